"""Build libtitan_b200.so (all sm_100a kernels + the C ABI) in-tree.

    python glm-5.3-kernels_b200/build.py [--force]

Output: glm-5.3-kernels_b200/lib/libtitan_b200.so.  One translation unit
(csrc/titan_b200.cu), cudart linked statically so the library needs nothing
but the NVIDIA driver at run time.  No fast-math: the INT8 writer's
quantisation must round exactly like IEEE fp32.

Also lib/_titan_pybind<EXT_SUFFIX>: the CPython fast-call bindings of the hot
launchers (csrc/titan_pybind.c, plain C against this interpreter's headers;
it does not link the library, titan_native binds it to the loaded copy).
"""
import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib" / "libtitan_b200.so"
INCLUDE = PKG.parent / "include"
PYBIND_SRC = CSRC / "titan_pybind.c"
PYBIND = PKG / "lib" / ("_titan_pybind" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date(target, srcs):
    if not target.exists():
        return False
    built = target.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in srcs)


def build_pybind(force=False):
    """Compile the CPython fast-call bindings (C, no CUDA).  Returns the path."""
    if not force and up_to_date(PYBIND, [PYBIND_SRC, *INCLUDE.glob("*.h")]):
        return PYBIND
    PYBIND.parent.mkdir(parents=True, exist_ok=True)
    tmp = PYBIND.with_name(PYBIND.name + ".tmp")
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    subprocess.run([cc, "-O2", "-fPIC", "-shared", "-std=gnu11", "-Wall", "-Werror",
                    "-I", sysconfig.get_paths()["include"], "-o", str(tmp), str(PYBIND_SRC)], check=True)
    os.replace(tmp, PYBIND)
    return PYBIND


def build(force=False, verbose=False):
    """Compile the library unless it is newer than every source, and the
    bindings.  Returns the library's path."""
    build_pybind(force)
    if not force and up_to_date(LIB, sources()):
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "titan_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
