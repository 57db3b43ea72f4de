# SPDX-License-Identifier: Apache-2.0
"""Binding of libtitan_b200.so, the C ABI declared in include/titan_b200.h.

The library is loaded lazily (ctypes) on the first kernel call, so importing
the titan_* modules touches neither the library nor CUDA (the reference's
import contract, tests/test_cpu_contracts.py:33-53).  The hot launchers are
then called through `entry()`: the CPython fast-call module _titan_pybind
(lib/, built with the library) bound to the entry points of the loaded
library — ctypes' per-argument conversion costs ~3.7 us for the MLA launcher,
more than the decode kernel's own host launch.  When that module is absent the
same entry points are called through ctypes.  There is no compute fallback: a
missing library or a failed launch raises.
"""
import ctypes
import importlib.machinery
import importlib.util
import os
import sysconfig
import threading
import types
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parent.parent
_DEFAULT_LIB = _PKG_ROOT / "lib" / "libtitan_b200.so"

_lock = threading.Lock()
_lib = None
_entry = None

# entry() name -> C entry point
_HOT = {
    "mla": "titan_mla_sparse_attention",
    "mla_sem": "titan_mla_sparse_attention_sem",
    "mla_paged": "titan_mla_sparse_attention_paged",
    "copy": "titan_copy_ex",
    "store_int8": "titan_store_int8",
    "moe_align": "titan_moe_align_small",
    "convert": "titan_convert_req_index_to_global",
    "device_pointer": "titan_device_pointer",
}

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/titan_b200.h.
SIGNATURES = {
    "titan_abi_version": (_int, []),
    "titan_last_error": (ctypes.c_char_p, []),
    "titan_store_int8": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _int, _i64, _vp]),
    "titan_mla_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "titan_mla_max_active_clusters": (_int, [_int]),
    "titan_mla_max_exclusive_clusters": (_int, [_int]),
    "titan_mla_sparse_attention": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
         ctypes.c_float, _i64, _vp, _i64, _vp],
    ),
    "titan_mla_semaphore_count": (_i64, [_i64, _i64]),
    "titan_mla_sparse_attention_sem": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
         ctypes.c_float, _i64, _vp, _i64, _vp, _i64, _vp],
    ),
    "titan_convert_req_index_to_global": (
        _int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp]),
    "titan_mla_sparse_attention_paged": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
         _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _i64, _vp, _i64, _vp, _i64, _vp],
    ),
    "titan_mla_noalloc_scratch_bytes": (_i64, []),
    "titan_mla_sparse_attention_noalloc": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
         ctypes.c_float, _i64, _vp],
    ),
    "titan_moe_align_small": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _int, _vp]),
    "titan_moe_split_align": (
        _int, [_vp, _int, _i64, _i64, _vp, _i64, _i64, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, _vp]),
    "titan_moe_split_align_smem_bytes": (_i64, [_i64]),
    "titan_device_error": (_int, [ctypes.POINTER(_int), _int, _vp]),
    "titan_selftest_bounded_wait": (_int, [ctypes.c_longlong, _vp]),
    "titan_selftest_bounded_spin": (_int, [ctypes.c_longlong, _vp]),
    "titan_moe_w4a16_packed_bytes": (_i64, [_i64, _i64, _i64]),
    "titan_pool_topk_expand": (_int, [_vp, _i64, _vp, _i64, _int, _int, _vp, _i64, _int, _vp]),
    "titan_moe_w4a16_gemm": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _int, _int, _int,
                                    _i64, _i64, _i64, _vp]),
    "titan_copy": (_int, [_vp, _vp, _i64, _vp]),
    "titan_copy_ex": (_int, [_vp, _vp, _i64, _int, _vp]),
    "titan_device_pointer": (_int, [_vp, ctypes.POINTER(_vp)]),
}


class TitanError(RuntimeError):
    """A launcher of libtitan_b200.so returned a non-zero status."""


def library_path():
    return Path(os.environ.get("TITAN_B200_LIB", str(_DEFAULT_LIB)))


def load():
    """Return the loaded library (loading it on first use)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise TitanError(
                    f"{path} is missing: build it with `python glm-5.3-kernels_b200/build.py` "
                    "(there is no CPU or Triton fallback)")
            lib = ctypes.CDLL(str(path))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def _load_pybind(lib):
    """_titan_pybind from the library's directory, bound to `lib`, or None."""
    path = library_path().parent / ("_titan_pybind" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not path.exists():
        return None
    loader = importlib.machinery.ExtensionFileLoader("_titan_pybind", str(path))
    spec = importlib.util.spec_from_file_location("_titan_pybind", str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    mod.bind(*(ctypes.cast(getattr(lib, c_name), ctypes.c_void_p).value for c_name in _HOT.values()))
    return mod


def _ctypes_device_pointer(ptr):
    out = ctypes.c_void_p()
    rc = load().titan_device_pointer(ptr, ctypes.byref(out))
    return rc, out.value or 0


def entry():
    """The hot launchers (`mla`, `mla_sem`, `mla_paged`, `copy`, `store_int8`,
    `moe_align`, `convert`; positional arguments as in include/titan_b200.h,
    returning the status) and `device_pointer(ptr) -> (status, address)`: the
    fast-call module, else the same calls through ctypes."""
    global _entry
    if _entry is not None:
        return _entry
    lib = load()
    with _lock:
        if _entry is None:
            fast = None if os.environ.get("TITAN_B200_CTYPES_ONLY") else _load_pybind(lib)
            if fast is None:
                calls = {name: getattr(lib, c_name) for name, c_name in _HOT.items()}
                calls["device_pointer"] = _ctypes_device_pointer
                fast = types.SimpleNamespace(**calls)
            _entry = fast
    return _entry


def check(status, what):
    if status != 0:
        msg = load().titan_last_error().decode(errors="replace")
        raise TitanError(f"{what} failed (status {status}): {msg}")


def stream_of(tensor):
    """Raw handle of torch's current stream on the tensor's device."""
    import torch
    return torch._C._cuda_getCurrentRawStream(tensor.device.index)


class on_device:
    """Make `device` current for the launch (no-op when it already is)."""

    __slots__ = ("index", "prev")

    def __init__(self, device):
        self.index = device.index

    def __enter__(self):
        import torch
        self.prev = torch.cuda.current_device()
        if self.prev != self.index:
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        import torch
        if self.prev != self.index:
            torch.cuda.set_device(self.prev)
        return False


def device_error(tensor, clear=True):
    """Synchronise and read the device error word (0 = none)."""
    out = _int(0)
    check(load().titan_device_error(ctypes.byref(out), 1 if clear else 0, stream_of(tensor)),
          "titan_device_error")
    return out.value
