#!/usr/bin/env python3
# SPDX-License-Identifier: Apache-2.0
"""Generate tests/golden/split_align_golden.npz from the REFERENCE's own code.

    python tests/golden/make_split_align_golden.py --reference <path to GLM-5.3-Kernels checkout>

Runs profiles/sm74/titan_prefill/moe_split_align.py (`buffers` + `split_align`,
five Triton kernels) under the Triton interpreter on the CPU, with every output
buffer pre-filled with -2 so entries the algorithm leaves untouched are pinned
too.  It needs `vllm.triton_utils` (the module's only import besides torch) and
the reference checkout; the tests only read the committed .npz.

Cases (routes int32 unless noted, 288 experts):
  uniform_m2304  whole-expert prefill, M = 2304 tokens x top-8 uniform experts
  zipf_m512      M = 512, Zipf(1.1) expert popularity, no duplicate per token
  invalid_m37    M = 37, ids drawn from [-3, 291): invalid ids are dropped
  int64_wrap     M = 64 int64 ids, some >= 2^32 (narrowed to int32 first)
  one_expert     M = 300, every route to expert 7 (2400 rows in one expert)
  single_route   M = 1, top-1
  small_e        M = 100 over 3 experts, t_max well above T
"""
import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
UNWRITTEN = -2


def zipf_routes(rng, M, E, topk, s):
    w = 1.0 / np.arange(1, E + 1) ** s
    w /= w.sum()
    return np.stack([rng.choice(E, size=topk, replace=False, p=w) for _ in range(M)])


def cases():
    rng = np.random.default_rng(20261202)
    E = 288
    out = {
        "uniform_m2304": (rng.integers(0, E, (2304, 8)).astype(np.int32), E, 2304 * 8),
        "zipf_m512": (zipf_routes(rng, 512, E, 8, 1.1).astype(np.int32), E, 512 * 8),
        "invalid_m37": (rng.integers(-3, E + 3, (37, 8)).astype(np.int32), E, 37 * 8 + 40),
        "one_expert": (np.full((300, 8), 7, dtype=np.int32), E, 300 * 8),
        "single_route": (np.array([[201]], dtype=np.int32), E, 1),
        "small_e": (rng.integers(0, 3, (100, 8)).astype(np.int32), 3, 2000),
    }
    wrap = rng.integers(0, E, (64, 8)).astype(np.int64)
    wrap[::3, 1] += 2 ** 32          # narrows to a valid id
    wrap[1::5, 2] = 2 ** 32 - 1      # narrows to -1: dropped
    wrap[2::7, 3] = -(2 ** 33) + 5   # narrows to 5
    out["int64_wrap"] = (wrap, E, 64 * 8)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--out", type=Path, default=HERE / "split_align_golden.npz")
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / "profiles" / "sm74"))
    from titan_prefill import moe_split_align as ref

    arrays = {"sizes": np.array(ref.SIZES, dtype=np.int32)}
    names = []
    for name, (routes, E, t_max) in cases().items():
        buf = ref.buffers(t_max, E, torch.device("cpu"))
        for t in buf["s"] + buf["e"]:
            t.fill_(UNWRITTEN)
        lists = ref.split_align(torch.from_numpy(routes), E, buf)
        arrays[f"{name}/routes"] = routes
        arrays[f"{name}/meta"] = np.array([E, t_max], dtype=np.int64)
        arrays[f"{name}/ntpp"] = np.array([n.item() for _, _, _, n in lists], dtype=np.int32)
        for k, (bs, s, e, _) in enumerate(lists):
            arrays[f"{name}/sorted{k}"] = s.numpy().copy()
            arrays[f"{name}/experts{k}"] = e.numpy().copy()
        names.append(name)
        print(name, "ntpp", arrays[f"{name}/ntpp"].tolist())
    arrays["names"] = np.array(names)
    np.savez_compressed(args.out, **arrays)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
