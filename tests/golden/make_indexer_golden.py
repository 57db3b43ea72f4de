#!/usr/bin/env python3
# SPDX-License-Identifier: Apache-2.0
"""Golden vectors of the indexer's pool expansion from the REFERENCE's own code.

    python tests/golden/make_indexer_golden.py --reference <GLM-5.3-Kernels checkout>

Runs the reference test's `expand_row` (tests/verify_indexer_sharding.py:68-76,
the CPU model of `kpool_ops.expand_pools_and_append_tail` /
`expand_pools_to_tokens`) on seeded pool lists and sequence lengths: 512
pools of 4 (the decode shape, 2051 entries), short and long contexts, -1
pools, every tail phase, pool size 1 and 4, with and without the tail.
Writes indexer_golden.npz next to this script.
"""
import argparse
import importlib.util
import random
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ref_verify_indexer",
                                                  args.reference / "tests" / "verify_indexer_sharding.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = random.Random(2026)
    out = {}
    cases = []
    for c in range(40):
        pool_size = 4 if c % 5 else 1
        k = 512 if c < 20 else rng.randint(1, 40)
        seq_len = rng.choice([0, 1, 2, 3, 4, 5, 7, 100, 2047, 2048, 2049, 2050, 2051, 8192 + rng.randint(0, 3),
                              262144 - rng.randint(0, 3)])
        npool = seq_len // pool_size
        pools = [rng.randrange(npool) if npool and rng.random() > 0.05 else -1 for _ in range(k)]
        tail = c % 3 != 0
        row = mod.expand_row(pools, seq_len, pool_size, tail)
        out[f"c{c}__pools"] = np.array(pools, np.int64)
        out[f"c{c}__meta"] = np.array([seq_len, pool_size, int(tail)], np.int64)
        out[f"c{c}__row"] = np.array(row, np.int64)
        cases.append(c)
    out["cases"] = np.array(cases, np.int64)
    np.savez_compressed(HERE / "indexer_golden.npz", **out)
    print("wrote indexer_golden.npz", len(cases), "cases")


if __name__ == "__main__":
    main()
