# SPDX-License-Identifier: Apache-2.0
"""Multi-process host logic of bench.py on CPU with world size 2 (gloo): token
sharding covers every request exactly once, the timing reduction takes the
max over ranks, and the reference arm runs on rank 0 only."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import bench
    d = bench.Dist(world, rank, 0, backend="gloo")
    try:
        blocks = {n: bench.token_block(n, world, rank) for n in (8, 4096, 3)}
        d.barrier()
        mx = d.max(float(10 * rank + 1))
        (Path(out_dir) / f"r{rank}.json").write_text(json.dumps({"blocks": blocks, "max": mx}))
    finally:
        d.close()


def test_sharding_and_max_over_ranks(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(world)]
    for n in ("8", "4096", "3"):
        covered = []
        for r in res:
            lo, hi = r["blocks"][n]
            covered += list(range(lo, hi))
        assert covered == list(range(int(n)))
    assert all(r["max"] == 11.0 for r in res)


def test_reference_arm_runs_on_rank0_only():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_token_block_edge_cases():
    sys.path.insert(0, str(ROOT))
    import bench
    assert [bench.token_block(8, 8, r) for r in range(8)] == [(r, r + 1) for r in range(8)]
    assert bench.token_block(8, 1, 0) == (0, 8)
    assert sum(hi - lo for lo, hi in (bench.token_block(5, 4, r) for r in range(4))) == 5
