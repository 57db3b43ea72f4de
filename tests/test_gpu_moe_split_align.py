# SPDX-License-Identifier: Apache-2.0
"""Split MoE block alignment on the GPU (csrc/titan_moe_split_align.cu) against
the reference-generated golden buffers and the CPU oracle, bit-exact.

Whole buffers are compared where the lists were pre-filled with a marker, so
entries the algorithm must leave untouched are checked too."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
GOLDEN = C.__file__.rsplit("/", 1)[0]


def _run(routes, E, t_max, device, dtype=None):
    from kernels import titan_moe_split_align as S
    buf = S.buffers(t_max, E, device)
    for t in buf["s"] + buf["e"]:
        t.fill_(O.SPLIT_UNWRITTEN)
    ids = torch.as_tensor(np.asarray(routes))
    if dtype is not None:
        ids = ids.to(dtype)
    out = S.split_align(ids.to(device), E, buf)
    return [(bs, s.cpu().numpy(), e.cpu().numpy(), int(n.item())) for bs, s, e, n in out]


def _assert_equal(got, want, what):
    for k, ((bs, s, e, n), (wbs, ws, we, wn)) in enumerate(zip(got, want)):
        assert bs == wbs and n == wn, (what, k, n, wn)
        assert np.array_equal(s, ws), (what, k, np.nonzero(s != ws)[0][:8])
        assert np.array_equal(e, we), (what, k, np.nonzero(e != we)[0][:8])


def test_golden_buffers(native_lib, cuda_device):
    gold = np.load(f"{GOLDEN}/split_align_golden.npz")
    for name in gold["names"]:
        E, t_max = (int(v) for v in gold[f"{name}/meta"])
        want = [(int(bs), gold[f"{name}/sorted{k}"], gold[f"{name}/experts{k}"], int(gold[f"{name}/ntpp"][k]))
                for k, bs in enumerate(gold["sizes"])]
        _assert_equal(_run(gold[f"{name}/routes"], E, t_max, cuda_device), want, str(name))


@pytest.mark.parametrize("M,topk,E,dist", [
    (1, 8, 288, "uniform"), (7, 8, 288, "uniform"), (333, 8, 288, "uniform"), (2304, 8, 288, "uniform"),
    (4096, 8, 288, "zipf"), (8192, 8, 288, "uniform"), (512, 8, 1024, "uniform"), (300, 8, 1, "uniform"),
    (1000, 6, 257, "zipf"), (64, 8, 288, "invalid"),
])
def test_against_oracle(native_lib, cuda_device, M, topk, E, dist):
    """Sizes from one token to T = 65,536 rows, 1 to 1024 experts (the
    shared-memory limit), skewed and invalid ids, and t_max above T."""
    rng = np.random.default_rng(M * 1000 + E)
    if dist == "zipf":
        w = 1.0 / np.arange(1, E + 1) ** 1.1
        routes = rng.choice(E, size=(M, topk), p=w / w.sum())
    elif dist == "invalid":
        routes = rng.integers(-5, E + 5, (M, topk))
    else:
        routes = rng.integers(0, E, (M, topk))
    routes = routes.astype(np.int32)
    t_max = M * topk + 17
    _assert_equal(_run(routes, E, t_max, cuda_device), O.moe_split_align(routes, E, t_max), (M, E, dist))
    if M <= 512:  # int64 ids give the same lists
        _assert_equal(_run(routes, E, t_max, cuda_device, torch.int64), O.moe_split_align(routes, E, t_max), "i64")


def test_reused_buffers_and_graph_replay(native_lib, cuda_device):
    """One buffer set serves successive calls (defined regions are rewritten each
    call), including replays of a CUDA graph that captured the launch."""
    from kernels import titan_moe_split_align as S
    E, M = 288, 2304
    buf = S.buffers(M * 8, E, cuda_device)
    ids = torch.zeros(M, 8, dtype=torch.int32, device=cuda_device)
    rng = np.random.default_rng(5)

    def check(routes):
        want = O.moe_split_align(routes, E, M * 8)
        for k in range(4):
            n = want[k][3]
            assert int(buf["ntpp"][k].item()) == n
            bs = want[k][0]
            assert np.array_equal(buf["s"][k][:n].cpu().numpy(), want[k][1][:n])
            assert np.array_equal(buf["e"][k][:n // bs].cpu().numpy(), want[k][2][:n // bs])

    for _ in range(2):
        routes = rng.integers(0, E, (M, 8)).astype(np.int32)
        ids.copy_(torch.from_numpy(routes))
        S.split_align(ids, E, buf)
        check(routes)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        S.split_align(ids, E, buf)
    for skew in (None, 1.1):
        if skew is None:
            routes = rng.integers(0, E, (M, 8)).astype(np.int32)
        else:
            w = 1.0 / np.arange(1, E + 1) ** skew
            routes = rng.choice(E, size=(M, 8), p=w / w.sum()).astype(np.int32)
        ids.copy_(torch.from_numpy(routes))
        graph.replay()
        torch.cuda.synchronize()
        check(routes)
    del graph


def test_errors(native_lib, cuda_device):
    from kernels import titan_moe_split_align as S
    buf = S.buffers(16, 288, cuda_device)
    with pytest.raises(AssertionError):
        S.split_align(torch.zeros(3, 8, dtype=torch.int32, device=cuda_device), 288, buf)  # T > t_max
    with pytest.raises(AssertionError):
        S.split_align(torch.zeros(1, 8, dtype=torch.int32, device=cuda_device), 287, buf)  # E mismatch
    with pytest.raises(AssertionError):
        S.split_align(torch.zeros(0, 8, dtype=torch.int32, device=cuda_device), 288, buf)  # T == 0


def test_int64_ids_narrowed_like_the_reference(native_lib, cuda_device):
    """int64 ids that do not fit in int32 are narrowed by wrapping, as the
    reference's `.to(torch.int32)` does (moe_split_align.py:207-209): 2^32 + 5
    becomes expert 5, -2^32 + 3 becomes 3, 2^31 becomes -2^31 (dropped)."""
    E, t_max = 288, 64
    wide = np.array([[2 ** 32 + 5, -(2 ** 32) + 3, 2 ** 31, 7, 2 ** 33 + 287, -1, 2 ** 32 + 288, 5]], np.int64)
    want = O.moe_split_align(wide, E, t_max)
    narrowed = torch.from_numpy(wide).to(torch.int32).numpy()
    assert narrowed.tolist() == [[5, 3, -2 ** 31, 7, 287, -1, 288, 5]]
    _assert_equal(want, O.moe_split_align(narrowed, E, t_max), "oracle wraps like torch")
    _assert_equal(_run(wide, E, t_max, cuda_device, torch.int64), want, "kernel")


def test_noncontiguous_ids_and_foreign_buffers(native_lib, cuda_device):
    """A strided id view gives the contiguous ids' lists; buffers on another
    device than the ids are refused."""
    from kernels import titan_moe_split_align as S
    rng = np.random.default_rng(11)
    wide = torch.from_numpy(rng.integers(0, 288, (64, 16)).astype(np.int32)).to(cuda_device)
    view = wide.reshape(-1)[::2]                          # 1-D, stride 2: reshape(-1) keeps the view
    assert not view.is_contiguous()
    buf = S.buffers(512, 288, cuda_device)
    got = [(bs, s.cpu().numpy(), e.cpu().numpy(), int(n.item())) for bs, s, e, n in S.split_align(view, 288, buf)]
    want = O.moe_split_align(view.cpu().numpy(), 288, 512)
    for (bs, s, e, n), (_, ws, we, wn) in zip(got, want):
        assert n == wn and np.array_equal(s[:n], ws[:n]) and np.array_equal(e[:n // bs], we[:n // bs])
    cpu_buf = S.buffers(512, 288, torch.device("cpu"))
    with pytest.raises(ValueError):
        S.split_align(view, 288, cpu_buf)


def test_eight_cta_cluster(native_lib, cuda_device, tmp_path):
    """The portable 8-CTA cluster (what a device that cannot hold a 16-CTA
    cluster runs), forced by TITAN_SPLIT_ALIGN_CLUSTER=8 in a fresh process:
    bit-exact against the oracle for several sizes, expert counts and skews."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    script = tmp_path / "split8.py"
    script.write_text(f"""
import sys
sys.path[:0] = [{str(root)!r}, {str(root / 'glm-5.3-kernels_b200')!r}]
import numpy as np, torch
from tests.test_gpu_moe_split_align import _run, _assert_equal
from oracle import oracle as O
dev = torch.device('cuda:0')
for M, E, zipf in ((1, 288, False), (333, 288, False), (2304, 288, True), (8192, 288, False), (512, 1024, False)):
    rng = np.random.default_rng(M + E)
    if zipf:
        w = 1.0 / np.arange(1, E + 1) ** 1.1
        routes = rng.choice(E, size=(M, 8), p=w / w.sum()).astype(np.int32)
    else:
        routes = rng.integers(-2, E + 2, (M, 8)).astype(np.int32)
    _assert_equal(_run(routes, E, M * 8 + 5, dev), O.moe_split_align(routes, E, M * 8 + 5), (M, E))
print('split8 ok')
""")
    env = dict(__import__("os").environ, TITAN_SPLIT_ALIGN_CLUSTER="8")
    r = subprocess.run([sys.executable, str(script)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "split8 ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
