# SPDX-License-Identifier: Apache-2.0
"""INT8 KV writer on the GPU vs the CPU oracle: bit-exact bytes."""
import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import oracle as O
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
GOLDEN = C.__file__.rsplit("/", 1)[0]


def _c_rows(x_bf16):
    bits = np.ascontiguousarray(O.tensor_bf16_bits(x_bf16))
    rows = np.zeros((bits.shape[0], 528), np.uint8)
    c_oracle().oracle_store_int8_rows(bits.ctypes.data, bits.shape[0], rows.ctypes.data)
    return rows


def test_golden_bytes(native_lib, cuda_device):
    from kernels.titan_kv import store_int8
    gold = np.load(f"{GOLDEN}/kv_golden.npz")
    x = C.kv_latents().to(cuda_device)
    for slot_dtype in (torch.int64, torch.int32):
        cache = torch.zeros(C.KV_BLOCKS, C.KV_BLOCK_SIZE, 528, dtype=torch.int8, device=cuda_device)
        store_int8(x, cache, C.kv_slots().to(slot_dtype).to(cuda_device))
        assert np.array_equal(cache.cpu().numpy().view(np.uint8), gold["cache"]), slot_dtype


@pytest.mark.parametrize("kernel", ["stream", "unaligned"])
def test_nonfinite_rows_every_kernel(native_lib, cuda_device, kernel):
    """The golden rows (NaN and inf rows among them) on the streaming kernel
    (>= 1024 rows: the 128 golden rows tiled 32 times, shuffled) and on the
    unaligned-row kernel: bytes equal the golden-pinned oracle's."""
    from kernels.titan_kv import store_int8
    gold = np.load(f"{GOLDEN}/kv_golden.npz")
    x = C.kv_latents()
    assert not torch.isfinite(x.float()).all(1).all()
    g = torch.Generator().manual_seed(5)
    if kernel == "stream":
        xs = x.repeat(32, 1)[torch.randperm(32 * x.shape[0], generator=g)]
        src = xs.to(cuda_device)
    else:
        xs = x
        wide = torch.zeros(x.shape[0], 520, dtype=torch.bfloat16)
        wide[:, 3:515] = x
        src = wide.to(cuda_device)[:, 3:515]            # rows 6 bytes off 16-byte alignment
    n = xs.shape[0]
    cache = torch.zeros((n + 255) // 256, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(src, cache, torch.arange(n, device=cuda_device))
    got = cache.view(-1, 528)[:n].cpu().numpy().view(np.uint8)
    want = O.store_int8_rows(O.tensor_bf16_bits(xs))
    assert np.array_equal(got, want)
    assert np.array_equal(_c_rows(xs), want)
    if kernel == "unaligned":
        flat = gold["cache"].reshape(-1, 528)
        keep = gold["slots"] >= 0
        assert np.array_equal(got[keep], flat[gold["slots"][keep]])


def test_uint8_cache_and_unaligned_rows(native_lib, cuda_device):
    """A uint8 cache and an x view whose rows are not 16-byte aligned (scalar kernel)."""
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(3)
    big = torch.randn(96, 520, generator=g).to(torch.bfloat16)
    x_cpu = big[:, 3:515]
    cache = torch.zeros(1, 128, 528, dtype=torch.uint8, device=cuda_device)
    slots = torch.randperm(128, generator=g)[:96]
    store_int8(big.to(cuda_device)[:, 3:515], cache, slots.to(cuda_device))
    want = np.zeros((1, 128, 528), np.uint8)
    O.store_int8(O.tensor_bf16_bits(x_cpu), want, slots.numpy())
    assert np.array_equal(cache.cpu().numpy(), want)


def test_negative_and_out_of_range_slots_leave_cache(native_lib, cuda_device):
    """tests/verify_mla.py:67-69: a negative slot modifies nothing.  A slot past
    the last block is skipped too."""
    from kernels.titan_kv import store_int8
    x = C.kv_latents()[:4].to(cuda_device)
    cache = torch.full((2, 4, 528), 7, dtype=torch.int8, device=cuda_device)
    before = cache.clone()
    store_int8(x, cache, torch.tensor([-1, -5, 8, 1 << 40], device=cuda_device))
    assert torch.equal(cache, before)
    store_int8(x[:0], cache, torch.empty(0, dtype=torch.int64, device=cuda_device))
    assert torch.equal(cache, before)


def test_block_strided_cache(native_lib, cuda_device):
    """Cache viewed out of a larger allocation: block stride != block_size * 528."""
    from kernels.titan_kv import store_int8
    x = C.kv_latents()[:64]
    storage = torch.zeros(3, 40, 528, dtype=torch.int8, device=cuda_device)
    cache = storage[:, 4:36]                       # [3, 32, 528], stride0 = 40 * 528
    slots = torch.arange(64) * 5 % 96                 # distinct slots (5 is coprime with 96)
    store_int8(x.to(cuda_device), cache, slots.to(cuda_device))
    want = np.zeros((3, 32, 528), np.uint8)
    O.store_int8(O.tensor_bf16_bits(x), want, slots.numpy())
    assert np.array_equal(cache.cpu().numpy().view(np.uint8), want)
    assert not storage[:, :4].any() and not storage[:, 36:].any()


@pytest.mark.parametrize("order", ["arange", "permutation"])
def test_full_cache_fill_bit_exact(native_lib, cuda_device, order):
    """The production cache fill (262,144 rows, slots in order) and the same
    fill with a random slot permutation, byte for byte against the C oracle,
    plus the reference test's
    quantisation criteria (tests/verify_mla.py:50-66)."""
    from kernels.titan_kv import store_int8
    n = 262144
    g = torch.Generator().manual_seed(20260910)
    x = torch.randn(n, 512, generator=g)
    x[:, :128] *= 0.05
    x[:, 256:384] *= 8
    x = x.to(torch.bfloat16)
    x[0] = 0
    slots = torch.arange(n) if order == "arange" else torch.randperm(n, generator=g)
    cache = torch.zeros(n // 256, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(x.to(cuda_device), cache, slots.to(cuda_device))
    got = cache.cpu().numpy().view(np.uint8).reshape(n, 528)
    rows = _c_rows(x)
    assert np.array_equal(got[slots.numpy()], rows)
    scales = rows[:, 512:516].copy().view(np.float32)[:, 0]
    xf = x.float().numpy()
    deq = (rows[:, :512].view(np.int8).astype(np.float32) * scales[:, None])
    deq = torch.from_numpy(deq).to(torch.bfloat16).float().numpy()
    nmse = float(((deq - xf) ** 2).sum() / (xf ** 2).sum())
    assert nmse < 3e-4


@pytest.mark.parametrize("n,slot_dtype", [(5000, torch.int32), (4097, torch.int64)])
def test_bulk_path_partial_chunks(native_lib, cuda_device, n, slot_dtype):
    """Contiguous latents above the bulk-path threshold with a row count that
    leaves a partial last chunk, some negative slots, random slot order."""
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, 512, generator=g).to(torch.bfloat16)
    slots = torch.randperm(8192, generator=g)[:n]
    slots[::97] = -1
    cache = torch.zeros(32, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(x.to(cuda_device), cache, slots.to(slot_dtype).to(cuda_device))
    want = np.zeros((32, 256, 528), np.uint8)
    O.store_int8(O.tensor_bf16_bits(x), want, slots.numpy())
    assert np.array_equal(cache.cpu().numpy().view(np.uint8), want)


def test_graph_capture_replay(native_lib, cuda_device):
    from kernels.titan_kv import store_int8
    x = C.kv_latents().to(cuda_device)
    slots = C.kv_slots().to(cuda_device)
    cache = torch.zeros(C.KV_BLOCKS, C.KV_BLOCK_SIZE, 528, dtype=torch.int8, device=cuda_device)
    store_int8(x, cache, slots)  # warm-up outside capture
    want = cache.clone()
    cache.zero_()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            store_int8(x, cache, slots)
    torch.cuda.current_stream().wait_stream(s)
    cache.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(cache, want)
    graph.reset()


def test_every_bf16_magnitude_as_row_max(native_lib, cuda_device):
    """One row per non-negative finite bf16 amax (32,640 rows, all scales the
    writer can produce, subnormal to near-max), other values uniform in
    [-amax, amax]: bytes bit-exact against the C oracle (IEEE division)."""
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(17)
    amax = torch.arange(0x7F80, dtype=torch.int32).mul(1 << 16).view(torch.float32)
    x = (torch.rand(amax.numel(), 512, generator=g, dtype=torch.float64) * 2 - 1) * amax[:, None].double()
    x = x.to(torch.float32).to(torch.bfloat16)
    x[:, 7] = amax.to(torch.bfloat16)                       # exact bf16: amax itself
    x[1::2, 7] = -x[1::2, 7]
    n = x.shape[0]
    cache = torch.zeros((n + 255) // 256, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(x.to(cuda_device), cache, torch.arange(n, device=cuda_device))
    got = cache.view(-1, 528)[:n].cpu().numpy().view(np.uint8)
    assert np.array_equal(got, _c_rows(x))


@pytest.mark.parametrize("n", [100, 3000])
def test_non_power_of_two_block_size(native_lib, cuda_device, n):
    """Blocks of 48 rows (the writer divides instead of shifting), on the
    small-batch (n < 1024) and the streaming (n >= 1024) kernels, with skipped
    slots: bytes bit-exact against the oracle, untouched rows stay zero."""
    from kernels.titan_kv import store_int8
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, 512, generator=g).to(torch.bfloat16)
    blocks = (n + 200) // 48 + 1
    slots = torch.randperm(blocks * 48, generator=g)[:n]
    slots[::17] = -1
    cache = torch.zeros(blocks, 48, 528, dtype=torch.int8, device=cuda_device)
    store_int8(x.to(cuda_device), cache, slots.to(cuda_device))
    want = np.zeros((blocks, 48, 528), np.uint8)
    O.store_int8(O.tensor_bf16_bits(x), want, slots.numpy())
    assert np.array_equal(cache.cpu().numpy().view(np.uint8), want)
