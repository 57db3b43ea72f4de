# SPDX-License-Identifier: Apache-2.0
"""Kernel-driven host <-> device staging (titan_copy) and the MLA reader
writing its output into pinned host memory (`out=`).

Copies must be bit-exact in every direction and size (16-byte vector body,
byte tail, unaligned offsets); pageable host memory is rejected on the host
before any launch; an attention call with a pinned host `out` gives the same
bits as the device-output call.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand_bytes(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)


@pytest.mark.parametrize("nbytes", [1, 15, 16, 17, 4096, 25088, 25095, 1 << 20, (64 << 20) + 48])
def test_copy_round_trip_bit_exact(nbytes, native_lib, cuda_device):
    from kernels.titan_io import copy_
    host = _rand_bytes(nbytes, nbytes).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    back = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
    copy_(dev, host)        # host -> device
    dev2 = torch.empty_like(dev)
    copy_(dev2, dev)        # device -> device
    copy_(back, dev2)       # device -> host
    dev3 = torch.empty_like(dev)
    copy_(dev3, host, src_ready=True)   # host-written source: loads start before the previous kernel ends
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), host)
    assert torch.equal(back, host)
    assert torch.equal(dev3.cpu(), host)


@pytest.mark.parametrize("shift", [1, 3, 8, 15])
def test_copy_unaligned_offsets(shift, native_lib, cuda_device):
    from kernels.titan_io import copy_
    n = 10000
    host = _rand_bytes(n + 32, shift).pin_memory()
    dev = torch.zeros(n + 32, dtype=torch.uint8, device=cuda_device)
    copy_(dev[shift:shift + n], host[0:n])
    copy_(dev[0:shift], host[n:n + shift])
    torch.cuda.synchronize()
    d = dev.cpu()
    assert torch.equal(d[shift:shift + n], host[0:n])
    assert torch.equal(d[0:shift], host[n:n + shift])
    assert not d[shift + n:].any()


def test_copy_rejects_pageable_and_overlap(native_lib, cuda_device):
    from kernels import titan_native
    from kernels.titan_io import copy_
    pageable = torch.zeros(64, dtype=torch.uint8)
    dev = torch.zeros(64, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError):
        copy_(dev, pageable)
    lib = titan_native.load()
    # Straight through the C ABI: the host-side check refuses, nothing launches.
    rc = lib.titan_copy(dev.data_ptr(), pageable.data_ptr(), 64, titan_native.stream_of(dev))
    assert rc == 1 and b"pageable" in lib.titan_last_error()
    rc = lib.titan_copy(dev.data_ptr() + 8, dev.data_ptr(), 32, titan_native.stream_of(dev))
    assert rc == 1 and b"overlap" in lib.titan_last_error()
    rc = lib.titan_copy_ex(dev.data_ptr(), dev.data_ptr() + 32, 16, 4, titan_native.stream_of(dev))
    assert rc == 1 and b"flags" in lib.titan_last_error()
    p = ctypes.c_void_p()
    assert lib.titan_device_pointer(pageable.data_ptr(), ctypes.byref(p)) == 1
    pinned = torch.zeros(64, dtype=torch.uint8).pin_memory()
    assert lib.titan_device_pointer(pinned.data_ptr(), ctypes.byref(p)) == 0 and p.value
    assert lib.titan_device_pointer(dev.data_ptr(), ctypes.byref(p)) == 0 and p.value == dev.data_ptr()
    torch.cuda.synchronize()


@pytest.mark.parametrize("tokens,splits", [(1, 0), (1, 1), (3, 0), (8, 0), (8, 1), (160, 0)])
def test_mla_pinned_host_output_matches(tokens, splits, native_lib, cuda_device):
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    g = torch.Generator().manual_seed(tokens * 10 + splits)
    rows, topk = 8192, 2176
    cache = torch.empty(rows // 256, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(torch.randn(rows, 512, generator=g).to(torch.bfloat16).to(cuda_device), cache,
               torch.arange(rows, device=cuda_device))
    kv = cache.view(rows, 1, 528)
    q = torch.randn(tokens, 16, 512, generator=g).to(torch.bfloat16).to(cuda_device)
    idx = torch.randint(-64, rows, (tokens, 1, topk), generator=g, dtype=torch.int32).to(cuda_device)
    ref = attn(q, kv, idx, 512 ** -0.5, num_kv_splits=splits)
    host = torch.full((tokens, 16, 512), float("nan"), dtype=torch.bfloat16).pin_memory()
    got = attn(q, kv, idx, 512 ** -0.5, num_kv_splits=splits, out=host)
    torch.cuda.synchronize()
    assert got is host
    assert torch.equal(host.view(torch.int16), ref.cpu().view(torch.int16))
    dev_out = torch.empty_like(ref)
    attn(q, kv, idx, 512 ** -0.5, num_kv_splits=splits, out=dev_out)
    assert torch.equal(dev_out.view(torch.int16), ref.view(torch.int16))
    with pytest.raises(AssertionError):
        attn(q, kv, idx, 512 ** -0.5, out=torch.empty(tokens, 16, 512, dtype=torch.bfloat16))  # pageable


def test_src_ready_copy_waits_for_the_previous_reader(native_lib, cuda_device):
    """With src_ready the copy's loads may start early, but its stores into a
    landing buffer still wait for the kernel reading that buffer: a chain of
    copy -> attention steps on one landing buffer gives every step's own result."""
    from kernels.titan_io import copy_
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    g = torch.Generator().manual_seed(5)
    rows, steps = 8192, 12
    cache = torch.empty(rows, 1, 528, dtype=torch.int8, device=cuda_device)
    store_int8(torch.randn(rows, 512, generator=g).to(torch.bfloat16).to(cuda_device), cache,
               torch.arange(rows, device=cuda_device))
    q = torch.randn(steps, 1, 16, 512, generator=g).to(torch.bfloat16)
    idx = torch.randint(-8, rows, (steps, 1, 1, 2176), generator=g, dtype=torch.int32)
    staging = torch.cat([q.reshape(steps, -1).view(torch.uint8), idx.reshape(steps, -1).view(torch.uint8)], 1)
    staging = staging.pin_memory()
    nq = q[0].numel() * 2
    landing = torch.empty(staging.shape[1], dtype=torch.uint8, device=cuda_device)
    outs = torch.empty(steps, 1, 16, 512, dtype=torch.bfloat16).pin_memory()
    for k in range(steps):
        copy_(landing, staging[k], src_ready=True)
        attn(landing[:nq].view(torch.bfloat16).view(1, 16, 512), cache, landing[nq:].view(torch.int32).view(1, 1, 2176),
             0.05, out=outs[k])
    torch.cuda.synchronize()
    for k in range(steps):
        ref = attn(q[k].to(cuda_device), cache, idx[k].to(cuda_device), 0.05)
        assert torch.equal(outs[k].view(torch.int16), ref.cpu().view(torch.int16)), k
