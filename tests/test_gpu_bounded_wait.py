# SPDX-License-Identifier: Apache-2.0
"""Failure reporting of the bounded waits, without a GPU fault.

Every wait in the kernels is bounded: a wait that runs out sets the device
error word (read by titan_device_error) and the kernel returns instead of
trapping.  The self-test kernels wait on an mbarrier that nothing completes
and on a counter that nothing increments, so their waits run out by
construction; the host then reads the status, and
the context is shown to be usable by a normal call checked against the
oracle.
"""
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_is_reported_and_context_survives(native_lib, cuda_device):
    from kernels import titan_native
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    probe = torch.zeros(1, device=cuda_device)
    assert titan_native.device_error(probe) == 0
    stream = titan_native.stream_of(probe)
    titan_native.check(native_lib.titan_selftest_bounded_wait(2_000_000, stream), "selftest")  # ~1 ms
    assert titan_native.device_error(probe, clear=False) == 1   # kDevErrMbarrierTimeout, reported
    assert titan_native.device_error(probe) == 1                 # read and clear
    assert titan_native.device_error(probe) == 0
    with pytest.raises(titan_native.TitanError):
        titan_native.check(native_lib.titan_selftest_bounded_wait(0, stream), "selftest")
    # The flat split merge's counter wait: a counter nothing increments.
    titan_native.check(native_lib.titan_selftest_bounded_spin(2_000_000, stream), "selftest")
    assert titan_native.device_error(probe) == 3                 # kDevErrSpinTimeout
    assert titan_native.device_error(probe) == 0
    with pytest.raises(titan_native.TitanError):
        titan_native.check(native_lib.titan_selftest_bounded_spin(0, stream), "selftest")

    g = torch.Generator().manual_seed(3)
    n = 4096
    latent = torch.randn(n, 512, generator=g).to(torch.bfloat16)
    cache = torch.zeros(n // 256, 256, 528, dtype=torch.int8, device=cuda_device)
    store_int8(latent.to(cuda_device), cache, torch.arange(n, device=cuda_device))
    q = torch.randn(2, 16, 512, generator=g).to(torch.bfloat16)
    idx = torch.randint(-8, n, (2, 1, 512), generator=g, dtype=torch.int32)
    out = attn(q.to(cuda_device), cache.view(n, 1, 528), idx.to(cuda_device), 512 ** -0.5, sm_count=148)
    ref = O.mla_sparse_attention(q, cache.view(n, 528).cpu(), idx, 512 ** -0.5)
    assert bool(((out.float().cpu() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all())
    assert titan_native.device_error(probe) == 0
