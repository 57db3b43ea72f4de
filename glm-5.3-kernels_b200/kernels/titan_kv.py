# SPDX-License-Identifier: Apache-2.0
"""Per-token symmetric INT8 latent KV writer for B200 (sm_100a); no calibration.

Drop-in for the reference `store_int8` (kernels/titan_kv.py:23-28).  Each
512-value latent becomes one 528-byte cache row: 512 int8 values, the fp32
scale at byte 512 and 12 zero bytes.  The kernel is `titan_store_int8` in
libtitan_b200.so (csrc/titan_kv.cu).
"""
import torch

try:
    from . import titan_native as _native
except ImportError:  # imported as a top-level module, like the reference's py-modules
    import titan_native as _native

ROW_BYTES = 528
LATENT_DIM = 512


def store_int8(x, cache, slots):
    """Quantise x[i] into the cache row of slots[i] (slots < 0 are skipped).

    x: [N, 512] bf16 latents (the GLM-5.3 latent dtype), last dim contiguous.  cache: [num_blocks, block_size, 528]
    int8 or uint8, updated in place.  slots: integer tensor, flattened; only
    the first slots.numel() rows of x are used.  Launches on the current stream.
    """
    # Argument contract of kernels/titan_kv.py:24-26.
    assert x.shape[-1] == LATENT_DIM and cache.shape[-1] == ROW_BYTES
    slots = slots.flatten()
    assert slots.numel() <= x.shape[0]
    assert cache.dim() == 3, "cache must be [num_blocks, block_size, 528]"
    assert x.is_cuda and cache.is_cuda and slots.is_cuda, "store_int8 runs on CUDA tensors only"
    assert x.device == cache.device == slots.device, "x, cache and slots must share a device"
    n = slots.numel()
    if n == 0:
        return
    assert x.dtype == torch.bfloat16, "store_int8 on B200 takes bf16 latents"
    if x.dim() != 2:
        x = x.reshape(-1, LATENT_DIM)
    if x.stride(-1) != 1:
        x = x.contiguous()
    if slots.dtype not in (torch.int32, torch.int64):
        slots = slots.to(torch.int64)
    cache8 = cache.view(torch.int8)
    lib = _native.entry()
    with _native.on_device(x.device):
        rc = lib.store_int8(
            x.data_ptr(), x.stride(0), cache8.data_ptr(), cache8.shape[0], cache8.shape[1],
            cache8.stride(0), cache8.stride(1), slots.data_ptr(), 1 if slots.dtype == torch.int64 else 0,
            n, _native.stream_of(x))
    _native.check(rc, "store_int8")
