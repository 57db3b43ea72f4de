# SPDX-License-Identifier: Apache-2.0
"""Kernel-driven host <-> device staging for latency-bound calls.

No counterpart in the reference (its callers keep every operand on the GPU).
A decode call moves ~25 KB in and 16 KB out; through the copy engine each
small pinned copy costs several microseconds of fixed latency.  `copy_` runs
libtitan_b200.so's `titan_copy` instead: a kernel on the current stream that
reads or writes the pinned host buffer through its device mapping.  For the
output side, `triton_mla_sparse_attention(..., out=<pinned host tensor>)`
lets the attention kernel store its result into host memory directly.
"""

import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native


def copy_(dst: torch.Tensor, src: torch.Tensor, *, src_ready: bool = False) -> torch.Tensor:
    """dst <- src, bytewise, by a kernel on the current stream of the CUDA side.

    Both tensors contiguous with the same number of bytes; one of them (or
    both) on a CUDA device, the other may be PINNED host memory.  Ordered
    after the stream's previous work; returns dst.  `src_ready=True` declares
    that no earlier work on the stream writes `src` (host-written input, say):
    the kernel then starts reading it before the preceding kernel has
    finished, and only its stores wait.
    """
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("copy_: tensors must be contiguous")
    nbytes = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != nbytes:
        raise ValueError("copy_: byte sizes differ")
    side = dst if dst.is_cuda else src
    if not side.is_cuda:
        raise ValueError("copy_: one side must be a CUDA tensor")
    for t in (dst, src):
        if t.is_cuda:
            if t.get_device() != side.get_device():
                raise ValueError("copy_: CUDA tensors on different devices")
        elif not t.is_pinned():
            raise ValueError("copy_: a host tensor must be pinned (tensor.pin_memory())")
    if nbytes == 0:
        return dst
    with _native.on_device(side.device):
        _native.check(_native.entry().copy(dst.data_ptr(), src.data_ptr(), nbytes, 1 if src_ready else 0,
                                           _native.stream_of(side)), "titan_io.copy_")
    return dst
