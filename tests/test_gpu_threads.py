# SPDX-License-Identifier: Apache-2.0
"""Launchers called from several host threads at once, on their own streams.

The Python bindings release the GIL around every launcher call, so threads
really overlap inside the library, including its one-time per-device setup
(kernel attributes, cluster capacity queries, the tensor-map encoder lookup,
the no-alloc scratch address).  A fresh process runs four threads that start
together, each writing its cache and running the MLA reader (several split
layouts), the no-alloc entry point (single pass: concurrent no-alloc calls
that need split scratch would share it) and a host staging copy on its own stream;
every result must equal the same work done afterwards on one thread.
"""
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

SCRIPT = textwrap.dedent(r"""
    import sys, threading
    sys.path[:0] = [{root!r}, {pkg!r}]
    import torch
    from kernels import titan_native
    from kernels.titan_io import copy_
    from kernels.titan_kv import store_int8
    from kernels.titan_mla import triton_mla_sparse_attention as attn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows, threads = 8192, 4
    inputs = []
    for k in range(threads):
        g = torch.Generator().manual_seed(100 + k)
        inputs.append((torch.randn(rows, 512, generator=g).to(torch.bfloat16).to(dev),
                       torch.randn(3, 16, 512, generator=g).to(torch.bfloat16).to(dev),
                       torch.randint(-16, rows, (3, 1, 2176), generator=g, dtype=torch.int32).to(dev),
                       torch.randint(0, 256, (25088,), generator=g, dtype=torch.uint8).pin_memory()))
    torch.cuda.synchronize()

    def work(k, results, barrier=None):
        lat, q, idx, host = inputs[k]
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            if barrier is not None:
                barrier.wait()
            cache = torch.empty(rows, 1, 528, dtype=torch.int8, device=dev)
            store_int8(lat, cache, torch.arange(rows, device=dev))
            outs = [attn(q, cache, idx, 0.05, num_kv_splits=s) for s in (0, 1, 16 >> k)]
            out_na = torch.empty_like(outs[0])
            rc = titan_native.load().titan_mla_sparse_attention_noalloc(
                q.data_ptr(), q.stride(0), q.stride(1), cache.data_ptr(), cache.stride(0), rows,
                idx.data_ptr(), idx.stride(0), 2176, out_na.data_ptr(), out_na.stride(0), out_na.stride(1),
                3, 16, 0.05, 1, torch._C._cuda_getCurrentRawStream(0))  # single pass: no shared scratch
            titan_native.check(rc, "noalloc")
            landing = torch.empty(host.numel(), dtype=torch.uint8, device=dev)
            copy_(landing, host)
        stream.synchronize()
        results[k] = [o.clone() for o in outs] + [out_na, cache.clone(), landing.cpu()]

    par = [None] * threads
    barrier = threading.Barrier(threads)
    ts = [threading.Thread(target=work, args=(k, par, barrier)) for k in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    seq = [None] * threads
    for k in range(threads):
        work(k, seq)
    for k in range(threads):
        assert par[k] is not None, k
        for a, b in zip(par[k], seq[k]):
            assert torch.equal(a.view(torch.uint8) if a.dtype != torch.uint8 else a,
                               b.view(torch.uint8) if b.dtype != torch.uint8 else b), k
        assert torch.equal(par[k][-1], inputs[k][3])
    assert titan_native.device_error(inputs[0][0]) == 0
    print("threads ok")
""")


def test_concurrent_first_use_from_threads(native_lib, cuda_device):
    code = SCRIPT.format(root=str(ROOT), pkg=str(ROOT / "glm-5.3-kernels_b200"))
    proc = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0 and "threads ok" in proc.stdout, proc.stdout[-2000:] + proc.stderr[-4000:]
