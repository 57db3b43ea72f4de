#!/usr/bin/env python3
# SPDX-License-Identifier: Apache-2.0
"""Generate the golden fixtures under tests/golden/ from the REFERENCE's own code.

    python tests/golden/make_golden.py --reference <path to GLM-5.3-Kernels checkout>

Runs only where the reference checkout exists (it is not needed at test time:
the tests read the committed .npz files).  Sources of truth:

* MoE align (moe_golden.npz): benchmarks/moe_align.py `cpu_reference`, checked
  equal to `cpu_pairwise`, over the reference's own 856-case sweep
  (`make_patterns` + 100 random routes per batch, random.Random(37),
  benchmarks/moe_align.py:49-66); plus kernels/titan_moe_align.py `_align_small`
  executed by the Triton interpreter on the 56 named patterns x int32/int64.
* KV writer (kv_golden.npz): kernels/titan_kv.py `store_int8` executed by the
  Triton interpreter on seeded bf16 latents with edge rows.
* Sparse MLA (mla_golden.npz): kernels/titan_mla.py `triton_mla_sparse_attention`
  executed by the Triton interpreter (final, split and merge kernels).
* Paged index conversion (index_golden.npz): vLLM's
  `triton_convert_req_index_to_global_index`, which the reference's backend
  calls before the reader (integration/titan_backend.py:49-52), executed by the
  Triton interpreter (vLLM version recorded in the file).

The interpreter needs four shims, all inside this script and none in the
reference's code: libdevice `nearbyint` (absent from the interpreter) is
np.rint (round half to even, as nearbyint in the default mode); bf16 casts
round to nearest even through torch (the interpreter stores bf16 as raw
uint16 bits and would otherwise convert integers to bits); `tl.dot` on
bf16 operands multiplies exactly in fp32 with fp32 accumulation (the
interpreter would otherwise multiply the raw bits); and elementwise
`tl.maximum` / `tl.minimum` drop a NaN operand (np.fmax / np.fmin), as
their default PropagateNan.NONE form does on the GPU, where they lower to
maxnum / minnum (the interpreter's `tl.max` reduction already drops NaN
with np.nanmax, but its elementwise forms would propagate it).  Fp32
division in the interpreter is IEEE division.  The autotuned MLA kernels are run with their
first listed config (the interpreter has no benchmarker).

MLA inputs are regenerated in the tests from the recorded seeds with torch's
CPU generator; each case stores a SHA-256 of its inputs so a changed generator
is caught instead of silently compared.
"""
import argparse
import hashlib
import importlib.util
import os
import random
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from tests.golden import cases as C  # noqa: E402


# ------------------------------------------------------------ interpreter shims
def install_interpreter_shims():
    import triton.language as tl
    import triton.runtime.interpreter as interp
    from triton.runtime.interpreter import TensorHandle

    def bf16_bits_to_f32(bits):
        return (bits.astype(np.uint32) << 16).view(np.float32)

    def f32_to_bf16_bits(f):
        t = torch.from_numpy(np.ascontiguousarray(f, dtype=np.float32)).to(torch.bfloat16)
        return t.view(torch.int16).numpy().view(np.uint16)

    def extern_elementwise(self, lib_name, lib_path, symbol, args, ret_type, is_pure):
        if symbol == "__nv_nearbyintf":
            a = args[0]
            return TensorHandle(np.rint(a.data).astype(a.data.dtype), a.dtype.scalar)
        raise NotImplementedError(symbol)

    orig_cast = interp.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if d == tl.bfloat16 and s != tl.bfloat16:
            return TensorHandle(f32_to_bf16_bits(src.data.astype(np.float32)).reshape(src.data.shape), d)
        if s == tl.bfloat16 and d != tl.bfloat16:
            return TensorHandle(bf16_bits_to_f32(src.data).astype(interp._get_np_dtype(dst_type)), d)
        return orig_cast(self, src, dst_type)

    orig_dot = interp.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            af = bf16_bits_to_f32(a.data) if a.dtype.scalar == tl.bfloat16 else a.data.astype(np.float32)
            bf = bf16_bits_to_f32(b.data) if b.dtype.scalar == tl.bfloat16 else b.data.astype(np.float32)
            return TensorHandle(np.matmul(af, bf, dtype=np.float32) + d.data, d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    B = interp.InterpreterBuilder
    # tl.maximum / tl.minimum with the default PropagateNan.NONE are maxnumf /
    # minnumf, which return the non-NaN operand when compiled for the GPU
    # (and the interpreter's own tl.max reduction already uses np.nanmax);
    # the interpreter's elementwise forms would propagate NaN instead.
    B.create_maxnumf = lambda self, lhs, rhs: self.binary_op(lhs, rhs, np.fmax)
    B.create_minnumf = lambda self, lhs, rhs: self.binary_op(lhs, rhs, np.fmin)
    B.create_extern_elementwise = extern_elementwise
    B.cast_impl = cast_impl
    B.create_si_to_fp = lambda self, src, dst_type: cast_impl(self, src, dst_type)
    B.create_fp_to_fp = lambda self, src, dst_type, rounding_mode: cast_impl(self, src, dst_type)
    B.create_fp_ext = lambda self, src, dst_type: cast_impl(self, src, dst_type)
    B.create_fp_trunc = lambda self, src, dst_type: cast_impl(self, src, dst_type)
    B.create_dot = create_dot
    orig_patch_lang = interp._patch_lang

    def patch_lang(fn):
        scope = orig_patch_lang(fn)
        interp._patch_builtin(tl.extra.cuda.libdevice, interp.interpreter_builder, scope)
        return scope

    interp._patch_lang = patch_lang


def load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def pin_autotuned(auto, **cfg):
    jit = auto.fn

    class Pinned:
        def __getitem__(self, grid):
            return lambda *a, **k: jit[grid](*a, **k, **cfg)

    return Pinned()


# ------------------------------------------------------------------ generators
def gen_moe(ref):
    bench = load_module("ref_moe_bench", ref / "benchmarks" / "moe_align.py")
    rng = random.Random(37)
    routes, batches, sorted_ids, expert_ids, postpad, origin = [], [], [], [], [], []
    for batch in range(1, 9):
        patterns = list(bench.make_patterns(batch, rng).values())
        patterns += [[rng.randrange(-2, 292) for _ in range(batch * 8)] for _ in range(100)]
        for k, flat in enumerate(patterns):
            want = bench.cpu_reference(flat)
            assert bench.cpu_pairwise(flat) == want
            r = np.full(64, -1, dtype=np.int64)
            r[:len(flat)] = flat
            s = np.full(512, -1, dtype=np.int32)
            s[:len(want[0])] = want[0]
            e = np.full(64, -2, dtype=np.int32)
            e[:len(want[1])] = want[1]
            routes.append(r)
            batches.append(batch)
            sorted_ids.append(s)
            expert_ids.append(e)
            postpad.append(want[2][0])
            origin.append(0 if k < 7 else 1)
    assert len(routes) == 856
    # The reference Triton kernel itself, on the named patterns, both dtypes.
    kmod = load_module("ref_titan_moe_align", ref / "kernels" / "titan_moe_align.py")
    interp_checked = 0
    rng = random.Random(37)
    for batch in range(1, 9):
        for name, flat in bench.make_patterns(batch, rng).items():
            want = bench.cpu_reference(flat)
            for dtype in (torch.int32, torch.int64):
                ids = torch.tensor(flat, dtype=dtype).view(batch, 8)
                out = _run_moe_kernel(kmod, ids)
                assert [o.tolist() for o in out] == [list(w) for w in want], (batch, name, dtype)
                interp_checked += 1
        _ = [[rng.randrange(-2, 292) for _ in range(batch * 8)] for _ in range(100)]
    return dict(routes=np.stack(routes), batch=np.array(batches, np.int32), sorted_ids=np.stack(sorted_ids),
                expert_ids=np.stack(expert_ids), postpad=np.array(postpad, np.int32), origin=np.array(origin, np.int8),
                interp_kernel_cases=np.array(interp_checked, np.int32))


def _run_moe_kernel(kmod, ids):
    # kernels/titan_moe_align.py:78-81 launch, with CPU tensors for the interpreter
    # (the public wrapper rejects non-CUDA input by design).
    import triton
    routes = ids.numel()
    sorted_ids = torch.empty(routes * 8, dtype=torch.int32)
    expert_ids = torch.empty(routes, dtype=torch.int32)
    postpad = torch.empty(1, dtype=torch.int32)
    kmod._align_small[(1,)](ids, sorted_ids, expert_ids, postpad, R=routes,
                            BR=triton.next_power_of_2(routes), BS=triton.next_power_of_2(routes * 8),
                            num_warps=1, num_stages=1)
    return sorted_ids, expert_ids, postpad


def gen_kv(ref):
    kv = load_module("ref_titan_kv", ref / "kernels" / "titan_kv.py")
    x = C.kv_latents()
    n = x.shape[0]
    cache = torch.zeros(C.KV_BLOCKS, C.KV_BLOCK_SIZE, 528, dtype=torch.int8)
    slots = C.kv_slots()
    kv.store_int8(x, cache, slots)
    # A second call with int32 slots into a fresh cache (same bytes expected).
    cache32 = torch.zeros_like(cache)
    kv.store_int8(x, cache32, slots.to(torch.int32))
    assert torch.equal(cache, cache32)
    return dict(x_bits=x.view(torch.int16).numpy().view(np.uint16), slots=slots.numpy(),
                cache=cache.numpy().view(np.uint8), n=np.array(n))


def gen_mla(ref):
    kvmod = load_module("ref_titan_kv2", ref / "kernels" / "titan_kv.py")
    mla = load_module("ref_titan_mla", ref / "kernels" / "titan_mla.py")
    mla._sparse_mla_kernel_final = pin_autotuned(mla._sparse_mla_kernel_final, BLOCK_N=64, num_warps=4,
                                                 num_stages=1)
    mla._sparse_mla_kernel_split = pin_autotuned(mla._sparse_mla_kernel_split, BLOCK_N=32, num_warps=4,
                                                 num_stages=2)
    out = {}
    for case in C.MLA_CASES:
        inp = C.mla_inputs(case)
        cache = torch.zeros(inp["latent"].shape[0] // 256, 256, 528, dtype=torch.int8)
        kvmod.store_int8(inp["latent"], cache, torch.arange(inp["latent"].shape[0]))
        rows = cache.view(-1, 1, 528)
        out[f"{case.name}__input_sha256"] = np.frombuffer(
            bytes.fromhex(C.mla_input_digest(inp)), dtype=np.uint8)
        out[f"{case.name}__cache_sha256"] = np.frombuffer(
            hashlib.sha256(cache.numpy().tobytes()).digest(), dtype=np.uint8)
        for splits in case.splits:
            o = mla.triton_mla_sparse_attention(inp["q"], rows, inp["indices"], case.sm_scale,
                                                num_kv_splits=splits, sm_count=148)
            out[f"{case.name}__s{splits}"] = o.view(torch.int16).numpy().view(np.uint16)
        print(f"  mla case {case.name}: splits {case.splits}", flush=True)
    return out


def gen_index():
    # vLLM's conversion kernel (the third-party function the reference's
    # backend calls, integration/titan_backend.py:49-52), run by the Triton
    # interpreter; installed vLLM 0.22 has no BLOCK_STRIDE_ROWS, so these
    # vectors pin the block_stride_rows == block_size mapping.
    import vllm
    from vllm.v1.attention.backends.mla.sparse_utils import triton_convert_req_index_to_global_index as conv
    out = {"vllm_version": np.frombuffer(vllm.__version__.encode(), dtype=np.uint8)}
    for case in C.INDEX_CASES:
        inp = C.index_inputs(case)
        res = conv(inp["req_id"], inp["block_table"], inp["token_indices"], BLOCK_SIZE=case.block_size,
                   NUM_TOPK_TOKENS=case.topk)
        for k, v in inp.items():
            out[f"{case.name}__{k}"] = v.numpy()
        out[f"{case.name}__out"] = res.numpy()
        print(f"  index case {case.name}", flush=True)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--out", type=Path, default=HERE)
    ap.add_argument("--only", choices=("moe", "kv", "mla", "index"), nargs="*")
    args = ap.parse_args()
    install_interpreter_shims()
    only = set(args.only or ("moe", "kv", "mla", "index"))
    if "moe" in only:
        np.savez_compressed(args.out / "moe_golden.npz", **gen_moe(args.reference))
        print("wrote moe_golden.npz")
    if "kv" in only:
        np.savez_compressed(args.out / "kv_golden.npz", **gen_kv(args.reference))
        print("wrote kv_golden.npz")
    if "mla" in only:
        np.savez_compressed(args.out / "mla_golden.npz", **gen_mla(args.reference))
        print("wrote mla_golden.npz")
    if "index" in only:
        np.savez_compressed(args.out / "index_golden.npz", **gen_index())
        print("wrote index_golden.npz")


if __name__ == "__main__":
    main()
