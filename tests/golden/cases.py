# SPDX-License-Identifier: Apache-2.0
"""Seeded inputs shared by the golden generator (make_golden.py) and the tests.

Everything here is deterministic torch-CPU generation; the golden fixtures
record a SHA-256 of the MLA inputs so a change in the generator is detected.
"""
import dataclasses
import hashlib

import numpy as np
import torch

KV_ROWS = 128
KV_BLOCKS = 2
KV_BLOCK_SIZE = 256


def _bf16(values):
    return torch.tensor(values, dtype=torch.float32).to(torch.bfloat16)


def kv_latents():
    """[128, 512] bf16 latents: random rows plus edge rows for the quantiser."""
    g = torch.Generator().manual_seed(20260910)
    x = torch.randn(KV_ROWS, 512, generator=g)
    x[:, :128] *= 0.05  # column groups scaled like tests/verify_mla.py:34
    x[:, 256:384] *= 8
    x = x.to(torch.bfloat16)
    x[0] = 0                                       # all-zero row -> scale 1e-12, q = 0
    x[1] = _bf16([1e-20] * 512)                    # scale floor 1e-12, q rounds to 0
    x[2] = _bf16((torch.linspace(-1e-10, 1e-10, 512)).tolist())  # floor scale, nonzero q
    ties = [127.0] + [(k % 126) + 0.5 for k in range(1, 256)] + [-((k % 126) + 0.5) for k in range(256)]
    x[3] = _bf16(ties)                             # scale == 1: exact half-way quotients
    quarter = [63.5] + [0.25 * (2 * (k % 120) + 1) for k in range(1, 512)]
    x[4] = _bf16(quarter)                          # scale == 0.5: ties at odd quarters
    x[5] = (torch.randn(512, generator=g) * 1e37).to(torch.bfloat16)   # near the top of the range
    sub = torch.tensor([1e-39, -2e-39, 5e-40, 3e-41] * 128)            # bf16 subnormals
    sub[::7] = 1e-3
    x[6] = sub.to(torch.bfloat16)
    x[7] = -3.0                                    # constant row -> all -127
    x[8] = (torch.randn(512, generator=g) * 0.01).to(torch.bfloat16)
    x[8, 17] = 40.0                                # one large outlier
    # Non-finite latents.  The reference's max / maximum / minimum drop NaN
    # operands (Triton's default PropagateNan.NONE), so a NaN value is
    # ignored by the row max and quantises to -127; an infinite value makes
    # the scale infinite, finite values then quantise to 0 and +-inf to -127.
    nan_bits = [0x7FC0, 0xFFC0, 0x7F81, 0x7FFF]    # quiet, negative, signalling, max-payload NaN
    x[9] = (torch.randn(512, generator=g)).to(torch.bfloat16)
    x[9, 5] = float("nan")                         # one NaN among finite values
    x[10] = (torch.randn(512, generator=g) * 3).to(torch.bfloat16)
    x[10, 100] = float("inf")                      # one +inf: scale = inf
    x[11] = (torch.randn(512, generator=g)).to(torch.bfloat16)
    x[11, 300] = float("-inf")
    x[11, 301] = float("nan")                      # -inf and NaN together
    x[12] = float("nan")                           # all NaN: scale floor, every value -127
    x[13] = (torch.randn(512, generator=g) * 1e30).to(torch.bfloat16)
    x[13, ::64] = float("inf")
    x[13, 1::64] = float("-inf")                   # several infinities of both signs
    x14 = x[14].view(torch.int16)
    for k, b in enumerate(nan_bits):               # NaN payloads and signs, as raw bf16 bits
        x14[64 * k + 3] = b - (1 << 16) if b >= 0x8000 else b
    return x


def kv_slots():
    """128 int64 slots into a [2, 256, 528] cache, 5 of them negative."""
    g = torch.Generator().manual_seed(7)
    slots = torch.randperm(KV_BLOCKS * KV_BLOCK_SIZE, generator=g)[:KV_ROWS].to(torch.int64)
    slots[[3, 40, 41, 77, 127]] = -1
    return slots


@dataclasses.dataclass(frozen=True)
class MlaCase:
    name: str
    seed: int
    kv_rows: int
    tokens: int
    heads: int
    topk: int
    pattern: str
    splits: tuple
    q_scale: float = 1.0
    sm_scale: float = 512 ** -0.5


MLA_CASES = (
    # The CPU-sized B=1 case: seed 0, [4096, 512] latents, q [1, 16, 512],
    # 2176 indices uniform in [0, 4096) with the last 128 set to -1.
    MlaCase("c1", 0, 4096, 1, 16, 2176, "tail128", (1, 4, 8, 16, 32)),
    # tests/verify_mla.py:72-78 masking: tail 2048.. = -1, token 1 2000.. = -1,
    # one positive out-of-range index; q scaled by 0.15.
    MlaCase("mask6", 20260910, 4096, 6, 16, 2176, "verify_mla", (1, 4, 8, 16), q_scale=0.15),
    MlaCase("h8", 11, 1024, 2, 8, 256, "random_neg", (1, 2)),
    MlaCase("h20", 12, 1024, 1, 20, 128, "random_neg", (1, 4)),
    MlaCase("blank", 13, 1024, 2, 16, 128, "all_neg", (1, 4)),
    MlaCase("dup", 14, 1024, 1, 16, 64, "duplicates", (1, 2)),
)


def mla_inputs(case):
    g = torch.Generator().manual_seed(case.seed)
    latent = torch.randn(case.kv_rows, 512, generator=g)
    if case.pattern == "verify_mla":
        latent[:, :128] *= 0.05
        latent[:, 256:384] *= 8
        latent[0] = 0
    latent = latent.to(torch.bfloat16)
    q = (torch.randn(case.tokens, case.heads, 512, generator=g) * case.q_scale).to(torch.bfloat16)
    idx = torch.randint(0, case.kv_rows, (case.tokens, 1, case.topk), generator=g, dtype=torch.int32)
    if case.pattern == "tail128":
        idx[:, :, -128:] = -1
    elif case.pattern == "verify_mla":
        idx[:, :, 2048:] = -1
        idx[1, :, 2000:] = -1
        idx[0, 0, 0] = case.kv_rows + 5
    elif case.pattern == "random_neg":
        drop = torch.rand(idx.shape, generator=g) < 0.2
        idx[drop] = -1
        idx[..., -5:] = case.kv_rows + 3
    elif case.pattern == "all_neg":
        idx[:] = -1
    elif case.pattern == "duplicates":
        idx[..., :16] = 7
        idx[..., 16:24] = 3
        idx[..., 40] = case.kv_rows
    return {"latent": latent, "q": q, "indices": idx}


def mla_input_digest(inp):
    h = hashlib.sha256()
    for key in ("latent", "q"):
        h.update(inp[key].contiguous().view(torch.int16).numpy().tobytes())
    h.update(inp["indices"].contiguous().numpy().astype(np.int32).tobytes())
    return h.hexdigest()


@dataclasses.dataclass(frozen=True)
class IndexCase:
    """Paged index conversion: T tokens of R requests, block tables of
    max_blocks entries, positions uniform in [-3, max_blocks * block_size + 40)."""
    name: str
    seed: int
    tokens: int
    reqs: int
    max_blocks: int
    block_size: int
    topk: int


INDEX_CASES = (
    IndexCase("bs64", 31, 6, 3, 5, 64, 256),
    IndexCase("bs16", 32, 4, 2, 20, 16, 128),
    IndexCase("bs48", 33, 3, 3, 8, 48, 128),
    IndexCase("bs64_topk2176", 34, 2, 2, 40, 64, 2176),
)


def index_inputs(case):
    g = torch.Generator().manual_seed(case.seed)
    req = torch.randint(0, case.reqs, (case.tokens,), generator=g, dtype=torch.int32)
    bt = torch.randint(0, 4096, (case.reqs, case.max_blocks), generator=g, dtype=torch.int32)
    hi = case.max_blocks * case.block_size + 40
    tok = torch.randint(-3, hi, (case.tokens, case.topk), generator=g, dtype=torch.int32)
    return {"req_id": req, "block_table": bt, "token_indices": tok}
