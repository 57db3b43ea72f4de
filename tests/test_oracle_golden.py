# SPDX-License-Identifier: Apache-2.0
"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py).  No GPU."""
import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import oracle as O
from tests.golden import cases as C

GOLDEN = C.__file__.rsplit("/", 1)[0]


@pytest.fixture(scope="module")
def kv_golden():
    return np.load(f"{GOLDEN}/kv_golden.npz")


@pytest.fixture(scope="module")
def moe_golden():
    return np.load(f"{GOLDEN}/moe_golden.npz")


@pytest.fixture(scope="module")
def mla_golden():
    return np.load(f"{GOLDEN}/mla_golden.npz")


def test_kv_inputs_regenerate(kv_golden):
    assert np.array_equal(O.tensor_bf16_bits(C.kv_latents()), kv_golden["x_bits"])
    assert np.array_equal(C.kv_slots().numpy(), kv_golden["slots"])


def test_kv_oracle_numpy_bit_exact(kv_golden):
    cache = np.zeros((C.KV_BLOCKS, C.KV_BLOCK_SIZE, 528), np.uint8)
    O.store_int8(kv_golden["x_bits"], cache, kv_golden["slots"])
    assert np.array_equal(cache, kv_golden["cache"])


def test_kv_oracle_c_bit_exact(kv_golden):
    bits = np.ascontiguousarray(kv_golden["x_bits"])
    rows = np.zeros((bits.shape[0], 528), np.uint8)
    c_oracle().oracle_store_int8_rows(bits.ctypes.data, bits.shape[0], rows.ctypes.data)
    flat = kv_golden["cache"].reshape(-1, 528)
    slots = kv_golden["slots"]
    keep = slots >= 0
    assert np.array_equal(rows[keep], flat[slots[keep]])
    # rows with a negative slot never reach the cache; untouched rows stay zero
    touched = np.zeros(flat.shape[0], bool)
    touched[slots[keep]] = True
    assert not flat[~touched].any()


def test_kv_reference_quantisation_criteria(kv_golden):
    """tests/verify_mla.py:50-66 criteria hold for the oracle's bytes."""
    x = O.bf16_bits_to_f32(kv_golden["x_bits"])
    rows = O.store_int8_rows(kv_golden["x_bits"])
    scales = rows[:, 512:516].copy().view(np.float32)[:, 0]
    finite = np.isfinite(x).all(1)
    expected = np.maximum(np.abs(x).max(1), 127e-12) / 127
    np.testing.assert_allclose(scales[finite], expected[finite].astype(np.float32), rtol=1e-6, atol=1e-12)
    ints = rows[:, :512].view(np.int8).astype(np.float32)
    assert np.abs(ints[finite] - np.clip(np.round(x[finite] / scales[finite, None]), -127, 127)).max() <= 1
    assert not rows[:, 516:].any()


def test_kv_nonfinite_rows(kv_golden):
    """Rows with NaN or inf, as the reference's NaN-dropping max / maximum /
    minimum treat them: NaN values are ignored by the row max and store -127;
    an infinite value makes the scale infinite, so finite values store 0 and
    +-inf (inf / inf = NaN) store -127; an all-NaN row keeps the 1e-12 floor."""
    x = O.bf16_bits_to_f32(kv_golden["x_bits"])
    flat = kv_golden["cache"].reshape(-1, 528)
    slots = kv_golden["slots"]
    seen_nan = seen_inf = 0
    for r in range(x.shape[0]):
        if np.isfinite(x[r]).all() or slots[r] < 0:
            continue
        row = flat[slots[r]]
        q = row[:512].view(np.int8)
        scale = row[512:516].copy().view(np.float32)[0]
        nan = np.isnan(x[r])
        assert (q[nan] == -127).all()
        if np.isinf(x[r]).any():
            seen_inf += 1
            assert np.isinf(scale) and scale > 0
            assert (q[np.isinf(x[r])] == -127).all() and (q[np.isfinite(x[r])] == 0).all()
        elif nan.all():
            assert scale == np.float32(1e-12)
        else:
            seen_nan += 1
            finite = ~nan
            assert scale == np.float32(np.abs(x[r][finite]).max() / np.float32(127))
            want = np.clip(np.rint(x[r][finite] / scale), -127, 127)
            assert np.array_equal(q[finite].astype(np.float32), want)
    assert seen_nan >= 2 and seen_inf >= 3


def _moe_cases(golden):
    for i in range(len(golden["batch"])):
        R = int(golden["batch"][i]) * 8
        yield (golden["routes"][i][:R], golden["sorted_ids"][i][:8 * R], golden["expert_ids"][i][:R],
               int(golden["postpad"][i]))


def test_moe_golden_case_count(moe_golden):
    assert len(moe_golden["batch"]) == 856          # tests/test_cpu_contracts.py:26
    assert int(moe_golden["interp_kernel_cases"]) == 112


def test_moe_oracle_vectorised_bit_exact(moe_golden):
    for routes, s, e, p in _moe_cases(moe_golden):
        so, eo, po = O.moe_align_small(routes)
        assert np.array_equal(so, s) and np.array_equal(eo, e) and po[0] == p


def test_moe_oracle_loops_bit_exact(moe_golden):
    for routes, s, e, p in _moe_cases(moe_golden):
        so, eo, po = O.moe_align_small_loops(routes.tolist())
        assert so == s.tolist() and eo == e.tolist() and po == [p]


def test_moe_oracle_c_bit_exact(moe_golden):
    lib = c_oracle()
    for routes, s, e, p in _moe_cases(moe_golden):
        ids = np.ascontiguousarray(routes, dtype=np.int64)
        R = ids.size
        so = np.empty(8 * R, np.int32)
        eo = np.empty(R, np.int32)
        po = np.empty(1, np.int32)
        assert lib.oracle_moe_align_small(ids.ctypes.data, R, so.ctypes.data, eo.ctypes.data, po.ctypes.data) == 0
        assert np.array_equal(so, s) and np.array_equal(eo, e) and po[0] == p


@pytest.mark.parametrize("case", C.MLA_CASES, ids=lambda c: c.name)
def test_mla_oracle_vs_reference_golden(case, mla_golden):
    inp = C.mla_inputs(case)
    assert bytes(mla_golden[f"{case.name}__input_sha256"]).hex() == C.mla_input_digest(inp)
    rows = O.store_int8_rows(O.tensor_bf16_bits(inp["latent"]))
    ref = O.mla_sparse_attention(inp["q"], rows, inp["indices"], case.sm_scale)
    for s in case.splits:
        gold = torch.from_numpy(O.bf16_bits_to_f32(mla_golden[f"{case.name}__s{s}"]).reshape(ref.shape))
        # Path tolerance: |a - b| <= 2e-2 + 1e-2 |b|.
        assert bool(((gold - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()), (case.name, s)
        if case.pattern == "all_neg":
            assert not gold.any()


def test_split_heuristic_restatement_table():
    """oracle.choose_num_kv_splits on hand-worked cases of the reference heuristic
    (kernels/titan_mla.py:441-449): decode at 70 and 148 SMs, B=8, T=37 (single
    pass) and T=0."""
    assert O.choose_num_kv_splits(1, 1, 2176, 70) == 32
    assert O.choose_num_kv_splits(1, 1, 2176, 148) == 32
    assert O.choose_num_kv_splits(8, 1, 2176, 148) == 16
    assert O.choose_num_kv_splits(37, 1, 2176, 148) == 1
    assert O.choose_num_kv_splits(0, 1, 2176, 148) == 1


def test_index_conversion_oracle_matches_vllm_goldens():
    """oracle.convert_req_index_to_global vs vLLM's own conversion kernel
    (Triton interpreter, tests/golden/make_golden.py), bit-exact."""
    gold = np.load(f"{GOLDEN}/index_golden.npz")
    assert bytes(gold["vllm_version"]).decode().startswith("0.")
    for case in C.INDEX_CASES:
        inp = C.index_inputs(case)
        for k, v in inp.items():
            assert np.array_equal(gold[f"{case.name}__{k}"], v.numpy()), (case.name, k)
        got = O.convert_req_index_to_global(inp["req_id"].numpy(), inp["block_table"].numpy(),
                                            inp["token_indices"].numpy(), case.block_size)
        want = gold[f"{case.name}__out"]
        assert np.array_equal(got, want), case.name
        assert (want == -1).any() and (want >= 0).any()


def _split_golden_cases():
    golden = np.load(f"{GOLDEN}/split_align_golden.npz")
    for name in golden["names"]:
        E, t_max = (int(v) for v in golden[f"{name}/meta"])
        yield str(name), golden[f"{name}/routes"], E, t_max, golden


def test_split_align_cover_table_is_cost_optimal():
    """Every r's cover reaches r rows, pads less than its smallest block and costs
    no more than any single-size cover (profiles/sm74/titan_prefill/moe_split_align.py:8-20)."""
    table = O.split_cover_table(600)
    for r in range(1, 601):
        n = table[r]
        covered = int(sum(int(c) * b for c, b in zip(n, O.SPLIT_SIZES)))
        smallest = min(b for c, b in zip(n, O.SPLIT_SIZES) if c)
        assert r <= covered < r + smallest
        cost = sum(int(c) * O.SPLIT_COST[b] for c, b in zip(n, O.SPLIT_SIZES))
        for b in O.SPLIT_SIZES:
            assert cost <= -(-r // b) * O.SPLIT_COST[b] + 1e-9


def test_split_align_oracle_bit_exact():
    """The split-align oracle equals the reference's five Triton kernels (run by the
    interpreter, tests/golden/make_split_align_golden.py) on whole buffers,
    untouched entries included: uniform, Zipf, invalid, int64-wrapped ids, one
    expert, a single route and three experts."""
    sizes = 0
    for name, routes, E, t_max, golden in _split_golden_cases():
        lists = O.moe_split_align(routes, E, t_max)
        assert [n for _, _, _, n in lists] == golden[f"{name}/ntpp"].tolist(), name
        for k, (bs, s, e, _) in enumerate(lists):
            assert bs == int(golden["sizes"][k])
            assert np.array_equal(s, golden[f"{name}/sorted{k}"]), (name, k)
            assert np.array_equal(e, golden[f"{name}/experts{k}"]), (name, k)
            sizes |= 1 << k if lists[k][3] else 0
    assert sizes == 0b1111  # every block size holds rows in some case


def test_split_align_product_cover_table_matches_oracle():
    from kernels import titan_moe_split_align as S
    assert np.array_equal(S.cover_table(3000).numpy(), O.split_cover_table(3000))
    assert S.SIZES == O.SPLIT_SIZES and S.COST == O.SPLIT_COST


def test_split_align_oracle_properties_at_prefill_size():
    """Size-independent checks of the split layout at M = 4096 x top-8 (uniform
    and Zipf experts): every valid route appears exactly once, in stable order
    within its expert; padding is the sentinel T only, at the tail of a block
    that holds at least one row; every block's expert id matches its rows; ntpp
    is a multiple of B."""
    rng = np.random.default_rng(11)
    E, M = 288, 4096
    w = 1.0 / np.arange(1, E + 1) ** 1.1
    for routes in (rng.integers(-2, E + 2, (M, 8)), rng.choice(E, size=(M, 8), p=w / w.sum())):
        flat = routes.reshape(-1)
        T = flat.size
        lists = O.moe_split_align(routes, E)
        seen = []
        for bs, s, e, n in lists:
            assert n % bs == 0
            rows, blocks = s[:n], e[:n // bs]
            for blk in range(n // bs):
                members = rows[blk * bs:(blk + 1) * bs]
                real = members[members != T]
                assert real.size > 0 and np.all(flat[real] == blocks[blk])
                pad = np.nonzero(members == T)[0]
                assert pad.size == 0 or pad[0] == bs - pad.size  # padding only at the block's tail
            seen.extend(rows[rows != T].tolist())
        valid = np.nonzero((flat >= 0) & (flat < E))[0]
        assert sorted(seen) == valid.tolist()
        order = {}
        for bs, s, e, n in lists:  # lists are taken largest block first, so ranks ascend across them
            for j in s[:n]:
                if j != T:
                    order.setdefault(flat[j], []).append(j)
        assert all(v == sorted(v) for v in order.values())
