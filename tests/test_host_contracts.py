# SPDX-License-Identifier: Apache-2.0
"""Host-side contract of the drop-in modules: import behaviour, argument
validation and exception types, the split heuristic.  No GPU, no kernel call."""
import importlib.util
import itertools
import sys
import types
from pathlib import Path
from unittest.mock import patch

import pytest
import torch

from oracle import oracle as O

PKG = Path(__file__).resolve().parents[1] / "glm-5.3-kernels_b200" / "kernels"


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_import_does_not_touch_cuda_or_library():
    """Like tests/test_cpu_contracts.py:33-53: executing the modules with a torch
    double whose torch.cuda raises on any attribute must succeed."""
    fake_torch = types.ModuleType("torch")
    fake_torch.Tensor = object

    class NoCUDA:
        def __getattr__(self, name):
            raise AssertionError(f"import-time torch.cuda access: {name}")

    fake_torch.cuda = NoCUDA()
    with patch.dict(sys.modules, {"torch": fake_torch}):
        sys.modules.pop("titan_native", None)
        native = _load("titan_native", PKG / "titan_native.py")
        assert native._lib is None
        with patch.dict(sys.modules, {"titan_native": native}):
            for filename, exported in (("titan_kv.py", "store_int8"),
                                       ("titan_mla.py", "triton_mla_sparse_attention"),
                                       ("titan_moe_align.py", "titan_moe_align_small"),
                                       ("titan_moe_split_align.py", "split_align")):
                mod = _load("isolated_" + filename[:-3], PKG / filename)
                assert callable(getattr(mod, exported))
        assert native._lib is None, "importing must not load the library"


def test_no_triton_or_vllm_imports():
    import re
    for f in PKG.glob("*.py"):
        text = f.read_text()
        assert not re.search(r"^\s*(import|from)\s+(triton|vllm)\b", text, re.M), f


# (cluster size, co-resident clusters, clusters with one CTA per SM) of the MLA
# kernel on a 148-SM B200, as titan_mla_max_active_clusters /
# titan_mla_max_exclusive_clusters report them.
B200_CLUSTER_TABLES = ((1, 296, 148), (2, 148, 74), (4, 71, 33), (8, 33, 15), (16, 14, 7))


def test_b200_split_policy_picks():
    """The automatic split counts for the decode batch sizes, and the launch
    layout (cluster size C, clusters per token NC) the launcher derives."""
    from kernels.titan_mla import _choose_kv_splits_b200, _launch_layout
    picks = {B: _choose_kv_splits_b200(B, 1, 2176, 148, B200_CLUSTER_TABLES) for B in range(1, 9)}
    assert picks == {1: 68, 2: 68, 3: 34, 4: 34, 5: 23, 6: 23, 7: 17, 8: 17}, picks
    assert _launch_layout(1, 68, B200_CLUSTER_TABLES) == (1, 68, True)     # flat merge
    assert _launch_layout(1, 80, B200_CLUSTER_TABLES) == (16, 5, False)    # last-arriver merge (NC <= C)
    assert _launch_layout(2, 40, B200_CLUSTER_TABLES) == (8, 5, False)
    assert _launch_layout(2, 48, B200_CLUSTER_TABLES) == (16, 3, False)    # last-arriver merge
    assert _launch_layout(4, 16, B200_CLUSTER_TABLES) == (16, 1, False)    # one cluster per token
    assert _launch_layout(8, 17, B200_CLUSTER_TABLES) == (1, 17, True)     # flat merge
    assert _launch_layout(4, 34, B200_CLUSTER_TABLES) == (1, 34, True)     # C = 2 would need the combine
    assert _launch_layout(3, 136, B200_CLUSTER_TABLES) == (1, 136, False)  # 408 CTAs: combine kernel
    assert _launch_layout(1, 8, B200_CLUSTER_TABLES) == (8, 1, False)
    assert _launch_layout(1, 12, B200_CLUSTER_TABLES) == (4, 3, False)     # last-arriver merge
    assert _launch_layout(1, 13, B200_CLUSTER_TABLES) == (1, 13, True)     # flat merge
    assert _launch_layout(1, 7, B200_CLUSTER_TABLES) == (1, 7, False)      # fewer than 8: combine
    assert _launch_layout(8, 16, B200_CLUSTER_TABLES) == (16, 1, False)
    assert _launch_layout(7, 16, B200_CLUSTER_TABLES) == (16, 1, False)    # one cluster per token
    assert _launch_layout(4, 24, B200_CLUSTER_TABLES) == (8, 3, False)
    for T in (148, 149, 4096):
        assert _choose_kv_splits_b200(T, 1, 2176, 148, B200_CLUSTER_TABLES) == 1
    assert _choose_kv_splits_b200(0, 1, 2176, 148, B200_CLUSTER_TABLES) == 1
    for B in range(1, 148):
        S = _choose_kv_splits_b200(B, 1, 2176, 148, B200_CLUSTER_TABLES)
        assert 1 <= S and B * S <= 148, (B, S)


def test_moe_argument_errors_are_value_errors():
    from kernels.titan_moe_align import titan_moe_align_small
    ok = torch.zeros(2, 8, dtype=torch.int32)
    with pytest.raises(ValueError):
        titan_moe_align_small(torch.zeros(9, 8, dtype=torch.int32))
    with pytest.raises(ValueError):
        titan_moe_align_small(torch.zeros(2, 4, dtype=torch.int32))
    with pytest.raises(ValueError):
        titan_moe_align_small(ok, block_size=16)
    with pytest.raises(ValueError):
        titan_moe_align_small(ok, num_experts=256)
    with pytest.raises(ValueError):
        titan_moe_align_small(ok, expert_map=torch.arange(288))
    with pytest.raises(ValueError):
        titan_moe_align_small(ok, ignore_invalid_experts=False)
    with pytest.raises(ValueError):  # CPU tensor: no CPU fallback
        titan_moe_align_small(ok)


def test_mla_argument_errors_are_assertions():
    from kernels.titan_mla import triton_mla_sparse_attention as attn
    q = torch.zeros(1, 16, 512, dtype=torch.bfloat16)
    kv = torch.zeros(64, 1, 528, dtype=torch.int8)
    idx = torch.zeros(1, 1, 64, dtype=torch.int32)
    with pytest.raises(AssertionError):
        attn(torch.zeros(1, 16, 320, dtype=torch.bfloat16), kv, idx, 0.1)      # dim_qk
    with pytest.raises(AssertionError):
        attn(q, torch.zeros(64, 2, 528, dtype=torch.int8), idx, 0.1)           # kv heads
    with pytest.raises(AssertionError):
        attn(q, kv, torch.zeros(1, 1, 48, dtype=torch.int32), 0.1)             # topk % 32
    with pytest.raises(AssertionError):
        attn(torch.zeros(1, 16, 576, dtype=torch.bfloat16), torch.zeros(64, 1, 528, dtype=torch.int8), idx, 0.1)
    with pytest.raises(AssertionError):
        attn(q, kv, idx, 0.1)                                                    # CPU tensors


def test_kv_argument_errors_are_assertions():
    from kernels.titan_kv import store_int8
    x = torch.zeros(4, 512, dtype=torch.bfloat16)
    cache = torch.zeros(1, 8, 528, dtype=torch.int8)
    with pytest.raises(AssertionError):
        store_int8(torch.zeros(4, 256, dtype=torch.bfloat16), cache, torch.arange(4))
    with pytest.raises(AssertionError):
        store_int8(x, torch.zeros(1, 8, 512, dtype=torch.int8), torch.arange(4))
    with pytest.raises(AssertionError):
        store_int8(x, cache, torch.arange(5))
    with pytest.raises(AssertionError):
        store_int8(x, cache, torch.arange(4))                                    # CPU tensors


def test_split_align_buffers_and_errors():
    """Buffer layout of profiles/sm74/titan_prefill/moe_split_align.py:187-201
    (lists sized t_max + B*E and (t_max + B*E) // B + 1, four-entry ntpp, the
    cover table of t_max + 1 rows); the reference's AssertionError on T = 0,
    T > t_max or a different E; a CPU tensor is refused (no CPU fallback)."""
    import torch
    from kernels import titan_moe_split_align as S
    buf = S.buffers(100, 288, torch.device("cpu"))
    assert buf["t_max"] == 100 and buf["E"] == 288 and buf["ntpp"].numel() == 4
    assert tuple(buf["tab"].shape) == (101, 4) and buf["tab"].dtype == torch.int32
    for k, bs in enumerate(S.SIZES):
        assert buf["s"][k].numel() == 100 + bs * 288 and buf["s"][k].dtype == torch.int32
        assert buf["e"][k].numel() == (100 + bs * 288) // bs + 1
    ids = torch.zeros(2, 8, dtype=torch.int32)
    for bad_ids, E in ((torch.zeros(0, 8, dtype=torch.int32), 288), (torch.zeros(13, 8, dtype=torch.int32), 288),
                       (ids, 287)):
        with pytest.raises(AssertionError):
            S.split_align(bad_ids, E, buf)
    with pytest.raises(ValueError):
        S.split_align(ids, 288, buf)
    with pytest.raises(ValueError):
        S.buffers(10, 1025, torch.device("cpu"))
