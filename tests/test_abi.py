# SPDX-License-Identifier: Apache-2.0
"""The C-ABI library loads and exports every entry point include/titan_b200.h
declares; host-side validation answers without a GPU."""
import ctypes
import re
from pathlib import Path

HEADER = Path(__file__).resolve().parents[1] / "include" / "titan_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(titan_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_path():
    names = declared_functions()
    for want in ("titan_store_int8", "titan_mla_sparse_attention", "titan_mla_workspace_bytes",
                 "titan_moe_align_small", "titan_last_error", "titan_abi_version", "titan_device_error"):
        assert want in names


def test_every_declared_symbol_is_exported(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), name


def test_python_binding_covers_header(native_lib):
    from kernels import titan_native
    assert set(titan_native.SIGNATURES) >= set(declared_functions())


def test_version_and_workspace(native_lib):
    assert native_lib.titan_abi_version() == 100
    assert native_lib.titan_mla_workspace_bytes(1, 16, 1) == 0
    # [T][S][Hp][512] fp32 partials + [T][S][Hp] fp32 LSE rounded up to 256 B
    assert native_lib.titan_mla_workspace_bytes(1, 16, 32) == 32 * 16 * 512 * 4 + 2048
    assert native_lib.titan_mla_workspace_bytes(2, 20, 4) == 2 * 4 * 32 * 512 * 4 + 1024


def test_invalid_arguments_rejected_on_host(native_lib):
    rc = native_lib.titan_moe_align_small(None, 0, 7, None, None, None, 1, None)
    assert rc == 1 and b"num_routes" in native_lib.titan_last_error()
    rc = native_lib.titan_moe_align_small(None, 0, 16, None, None, None, 3, None)
    assert rc == 1 and b"num_warps" in native_lib.titan_last_error()
    rc = native_lib.titan_mla_sparse_attention(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, 1, 16,
                                               ctypes.c_float(0.1), 0, None, 0, None)
    assert rc == 1
    rc = native_lib.titan_store_int8(None, 512, None, 1, 256, 0, 0, None, 1, -1, None)
    assert rc == 1
    assert native_lib.titan_store_int8(None, 512, None, 1, 256, 0, 0, None, 1, 0, None) == 0  # nothing to do


def test_split_align_invalid_arguments_rejected_on_host(native_lib):
    """Host validation of titan_moe_split_align: routes within (0, t_max], expert
    count within the shared-memory limit, a cover table of T + 1 rows, pointers."""
    lists = (ctypes.c_void_p * 4)(16, 16, 16, 16)
    split = native_lib.titan_moe_split_align
    assert split(16, 0, 0, 288, 16, 1, 8, lists, lists, 16, None) == 1
    assert b"num_routes" in native_lib.titan_last_error()
    assert split(16, 0, 9, 288, 16, 10, 8, lists, lists, 16, None) == 1   # T > t_max
    assert split(16, 0, 8, 1025, 16, 9, 8, lists, lists, 16, None) == 1
    assert b"num_experts" in native_lib.titan_last_error()
    assert split(16, 0, 8, 288, 16, 8, 8, lists, lists, 16, None) == 1    # table too short
    assert b"cover table" in native_lib.titan_last_error()
    assert split(None, 0, 8, 288, 16, 9, 8, lists, lists, 16, None) == 1
    assert b"null" in native_lib.titan_last_error()
    assert native_lib.titan_moe_split_align_smem_bytes(288) == (32 * 289 + 10 * 288) * 4


def test_fast_call_binding_is_built_and_bound(native_lib):
    """The hot launchers go through the CPython fast-call module (bound to the
    loaded library), which validates argument count and types before calling."""
    import pytest
    from kernels import titan_native
    e = titan_native.entry()
    assert type(e).__name__ == "module" and e.__name__ == "_titan_pybind"
    for name in titan_native._HOT:
        assert callable(getattr(e, name))
    # Same host-side validation as through ctypes: status 1, nothing launched.
    assert e.moe_align(None, 0, 7, None, None, None, 1, None) == 1
    assert b"num_routes" in native_lib.titan_last_error()
    assert e.mla(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, 1, 16, 0.1, 0, None, 0, None) == 1
    assert e.store_int8(None, 512, None, 1, 256, 0, 0, None, 1, 0, None) == 0
    assert e.copy(None, None, 0, 0, None) == 0
    assert e.copy(None, None, 16, 0, None) == 1 and b"null" in native_lib.titan_last_error()
    assert e.copy(None, None, 16, 2, None) == 1 and b"flags" in native_lib.titan_last_error()
    with pytest.raises(TypeError):
        e.mla_sem(*([0] * 20))                   # one argument short
    with pytest.raises(TypeError):
        e.copy(0, 0, 1.5, 0, 0)                  # float where an int64 belongs
    with pytest.raises(TypeError):
        e.store_int8("x", 512, None, 1, 256, 0, 0, None, 1, 0, None)
