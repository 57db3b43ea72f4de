# SPDX-License-Identifier: Apache-2.0
"""CPU oracle of the sparse-MLA decode path (test infrastructure only).

`oracle.oracle` holds the numpy / torch-CPU restatements; `oracle.c_oracle()`
loads the C restatement (titan_oracle.c) built by `oracle/build.py`.
"""
import ctypes
from pathlib import Path

from .build import build as _build

_c = None


def c_oracle():
    """ctypes handle of the C restatement (built on first use with gcc)."""
    global _c
    if _c is None:
        lib = ctypes.CDLL(str(_build()))
        lib.oracle_store_int8_rows.restype = None
        lib.oracle_store_int8_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.oracle_moe_align_small.restype = ctypes.c_int
        lib.oracle_moe_align_small.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p]
        _c = lib
    return _c
