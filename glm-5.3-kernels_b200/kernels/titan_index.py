# SPDX-License-Identifier: Apache-2.0
"""Request-local top-k positions -> global cache rows, on B200.

Drop-in for the conversion the reference's attention backend calls before the
sparse MLA reader (integration/titan_backend.py:48-52): vLLM's
`triton_convert_req_index_to_global_index` (vLLM
v1/attention/backends/mla/sparse_utils.py, a third-party dependency of the
reference, not in its tree), with the `BLOCK_STRIDE_ROWS` argument the
reference passes for padded block layouts.  The kernel is
`titan_convert_req_index_to_global` in libtitan_b200.so
(csrc/titan_index.cu).  To skip the conversion altogether, call
titan_mla.triton_mla_sparse_attention_paged, which translates inside the
gather.
"""
import torch

try:
    from . import titan_native as _native
except ImportError:
    import titan_native as _native


def triton_convert_req_index_to_global_index(
    req_id: torch.Tensor,
    block_table: torch.Tensor,
    token_indices: torch.Tensor,
    BLOCK_SIZE: int = 64,
    NUM_TOPK_TOKENS: int = 2048,
    BLOCK_N: int = 128,
    HAS_PREFILL_WORKSPACE: bool = False,
    prefill_workspace_request_ids: torch.Tensor | None = None,
    prefill_workspace_starts: torch.Tensor | None = None,
    return_valid_counts: bool = False,
    *,
    BLOCK_STRIDE_ROWS: int | None = None,
) -> torch.Tensor:
    """out[t, j] = block_table[req_id[t], tok // BLOCK_SIZE] * BLOCK_STRIDE_ROWS + tok % BLOCK_SIZE
    with tok = token_indices[t, j]; -1 where tok < 0 or the block index is
    past the table (and, a widening, where req_id[t] is not a row of
    block_table).  BLOCK_STRIDE_ROWS defaults to BLOCK_SIZE.  Same argument
    checks as vLLM's function; the prefill-workspace and valid-count options
    are not used by the reference's backend and are rejected.
    """
    assert req_id.dtype == torch.int32
    assert block_table.dtype == torch.int32
    assert token_indices.dtype == torch.int32
    assert token_indices.shape[1] == NUM_TOPK_TOKENS
    assert NUM_TOPK_TOKENS % BLOCK_N == 0, (
        f"NUM_TOPK_TOKENS ({NUM_TOPK_TOKENS}) must be divisible by BLOCK_N ({BLOCK_N})")
    assert not HAS_PREFILL_WORKSPACE and not return_valid_counts, \
        "prefill workspaces and valid counts are not supported by the B200 conversion"
    assert req_id.is_cuda and block_table.is_cuda and token_indices.is_cuda, "CUDA tensors only"
    stride_rows = BLOCK_SIZE if BLOCK_STRIDE_ROWS is None else BLOCK_STRIDE_ROWS
    num_tokens = req_id.shape[0]
    ti = token_indices if token_indices.stride(1) == 1 else token_indices.contiguous()
    req = req_id if req_id.is_contiguous() else req_id.contiguous()
    out = torch.empty((num_tokens, NUM_TOPK_TOKENS), dtype=torch.int32, device=token_indices.device)
    lib = _native.entry()
    with _native.on_device(token_indices.device):
        rc = lib.convert(
            req.data_ptr(), block_table.shape[0], block_table.data_ptr(), block_table.stride(0),
            block_table.stride(1), block_table.shape[1], ti.data_ptr(), ti.stride(0), NUM_TOPK_TOKENS,
            out.data_ptr(), out.stride(0), num_tokens, int(BLOCK_SIZE), int(stride_rows),
            _native.stream_of(token_indices))
    _native.check(rc, "triton_convert_req_index_to_global_index")
    return out
