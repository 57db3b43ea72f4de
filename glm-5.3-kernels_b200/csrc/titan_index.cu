// Request-local top-k positions -> global cache rows, for paged KV caches.
//
// The reference's attention backend converts the indexer's request-local
// positions before calling the sparse MLA reader (integration/titan_backend.py:
// 48-54), with vLLM's `triton_convert_req_index_to_global_index` (vLLM
// v1/attention/backends/mla/sparse_utils.py; a third-party dependency, not in
// the reference tree).  Mapping, per token t and position tok = idx[t, j]:
//   blk = tok / block_size, off = tok % block_size
//   out = block_table[req_id[t], blk] * block_stride_rows + off
//   out = -1 if tok < 0 or blk >= max_blocks (vLLM's guards), and here also
//   if req_id[t] is outside [0, num_reqs) (vLLM would read out of bounds).
// block_stride_rows = block_size for a contiguous cache (the mapping of the
// vLLM 0.22 kernel); the reference's backend passes the row stride of a
// padded block layout.  The output is the int32 value of that expression
// (two's-complement wrap like the Triton int32 arithmetic).
//
// B200 design: one thread per position, 16-byte loads and stores of four
// positions when the rows are 16-byte aligned; the block-table row of the
// token is loaded once per thread group of four.  The fused alternative,
// which translates inside the MLA gather, is titan_mla_sparse_attention_paged.
#include "titan_common.cuh"

namespace titan {

constexpr int kIndexThreads = 256;

__device__ __forceinline__ int32_t req_to_global(int32_t tok, const int32_t *bt_row, int64_t bt_st1, int64_t max_blocks,
                                                 int64_t block_size, int block_shift, int64_t block_stride_rows) {
  if (bt_row == nullptr || tok < 0) return -1;
  const int64_t blk = block_shift >= 0 ? ((int64_t)tok >> block_shift) : (int64_t)tok / block_size;
  if (blk >= max_blocks) return -1;
  const int64_t base = (int64_t)__ldg(bt_row + blk * bt_st1);
  return (int32_t)(uint32_t)(uint64_t)(base * block_stride_rows + ((int64_t)tok - blk * block_size));
}

// grid (num_tokens, ceil(topk / (4 * kIndexThreads))): thread handles positions 4 i .. 4 i + 3.
__global__ void __launch_bounds__(kIndexThreads)
    req_index_to_global_kernel(const int32_t *__restrict__ req_id, int64_t num_reqs,
                               const int32_t *__restrict__ block_table, int64_t bt_st0, int64_t bt_st1,
                               int64_t max_blocks, const int32_t *__restrict__ idx, int64_t idx_st, int64_t topk,
                               int32_t *__restrict__ out, int64_t out_st, int64_t block_size, int block_shift,
                               int64_t block_stride_rows, bool vec) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int64_t t = blockIdx.x;
  const int64_t j0 = ((int64_t)blockIdx.y * kIndexThreads + threadIdx.x) * 4;
  if (j0 >= topk) return;
  const int req = __ldg(req_id + t);
  const int32_t *bt_row = (req >= 0 && req < num_reqs) ? block_table + (int64_t)req * bt_st0 : nullptr;
  const int32_t *src = idx + t * idx_st + j0;
  int32_t *dst = out + t * out_st + j0;
  if (vec && j0 + 4 <= topk) {
    const int4 v = __ldg(reinterpret_cast<const int4 *>(src));
    int4 o;
    o.x = req_to_global(v.x, bt_row, bt_st1, max_blocks, block_size, block_shift, block_stride_rows);
    o.y = req_to_global(v.y, bt_row, bt_st1, max_blocks, block_size, block_shift, block_stride_rows);
    o.z = req_to_global(v.z, bt_row, bt_st1, max_blocks, block_size, block_shift, block_stride_rows);
    o.w = req_to_global(v.w, bt_row, bt_st1, max_blocks, block_size, block_shift, block_stride_rows);
    *reinterpret_cast<int4 *>(dst) = o;
  } else {
    for (int k = 0; k < 4 && j0 + k < topk; ++k)
      dst[k] = req_to_global(__ldg(src + k), bt_row, bt_st1, max_blocks, block_size, block_shift, block_stride_rows);
  }
}

}  // namespace titan

extern "C" int titan_convert_req_index_to_global(const int32_t *req_id, int64_t num_reqs, const int32_t *block_table,
                                                 int64_t block_table_stride_req, int64_t block_table_stride_block,
                                                 int64_t max_blocks_per_req, const int32_t *token_indices,
                                                 int64_t indices_stride_token, int64_t topk, int32_t *out,
                                                 int64_t out_stride_token, int64_t num_tokens, int64_t block_size,
                                                 int64_t block_stride_rows, titan_stream_t stream) {
  using namespace titan;
  if (num_tokens < 0 || topk < 0 || num_reqs < 0 || max_blocks_per_req < 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "convert_req_index: negative size");
  if (block_size <= 0 || block_stride_rows < 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "convert_req_index: block_size must be > 0, block_stride_rows >= 0");
  if (num_tokens == 0 || topk == 0) return TITAN_OK;
  if (req_id == nullptr || token_indices == nullptr || out == nullptr ||
      (block_table == nullptr && num_reqs > 0 && max_blocks_per_req > 0))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "convert_req_index: null pointer");
  if (num_tokens > 0x7fffffffLL) return fail(TITAN_ERR_INVALID_ARGUMENT, "convert_req_index: too many tokens");
  const int64_t per_cta = 4 * kIndexThreads;
  const int64_t tiles = (topk + per_cta - 1) / per_cta;
  if (tiles > 65535) return fail(TITAN_ERR_INVALID_ARGUMENT, "convert_req_index: topk too large");
  int block_shift = -1;
  for (int sh = 0; sh < 62; ++sh)
    if ((1ll << sh) == block_size) block_shift = sh;
  const bool vec = (uintptr_t)token_indices % 16 == 0 && (uintptr_t)out % 16 == 0 && indices_stride_token % 4 == 0 &&
                   out_stride_token % 4 == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_tokens, (unsigned)tiles, 1);
  cfg.blockDim = dim3(kIndexThreads);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, req_index_to_global_kernel, req_id, num_reqs, block_table,
                                     block_table_stride_req, block_table_stride_block, max_blocks_per_req,
                                     token_indices, indices_stride_token, topk, out, out_stride_token, block_size,
                                     block_shift, block_stride_rows, vec);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "convert_req_index launch: %s", cudaGetErrorString(e));
  return TITAN_OK;
}
