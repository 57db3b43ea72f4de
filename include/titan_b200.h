/*
 * titan_b200.h — C ABI of the B200 (sm_100a) GLM-5.3 sparse-MLA decode path.
 *
 * The path's operations, each an `extern "C"` launcher that takes plain
 * device pointers, sizes, strides and a CUDA stream, launches on that stream,
 * never synchronises and never allocates.  The caller owns every buffer.
 *
 *   titan_store_int8              replaces kernels/titan_kv.py:23-28
 *   titan_mla_sparse_attention    replaces kernels/titan_mla.py:452-581
 *   titan_moe_align_small         replaces kernels/titan_moe_align.py:49-81
 *   titan_moe_split_align         replaces profiles/sm74/titan_prefill/moe_split_align.py:204-223
 *   titan_convert_req_index_to_global / titan_mla_sparse_attention_paged
 *                                 replace the index conversion before the
 *                                 reader, integration/titan_backend.py:48-54
 *
 * The Python modules titan_kv / titan_mla / titan_moe_align / titan_index /
 * titan_moe_split_align keep the reference's names, argument meaning and
 * exception types and call these entry points (through ctypes, or the
 * CPython fast-call module for the hot launchers).
 *
 * Return value: TITAN_OK (0) or a non-zero TITAN_ERR_* code; the message of
 * the last failure on the calling thread is available from titan_last_error().
 *
 * Byte layout of one INT8 KV row ("528-byte row", kernels/titan_kv.py:19-21,
 * kernels/titan_mla.py:4-7): bytes [0,512) int8 latent values, bytes [512,516)
 * little-endian fp32 scale, bytes [516,528) zero.
 */
#ifndef TITAN_B200_H
#define TITAN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t / CUstream handle (0 = legacy default stream). */
typedef struct CUstream_st *titan_stream_t;

#define TITAN_OK 0
#define TITAN_ERR_INVALID_ARGUMENT 1 /* shape / dtype / alignment rejected on the host */
#define TITAN_ERR_CUDA 2             /* a CUDA runtime call failed */
#define TITAN_ERR_UNSUPPORTED 3      /* valid for the reference but not built here */

#define TITAN_LATENT_DIM 512
#define TITAN_ROW_BYTES 528
#define TITAN_HEAD_GROUP 16
#define TITAN_MOE_NUM_EXPERTS 288
#define TITAN_MOE_TOPK 8
#define TITAN_MOE_BLOCK 8

/* ABI version (major * 100 + minor). */
int titan_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char *titan_last_error(void);

/*
 * INT8 latent KV writer.  Replaces `store_int8(x, cache, slots)`,
 * kernels/titan_kv.py:23-28 (kernel body :7-21).
 *
 * For i < n_slots with s = slots[i] >= 0: quantise x[i, 0:512] (bf16) to the
 * 528-byte row at cache + (s / block_size) * cache_stride0 + (s % block_size) *
 * cache_stride1.  scale = max(max|x| / 127, 1e-12) (IEEE fp32 division),
 * q = clamp(nearbyint(x / scale), -127, 127).  Negative slots are skipped.
 * Slots whose block index is >= num_blocks are skipped as well (the reference
 * would write out of bounds there).
 *
 *   x               bf16, row i at x + i * x_row_stride elements; last dim contiguous
 *   cache           int8 (or uint8) base pointer
 *   cache_stride0   bytes between blocks;  cache_stride1  bytes between slots of a block
 *   slots           int64 (slots_is_int64 = 1) or int32 (0), n_slots entries
 */
int titan_store_int8(const void *x, int64_t x_row_stride,
                     void *cache, int64_t num_blocks, int64_t block_size,
                     int64_t cache_stride0, int64_t cache_stride1,
                     const void *slots, int slots_is_int64, int64_t n_slots,
                     titan_stream_t stream);

/*
 * Workspace bytes titan_mla_sparse_attention needs for a split-KV launch
 * (0 when num_kv_splits == 1).  Mirrors the reference's `mid_out` buffer,
 * kernels/titan_mla.py:533-537 (layout differs: fp32 partial outputs plus a
 * separate natural-log LSE array).
 */
int64_t titan_mla_workspace_bytes(int64_t num_tokens, int64_t num_heads,
                                  int64_t num_kv_splits);

/*
 * Diagnostic: how many thread-block clusters of `cluster_size` CTAs (1..16) of
 * the MLA kernel the current device can hold at once (-1 on error).  The
 * launcher uses the same query to pick its cluster size.
 */
int titan_mla_max_active_clusters(int cluster_size);

/*
 * Diagnostic: like titan_mla_max_active_clusters, but counting clusters whose
 * CTAs each have an SM to themselves (-1 on error).  Clusters beyond this
 * count share SMs with other MLA CTAs; the automatic split policy of the
 * Python layer avoids that.
 */
int titan_mla_max_exclusive_clusters(int cluster_size);

/*
 * Sparse NoPE MLA attention over an INT8 528-byte-row cache.  Replaces
 * `triton_mla_sparse_attention(q, kv, indices, sm_scale, num_kv_splits,
 * sm_count)`, kernels/titan_mla.py:452-581 (kernels :59-429).
 *
 *   q        bf16 [num_tokens, num_heads, 512]; strides in elements, last dim contiguous
 *   kv       int8 rows; row r at kv + r * kv_row_stride bytes, r in [0, seq_kv)
 *   indices  int32 [num_tokens, topk]; token stride in elements, last dim contiguous.
 *            An index outside [0, seq_kv) is masked (contributes nothing).
 *   out      bf16 [num_tokens, num_heads, 512]; strides in elements
 *   sm_scale softmax scale (not pre-multiplied by log2 e)
 *   num_kv_splits  >= 1; 1 = single pass, otherwise split-KV + combine
 *   workspace      >= titan_mla_workspace_bytes(...) bytes of device memory, 16-byte aligned
 *
 * kv and kv_row_stride must be 16-byte aligned (rows are read with 16-byte
 * loads).  A token whose indices are all masked produces exact zeros.
 */
int titan_mla_sparse_attention(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                               const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                               const int32_t *indices, int64_t indices_stride_token, int64_t topk,
                               void *out, int64_t out_stride_token, int64_t out_stride_head,
                               int64_t num_tokens, int64_t num_heads, float sm_scale,
                               int64_t num_kv_splits, void *workspace, int64_t workspace_bytes,
                               titan_stream_t stream);

/*
 * Arrival counters for titan_mla_sparse_attention_sem: the number of int32
 * entries (num_tokens * ceil(num_heads / 16) * 16).
 */
int64_t titan_mla_semaphore_count(int64_t num_tokens, int64_t num_heads);

/*
 * titan_mla_sparse_attention with the split merge done inside the split
 * kernel.  Same arguments and results (within the fp32 summation-order
 * tolerance) as titan_mla_sparse_attention, which this also replaces
 * (kernels/titan_mla.py:452-581: the split kernel :258-354 and the combine
 * kernel :357-429 become one launch).  When the splits of a token form several
 * thread-block clusters and at most as many clusters as CTAs per cluster,
 * each cluster CTA publishes its partial slice and takes a ticket from an
 * arrival counter; the last CTA of each cluster rank merges that rank's slice
 * over all clusters and writes the bf16 output, then resets its counter to
 * zero.  Otherwise, for 8 <= num_kv_splits <= 160 and a grid of at most the
 * CTAs that fit on the device at once, the launch is cooperative and without
 * clusters: the split CTAs of a token publish their partials, meet at the
 * token's counter (bounded wait: device error 3 if it runs out) and each
 * merges a share of the columns; the last CTA to leave zeroes the counters.
 * Larger grids fall back to the combine kernel.
 *
 *   semaphores       int32 [semaphore_count] device array, all zero before the
 *                    first call; every call leaves it zero again.  Calls that
 *                    share one array must be ordered on the GPU (same stream,
 *                    or event-ordered): overlapping calls race on the counters.
 *   semaphore_count  >= titan_mla_semaphore_count(num_tokens, num_heads)
 */
int titan_mla_sparse_attention_sem(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                   const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                   const int32_t *indices, int64_t indices_stride_token, int64_t topk,
                                   void *out, int64_t out_stride_token, int64_t out_stride_head,
                                   int64_t num_tokens, int64_t num_heads, float sm_scale,
                                   int64_t num_kv_splits, void *workspace, int64_t workspace_bytes,
                                   int32_t *semaphores, int64_t semaphore_count, titan_stream_t stream);

/*
 * Request-local top-k positions -> global cache rows (paged KV cache).
 * Replaces the conversion the reference's backend runs before the sparse MLA
 * reader (integration/titan_backend.py:48-54), vLLM's
 * `triton_convert_req_index_to_global_index` (v1/attention/backends/mla/
 * sparse_utils.py, a third-party dependency of the reference):
 *   out[t, j] = block_table[req_id[t], tok / block_size] * block_stride_rows
 *               + tok % block_size,   tok = token_indices[t, j]
 *   out[t, j] = -1 if tok < 0, tok / block_size >= max_blocks_per_req, or
 *               req_id[t] outside [0, num_reqs) (the last one is a widening:
 *               vLLM reads out of bounds there).
 * block_stride_rows = block_size for a contiguous cache.  All arrays int32;
 * strides in elements; block_table_stride_block is the stride between the
 * blocks of one request (1 when contiguous).
 */
int titan_convert_req_index_to_global(const int32_t *req_id, int64_t num_reqs, const int32_t *block_table,
                                      int64_t block_table_stride_req, int64_t block_table_stride_block,
                                      int64_t max_blocks_per_req, const int32_t *token_indices,
                                      int64_t indices_stride_token, int64_t topk, int32_t *out,
                                      int64_t out_stride_token, int64_t num_tokens, int64_t block_size,
                                      int64_t block_stride_rows, titan_stream_t stream);

/*
 * titan_mla_sparse_attention_sem on request-local positions: the gather
 * translates each position with the mapping of
 * titan_convert_req_index_to_global (a translated row outside [0, seq_kv) is
 * masked, like any index), so the conversion kernel, its launch and its
 * global-index round trip disappear (the reference runs the conversion and
 * the reader back to back, integration/titan_backend.py:49-54).  Results are
 * bit-identical to the conversion followed by the sem/combine entry point.
 * semaphores may be null (combine kernel for multi-cluster splits).
 */
int titan_mla_sparse_attention_paged(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                     const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                     const int32_t *token_indices, int64_t indices_stride_token, int64_t topk,
                                     const int32_t *req_id, int64_t num_reqs, const int32_t *block_table,
                                     int64_t block_table_stride_req, int64_t block_table_stride_block,
                                     int64_t max_blocks_per_req, int64_t block_size, int64_t block_stride_rows,
                                     void *out, int64_t out_stride_token, int64_t out_stride_head,
                                     int64_t num_tokens, int64_t num_heads, float sm_scale,
                                     int64_t num_kv_splits, void *workspace, int64_t workspace_bytes,
                                     int32_t *semaphores, int64_t semaphore_count, titan_stream_t stream);

/*
 * Allocation-free variant of titan_mla_sparse_attention (no counterpart in the
 * reference).  For callers that cannot allocate device memory — a plugin whose
 * host engine owns the whole device pool, or work issued while another thread
 * captures a stream in global capture mode, where cudaMalloc is refused.  The
 * split-KV scratch is a static device array of titan_mla_noalloc_scratch_bytes()
 * bytes (8 MiB) that every GPU loading the library holds until exit; a call that
 * needs more (titan_mla_workspace_bytes(T, H, num_kv_splits) > 8 MiB) fails with
 * TITAN_ERR_INVALID_ARGUMENT.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls on a device share the one array: calls that overlap on the
 * GPU (different streams, no ordering) race.  Nothing in the scratch needs to
 * start at zero; each call overwrites what it reads.  Allocates nothing.
 */
int64_t titan_mla_noalloc_scratch_bytes(void);
int titan_mla_sparse_attention_noalloc(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                       const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                       const int32_t *indices, int64_t indices_stride_token, int64_t topk,
                                       void *out, int64_t out_stride_token, int64_t out_stride_head,
                                       int64_t num_tokens, int64_t num_heads, float sm_scale,
                                       int64_t num_kv_splits, titan_stream_t stream);

/*
 * Small stable MoE route alignment (B1..8, top-8, 288 experts, block 8).
 * Replaces `titan_moe_align_small(topk_ids, ...)`, kernels/titan_moe_align.py:49-81
 * (kernel :12-46).
 *
 *   topk_ids    int32 (ids_is_int64 = 0) or int64 (1), num_routes = 8 * B entries, contiguous
 *   sorted_ids  int32 [8 * num_routes]   (padding entries hold num_routes)
 *   expert_ids  int32 [num_routes]       (unused blocks hold -1)
 *   postpad     int32 [1]                (sum of per-expert counts rounded up to 8)
 *   num_warps   1, 2 or 4: CTA size; does not change the outputs
 *
 * Routes outside [0, 288) are ignored.
 */
int titan_moe_align_small(const void *topk_ids, int ids_is_int64, int64_t num_routes,
                          int32_t *sorted_ids, int32_t *expert_ids, int32_t *postpad,
                          int num_warps, titan_stream_t stream);

/*
 * Split MoE block alignment for whole-expert prefill: the routed rows sorted
 * by expert into four block lists, block sizes {64, 48, 32, 16}, one Marlin
 * launch per list.  Replaces `split_align(topk_ids, E, buf)`,
 * profiles/sm74/titan_prefill/moe_split_align.py:204-223 (kernels :44-169).
 * One launch of one 16-CTA thread-block cluster (8 CTAs where the device
 * cannot hold 16; the environment variable TITAN_SPLIT_ALIGN_CLUSTER=8, read
 * at the first call on a device, forces 8); no scratch memory.
 *
 *   topk_ids     int32 (ids_is_int64 = 0) or int64 (1), num_routes = M * topk
 *                entries, contiguous; int64 ids are narrowed to int32 first
 *   num_experts  E in [1, TITAN_SPLIT_ALIGN_MAX_EXPERTS]; ids outside [0, E) are dropped
 *   cover_tab    int32 [cover_rows][4] on the device: blocks of each size in the
 *                cheapest cover of r rows (moe_split_align.py:172-185);
 *                cover_rows >= num_routes + 1.  Every block of a cover must
 *                hold at least one row (true of the cost-optimal table, whose
 *                covers pad less than their smallest block): the padding and
 *                the rows then land in disjoint entries, which the kernel
 *                writes without ordering them.
 *   t_max        capacity the lists were allocated for, num_routes <= t_max:
 *   sorted_ids   host array of 4 device pointers, list k int32 [t_max + B_k * E]
 *   expert_ids   host array of 4 device pointers, list k int32 [(t_max + B_k * E) / B_k + 1]
 *   ntpp         int32 [4]: rows of each list (padding included)
 *
 * Padded entries of sorted_ids hold num_routes; entries beyond what the
 * algorithm writes are left untouched.  Calls sharing lists must be ordered.
 */
#define TITAN_SPLIT_ALIGN_MAX_EXPERTS 1024
int titan_moe_split_align(const void *topk_ids, int ids_is_int64, int64_t num_routes, int64_t num_experts,
                          const int32_t *cover_tab, int64_t cover_rows, int64_t t_max,
                          int32_t *const *sorted_ids, int32_t *const *expert_ids, int32_t *ntpp,
                          titan_stream_t stream);
/* Dynamic shared memory the split-align kernel uses for num_experts experts. */
int64_t titan_moe_split_align_smem_bytes(int64_t num_experts);

/*
 * Host <-> device staging (no counterpart in the reference, whose callers keep
 * every operand on the GPU).  titan_copy moves `bytes` from src to dst with a
 * kernel launched on `stream` (ordered after the stream's previous kernel, as
 * a programmatic dependent); either side may be device memory or PINNED host
 * memory (cudaHostAlloc / cudaMallocHost / torch pin_memory), which the kernel
 * reads or writes through its device mapping: one PCIe round trip instead of
 * a copy engine's fixed latency, for the small per-call transfers of decode.
 * Pageable host memory and overlapping buffers are rejected
 * (TITAN_ERR_INVALID_ARGUMENT).
 *
 * titan_device_pointer returns the device-accessible address of `ptr` (the
 * device mapping of pinned host memory; device memory unchanged), e.g. to
 * hand a pinned host buffer to titan_mla_sparse_attention as `out` so the
 * reader stores its result straight into host memory.
 */
int titan_copy(void *dst, const void *src, int64_t bytes, titan_stream_t stream);
/* titan_copy with flags.  TITAN_COPY_SRC_READY: no earlier work on the stream
 * writes src (e.g. host-written input in pinned memory), so the kernel issues
 * its first round of loads before waiting for the preceding kernel, hiding
 * the source's latency behind that kernel's tail; stores still wait. */
#define TITAN_COPY_SRC_READY 1
int titan_copy_ex(void *dst, const void *src, int64_t bytes, int flags, titan_stream_t stream);
int titan_device_pointer(const void *ptr, void **device_ptr_out);

/*
 * Device-side error word: kernels set it instead of trapping when a bounded
 * wait gives up.  Reads (and, if clear_after is non-zero, resets) the word of
 * the current device; synchronises the stream first.  0 = no error, 1 = an
 * mbarrier wait (a TMA or bulk copy that did not land) ran out, 2 = a count
 * exceeded a fixed-size list (the excess was dropped), 3 = a CTA of a flat
 * split merge gave up waiting for the other CTAs of its token.  The first
 * error since the last reset is kept.
 */
int titan_device_error(int *error_out, int clear_after, titan_stream_t stream);

/*
 * W4A16 MoE GEMM over one split-align block list, on the tcgen05 tensor cores.
 * Replaces one `moe_wna16_marlin_gemm` call of the split Marlin path,
 * profiles/sm74/titan_prefill/marlin.py:417-444 (uint4b8 weights, group 128,
 * bf16 activations, fp32 accumulation).  For each block b < ntpp[0] /
 * block_size with e = expert_ids[b] and routed rows s = sorted_ids[b * bs + j]
 * (ids >= size_m * top_k are padding and are skipped):
 *   C[s, n] = sum_k A[s / top_k, k] * bf16((q[e,n,k] - 8) * scales[e, k/128, n])
 *   times topk_weights[s] when mul_topk_weights.
 *   a            bf16 [size_m rows][k], rows a_stride elements apart (16-byte aligned)
 *   c            bf16, rows c_stride elements apart; only listed rows are written
 *   wq_packed    uint8, E x n x k / 2 bytes: per expert, 128-feature tiles in
 *                pairs, per pair and 128-wide k step (one scale group) the
 *                pair's 8 KB tiles back to back, each [k quarter][row][16 B]
 *                (kernels/titan_moe_gemm.py pack_weights); 16-byte aligned;
 *                titan_moe_w4a16_packed_bytes
 *   scales       bf16 [E][k/128][n], 16-byte aligned
 *   sorted_ids, expert_ids (max_blocks entries), ntpp: one list of
 *                titan_moe_split_align; block_size in {16, 32, 48, 64}
 *   n % 128 == 0, k % 128 == 0.  One persistent launch, no scratch memory.
 */
int64_t titan_moe_w4a16_packed_bytes(int64_t num_experts, int64_t n, int64_t k);
int titan_moe_w4a16_gemm(const void *a, int64_t a_stride, int64_t size_m, void *c, int64_t c_stride,
                         const void *wq_packed, const void *scales, const int32_t *sorted_ids,
                         const int32_t *expert_ids, int64_t max_blocks, const int32_t *ntpp,
                         const float *topk_weights, int block_size, int top_k, int mul_topk_weights,
                         int64_t num_experts, int64_t n, int64_t k, titan_stream_t stream);

/*
 * Pool top-k of the sparse indexer and its expansion into the MLA reader's
 * token indices.  Replaces the CUDA top-k over pool logits and
 * `kpool_ops.expand_pools_and_append_tail` of the reference's indexer
 * (integration/patch_decode_indexer.py:49-104, integration/
 * patch_indexer_sharding.py:58-104; expansion as tests/
 * verify_indexer_sharding.py:68-76 `expand_row`).  For each of num_rows
 * query rows: valid pools p < min(seq_lens[t] / pool_size, ld); the k pools of
 * largest logits[t * ld + p] by logit descending (equal: smaller pool first;
 * NaN above every number), -1 where fewer are valid; out[t][pool i + o] =
 * pool_i * pool_size + o (-1 for -1), then pool_size - 1 tail entries
 * (seq_len / pool) * pool + o for o < seq_len % pool (else -1), then -1 up
 * to `width` (>= k * pool_size + pool_size - 1; 2176 for k = 512, pool 4).
 * k <= 1024, pool_size <= 64.  One CTA per row.
 */
int titan_pool_topk_expand(const float *logits, int64_t ld, const int32_t *seq_lens, int64_t num_rows, int k,
                           int pool_size, int32_t *out, int64_t out_stride, int width, titan_stream_t stream);

/*
 * Self-test of the bounded waits (no counterpart in the reference): one warp
 * waits on an mbarrier that nothing completes, gives up after about
 * `limit_cycles` SM clocks (1 .. 4e9), sets the device error word to 1
 * (mbarrier timeout) and returns; the context stays usable.  Lets a test show
 * that a wait that runs out is reported through titan_device_error.
 */
int titan_selftest_bounded_wait(long long limit_cycles, titan_stream_t stream);

/*
 * Self-test of the bounded counter wait of the flat split merge (no
 * counterpart in the reference): one thread waits for a device counter that
 * nothing increments, gives up after about `limit_cycles` SM clocks (1 ..
 * 4e9), sets the device error word to 3 and returns; the context stays usable.
 */
int titan_selftest_bounded_spin(long long limit_cycles, titan_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TITAN_B200_H */
