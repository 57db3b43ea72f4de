// Sparse NoPE MLA decode over the INT8 528-byte-row cache.
//
// Semantics follow kernels/titan_mla.py (the reference Triton path):
//   :59-182  per (token, 16-head group), over top-k positions of one range:
//            s_j = (q . k_j) * scale_j * sm_scale * log2(e)   (k_j int8 -> bf16, exact)
//            masked (index < 0, >= seq_kv, or past the range) -> -1e30, p = 0
//            online softmax in base 2; acc += bf16(p_j * scale_j) * k_j
//   :185-255 single range (num_kv_splits == 1): out = bf16(acc / l), l == 0 -> zeros
//   :258-354 split range s of ceil(topk / S): partial acc / l (fp32) and
//            lse = (m + log2 l) * ln 2
//   :357-429 combine: sum_s exp(lse_s - M) o_s / sum_s exp(lse_s - M), bf16
//
// B200 design: one CTA (8 warps) per (token, split, 16-head group).
//  * Row gather by the tensor memory accelerator: per 32-row tile, lane 0 of
//    each of the eight warps issues one `cp.async.bulk.tensor ...
//    tile::gather4` load (four rows by row index, 544-byte boxes) into a
//    three-stage shared-memory ring, two tiles ahead of the math, completing
//    on the stage's mbarrier.
//    Rows outside [0, seq_kv) read as zeros (TMA bounds fill); a group whose
//    four rows are all masked is not issued.  The row scale arrives with the
//    row (bytes 512..515).  Warp w owns latent dims [64 w, 64 w + 64); lane
//    (g, c) reads 16 bytes of each of its four rows at byte 64 w + 16 c:
//    exactly its MMA B fragments, bank-conflict free in the 544-byte pitch.
//    The indices reach shared memory through warp 0's 4-byte cp.async ring
//    five tiles ahead (paged: positions eight and block-table entries five
//    tiles ahead), so no thread waits on a load issued one tile earlier.
//  * QK: mma.sync m16n8k16 with fp32 accumulate (A = 16 heads x 16 dims of q
//    in registers).  Decode-length CTAs keep the reference's bf16 operands
//    (int8 -> bf16 exact through the fp32 magic number); single-pass CTAs of
//    at least kF16MinTiles tiles (prefill shapes) use f16: int8 -> f16 exact
//    in one PRMT + one packed add per pair, q scaled by a power of two per
//    warp and head, undone in the score reduction.  The k dimension is
//    permuted identically for q and k so that each lane's 16 contiguous bytes
//    feed four k-steps.  The 8 warps' partial scores meet in shared memory;
//    16 lanes per head run the online softmax, whose running max moves only
//    by steps above kLazyMax (log2 units); tiles whose rows are all masked
//    are skipped.
//  * PV: the K fragments are transposed in registers with movmatrix (rows
//    become the reduction dim), A = bf16(p * scale) (f16 path: f16(p * scale
//    * 2^-e), e the exponent of the largest row scale so far) from shared
//    memory; each accumulator lane then owns 16 contiguous output dims.
//  * Split merge: the C <= 16 splits of a (token, head group) that form one
//    thread-block cluster merge through distributed shared memory, each CTA
//    reducing 512 / C dims; a single cluster writes the bf16 output directly.
//    With more clusters than one, each cluster writes one partial (o, lse);
//    given arrival counters, the last CTA of each rank to finish merges that
//    rank's slice over all partials (no second kernel).  When that does not
//    apply (more partials than CTAs per cluster), counters are given and the
//    grid fits on the device, the launch drops the clusters and is
//    cooperative: every split CTA writes its partial, the CTAs of a token
//    meet at a counter barrier and each merges a share of the output (flat
//    merge).  Otherwise a combine kernel, launched as a programmatic
//    dependent, merges the partials.
#include <cuda.h>  // CUtensorMap

#include "titan_common.cuh"

namespace titan {
namespace mla {

constexpr int kD = TITAN_LATENT_DIM;       // 512
constexpr int kHeads = TITAN_HEAD_GROUP;    // 16 heads per CTA
constexpr int kWarps = 8;                   // 64 dims per warp
constexpr int kThreads = kWarps * 32;
constexpr int kBN = 32;                     // rows per tile (four 8-row n-tiles)
constexpr int kRedStride = 40;              // floats per head row of a warp's partial scores
constexpr int kPStrideWords = 36;           // 32-bit words per head row of P (f16, 32 rows + pad)
constexpr int kMaxCluster = 16;
constexpr int kRing = 3;                    // row-gather ring: tiles in flight ahead of the math + 1
constexpr int kIdxRing = 8;                 // index ring: indices are staged up to eight tiles ahead
constexpr int kRowPitch = 544;              // gathered row in shared memory: 528 B + 16 B of bounds fill
constexpr int kGroupBytes = 4 * kRowPitch;  // one gather4 load: 2176 B, a multiple of 128
constexpr int kGroups = kBN / 4;            // gather4 loads per tile
constexpr float kNegLarge = -1.0e30f;       // finite mask sentinel, kernels/titan_mla.py:112
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazyMax = 8.0f;            // the running max moves when a tile exceeds it by more (log2 units)
constexpr int kF16MinTiles = 16;            // single-pass CTAs of at least this many tiles use the f16 arithmetic

struct Smem {
  float red[kWarps][kHeads * kRedStride];  // partial scores of each warp
  uint32_t p[kHeads * kPStrideWords];      // f16(p * scale * 2^-e), n-order
  float rcv[kHeads * kD];                  // cluster merge: [C][16][512/C] slices pushed by the peers
  union alignas(128) {
    float stage[kHeads * kD];              // cluster merge: this CTA's acc as [owner][16][512/C]
    struct {
      uint8_t rows[kRing][kGroups][kGroupBytes];  // tile loop: stage = 8 gather4 groups of 4 rows
      int32_t idx[kIdxRing][kBN];          // row indices (paged: request-local positions) of tile j, slot j % kIdxRing
      int32_t base[kIdxRing][kBN];         // paged: block-table entry of each position of tile j
    } ring;                                // (dead before the merge stages its accumulator)
  } u;
  float2 cml[kMaxCluster][kHeads];         // cluster merge: (m, l) pushed by each peer
  alignas(8) uint8_t vbits[kRing][kGroups];  // per stage and gather4 group: bit k = slot k valid
  float scale[kBN];                        // row scales of the current tile, n-order (masked: unused)
  float qf[kWarps][kHeads];                // 2^-kq: undoes warp w's f16 scaling of head h's q
  float alpha[kHeads];
  float2 ml[kHeads];                       // final (m, l) of this CTA
  float cw[kMaxCluster][kHeads];           // cluster merge weights
  float cM[kHeads], cL[kHeads];
  alignas(8) uint64_t merge_bar;           // counts the bytes the cluster pushes here
  uint64_t row_bar[kRing];                 // per ring stage: one arrival per warp + its gather4 bytes
  int last;                                // cross-cluster merge: this CTA arrived last; flat merge: its wait ended
};

// Two CTAs per SM: 228 KB of shared memory per SM, 1 KB reserved per CTA.
static_assert(2 * (sizeof(Smem) + 1024) <= 228 * 1024, "the reader must fit twice per SM");
static_assert(kGroups == kWarps, "warp w issues gather4 group w");
static_assert(offsetof(Smem, p) % 16 == 0 && (kPStrideWords * 4) % 16 == 0, "ldmatrix reads 16-byte rows of P");
static_assert(offsetof(Smem, u) % 128 == 0 && kGroupBytes % 128 == 0, "gather4 destinations are 128-byte aligned");

struct Params {
  const __nv_bfloat16 *q;
  int64_t q_st, q_sh;
  const uint8_t *kv;
  int64_t kv_rs, seq_kv;
  const int32_t *idx;
  int64_t idx_st, topk;
  __nv_bfloat16 *out;
  int64_t out_st, out_sh;
  float *part_o;    // [T][NC][Hp][512]  (partials, one per cluster)
  float *part_lse;  // [T][NC][Hp]
  int T, H, Hp;
  int S;            // splits per (token, head group)
  int C;            // splits per cluster (1, 2, 4, 8 or 16; divides S)
  int logC;         // log2(C)
  int NC;           // clusters per (token, head group) = S / C = partials to combine
  int64_t split_topk;
  float scale_log2;  // sm_scale * log2(e)
  int *sem;          // [T][groups][16] arrival counters (zero between calls) or null: combine kernel
                     // (cluster launches: one per cluster rank; flat merge: arrivals, departures)
  // Paged launches (kPaged): idx holds request-local token positions; row =
  // block_table[req_id[t], tok / block_size] * block_stride_rows + tok % block_size.
  const int32_t *req_id;
  const int32_t *block_table;
  int64_t bt_st0, bt_st1;
  int num_reqs, max_blocks, block_size, block_shift;  // block_shift >= 0: block_size is 2^block_shift
  int64_t block_stride_rows;
};

// Float position of logical dim dd (0 <= dd < D = 512 / C) in the row of
// (head hl, owner) of the cluster-merge stage and receive buffers.  The
// 16-byte chunks of a row are XOR-swizzled (a bijection within the row): a
// quarter-warp's 16-byte staging stores, which cover two heads and two owners
// (C = 16) or two chunk halves (C < 16) at equal offsets, then fall on eight
// distinct bank groups instead of two.
__device__ __forceinline__ int merge_pos(int hl, int owner, int dd) {
  const int chunk = dd >> 2;
  return ((chunk ^ ((hl & 1) << 1) ^ ((chunk >> 3) & 1) ^ (owner & 1)) << 2) | (dd & 3);
}

// Last-arriver merge of the NC <= C cluster partials of (token t, head group
// hg) over the dims of cluster rank `rank` (D = 512 / C = 32 kPer dims), same
// arithmetic as the combine kernel below.  16 lanes per head: lane j holds
// partial j's LSE and owns pairs j + 16 k, k < kPer; every load is issued
// before the first use.
template <int kPer>
__device__ __forceinline__ void merge_cluster_partials(const Params &p, int t, int hg, uint32_t rank, int tid) {
  constexpr int kSlots = kMaxCluster / kPer;  // = C, upper bound of NC
  constexpr float kLog2e = 1.4426950408889634f;
  const int h = tid >> 4, j = tid & 15;
  const int hh = hg * kHeads + h;
  const bool live = hh < p.H;
  const int64_t split_stride = (int64_t)p.Hp * kD;
  const int dim = (int)rank * (32 * kPer) + 2 * j;
  const float *o_src = p.part_o + ((int64_t)t * p.NC * p.Hp + hh) * kD + dim;
  const float lse = (live && j < p.NC) ? __ldcg(p.part_lse + ((int64_t)t * p.NC + j) * p.Hp + hh) : -INFINITY;
  float2 ov[kSlots][kPer];
#pragma unroll
  for (int s = 0; s < kSlots; ++s)
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      ov[s][k] = (live && s < p.NC) ? __ldcg(reinterpret_cast<const float2 *>(o_src + s * split_stride + 32 * k))
                                    : make_float2(0.f, 0.f);
  float m = fmaxf(kNegLarge, lse);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float w = ex2_approx((lse - m) * kLog2e);
  float L = w;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  const float inv = L > 0.0f ? 1.0f / L : 1.0f;
  float2 sum[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) sum[k] = make_float2(0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kSlots; ++s) {
    const float ws = __shfl_sync(0xffffffffu, w, s, 16);  // partial s's weight, from lane s of this head
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      sum[k].x += ws * ov[s][k].x;
      sum[k].y += ws * ov[s][k].y;
    }
  }
  if (live) {
    __nv_bfloat16 *dst = p.out + (int64_t)t * p.out_st + (int64_t)hh * p.out_sh + dim;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      *reinterpret_cast<uint32_t *>(dst + 32 * k) = pack_bf16x2(sum[k].x * inv, sum[k].y * inv);
  }
}

// Flat split merge (cluster-less launches given arrival counters): the S
// CTAs of (token t, head group hg) have each written a normalised partial and
// its LSE; they meet at a counter barrier, then each merges a share of the
// 256 units (head, 32-dim block) of the token over all S partials: CTA
// `split` takes units split, split + S, ...  Thread (group g, item = (unit
// slot, float4 column)) loads partials g, g + groups, ... with their LSEs in
// one round trip (each warp load is four whole 128-byte lines) and weighs
// them against its own largest LSE m_g; the groups then meet in shared
// memory: out = sum_g acc_g e^(m_g - M) / sum_g l_g e^(m_g - M), M = max m_g,
// the combine kernel's result up to rounding.  The launcher uses this only
// for 8 <= S <= 160 and grids that fit on the device at once, launched
// cooperatively so that every CTA a waiter waits for is resident.  Counters:
// [0] arrivals, [1] departures; the last CTA to depart (every CTA has
// finished waiting by then) zeroes both for the next call.
constexpr int kFlatPre = 15;    // partials per thread (at most 15 for 8 <= S <= 160), all loaded at once
constexpr int kFlatMinS = 8;     // 8 x 32 = 256 (unit slot, column) items at most
constexpr int kFlatMaxS = 160;
constexpr int kFlatUnits = kHeads * (kD / 32);
static_assert(6 * kThreads <= kHeads * kD, "the group sums and (m, l) pairs fit the dead staging area");
// Every split count the flat merge takes gives each thread at most kFlatPre
// partials (all loaded in one round trip) and at least one thread group.
constexpr bool flat_shares_fit() {
  for (int S = kFlatMinS; S <= kFlatMaxS; ++S) {
    const int groups = kThreads / (8 * ((kFlatUnits + S - 1) / S));
    if (groups < 1 || (S + groups - 1) / groups > kFlatPre) return false;
  }
  return true;
}
static_assert(flat_shares_fit(), "flat merge shares exceed the preloaded partials");

__device__ __forceinline__ void merge_flat_share(const Params &p, Smem &sm, int t, int hg, int split, int tid) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int S = p.NC;
  const int slots = (kFlatUnits + S - 1) / S;  // units of the widest share (<= 32)
  const int items = 8 * slots;
  const int groups = kThreads / items;  // ceil(S / groups) <= kFlatPre for every S the launcher allows
  const int grp = tid / items, item = tid - grp * items;
  const int u = split + S * (item >> 3), q4 = item & 7;
  const int h = u & (kHeads - 1), blk = u >> 4;  // head and 32-dim block of unit u
  const int hh = hg * kHeads + h;
  const bool mine = grp < groups && u < kFlatUnits && hh < p.H;
  const int64_t split_stride = (int64_t)p.Hp * kD;
  const float *o_t = p.part_o + ((int64_t)t * S * p.Hp + hh) * kD + 32 * blk + 4 * q4;
  const float *lse_t = p.part_lse + (int64_t)t * S * p.Hp + hh;

  float4 o_pre[kFlatPre];
  float lse_pre[kFlatPre];
#pragma unroll
  for (int k = 0; k < kFlatPre; ++k) {
    const int s = grp + groups * k;
    const bool ld = mine && s < S;
    o_pre[k] = ld ? __ldcg(reinterpret_cast<const float4 *>(o_t + s * split_stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
    lse_pre[k] = ld ? __ldcg(lse_t + (int64_t)s * p.Hp) : -INFINITY;
  }
  float m = kNegLarge;
#pragma unroll
  for (int k = 0; k < kFlatPre; ++k) m = fmaxf(m, lse_pre[k]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float l = 0.0f;
#pragma unroll
  for (int k = 0; k < kFlatPre; ++k) {
    const float w = ex2_approx((lse_pre[k] - m) * kLog2e);
    l += w;
    acc.x += w * o_pre[k].x;
    acc.y += w * o_pre[k].y;
    acc.z += w * o_pre[k].z;
    acc.w += w * o_pre[k].w;
  }
  float4 *part = reinterpret_cast<float4 *>(sm.u.stage);  // [groups][items] sums; the ring is dead
  float2 *part_ml = reinterpret_cast<float2 *>(sm.u.stage + 4 * kThreads);  // [groups][items] (m_g, l_g)
  if (grp < groups) {
    part[tid] = acc;
    part_ml[tid] = make_float2(m, l);
  }
  __syncthreads();
  if (grp == 0 && mine) {
    float M = m;
    for (int g2 = 1; g2 < groups; ++g2) M = fmaxf(M, part_ml[g2 * items + item].x);
    const float a0 = ex2_approx((m - M) * kLog2e);
    float L = l * a0;
    acc.x *= a0;
    acc.y *= a0;
    acc.z *= a0;
    acc.w *= a0;
    for (int g2 = 1; g2 < groups; ++g2) {
      const float2 ml = part_ml[g2 * items + item];
      const float4 v = part[g2 * items + item];
      const float a = ex2_approx((ml.x - M) * kLog2e);
      L += ml.y * a;
      acc.x += a * v.x;
      acc.y += a * v.y;
      acc.z += a * v.z;
      acc.w += a * v.w;
    }
    const float inv = L > 0.0f ? 1.0f / L : 1.0f;
    uint2 r;
    r.x = pack_bf16x2(acc.x * inv, acc.y * inv);
    r.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2 *>(p.out + (int64_t)t * p.out_st + (int64_t)hh * p.out_sh + 32 * blk + 4 * q4) = r;
  }
}

__device__ __forceinline__ void merge_flat(const Params &p, Smem &sm, int t, int hg, int split, int tid) {
  const int S = p.NC;
  __syncthreads();  // every partial store of this CTA precedes thread 0's release below
  int *ctr = p.sem + ((int64_t)t * gridDim.y + hg) * kMaxCluster;
  int departed = 0;
  if (tid == 0) {
    // The last to arrive knows it from its own ticket; the others poll.
    sm.last = atom_add_acq_rel_gpu(ctr, 1) == S - 1 || spin_until_at_least(ctr, S, kLongWaitCycles);
    // Departure ticket: relaxed, yet ordered after the arrival / wait by
    // their acquire; the result is first read after the merge, so the round
    // trip overlaps it.
    departed = atom_add_relaxed_gpu(ctr + 1, 1);
  }
  __syncthreads();
  if (sm.last) merge_flat_share(p, sm, t, hg, split, tid);  // else: the error word says so
  if (tid == 0 && departed == S - 1) {
    st_relaxed_gpu(ctr, 0);
    st_relaxed_gpu(ctr + 1, 0);
  }
}

// kCluster: launched with clusters of C >= 2 CTAs (the cluster merge is
// compiled only into these instantiations; C == 1 launches carry none of it).
// kF16: the f16 arithmetic (exact int8 -> f16 in one PRMT + one packed add
// per pair, q scaled per warp and head, P relative to the largest row scale),
// for single-pass CTAs that walk many tiles (prefill shapes): fewer
// instructions per tile, at a fixed cost per CTA that short (decode) CTAs do
// not recover; those keep the reference's bf16 arithmetic.
template <bool kPartialOut, bool kPaged, bool kCluster, bool kF16 = false>
__global__ void __launch_bounds__(kThreads, 2)
    sparse_mla_kernel(const Params p, const __grid_constant__ CUtensorMap rows_map) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  // Long single-pass (f16) launches take the tokens last first: in a causal
  // prefill a token's valid indices grow with its position, so the longest
  // CTAs start first and the short ones fill the last wave (T = 4096:
  // 1.396 -> 1.386 ms).  Decode launches keep the natural order (reversed,
  // B=1 was 0.03 us slower).
  const int tb = blockIdx.x / p.S;
  const int split = blockIdx.x - tb * p.S;
  const int t = kF16 ? p.T - 1 - tb : tb;
  const int hg = blockIdx.y;

  // Ring-stage barriers (one arrival per warp, plus the gather bytes, per
  // use) and, for clusters, the merge barrier.  Cluster peers must be
  // running, with their merge barrier initialised, before anyone writes into
  // their shared memory: initialise, publish to the cluster, arrive now, wait
  // right before the first remote store.  None of this, nor the prefetch of
  // the rows' tensor map, reads memory another kernel writes, so it runs
  // before the programmatic-dependency wait, overlapping the previous grid's
  // tail.
  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) mbar_init(&sm.row_bar[s], kWarps);
    if (kCluster) mbar_init(&sm.merge_bar, 1);
    fence_mbar_init();
  }
  if (tid == 32) prefetch_tensormap(&rows_map);
  __syncthreads();
  if constexpr (kCluster) cluster_arrive_relaxed();
  // Launched as a programmatic dependent of whatever ran before on the stream:
  // CTAs may be resident early, but nothing is read before the previous grid
  // has completed and flushed.
  pdl_wait_primary();
  pdl_launch_dependents();  // the combine (or the next call) may become resident now

  const int64_t start = (int64_t)split * p.split_topk;
  const int64_t end = min(start + p.split_topk, p.topk);
  const int n_rows = end > start ? (int)(end - start) : 0;
  const int n_tiles = (n_rows + kBN - 1) / kBN;
  const int32_t *idx_row = p.idx + (int64_t)t * p.idx_st;
  const int64_t seq_kv = p.seq_kv;

  auto row_ok = [&](int r) { return r >= 0 && (int64_t)r < seq_kv; };
  // Paged: the request of this token (positions of an unknown request, a
  // negative position or a block past the table give row -1; the gather masks
  // rows outside [0, seq_kv) as for any index).  Same mapping as the
  // standalone titan_convert_req_index_to_global.
  const int req = kPaged ? __ldg(p.req_id + t) : 0;
  const bool req_ok = req >= 0 && req < p.num_reqs;
  const int32_t *bt_req = p.block_table + (int64_t)(req_ok ? req : 0) * p.bt_st0;

  // Tile layout in a ring stage: the row at n-order position 8 nt + g (n-tile
  // nt, row g of the MMA B fragment) sits in gather4 group (g >> 1) + 4 (nt >> 1)
  // at slot 2 (g & 1) + (nt & 1).  With the 544-byte pitch (= 32 mod 128) the
  // two rows a quarter-warp reads are 64 bytes apart in the banks: the
  // lanes' 16-byte loads are conflict free.  Group w therefore holds the
  // positions b, b + 8, b + 1, b + 9 with b = 16 (w >> 2) + 2 (w & 3).
  auto row_offset = [](int nt, int gg) {
    return ((gg >> 1) + 4 * (nt >> 1)) * kGroupBytes + (2 * (gg & 1) + (nt & 1)) * kRowPitch;
  };
  auto row_valid = [](uint64_t vb, int nt, int gg) {
    return (uint32_t)(vb >> (8 * ((gg >> 1) + 4 * (nt >> 1)) + 2 * (gg & 1) + (nt & 1))) & 1u;
  };
  const int grp_b = 16 * (warp >> 2) + 2 * (warp & 3);  // first position of this warp's group

  // Warp 0 stages the 32 indices (paged: positions) of tile j into slot j % 8
  // with 4-byte cp.async five (paged: eight) tiles ahead of the row gather,
  // one commit group per iteration; paged, it also stages the block-table
  // entry of each position five tiles ahead (reading the position from the
  // ring).  Warp 0 waits for a slot two iterations after its copy
  // (cp.async.wait_group 1) and the CTA barriers of that iteration publish it
  // to every warp, which reads it one iteration later: no thread waits on a
  // load issued one tile earlier.
  auto copy_idx = [&](int j) {
    if (j < n_tiles) {
      const int64_t pos = start + (int64_t)j * kBN + lane;
      int32_t *dst = &sm.u.ring.idx[j % kIdxRing][lane];
      if (pos < end)
        cp_async_4_zfill(dst, idx_row + pos, 4u);
      else
        *dst = -1;
    }
  };
  auto copy_base = [&](int j) {
    if (j < n_tiles) {
      const int x = sm.u.ring.idx[j % kIdxRing][lane];
      const int blk = p.block_shift >= 0 ? (x >> p.block_shift) : x / p.block_size;
      if (req_ok && x >= 0 && blk < p.max_blocks)
        cp_async_4_zfill(&sm.u.ring.base[j % kIdxRing][lane], bt_req + (int64_t)blk * p.bt_st1, 4u);
    }
  };
  // Row of tile-j position `pos` (paged: translated; -1 when masked).
  auto row_at = [&](int j, int pos) {
    const int x = sm.u.ring.idx[j % kIdxRing][pos];
    if constexpr (!kPaged) {
      return x;
    } else {
      const int blk = p.block_shift >= 0 ? (x >> p.block_shift) : x / p.block_size;
      int row = -1;
      if (req_ok && x >= 0 && blk < p.max_blocks) {
        const int64_t v = (int64_t)sm.u.ring.base[j % kIdxRing][pos] * p.block_stride_rows + (x - blk * p.block_size);
        row = (v >= 0 && v <= 0x7fffffffLL) ? (int)v : -1;
      }
      return row;
    }
  };
  // Gather of tile j (< n_tiles) into stage st: lane 0 of warp w issues
  // group w (one gather4; none when its four rows are all masked), arrives on
  // the stage barrier with the bytes it issued and records the group's
  // validity (bit k = slot k) in vbits[st][w].
  auto issue_rows = [&](int st, int r0, int r1, int r2, int r3) {  // lane 0
    {
      const uint32_t v = (uint32_t)row_ok(r0) | (uint32_t)row_ok(r1) << 1 | (uint32_t)row_ok(r2) << 2 |
                         (uint32_t)row_ok(r3) << 3;
      // Masked rows go to the gather as row -1 (read as zeros, never used),
      // whatever their index was.
      r0 = (v & 1u) ? r0 : -1;
      r1 = (v & 2u) ? r1 : -1;
      r2 = (v & 4u) ? r2 : -1;
      r3 = (v & 8u) ? r3 : -1;
      mbar_arrive_expect_tx(&sm.row_bar[st], v ? (uint32_t)kGroupBytes : 0u);
      if (v) tma_gather4(&sm.u.ring.rows[st][warp][0], &rows_map, 0, r0, r1, r2, r3, &sm.row_bar[st]);
      sm.vbits[st][warp] = (uint8_t)v;
    }
  };
  auto issue = [&](int j, int st) {  // rows from the index ring
    if (lane == 0)
      issue_rows(st, row_at(j, grp_b), row_at(j, grp_b + 8), row_at(j, grp_b + 1), row_at(j, grp_b + 9));
  };
  // Global indices, tiles 0 and 1: lane 0 loads its group's eight indices
  // straight from global memory, all in flight together, and issues both
  // gathers: no shared-memory hop and no CTA barrier before the first rows
  // are requested (B=1 -0.05 us, B=8 -0.2 us).  Paged launches stage tiles 0
  // and 1 through the ring like the rest: there a lane would chain positions,
  // table entries and the gather while warp 0's ring work waits behind it.
  auto issue_first_two = [&]() {
    if (lane == 0) {
      const int pos[4] = {grp_b, grp_b + 8, grp_b + 1, grp_b + 9};
      int x[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t gp = start + (int64_t)(k >> 2) * kBN + pos[k & 3];
        x[k] = gp < end ? __ldg(idx_row + gp) : -1;
      }
      if (n_tiles > 0) issue_rows(0, x[0], x[1], x[2], x[3]);
      if (n_tiles > 1) issue_rows(1, x[4], x[5], x[6], x[7]);
    }
  };

  // Tiles 0 and 1 in flight; the index ring holds tiles 2..4 (paged:
  // positions of tiles 2..7 and block-table entries of tiles 2..4).
  if constexpr (kPaged) {
    if (warp == 0) {
#pragma unroll 1
      for (int j = 0; j < 8; ++j) copy_idx(j);
      cp_async_commit();
      cp_async_wait<0>();
      __syncwarp();
#pragma unroll 1
      for (int j = 0; j < 5; ++j) copy_base(j);
      cp_async_commit();
      cp_async_wait<0>();
    }
  } else {
    if (warp == 0 && n_tiles > 2) {  // ring copies first: in flight with the direct loads
#pragma unroll 1
      for (int j = 2; j < 5; ++j) copy_idx(j);
      cp_async_commit();
    }
    issue_first_two();
  }

  if constexpr (kPaged) {
    __syncthreads();
    if (n_tiles > 0) issue(0, 0);
    if (n_tiles > 1) issue(1, 1);
  } else {
    if (warp == 0 && n_tiles > 2) cp_async_wait<0>();
    __syncthreads();
  }

  // q of this warp's 64 dims for heads g and g + 8 (A operand of QK), loaded
  // after the gathers of tiles 0 and 1 are issued: loads issued ahead of the
  // index loads delay the index -> row chain (B=1 +0.55 us when q went
  // first), while here their latency hides behind the rows in flight.
  const int dim0 = warp * 64 + c * 16;
  uint4 qr[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  {
    const int h0 = hg * kHeads + g, h1 = h0 + 8;
    const __nv_bfloat16 *qt = p.q + (int64_t)t * p.q_st;
    if (h0 < p.H) {
      const uint4 *src = reinterpret_cast<const uint4 *>(qt + (int64_t)h0 * p.q_sh + dim0);
      qr[0] = src[0];
      qr[1] = src[1];
    }
    if (h1 < p.H) {
      const uint4 *src = reinterpret_cast<const uint4 *>(qt + (int64_t)h1 * p.q_sh + dim0);
      qr[2] = src[0];
      qr[3] = src[1];
    }
  }

  // q fragments (A operand of QK): k-step s of this lane uses dims
  // 16 c + 4 s + {0, 1} (regs 0, 1: heads g, g + 8) and + {2, 3} (regs 2, 3),
  // the same permutation as the K fragments.  bf16 as given; for the f16
  // MMAs, q is scaled per warp and head by a power of two 2^kq that puts the
  // warp's largest |q| of the head in [2^14, 2^15): every bf16 value then
  // converts exactly unless it is below 2^-24 of that largest value (f16
  // subnormal range; absolute error <= 2^-25 of it), and the score reduction
  // multiplies this warp's partial scores by 2^-kq (qf, published to the
  // reducing threads by the first tile's first barrier).
  uint32_t qa[4][4];
  {
    const uint32_t w[2][8] = {{qr[0].x, qr[0].y, qr[0].z, qr[0].w, qr[1].x, qr[1].y, qr[1].z, qr[1].w},
                              {qr[2].x, qr[2].y, qr[2].z, qr[2].w, qr[3].x, qr[3].y, qr[3].z, qr[3].w}};
    float qscale[2] = {1.0f, 1.0f};
    if constexpr (kF16) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t mx = 0;  // largest |q| as bf16 bits (integer order = value order)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx = max(mx, max(w[h][k] & 0x7FFFu, (w[h][k] >> 16) & 0x7FFFu));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const int e = mx == 0 ? 0 : max((int)(mx >> 7) - 127, -126);  // floor(log2(largest |q|))
        const int kq = min(14 - e, 126);
        qscale[h] = exp2i(kq);
        if (c == 0) sm.qf[warp][g + 8 * h] = exp2i(-kq);
      }
    }
#pragma unroll
    for (int s2 = 0; s2 < 4; ++s2)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t wd = w[h][2 * s2 + half];
          if constexpr (kF16)
            qa[s2][2 * half + h] = pack_f16x2(__uint_as_float(wd << 16) * qscale[h],
                                              __uint_as_float(wd & 0xFFFF0000u) * qscale[h]);
          else
            qa[s2][2 * half + h] = wd;
        }
  }

  // Softmax state of head red_h: m_run replicated over its 16 lanes, l_run
  // one share per lane until the loop ends.
  float m_run = kNegLarge, l_run = 0.0f;
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;

  const int red_h = tid >> 4;        // head reduced by this thread
  const int red_j = (tid & 15) * 2;  // its two n-order positions
  const int red_nt = red_j >> 3;
  const int red_n = red_j & 7;
  float qf[kWarps];                  // 2^-kq of each warp for head red_h (read at the first tile)
  // f16: the accumulator holds sum(p_r s_r v_r) / 2^e_acc: P enters the PV
  // MMA as p_r s_r 2^-e with e the exponent of the largest row scale seen so
  // far (s_r 2^-e < 2), so every P value is a normal f16 unless its
  // contribution is below 2^-14 of that largest scale.
  int e_acc = -127;

  // A ring wait that gives up (a gather that never landed: the device error
  // word is set) ends the tile loop for the whole CTA at the next barrier:
  // no further gathers are issued and the remaining tiles are skipped; the
  // gathers already in flight are then waited for with short bounded waits,
  // so none lands after the CTA has exited.  The CTA still completes the
  // split-merge protocol below with the state it has (cluster pushes, ticket
  // and counter reset), so its cluster peers are not left to time out and
  // the next call's arrival counters start from zero; that call's outputs
  // are undefined and the error word reports it.
  int st = 0, st_issue = 2;  // ring stage of tile i and of tile i + 2
  int i_end = n_tiles;       // tiles started (fewer after a give-up)
  bool gave_up = false;
  for (int i = 0; i < n_tiles; ++i) {
    // Tile i + 2 goes in flight (its indices were published by the last
    // iteration's barriers); warp 0 stages later tiles' indices.
    if (i + 2 < n_tiles) issue(i + 2, st_issue);
    if (warp == 0) {
      cp_async_wait<1>();  // copies of two iterations back have landed; this iteration's barriers publish them
      if constexpr (kPaged) {
        copy_base(i + 5);  // block-table entries, five tiles ahead
        copy_idx(i + 8);   // positions, eight tiles ahead
      } else {
        copy_idx(i + 5);
      }
      cp_async_commit();
    }
    // Tile i's rows (this stage's k-th use has parity k & 1).
    const bool landed = mbar_wait_bounded(&sm.row_bar[st], (uint32_t)(i / kRing) & 1u, kLongWaitCycles);
    // A tile whose 32 rows are all masked (no gather was issued for it; its
    // validity bits were published by earlier barriers) contributes nothing:
    // one barrier keeps the index-ring hand-over, the math is skipped.
    if (*reinterpret_cast<const uint64_t *>(sm.vbits[st]) == 0) {
      if (__syncthreads_or(!landed)) {
        i_end = i + 1;
        gave_up = true;
        break;
      }
      st = st == kRing - 1 ? 0 : st + 1;
      st_issue = st_issue == kRing - 1 ? 0 : st_issue + 1;
      continue;
    }
    const uint8_t *stage = sm.u.ring.rows[st][0];
    uint4 kb_cur[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
      kb_cur[nt] = *reinterpret_cast<const uint4 *>(stage + row_offset(nt, g) + warp * 64 + c * 16);
    // Warp 0 packs the 32 row scales (bytes 512..515 of each row) n-order for
    // the reduction below; the next iteration rewrites them only after this
    // iteration's second barrier.
    if (warp == 0) sm.scale[lane] = *reinterpret_cast<const float *>(stage + row_offset(lane >> 3, lane & 7) + 512);

    // ---- QK^T over this warp's 64 dims; keep the f16 B fragments for PV.
    uint32_t kf[4][4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      if constexpr (kF16) {
        i8x4_to_f16x4(kb_cur[nt].x, kf[nt][0][0], kf[nt][0][1]);
        i8x4_to_f16x4(kb_cur[nt].y, kf[nt][1][0], kf[nt][1][1]);
        i8x4_to_f16x4(kb_cur[nt].z, kf[nt][2][0], kf[nt][2][1]);
        i8x4_to_f16x4(kb_cur[nt].w, kf[nt][3][0], kf[nt][3][1]);
      } else {
        i8x4_to_bf16x4(kb_cur[nt].x, kf[nt][0][0], kf[nt][0][1]);
        i8x4_to_bf16x4(kb_cur[nt].y, kf[nt][1][0], kf[nt][1][1]);
        i8x4_to_bf16x4(kb_cur[nt].z, kf[nt][2][0], kf[nt][2][1]);
        i8x4_to_bf16x4(kb_cur[nt].w, kf[nt][3][0], kf[nt][3][1]);
      }
    }
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
    for (int s = 0; s < 4; ++s)  // k-step outer: four independent accumulator chains interleave
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        if constexpr (kF16)
          mma_f16_16816(sacc[nt], qa[s], kf[nt][s][0], kf[nt][s][1]);
        else
          mma_bf16_16816(sacc[nt], qa[s], kf[nt][s][0], kf[nt][s][1]);
      }
    {
      float *red = sm.red[warp];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        *reinterpret_cast<float2 *>(&red[g * kRedStride + nt * 8 + 2 * c]) = make_float2(sacc[nt][0], sacc[nt][1]);
        *reinterpret_cast<float2 *>(&red[(g + 8) * kRedStride + nt * 8 + 2 * c]) = make_float2(sacc[nt][2], sacc[nt][3]);
      }
    }
    if (__syncthreads_or(!landed)) {  // partial scores, row scales; or a thread's wait gave up
      i_end = i + 1;
      gave_up = true;
      break;
    }

    // ---- Reduce the 8 partial scores, scale, mask, online softmax, P.
    {
      if (kF16 && i == 0) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) qf[w] = sm.qf[w][red_h];
      }
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {  // f16: each warp's partial in its own q scaling
        const float2 v = *reinterpret_cast<const float2 *>(&sm.red[w][red_h * kRedStride + red_j]);
        s0 = kF16 ? fmaf(v.x, qf[w], s0) : s0 + v.x;
        s1 = kF16 ? fmaf(v.y, qf[w], s1) : s1 + v.y;
      }
      const uint64_t vb = *reinterpret_cast<const uint64_t *>(sm.vbits[st]);
      const bool v0 = row_valid(vb, red_nt, red_n), v1 = row_valid(vb, red_nt, red_n + 1);
      const float2 sc = *reinterpret_cast<const float2 *>(&sm.scale[red_j]);
      const float sc0 = sc.x, sc1 = sc.y;
      const float x0 = v0 ? (s0 * sc0) * p.scale_log2 : kNegLarge;
      const float x1 = v1 ? (s1 * sc1) * p.scale_log2 : kNegLarge;
      float mx = fmaxf(x0, x1);
      // Largest valid row scale of the tile, as bits (positive floats: bit
      // order = value order; masked rows may hold stale bytes and count as 0).
      uint32_t top = max(v0 ? __float_as_uint(sc0) : 0u, v1 ? __float_as_uint(sc1) : 0u);
      // The running max moves only when the tile's max exceeds it by more
      // than kLazyMax (log2 units): p stays <= 2^kLazyMax, and most tiles
      // leave the accumulator unscaled (alpha == 1 skips the rescale below).
      // Any reference value gives the same softmax: acc and l share it.
      // The head-wide max (and, f16, largest row scale) is needed only when
      // some lane would move m_run (or e_acc): a warp vote decides, and the
      // shuffle reductions run only then (always at the first tile).  Without
      // them every lane's own max leaves m_run and e_acc unchanged, as the
      // head-wide values would.
      const bool grow = mx > m_run + kLazyMax || (kF16 && (int)(top >> 23) - 127 > e_acc);
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          if constexpr (kF16) top = max(top, __shfl_xor_sync(0xffffffffu, top, o));
        }
      }
      const float m_cand = fmaxf(m_run, mx);
      const float m_new = m_cand > m_run + kLazyMax ? m_cand : m_run;
      const int e_new = kF16 ? max(e_acc, (int)(top >> 23) - 127) : 0;
      const float am = m_new == m_run ? 1.0f : ex2_approx(m_run - m_new);
      const float alpha = kF16 ? am * exp2i(e_acc - e_new) : am;
      const float p0 = v0 ? ex2_approx(x0 - m_new) : 0.0f;
      const float p1 = v1 ? ex2_approx(x1 - m_new) : 0.0f;
      l_run = l_run * am + (p0 + p1);  // this lane's share; the head's 16 lanes are summed after the loop
      m_run = m_new;
      // P = bf16(p s_r), rounded as kernels/titan_mla.py:175-176 does; f16:
      // p s_r 2^-e_new (11 significant bits against bf16's 8).
      if constexpr (kF16) {
        const float pe = exp2i(-e_new);
        sm.p[red_h * kPStrideWords + (red_j >> 1)] = pack_f16x2(v0 ? p0 * (sc0 * pe) : 0.0f, v1 ? p1 * (sc1 * pe) : 0.0f);
      } else {
        sm.p[red_h * kPStrideWords + (red_j >> 1)] = pack_bf16x2(v0 ? p0 * sc0 : 0.0f, v1 ? p1 * sc1 : 0.0f);
      }
      e_acc = e_new;
      if ((tid & 15) == 0) sm.alpha[red_h] = alpha;
    }
    __syncthreads();

    // ---- PV: acc[16 heads x 64 dims] += P[16 x 32] . V[32 x 64].
    {
      const float al0 = sm.alpha[g], al1 = sm.alpha[g + 8];
      if (__any_sync(0xffffffffu, (al0 != 1.0f) | (al1 != 1.0f))) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          acc[n][0] *= al0;
          acc[n][1] *= al0;
          acc[n][2] *= al1;
          acc[n][3] *= al1;
        }
      }
      // P's A fragments.  Long (f16) CTAs take them with one ldmatrix per
      // k-step: lane i addresses row (i & 7) + 8 ((i >> 3) & 1), column block
      // i >> 4 (rows 144 bytes apart: conflict free); prefill T = 4096
      // 1.405 -> 1.394 ms.  Decode CTAs keep four 4-byte loads, whose first
      // values reach the MMA sooner (ldmatrix there: B=1 +0.06 us, B=8
      // +0.13 us).
      const uint32_t *p_row = &sm.p[((lane & 7) + 8 * ((lane >> 3) & 1)) * kPStrideWords + 4 * (lane >> 4)];
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        uint32_t a[4];
        if constexpr (kF16) {
          ldmatrix_x4(a, p_row + 8 * ks);
        } else {
          a[0] = sm.p[g * kPStrideWords + 8 * ks + c];
          a[1] = sm.p[(g + 8) * kPStrideWords + 8 * ks + c];
          a[2] = sm.p[g * kPStrideWords + 8 * ks + 4 + c];
          a[3] = sm.p[(g + 8) * kPStrideWords + 8 * ks + 4 + c];
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const uint32_t b0 = movmatrix_trans(kf[2 * ks][s][x]);
            const uint32_t b1 = movmatrix_trans(kf[2 * ks + 1][s][x]);
            if constexpr (kF16)
              mma_f16_16816(acc[2 * s + x], a, b0, b1);
            else
              mma_bf16_16816(acc[2 * s + x], a, b0, b1);
          }
        }
      }
    }
    st = st == kRing - 1 ? 0 : st + 1;
    st_issue = st_issue == kRing - 1 ? 0 : st_issue + 1;
  }
  // After a give-up at tile i_end - 1, that tile's gather and those of the
  // next two tiles (already issued) may still be in flight: short bounded
  // waits by every thread on their stages.
  if (gave_up)
    for (int k = i_end - 1; k < n_tiles && k < i_end + kRing - 1; ++k)
      mbar_wait_bounded(&sm.row_bar[k % kRing], (uint32_t)(k / kRing) & 1u, kShortWaitCycles);
  // Every issued gather was waited for; warp 0's index copies beyond the
  // last tile are empty groups.  The ring is dead from here.
  cp_async_wait<0>();
  if constexpr (kF16) {  // back to the scale of the cache values: acc = sum(p_r s_r v_r)
    const float es = exp2i(e_acc);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      acc[n][0] *= es;
      acc[n][1] *= es;
      acc[n][2] *= es;
      acc[n][3] *= es;
    }
  }

  // The softmax denominator of head red_h: the sum of its 16 lanes' shares
  // (each rescaled with the head's common factors along the way).
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) l_run += __shfl_xor_sync(0xffffffffu, l_run, o);

  // ---- Epilogue.  Lane (g, c) of warp w holds, for heads g and g + 8,
  // dims 64 w + 16 c + j at acc[2 s + x][2 half + e] with j = 4 s + 2 x + e.
  if ((tid & 15) == 0) sm.ml[red_h] = make_float2(m_run, l_run);
  const int C = kCluster ? p.C : 1;
  const int cl = split / C;  // partial index when kPartialOut
  if constexpr (!kCluster && kPartialOut) {
    // Partial of this split: the normalised accumulator goes through shared
    // memory (the cluster merge's swizzled [16][512] staging, conflict free)
    // and leaves as fully coalesced 512-byte warp stores; stored straight
    // from the MMA fragments every warp store touched 16 half-written lines.
    __syncthreads();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int hl = g + 8 * half;
      const float l = sm.ml[hl].y;
      const float inv = l > 0.0f ? 1.0f / l : 1.0f;
      float *row = &sm.u.stage[hl * kD];
#pragma unroll
      for (int s = 0; s < 4; ++s)
        *reinterpret_cast<float4 *>(row + merge_pos(hl, 0, dim0 + 4 * s)) =
            make_float4(acc[2 * s][2 * half] * inv, acc[2 * s][2 * half + 1] * inv, acc[2 * s + 1][2 * half] * inv,
                        acc[2 * s + 1][2 * half + 1] * inv);
    }
    __syncthreads();
    float *dst = p.part_o + (((int64_t)t * p.NC + cl) * p.Hp + hg * kHeads) * kD;
#pragma unroll
    for (int k = 0; k < kHeads * kD / 4 / kThreads; ++k) {
      const int e = tid + kThreads * k;  // float4 e of the CTA's 16 x 512 block
      const int hl = e / (kD / 4), q4 = e % (kD / 4);
      if (hg * kHeads + hl < p.H)
        *reinterpret_cast<float4 *>(dst + hl * kD + 4 * q4) =
            *reinterpret_cast<const float4 *>(&sm.u.stage[hl * kD + merge_pos(hl, 0, 4 * q4)]);
    }
    if (tid < kHeads && hg * kHeads + tid < p.H) {
      const float2 ml = sm.ml[tid];
      // (m + log2 l) * ln 2; l == 0 gives -inf, which the merge weighs as 0.
      p.part_lse[((int64_t)t * p.NC + cl) * p.Hp + hg * kHeads + tid] = (ml.x + lg2_approx(ml.y)) * kLn2;
    }
    if (p.sem != nullptr) merge_flat(p, sm, t, hg, split, tid);
    return;
  }
  if constexpr (!kCluster) {
    __syncthreads();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int hl = g + 8 * half;
      const int h = hg * kHeads + hl;
      if (h >= p.H) continue;
      const float l = sm.ml[hl].y;
      const float inv = l > 0.0f ? 1.0f / l : 1.0f;
      float v[16];
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          v[4 * s + 2 * x + 0] = acc[2 * s + x][2 * half + 0] * inv;
          v[4 * s + 2 * x + 1] = acc[2 * s + x][2 * half + 1] * inv;
        }
      uint4 o0, o1;
      o0.x = pack_bf16x2(v[0], v[1]);
      o0.y = pack_bf16x2(v[2], v[3]);
      o0.z = pack_bf16x2(v[4], v[5]);
      o0.w = pack_bf16x2(v[6], v[7]);
      o1.x = pack_bf16x2(v[8], v[9]);
      o1.y = pack_bf16x2(v[10], v[11]);
      o1.z = pack_bf16x2(v[12], v[13]);
      o1.w = pack_bf16x2(v[14], v[15]);
      uint4 *dst = reinterpret_cast<uint4 *>(p.out + (int64_t)t * p.out_st + (int64_t)h * p.out_sh + dim0);
      dst[0] = o0;
      dst[1] = o1;
    }
    return;
  }

  // Cluster merge (push): CTA `rank` owns dims [rank * D, rank * D + D),
  // D = 512 / C.  Every CTA stores its (m, l) into all peers and each of its
  // 16-dim acc pieces into the owner's slot for it; after one cluster barrier
  // each owner reduces its slice from its own shared memory.
  const uint32_t rank = cluster_ctarank();
  const int D = kD / C;
  cluster_wait();  // all peers have started and initialised their merge barrier
  // Bytes this CTA receives: from each of the C CTAs, its 16 x D slice of acc
  // and its 16 (m, l) pairs.
  if (tid == 0) mbar_arrive_expect_tx(&sm.merge_bar, (uint32_t)(C * kHeads * (D * 4 + 8)));
  {
    // Thread (head red_h, lane r of its 16) sends that head's (m, l) to peer
    // r: all C x 16 pairs leave at once.
    const int r = tid & 15;
    if (r < C)
      st_async_f32x2(dsmem_addr(&sm.cml[rank][red_h], (uint32_t)r), make_float2(m_run, l_run),
                     dsmem_addr(&sm.merge_bar, (uint32_t)r));
  }
  {
    // Stage acc locally as [owner][head][dd] (dd swizzled, merge_pos) so each
    // owner's slice is one contiguous 16 x D block, then ship each block with
    // one bulk copy; the owner reads it back through the same swizzle.
    const int owner = dim0 / D;  // 16 | D, so a lane's 16 dims have one owner
    const int dd = dim0 - owner * D;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int hl = g + 8 * half;
      float *row = &sm.u.stage[(owner * kHeads + hl) * D];
#pragma unroll
      for (int s = 0; s < 4; ++s)
        *reinterpret_cast<float4 *>(row + merge_pos(hl, owner, dd + 4 * s)) =
            make_float4(acc[2 * s][2 * half], acc[2 * s][2 * half + 1], acc[2 * s + 1][2 * half],
                        acc[2 * s + 1][2 * half + 1]);
    }
  }
  fence_proxy_async_smem();  // make the staged block visible to the bulk-copy engine
  __syncthreads();
  if (tid < C) {
    const uint32_t bytes = (uint32_t)(kHeads * D * 4);
    bulk_s2cluster(dsmem_addr(&sm.rcv[(int)rank * kHeads * D], (uint32_t)tid), &sm.u.stage[tid * kHeads * D], bytes,
                   dsmem_addr(&sm.merge_bar, (uint32_t)tid));
    bulk_commit();
  }
  // Every byte this CTA owns (C slices and C (m, l) sets) has landed once the
  // barrier's phase completes; only after that may it read them or exit.  No
  // cluster-wide barrier follows, and only local shared memory is read.
  mbar_wait_bounded(&sm.merge_bar, 0u, kLongWaitCycles);
  // Merge weights: 16 lanes per head (head mh), lane mr holds peer mr's (m, l).
  const int mh = tid >> 4, mr = tid & 15;
  const float2 mml = mr < C ? sm.cml[mr][mh] : make_float2(kNegLarge, 0.0f);
  float M = mml.x;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float w = mr < C ? ex2_approx(mml.x - M) : 0.0f;
  float L = w * mml.y;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  // Output pair (head h, dims d, d + 1 of this rank's slice) = sum over the
  // peers of weight * partial, divided by L.
  auto emit = [&](int h, int dd, float2 sum, float Lh) {
    const int hh = hg * kHeads + h;
    const int d = (int)rank * D + dd;
    if (hh < p.H) {
      const float inv = Lh > 0.0f ? 1.0f / Lh : 1.0f;
      if constexpr (!kPartialOut) {
        *reinterpret_cast<uint32_t *>(p.out + (int64_t)t * p.out_st + (int64_t)hh * p.out_sh + d) =
            pack_bf16x2(sum.x * inv, sum.y * inv);
      } else {
        *reinterpret_cast<float2 *>(p.part_o + (((int64_t)t * p.NC + cl) * p.Hp + hh) * kD + d) =
            make_float2(sum.x * inv, sum.y * inv);
      }
    }
  };
  if (C == kMaxCluster) {
    // 16 x 16 pairs = one per thread, of the head whose weights this thread's
    // 16-lane group holds: they stay in registers (width-16 shuffles), no
    // barrier before the reduction.
    const int dd = 2 * mr;
    float2 v[kMaxCluster];
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r)  // issue every load before any use
      v[r] = *reinterpret_cast<const float2 *>(&sm.rcv[(r * kHeads + mh) * D + merge_pos(mh, (int)rank, dd)]);
    float2 sum = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      const float wr = __shfl_sync(0xffffffffu, w, r, 16);
      sum.x += wr * v[r].x;
      sum.y += wr * v[r].y;
    }
    emit(mh, dd, sum, L);
    if constexpr (kPartialOut) {
      if (mr == 0 && hg * kHeads + mh < p.H)
        p.part_lse[((int64_t)t * p.NC + cl) * p.Hp + hg * kHeads + mh] = (M + lg2_approx(L)) * kLn2;
    }
  } else {
    if (mr < C) sm.cw[mr][mh] = w;
    if (mr == 0) {
      sm.cM[mh] = M;
      sm.cL[mh] = L;
    }
    __syncthreads();
    const int pair_shift = 8 - p.logC;       // log2(D / 2)
    const int pairs = kHeads << pair_shift;  // float2 outputs of this CTA
    for (int pp = tid; pp < pairs; pp += kThreads) {
      const int h = pp >> pair_shift;
      const int dd = 2 * (pp - (h << pair_shift));
      float2 v[kMaxCluster];
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)  // issue every load before any use
        if (r < C) v[r] = *reinterpret_cast<const float2 *>(&sm.rcv[(r * kHeads + h) * D + merge_pos(h, (int)rank, dd)]);
      float2 sum = make_float2(0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < C) {
          const float wr = sm.cw[r][h];
          sum.x += wr * v[r].x;
          sum.y += wr * v[r].y;
        }
      emit(h, dd, sum, sm.cL[h]);
    }
    if constexpr (kPartialOut) {
      // Every rank writes the (identical) LSE of its cluster, so the rank-r
      // counter below orders everything the rank-r merge reads.
      if (tid < kHeads && hg * kHeads + tid < p.H)
        p.part_lse[((int64_t)t * p.NC + cl) * p.Hp + hg * kHeads + tid] =
            (sm.cM[tid] + lg2_approx(sm.cL[tid])) * kLn2;
    }
  }
  if constexpr (kPartialOut) {
    if (p.sem != nullptr) {
      // Cross-cluster merge in this kernel: the CTAs of rank r in the NC
      // clusters of (t, hg) take a ticket after publishing their slice; the
      // last one merges dims [r D, r D + D) over all NC partials and resets
      // the counter for the next call.  The launcher guarantees NC <= C.
      __syncthreads();
      if (tid == 0) {
        // acq_rel ticket after the CTA barrier: releases this CTA's slice and
        // LSE, and the last arriver acquires every other CTA's.
        int *ctr = p.sem + ((int64_t)t * gridDim.y + hg) * kMaxCluster + rank;
        const int last = atom_add_acq_rel_gpu(ctr, 1) == p.NC - 1;
        if (last) st_relaxed_gpu(ctr, 0);
        sm.last = last;
      }
      __syncthreads();
      if (sm.last) {
        switch (p.logC) {
          case 1: merge_cluster_partials<8>(p, t, hg, rank, tid); break;
          case 2: merge_cluster_partials<4>(p, t, hg, rank, tid); break;
          case 3: merge_cluster_partials<2>(p, t, hg, rank, tid); break;
          default: merge_cluster_partials<1>(p, t, hg, rank, tid); break;
        }
      }
    }
  }
  if (tid < C) bulk_wait_read_all();  // the stage is read by the copy engine until here
}

// Combine: one CTA per (token, head group, 16-dim chunk), 256 threads.
// Same merge as kernels/titan_mla.py:403-427 (natural-log LSE, max sentinel
// -1e30, empty sum -> zeros), evaluated in parallel over the splits:
//   1. 16 lanes per head stream the S LSE values: head max M and sum of
//      exp(lse - M) by shuffle reduction;
//   2. 4 split groups x 16 heads x 4 float4 columns accumulate
//      sum_s exp(lse_s - M) * o_s with independent loads, then meet in smem.
constexpr int kCombineDims = 16;
constexpr int kCombineGroups = 4;
constexpr int kCombineThreads = 256;

__global__ void __launch_bounds__(kCombineThreads) sparse_mla_combine_kernel(const Params p) {
  pdl_wait_primary();
  pdl_launch_dependents();
  __shared__ float s_max[kHeads];
  __shared__ float s_inv[kHeads];
  __shared__ float4 s_part[kCombineGroups][kHeads * kCombineDims / 4];
  constexpr float kLog2e = 1.4426950408889634f;
  const int t = blockIdx.x, hg = blockIdx.y, chunk = blockIdx.z;
  const int tid = threadIdx.x;
  const int S = p.NC;  // partials to merge
  const float *lse_t = p.part_lse + (int64_t)t * S * p.Hp + hg * kHeads;
  const int grp = tid >> 6;            // split group
  const int pair = tid & 63;           // (head, float4 column)
  const int h = pair >> 2, c4 = pair & 3;
  const int hh = hg * kHeads + h;
  const int dim = chunk * kCombineDims + c4 * 4;
  const float *o_t = p.part_o + ((int64_t)t * S * p.Hp + hh) * kD + dim;
  const int64_t split_stride = (int64_t)p.Hp * kD;

  // 0. issue this thread's partial loads before the max/sum phase (all of
  // them for up to 4 x kPre partials: 17 at B = 8), so the weighted sum
  // below waits on no further load round trip
  constexpr int kPre = 5;
  float4 o_pre[kPre];
  float lse_pre[kPre];
#pragma unroll
  for (int k = 0; k < kPre; ++k) {
    const int s = grp + kCombineGroups * k;
    o_pre[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    lse_pre[k] = -INFINITY;
    if (s < S && hh < p.H) {
      o_pre[k] = *reinterpret_cast<const float4 *>(o_t + s * split_stride);
      lse_pre[k] = lse_t[(int64_t)s * p.Hp + h];
    }
  }

  {  // 1. per-head max and normaliser
    const int hr = tid >> 4, j = tid & 15;
    const bool live = hg * kHeads + hr < p.H;
    float m = kNegLarge;
    if (live)
      for (int s = j; s < S; s += 16) m = fmaxf(m, lse_t[(int64_t)s * p.Hp + hr]);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
    if (live)
      for (int s = j; s < S; s += 16) sum += ex2_approx((lse_t[(int64_t)s * p.Hp + hr] - m) * kLog2e);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (j == 0) {
      s_max[hr] = m;
      s_inv[hr] = sum > 0.0f ? 1.0f / sum : 1.0f;
    }
  }
  __syncthreads();

  // 2. weighted sum of the partial outputs
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (hh < p.H) {
    const float m = s_max[h];
#pragma unroll
    for (int k = 0; k < kPre; ++k) {
      const float w = ex2_approx((lse_pre[k] - m) * kLog2e);
      acc.x += w * o_pre[k].x;
      acc.y += w * o_pre[k].y;
      acc.z += w * o_pre[k].z;
      acc.w += w * o_pre[k].w;
    }
#pragma unroll 4
    for (int s = grp + kCombineGroups * kPre; s < S; s += kCombineGroups) {
      const float w = ex2_approx((lse_t[(int64_t)s * p.Hp + h] - m) * kLog2e);
      const float4 o = *reinterpret_cast<const float4 *>(o_t + s * split_stride);
      acc.x += w * o.x;
      acc.y += w * o.y;
      acc.z += w * o.z;
      acc.w += w * o.w;
    }
  }
  s_part[grp][pair] = acc;
  __syncthreads();
  if (grp == 0 && hh < p.H) {
#pragma unroll
    for (int g2 = 1; g2 < kCombineGroups; ++g2) {
      const float4 v = s_part[g2][pair];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const float inv = s_inv[h];
    uint2 r;
    r.x = pack_bf16x2(acc.x * inv, acc.y * inv);
    r.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2 *>(p.out + (int64_t)t * p.out_st + (int64_t)hh * p.out_sh + dim) = r;
  }
}

static cudaError_t launch_combine(const Params &prm, int groups, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)prm.T, (unsigned)groups, (unsigned)(kD / kCombineDims));
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sparse_mla_combine_kernel, prm);
}

// Tensor map of the cache for the row gather: a 2-D tensor of uint32 words,
// 132 per row (528 bytes), rows kv_row_stride bytes apart; boxes of 136 words
// by one row (the 16 bytes past the row read as zeros and are never used).
// Rows at or beyond min(seq_kv, 2^31) are outside the map (int32 indices
// cannot reach further).  Encoded through the driver entry point; the last
// encoding of each host thread is reused.
static int rows_tensor_map(const void *kv, int64_t seq_kv, int64_t kv_row_stride, const void *dummy, CUtensorMap *out) {
  const EncodeTiledFn encode = tensor_map_encoder();
  if (encode == nullptr) return fail(TITAN_ERR_CUDA, "mla: cuTensorMapEncodeTiled is unavailable");
  // seq_kv == 0: no row is valid and nothing is loaded; any aligned address
  // makes a well-formed map.
  const void *base = seq_kv > 0 ? kv : dummy;
  const int64_t rows = seq_kv > 0 ? (seq_kv < 0x7fffffffLL ? seq_kv : 0x7fffffffLL) : 1;
  const int64_t stride = seq_kv > 0 ? kv_row_stride : TITAN_ROW_BYTES;
  static thread_local const void *last_base = nullptr;
  static thread_local int64_t last_rows = -1, last_stride = -1;
  static thread_local CUtensorMap last_map;
  if (base == last_base && rows == last_rows && stride == last_stride) {
    *out = last_map;
    return TITAN_OK;
  }
  const cuuint64_t dims[2] = {TITAN_ROW_BYTES / 4, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)stride};
  const cuuint32_t box[2] = {kRowPitch / 4, 1};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box, elem,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TITAN_ERR_CUDA, "mla: cuTensorMapEncodeTiled failed (%d) for rows=%lld stride=%lld", (int)r,
                (long long)rows, (long long)stride);
  last_base = base;
  last_rows = rows;
  last_stride = stride;
  last_map = *out;
  return TITAN_OK;
}

// Per-device one-time setup: dynamic shared-memory opt-in, non-portable
// cluster size opt-in, and the largest cluster size the device can schedule
// for this kernel (queried, not assumed).
static std::atomic<bool> g_dev_ready[64];
static int g_cluster_capacity[64][kMaxCluster + 1];  // [dev][C] co-resident clusters of C CTAs

static int prepare_device(size_t smem, const int **capacity) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "mla: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TITAN_ERR_CUDA, "mla: device ordinal %d out of range", dev);
  if (!g_dev_ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(setup_mutex());
    if (g_dev_ready[dev].load(std::memory_order_relaxed)) {
      *capacity = g_cluster_capacity[dev];
      return TITAN_OK;
    }
    void (*kernels[10])(const Params, const CUtensorMap) = {
        sparse_mla_kernel<false, false, false>,      sparse_mla_kernel<true, false, false>,
        sparse_mla_kernel<false, true, false>,       sparse_mla_kernel<true, true, false>,
        sparse_mla_kernel<false, false, true>,       sparse_mla_kernel<true, false, true>,
        sparse_mla_kernel<false, true, true>,        sparse_mla_kernel<true, true, true>,
        sparse_mla_kernel<false, false, false, true>, sparse_mla_kernel<false, true, false, true>};
    for (auto k : kernels) {
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "mla: kernel attributes: %s", cudaGetErrorString(e));
    }
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sparse_mla_kernel<false, false, false>, kThreads, smem) !=
            cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    for (int cs = 0; cs <= kMaxCluster; ++cs) g_cluster_capacity[dev][cs] = 0;
    g_cluster_capacity[dev][1] = sms * per_sm;  // co-resident CTAs without clusters
    for (int cs = 2; cs <= kMaxCluster; cs <<= 1) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)cs, 1, 1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)cs;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, sparse_mla_kernel<true, false, true>, &cfg) != cudaSuccess) {
        cudaGetLastError();  // clear a rejected query: that size is not schedulable
        n = 0;
      }
      g_cluster_capacity[dev][cs] = n;
    }
    g_dev_ready[dev].store(true, std::memory_order_release);
  }
  *capacity = g_cluster_capacity[dev];
  return TITAN_OK;
}

// Cluster size for `clusters_per_split_unit` (= tokens x head groups) units of
// S splits: the largest power of two <= 16 that divides S and whose clusters
// all fit on the device at once (else the grid would run in waves and the
// cluster merge would wait on the second wave).
static int choose_cluster(int64_t units, int64_t S, const int *capacity) {
  int C = 1;
  for (int cs = 2; cs <= kMaxCluster; cs <<= 1) {
    if (S % cs != 0) break;
    if (units * (S / cs) <= capacity[cs]) C = cs;
  }
  return C;
}

}  // namespace mla
}  // namespace titan

namespace titan {
namespace mla {

// Co-resident clusters of `cluster_size` MLA CTAs; with `exclusive`, counted
// as if each CTA had an SM to itself (the query is made with enough dynamic
// shared memory that a second CTA cannot fit on the SM).
static int max_active_clusters(int cluster_size, bool exclusive) {
  if (cluster_size < 1 || cluster_size > kMaxCluster) return -1;
  const int *capacity = nullptr;
  if (prepare_device(sizeof(Smem), &capacity) != TITAN_OK) return -1;
  size_t smem = sizeof(Smem);
  // The exclusive query raises and restores the kernel's shared-memory
  // ceiling: one query at a time.
  std::unique_lock<std::mutex> lock(setup_mutex(), std::defer_lock);
  if (exclusive) {
    lock.lock();
    int dev = 0, per_sm = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    smem = (size_t)per_sm / 2 + 1024;
    if (smem < sizeof(Smem)) smem = sizeof(Smem);
    if (smem > (size_t)optin) return -1;
    // Raise the opt-in ceiling so the query is legal; launches still request
    // sizeof(Smem).
    if (cudaFuncSetAttribute(sparse_mla_kernel<true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cluster_size, 1, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, sparse_mla_kernel<true, false, true>, &cfg);
  if (exclusive)  // back to the launch setting
    cudaFuncSetAttribute(sparse_mla_kernel<true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(Smem));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return n;
}

}  // namespace mla
}  // namespace titan

extern "C" int titan_mla_max_active_clusters(int cluster_size) {
  return titan::mla::max_active_clusters(cluster_size, false);
}

extern "C" int titan_mla_max_exclusive_clusters(int cluster_size) {
  return titan::mla::max_active_clusters(cluster_size, true);
}

extern "C" int64_t titan_mla_workspace_bytes(int64_t num_tokens, int64_t num_heads, int64_t num_kv_splits) {
  using namespace titan::mla;
  if (num_kv_splits <= 1 || num_tokens <= 0 || num_heads <= 0) return 0;
  const int64_t hp = (num_heads + kHeads - 1) / kHeads * kHeads;
  const int64_t o_bytes = num_tokens * num_kv_splits * hp * kD * 4;
  const int64_t lse_bytes = num_tokens * num_kv_splits * hp * 4;
  return o_bytes + ((lse_bytes + 255) / 256) * 256;
}

extern "C" int64_t titan_mla_semaphore_count(int64_t num_tokens, int64_t num_heads) {
  using namespace titan::mla;
  if (num_tokens <= 0 || num_heads <= 0) return 0;
  return num_tokens * ((num_heads + kHeads - 1) / kHeads) * kMaxCluster;
}

namespace titan {
namespace mla {

// Request-local indices of a paged launch (see Params).
struct PagedIndex {
  const int32_t *req_id;
  int64_t num_reqs;
  const int32_t *block_table;
  int64_t bt_st0, bt_st1, max_blocks, block_size, block_stride_rows;
};

// Shared launcher of titan_mla_sparse_attention (sem == nullptr: partials of
// several clusters are merged by the combine kernel),
// titan_mla_sparse_attention_sem (the split kernel merges them itself) and
// titan_mla_sparse_attention_paged (paged != nullptr: indices are
// request-local positions translated in the gather).
static int launch_mla(const void *q, int64_t q_stride_token, int64_t q_stride_head, const void *kv,
                      int64_t kv_row_stride, int64_t seq_kv, const int32_t *indices, int64_t indices_stride_token,
                      int64_t topk, void *out, int64_t out_stride_token, int64_t out_stride_head, int64_t num_tokens,
                      int64_t num_heads, float sm_scale, int64_t num_kv_splits, void *workspace,
                      int64_t workspace_bytes, int32_t *sem, int64_t sem_count, const PagedIndex *paged,
                      titan_stream_t stream) {
  if (num_tokens < 0 || num_heads <= 0 || topk < 0 || seq_kv < 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: invalid sizes");
  if (num_tokens == 0) return TITAN_OK;
  if (num_kv_splits < 1) return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: num_kv_splits must be >= 1");
  // indices may be null only when there is nothing to read (topk == 0), kv
  // only when no index can be valid (seq_kv == 0).
  if (q == nullptr || out == nullptr || (indices == nullptr && topk > 0) || (kv == nullptr && seq_kv > 0))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: null pointer");
  if ((uintptr_t)kv % 16 || kv_row_stride % 16)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: kv base and row stride must be 16-byte aligned");
  if ((uintptr_t)q % 16 || (q_stride_token * 2) % 16 || (q_stride_head * 2) % 16)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: q rows must be 16-byte aligned");
  if ((uintptr_t)out % 16 || (out_stride_token * 2) % 16 || (out_stride_head * 2) % 16)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: out rows must be 16-byte aligned");
  const int64_t groups = (num_heads + kHeads - 1) / kHeads;
  if (groups > 65535) return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: too many heads");
  if (num_tokens * num_kv_splits > 0x7fffffffLL) return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: grid too large");
  const int64_t need = titan_mla_workspace_bytes(num_tokens, num_heads, num_kv_splits);
  if (num_kv_splits > 1) {
    if (workspace == nullptr || workspace_bytes < need)
      return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: workspace too small (%lld < %lld bytes)",
                  (long long)workspace_bytes, (long long)need);
    if ((uintptr_t)workspace % 16) return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: workspace must be 16-byte aligned");
  }

  const size_t smem = sizeof(Smem);
  const int *capacity = nullptr;
  int rc = prepare_device(smem, &capacity);
  if (rc != TITAN_OK) return rc;
  // NC clusters (partials) of C splits per (token, head group).
  int C = choose_cluster(num_tokens * groups, num_kv_splits, capacity);
  int64_t NC = num_kv_splits / C;
  // The split kernel merges cluster partials itself only when every lane of
  // the last CTA loads at most 16 partial values (NC <= C).  Otherwise, with
  // counters given and a grid that is resident all at once, the CTAs of a
  // token merge among themselves without clusters (merge_flat); else the
  // combine kernel merges.
  const bool in_kernel_merge = sem != nullptr && C >= 2 && NC > 1 && NC <= C;
  const bool flat_merge = sem != nullptr && !in_kernel_merge && NC > 1 && num_kv_splits >= kFlatMinS &&
                          num_kv_splits <= kFlatMaxS && num_tokens * groups * num_kv_splits <= capacity[1];
  if (flat_merge) {
    C = 1;
    NC = num_kv_splits;
  }
  if (sem != nullptr && sem_count < titan_mla_semaphore_count(num_tokens, num_heads))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: %lld semaphores given, %lld needed", (long long)sem_count,
                (long long)titan_mla_semaphore_count(num_tokens, num_heads));

  Params prm;
  prm.q = static_cast<const __nv_bfloat16 *>(q);
  prm.q_st = q_stride_token;
  prm.q_sh = q_stride_head;
  prm.kv = static_cast<const uint8_t *>(kv);
  prm.kv_rs = kv_row_stride;
  prm.seq_kv = seq_kv;
  prm.idx = indices;
  prm.idx_st = indices_stride_token;
  prm.topk = topk;
  prm.out = static_cast<__nv_bfloat16 *>(out);
  prm.out_st = out_stride_token;
  prm.out_sh = out_stride_head;
  prm.T = (int)num_tokens;
  prm.H = (int)num_heads;
  prm.Hp = (int)(groups * kHeads);
  prm.S = (int)num_kv_splits;
  prm.C = C;
  prm.logC = 0;
  while ((1 << prm.logC) < C) ++prm.logC;
  prm.NC = (int)NC;
  prm.split_topk = (topk + num_kv_splits - 1) / num_kv_splits;
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  prm.part_o = nullptr;
  prm.part_lse = nullptr;
  prm.sem = in_kernel_merge || flat_merge ? sem : nullptr;
  prm.req_id = nullptr;
  prm.block_table = nullptr;
  prm.bt_st0 = prm.bt_st1 = 0;
  prm.num_reqs = prm.max_blocks = 0;
  prm.block_size = 1;
  prm.block_shift = 0;
  prm.block_stride_rows = 0;
  if (paged != nullptr) {
    prm.req_id = paged->req_id;
    prm.block_table = paged->block_table;
    prm.bt_st0 = paged->bt_st0;
    prm.bt_st1 = paged->bt_st1;
    prm.num_reqs = (int)paged->num_reqs;
    prm.max_blocks = (int)paged->max_blocks;
    prm.block_size = (int)paged->block_size;
    prm.block_shift = -1;
    for (int sh = 0; sh < 31; ++sh)
      if ((1ll << sh) == paged->block_size) prm.block_shift = sh;
    prm.block_stride_rows = paged->block_stride_rows;
  }
  if (NC > 1) {
    const int64_t o_bytes = num_tokens * NC * prm.Hp * kD * 4;
    prm.part_o = static_cast<float *>(workspace);
    prm.part_lse = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + o_bytes);
  }

  CUtensorMap rows_map;
  rc = rows_tensor_map(kv, seq_kv, kv_row_stride, q, &rows_map);
  if (rc != TITAN_OK) return rc;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(num_tokens * num_kv_splits), (unsigned)groups, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (flat_merge) {
    // The CTAs of a token wait for one another: a cooperative launch makes
    // the runtime guarantee that the whole grid is resident at once, also
    // next to other work on other streams.
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
  } else {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)C;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = C > 1 || flat_merge ? 2 : 1;
  cudaError_t e;
  // Single-pass CTAs that walk at least kF16MinTiles tiles (prefill shapes)
  // take the f16 arithmetic.
  const bool f16 = C == 1 && NC == 1 && (prm.split_topk + kBN - 1) / kBN >= kF16MinTiles;
  if (f16)
    e = paged != nullptr ? cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, true, false, true>, prm, rows_map)
                         : cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, false, false, true>, prm, rows_map);
  else if (paged != nullptr)
    e = C > 1 ? (NC > 1 ? cudaLaunchKernelEx(&cfg, sparse_mla_kernel<true, true, true>, prm, rows_map)
                        : cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, true, true>, prm, rows_map))
              : (NC > 1 ? cudaLaunchKernelEx(&cfg, sparse_mla_kernel<true, true, false>, prm, rows_map)
                        : cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, true, false>, prm, rows_map));
  else
    e = C > 1 ? (NC > 1 ? cudaLaunchKernelEx(&cfg, sparse_mla_kernel<true, false, true>, prm, rows_map)
                        : cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, false, true>, prm, rows_map))
              : (NC > 1 ? cudaLaunchKernelEx(&cfg, sparse_mla_kernel<true, false, false>, prm, rows_map)
                        : cudaLaunchKernelEx(&cfg, sparse_mla_kernel<false, false, false>, prm, rows_map));
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "mla launch (C=%d): %s", C, cudaGetErrorString(e));
  if (NC == 1 || in_kernel_merge || flat_merge) return TITAN_OK;
  // Combine the NC cluster partials: 32 CTAs per (token, head group).
  e = launch_combine(prm, (int)groups, s);
  if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "mla combine launch: %s", cudaGetErrorString(e));
  return TITAN_OK;
}

}  // namespace mla
}  // namespace titan

extern "C" int titan_mla_sparse_attention(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                          const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                          const int32_t *indices, int64_t indices_stride_token, int64_t topk,
                                          void *out, int64_t out_stride_token, int64_t out_stride_head,
                                          int64_t num_tokens, int64_t num_heads, float sm_scale,
                                          int64_t num_kv_splits, void *workspace, int64_t workspace_bytes,
                                          titan_stream_t stream) {
  return titan::mla::launch_mla(q, q_stride_token, q_stride_head, kv, kv_row_stride, seq_kv, indices,
                                indices_stride_token, topk, out, out_stride_token, out_stride_head, num_tokens,
                                num_heads, sm_scale, num_kv_splits, workspace, workspace_bytes, nullptr, 0, nullptr,
                                stream);
}

extern "C" int titan_mla_sparse_attention_sem(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                              const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                              const int32_t *indices, int64_t indices_stride_token, int64_t topk,
                                              void *out, int64_t out_stride_token, int64_t out_stride_head,
                                              int64_t num_tokens, int64_t num_heads, float sm_scale,
                                              int64_t num_kv_splits, void *workspace, int64_t workspace_bytes,
                                              int32_t *semaphores, int64_t semaphore_count, titan_stream_t stream) {
  if (semaphores == nullptr || (uintptr_t)semaphores % 4)
    return titan::fail(TITAN_ERR_INVALID_ARGUMENT, "mla: semaphores must be a non-null int32 array");
  return titan::mla::launch_mla(q, q_stride_token, q_stride_head, kv, kv_row_stride, seq_kv, indices,
                                indices_stride_token, topk, out, out_stride_token, out_stride_head, num_tokens,
                                num_heads, sm_scale, num_kv_splits, workspace, workspace_bytes, semaphores,
                                semaphore_count, nullptr, stream);
}

extern "C" int titan_mla_sparse_attention_paged(
    const void *q, int64_t q_stride_token, int64_t q_stride_head, const void *kv, int64_t kv_row_stride,
    int64_t seq_kv, const int32_t *token_indices, int64_t indices_stride_token, int64_t topk, const int32_t *req_id,
    int64_t num_reqs, const int32_t *block_table, int64_t block_table_stride_req, int64_t block_table_stride_block,
    int64_t max_blocks_per_req, int64_t block_size, int64_t block_stride_rows, void *out, int64_t out_stride_token,
    int64_t out_stride_head, int64_t num_tokens, int64_t num_heads, float sm_scale, int64_t num_kv_splits,
    void *workspace, int64_t workspace_bytes, int32_t *semaphores, int64_t semaphore_count, titan_stream_t stream) {
  using namespace titan;
  if (num_tokens > 0 && topk > 0 && (req_id == nullptr || (block_table == nullptr && num_reqs > 0 && max_blocks_per_req > 0)))
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla paged: null req_id or block_table");
  if (block_size <= 0 || block_size > 0x40000000LL || num_reqs < 0 || max_blocks_per_req < 0 ||
      max_blocks_per_req > 0x7fffffffLL || num_reqs > 0x7fffffffLL || block_stride_rows < 0)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla paged: invalid block geometry");
  if (semaphores != nullptr && (uintptr_t)semaphores % 4)
    return fail(TITAN_ERR_INVALID_ARGUMENT, "mla: semaphores must be an int32 array");
  const mla::PagedIndex paged = {req_id, num_reqs, block_table, block_table_stride_req, block_table_stride_block,
                                 max_blocks_per_req, block_size, block_stride_rows};
  return mla::launch_mla(q, q_stride_token, q_stride_head, kv, kv_row_stride, seq_kv, token_indices,
                         indices_stride_token, topk, out, out_stride_token, out_stride_head, num_tokens, num_heads,
                         sm_scale, num_kv_splits, workspace, workspace_bytes, semaphores, semaphore_count, &paged,
                         stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of titan_mla_sparse_attention.
//
// The split-KV path needs scratch memory for the per-cluster partial outputs.
// Callers that cannot allocate device memory themselves — a plugin running
// inside a host engine whose pool owns all device memory, or code issuing
// work while a stream is being captured in global capture mode, where
// cudaMalloc is not permitted — use this entry point instead: the scratch is a
// file-scope device array of kNoAllocScratchBytes (8 MiB) that every GPU which
// loads this library holds until the process exits.
namespace titan {
namespace mla {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static std::atomic<void *> g_noalloc_scratch_ptr[64];

}  // namespace mla
}  // namespace titan

extern "C" int64_t titan_mla_noalloc_scratch_bytes(void) { return titan::mla::kNoAllocScratchBytes; }

extern "C" int titan_mla_sparse_attention_noalloc(const void *q, int64_t q_stride_token, int64_t q_stride_head,
                                                  const void *kv, int64_t kv_row_stride, int64_t seq_kv,
                                                  const int32_t *indices, int64_t indices_stride_token,
                                                  int64_t topk, void *out, int64_t out_stride_token,
                                                  int64_t out_stride_head, int64_t num_tokens, int64_t num_heads,
                                                  float sm_scale, int64_t num_kv_splits, titan_stream_t stream) {
  using namespace titan;
  using namespace titan::mla;
  const int64_t need = titan_mla_workspace_bytes(num_tokens, num_heads, num_kv_splits);
  if (need > kNoAllocScratchBytes)
    return fail(TITAN_ERR_INVALID_ARGUMENT,
                "mla noalloc: this call needs %lld bytes of split scratch but the static scratch holds %lld; "
                "lower num_kv_splits or num_tokens, or call titan_mla_sparse_attention with a workspace",
                (long long)need, (long long)kNoAllocScratchBytes);
  void *scratch = nullptr;
  if (need > 0) {
    // Host code cannot use the array's name as a device address: look up the
    // address once per device, with that device current.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(TITAN_ERR_CUDA, "mla noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(TITAN_ERR_CUDA, "mla noalloc: device ordinal %d out of range", dev);
    scratch = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
    if (scratch == nullptr) {
      e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
      if (e != cudaSuccess || scratch == nullptr)
        return fail(TITAN_ERR_CUDA, "mla noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_noalloc_scratch_ptr[dev].store(scratch, std::memory_order_release);  // same address from any thread
    }
  }
  return titan_mla_sparse_attention(q, q_stride_token, q_stride_head, kv, kv_row_stride, seq_kv, indices,
                                    indices_stride_token, topk, out, out_stride_token, out_stride_head, num_tokens,
                                    num_heads, sm_scale, num_kv_splits, scratch, need > 0 ? kNoAllocScratchBytes : 0,
                                    stream);
}
