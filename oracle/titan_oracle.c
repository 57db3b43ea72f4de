/*
 * titan_oracle.c — C restatement of the byte-exact parts of the path.
 * TEST INFRASTRUCTURE ONLY: used by tests/ to cross-check oracle.py and the
 * CUDA kernels; the product never links it.
 *
 * oracle_store_int8_rows  follows kernels/titan_kv.py:15-21 in IEEE fp32
 *                         (compile without fast-math; rintf in the default
 *                         round-to-nearest-even mode is nearbyint); NaN
 *                         operands are dropped by max / maximum / minimum as
 *                         in the reference (Triton's maxnum / minnum).
 * oracle_moe_align_small  follows kernels/titan_moe_align.py:17-46 (the
 *                         pairwise rank/count/offset formulation of
 *                         benchmarks/moe_align.py:34-46).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

void oracle_store_int8_rows(const uint16_t *x_bits, int64_t n, uint8_t *rows_out) {
  for (int64_t i = 0; i < n; ++i) {
    const uint16_t *x = x_bits + i * 512;
    uint8_t *row = rows_out + i * 528;
    float amax = 0.0f; /* a NaN never compares greater: the row max ignores it */
    for (int d = 0; d < 512; ++d) {
      float a = fabsf(bf16_to_f32(x[d]));
      if (a > amax) amax = a;
    }
    volatile float q127 = 127.0f; /* keep the division a runtime IEEE divide */
    float scale = amax / q127;
    if (!(scale >= 1.0e-12f)) scale = 1.0e-12f;
    for (int d = 0; d < 512; ++d) {
      /* fmaxf / fminf return the non-NaN operand, like the reference's
         maximum / minimum: a NaN quotient clamps to -127. */
      float y = rintf(bf16_to_f32(x[d]) / scale);
      y = fminf(fmaxf(y, -127.0f), 127.0f);
      row[d] = (uint8_t)(int8_t)y;
    }
    memcpy(row + 512, &scale, 4);
    memset(row + 516, 0, 12);
  }
}

int oracle_moe_align_small(const int64_t *ids, int R, int32_t *sorted_ids, int32_t *expert_ids,
                           int32_t *postpad) {
  if (R <= 0 || R > 64) return -1;
  int valid[64], e[64], rank[64], count[64], first[64], padded[64], offset[64];
  for (int j = 0; j < R; ++j) {
    valid[j] = ids[j] >= 0 && ids[j] < 288;
    e[j] = valid[j] ? (int)ids[j] : 288;
  }
  for (int j = 0; j < R; ++j) {
    rank[j] = 0;
    count[j] = 0;
    for (int k = 0; k < R; ++k) {
      const int same = valid[k] && e[k] == e[j];
      count[j] += same;
      rank[j] += same && k < j;
    }
    first[j] = valid[j] && rank[j] == 0;
    padded[j] = (count[j] + 7) / 8 * 8;
  }
  int total = 0;
  for (int j = 0; j < R; ++j) {
    offset[j] = 0;
    for (int k = 0; k < R; ++k)
      if (first[k] && e[k] < e[j]) offset[j] += padded[k];
    if (first[j]) total += padded[j];
  }
  for (int i = 0; i < R * 8; ++i) sorted_ids[i] = R;
  for (int i = 0; i < R; ++i) expert_ids[i] = -1;
  for (int j = 0; j < R; ++j) {
    if (valid[j]) sorted_ids[offset[j] + rank[j]] = j;
    if (first[j])
      for (int b = 0; b < padded[j] / 8; ++b) expert_ids[offset[j] / 8 + b] = e[j];
  }
  postpad[0] = total;
  return 0;
}
