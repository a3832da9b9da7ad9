/*
 * ORACLE — test infrastructure only.  A plain-C, single-threaded restatement of
 * the BatchStream reference arithmetic for the paged-attention path.  Only the
 * tests, the smoke check and bench.py's CPU-baseline leg may load it, and only to
 * check or time against; the product never calls it.
 *
 * Pinned against golden vectors produced by the reference itself (the compiled
 * C++ op and the Python op; see tests/golden/make_golden.py).
 *
 * Functions and the reference code each one restates:
 *   oracle_decode_bf16   csrc/paged_attention.cpp:47-105 (score_one_head,
 *                        torch::softmax, sum_values_one_head, bf16 output)
 *   oracle_decode_f32    src/server/torch_model.py:58-80 (_read_blocks +
 *                        attend with no mask, fp32 throughout)
 *   oracle_prefill       src/server/torch_model.py:39-55, 58-64, 295-297
 *                        (gather, causal-within-chunk mask, attend), for bf16
 *                        (rounding points of torch's bf16 matmuls) and fp32
 *   oracle_slot_mapping  src/server/block_allocator.py:28-30 (locate) as used by
 *                        PagedKVCache.append, torch_model.py:149-153
 *
 * Layouts: query [H, D]; pools [Hkv, NB, bs, D]; block tables int64 (the
 * reference's list[int]).  bf16 values travel as uint16 bit patterns.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* bf16 is the upper half of an IEEE float32. */
static float bf16_to_f32(uint16_t b) {
  uint32_t w = (uint32_t)b << 16;
  float f;
  memcpy(&f, &w, sizeof f);
  return f;
}

/* Round-to-nearest-even float32 -> bf16 (NaN stays NaN). */
static uint16_t f32_to_bf16(float f) {
  uint32_t w;
  memcpy(&w, &f, sizeof w);
  if ((w & 0x7f800000u) == 0x7f800000u && (w & 0x007fffffu)) return (uint16_t)((w >> 16) | 0x40u);
  w += 0x7fffu + ((w >> 16) & 1u);
  return (uint16_t)(w >> 16);
}

static float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* softmax over n fp32 values in place: exp(x - max) / sum (fp32). */
static void softmax_inplace(float* x, int64_t n) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) mx = x[i] > mx ? x[i] : mx;
  float sum = 0.f;
  for (int64_t i = 0; i < n; ++i) {
    x[i] = (x[i] == -INFINITY) ? 0.f : expf(x[i] - mx);
    sum += x[i];
  }
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] / sum;
}

/* Row of token `pos` of kv head h in a pool, through the block table. */
static int64_t pool_row(const int64_t* table, int64_t pos, int64_t bs, int64_t NB, int64_t h) {
  return (h * NB + table[pos / bs]) * bs + pos % bs;
}

/*
 * One decode token, bf16 pool: returns 0, or -1 when scratch allocation fails.
 * score = bf16(bf16(q . k) * scale); w = softmax(score) in fp32; out = bf16(sum
 * bf16(w) * v) with the dot products and the weighted sum accumulated in fp32 in
 * position order, exactly the order of the reference loops.
 */
int oracle_decode_bf16(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int64_t H,
                       int64_t Hkv, int64_t NB, int64_t bs, int64_t D, const int64_t* table,
                       int64_t length, int64_t groups, double scaling, uint16_t* out) {
  float* w = (float*)malloc(sizeof(float) * (size_t)length);
  float* acc = (float*)malloc(sizeof(float) * (size_t)D);
  if (!w || !acc) {
    free(w);
    free(acc);
    return -1;
  }
  const float scale = (float)scaling;
  (void)Hkv;
  for (int64_t h = 0; h < H; ++h) {
    const int64_t kvh = h / groups;
    const uint16_t* qh = q + h * D;
    for (int64_t p = 0; p < length; ++p) {
      const uint16_t* k = keys + pool_row(table, p, bs, NB, kvh) * D;
      float dot = 0.f;
      for (int64_t d = 0; d < D; ++d) dot += bf16_to_f32(qh[d]) * bf16_to_f32(k[d]);
      w[p] = round_bf16(round_bf16(dot) * scale);
    }
    softmax_inplace(w, length);
    for (int64_t d = 0; d < D; ++d) acc[d] = 0.f;
    for (int64_t p = 0; p < length; ++p) {
      const uint16_t* v = values + pool_row(table, p, bs, NB, kvh) * D;
      const float wt = round_bf16(w[p]);
      for (int64_t d = 0; d < D; ++d) acc[d] += wt * bf16_to_f32(v[d]);
    }
    for (int64_t d = 0; d < D; ++d) out[h * D + d] = f32_to_bf16(acc[d]);
  }
  free(w);
  free(acc);
  return 0;
}

/* One decode token, fp32 pool and query: softmax(q K^T * scale) V in fp32. */
int oracle_decode_f32(const float* q, const float* keys, const float* values, int64_t H,
                      int64_t Hkv, int64_t NB, int64_t bs, int64_t D, const int64_t* table,
                      int64_t length, int64_t groups, double scaling, float* out) {
  float* w = (float*)malloc(sizeof(float) * (size_t)length);
  if (!w) return -1;
  const float scale = (float)scaling;
  (void)Hkv;
  for (int64_t h = 0; h < H; ++h) {
    const int64_t kvh = h / groups;
    const float* qh = q + h * D;
    for (int64_t p = 0; p < length; ++p) {
      const float* k = keys + pool_row(table, p, bs, NB, kvh) * D;
      float dot = 0.f;
      for (int64_t d = 0; d < D; ++d) dot += qh[d] * k[d];
      w[p] = dot * scale;
    }
    softmax_inplace(w, length);
    for (int64_t d = 0; d < D; ++d) {
      float acc = 0.f;
      for (int64_t p = 0; p < length; ++p) {
        acc += w[p] * values[pool_row(table, p, bs, NB, kvh) * D + d];
      }
      out[h * D + d] = acc;
    }
  }
  free(w);
  return 0;
}

/*
 * A prefill chunk of n query tokens at positions past .. past + n - 1 of one
 * sequence whose past + n tokens are already in the pool.  Query token i sees
 * tokens 0 .. past + i (the reference's _causal_mask).  q and out are [n, H, D]
 * (token-major, the layout of the model's flat batch); dtype 0 = bf16 (uint16
 * storage, rounding points of torch's bf16 matmuls: scores rounded, scaled and
 * rounded; weights rounded; output rounded), 1 = fp32.
 */
int oracle_prefill(const void* q, const void* keys, const void* values, int32_t dtype, int64_t n,
                   int64_t past, int64_t H, int64_t Hkv, int64_t NB, int64_t bs, int64_t D,
                   const int64_t* table, int64_t groups, double scaling, void* out) {
  const int64_t total = past + n;
  float* w = (float*)malloc(sizeof(float) * (size_t)total);
  float* acc = (float*)malloc(sizeof(float) * (size_t)D);
  float* qf = (float*)malloc(sizeof(float) * (size_t)D);
  if (!w || !acc || !qf) {
    free(w);
    free(acc);
    free(qf);
    return -1;
  }
  const float scale = (float)scaling;
  (void)Hkv;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t visible = past + i + 1;
    for (int64_t h = 0; h < H; ++h) {
      const int64_t kvh = h / groups;
      const int64_t qoff = (i * H + h) * D;
      for (int64_t d = 0; d < D; ++d) {
        qf[d] = dtype == 0 ? bf16_to_f32(((const uint16_t*)q)[qoff + d]) : ((const float*)q)[qoff + d];
      }
      for (int64_t p = 0; p < total; ++p) {
        if (p >= visible) {
          w[p] = -INFINITY;
          continue;
        }
        const int64_t row = pool_row(table, p, bs, NB, kvh) * D;
        float dot = 0.f;
        if (dtype == 0) {
          const uint16_t* k = (const uint16_t*)keys + row;
          for (int64_t d = 0; d < D; ++d) dot += qf[d] * bf16_to_f32(k[d]);
          w[p] = round_bf16(round_bf16(dot) * scale);
        } else {
          const float* k = (const float*)keys + row;
          for (int64_t d = 0; d < D; ++d) dot += qf[d] * k[d];
          w[p] = dot * scale;
        }
      }
      softmax_inplace(w, total);
      for (int64_t d = 0; d < D; ++d) acc[d] = 0.f;
      for (int64_t p = 0; p < visible; ++p) {
        const int64_t row = pool_row(table, p, bs, NB, kvh) * D;
        if (dtype == 0) {
          const float wt = round_bf16(w[p]);
          const uint16_t* v = (const uint16_t*)values + row;
          for (int64_t d = 0; d < D; ++d) acc[d] += wt * bf16_to_f32(v[d]);
        } else {
          const float* v = (const float*)values + row;
          for (int64_t d = 0; d < D; ++d) acc[d] += w[p] * v[d];
        }
      }
      for (int64_t d = 0; d < D; ++d) {
        if (dtype == 0) {
          ((uint16_t*)out)[qoff + d] = f32_to_bf16(acc[d]);
        } else {
          ((float*)out)[qoff + d] = acc[d];
        }
      }
    }
  }
  free(w);
  free(acc);
  free(qf);
  return 0;
}

/*
 * Slot of each new token: rows r = 0 .. R-1 hold n_new[r] tokens after
 * start_pos[r] cached ones; tables is [R, table_stride] (int64).  Writes
 * slot_mapping[T] = table[r][pos / bs] * bs + pos % bs and positions[T].
 * Returns the number of tokens written.
 */
int64_t oracle_slot_mapping(const int64_t* tables, int64_t table_stride, const int64_t* start_pos,
                            const int64_t* n_new, int64_t R, int64_t bs, int64_t* positions,
                            int64_t* slot_mapping) {
  int64_t t = 0;
  for (int64_t r = 0; r < R; ++r) {
    for (int64_t i = 0; i < n_new[r]; ++i, ++t) {
      const int64_t pos = start_pos[r] + i;
      positions[t] = pos;
      slot_mapping[t] = tables[r * table_stride + pos / bs] * bs + pos % bs;
    }
  }
  return t;
}
