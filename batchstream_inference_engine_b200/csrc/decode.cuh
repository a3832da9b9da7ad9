// Split-K ragged decode attention: the parts shared by the tensor-core and the
// SIMT kernels.
//
// Work layout ("stream-K" over KV blocks).  A *segment* is one (sequence, kv
// head) pair; it holds nb = ceil(len / block_size) *units* (KV blocks).  Segments
// are laid out sequence-major, kv-head minor, so unit u of the whole batch lives
// in segment s with U(s) <= u < U(s) + nb.  The W units are cut into C equal
// contiguous spans, one per CTA (the first W % C CTAs take one unit more), so
// every CTA streams the same number of KV bytes whatever the length mix.  A CTA
// that sees a whole segment writes the final output rows directly.  A segment cut
// by span boundaries gets one partial record (unnormalised O, row max, row sum)
// per CTA that touched it; the last of those CTAs to finish (atomic counter, no
// waiting) merges the records and writes the output, then resets the counter to 0
// so the workspace is ready for the next launch.
//
// Arithmetic follows the reference op (csrc/paged_attention.cpp:47-74 of the
// BatchStream sources): scores are fp32 dot products, rounded to bf16, scaled,
// rounded to bf16 again; softmax runs in fp32; the probabilities are rounded to
// bf16 before they weight V; the weighted sum accumulates in fp32 and is cast to
// the output dtype at the end.  The online softmax keeps everything in base 2
// (scores multiplied by log2(e)).
#pragma once

#include "common.cuh"

namespace bsb {

constexpr float kLog2e = 1.4426950408889634f;

// A segment cut across CTAs, to be merged after the decode kernel: written by
// the CTA that holds its last unit (every CTA writes its entry every launch).
struct MergeTask {
  int64_t seg_unit, q, rem;  // first unit, and the span split of the launch
  int32_t seq, kvh, nb, valid;
};

struct DecodeArgs {
  const void* q;         // [B, H, D]; heads of one sequence contiguous (stride D)
  int64_t q_stride_seq;  // elements between sequences
  void* out;             // [B, H, D] with the same head/dim layout
  int64_t o_stride_seq;
  const void* k_pool;  // [Hkv, NB, bs, D] contiguous
  const void* v_pool;
  const int32_t* block_tables;  // [rows, bt_stride]
  int64_t bt_stride;
  int32_t bt_rows;
  const int32_t* seq_rows;  // optional [B] row of each sequence in block_tables
  const int32_t* context_lens;  // [B]
  int32_t num_seqs, num_heads, num_kv_heads, groups, head_dim, block_size, num_blocks,
      max_blocks;  // max_blocks = usable entries per table row
  float scale;
  float* partials;  // [2 * C, rec_stride]
  int32_t rec_stride;
  int32_t* seg_counters;  // [B * Hkv], zero between launches
  uint32_t* status;
  // Non-zero when context_lens, block_tables and seq_rows were final before the
  // kernel launched just ahead of this one: the span search may then overlap it
  // (programmatic dependent launch); query and pools are read only after it.
  int32_t lens_ready;
  // With lens_ready: the kernel just ahead wrote at most each sequence's last
  // pool block, so other blocks and the query may be loaded before it ends.
  int32_t after_append;
  // [grid] merge tasks.  When set (tensor-core kernel), cut segments are merged
  // by decode_merge_kernel after the decode kernel instead of by the last CTA
  // to finish (atomic counters).
  MergeTask* tasks;
  // Limit of each pipeline wait of the tensor-core kernel (0: kWaitLimitNs).
  uint64_t wait_limit_ns;
  // Test hook of the bounded-wait error path (bs_set_wait_probe): when set,
  // warp 0 of CTA 0 never arms or fills its stages, so its first wait runs
  // out with no copy in flight.  Zero in every production call.
  int32_t probe_unarmed;
};

// Applies the process-wide wait settings of bs_set_wait_probe (capi.cu) to a
// launch.
void apply_wait_probe(DecodeArgs& a);

// Units of a sequence from its raw length and table row (already loaded);
// invalid ones count as 0 units with len = 0.
__device__ __forceinline__ int32_t units_of(const DecodeArgs& a, int32_t raw_len, int32_t raw_row,
                                            int32_t& len, int32_t& row) {
  len = raw_len;
  row = raw_row;
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  if (row < 0 || row >= a.bt_rows || len <= 0 || len > cap) {
    len = 0;
    return 0;
  }
  return (len + a.block_size - 1) / a.block_size;
}

// Units of a sequence with raw length `raw_len` and table row `raw_row` after
// validation; also returns the clamped length.
__device__ __forceinline__ int32_t seq_units_raw(const DecodeArgs& a, int32_t raw_len,
                                                 int32_t raw_row, int32_t& len, int32_t& row,
                                                 bool report) {
  len = raw_len;
  row = raw_row;
  if (len == 0) return 0;  // padding row: nothing read, its output row left as is
  if (row < 0 || row >= a.bt_rows) {
    if (report) set_status(a.status, kStatusBadRow);
    len = 0;
    return 0;
  }
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  if (len < 0 || len > cap) {
    if (report) set_status(a.status, kStatusBadLength);
    len = 0;
    return 0;
  }
  return (len + a.block_size - 1) / a.block_size;
}

// Units of sequence i after validation; also returns the clamped length.
__device__ __forceinline__ int32_t seq_units(const DecodeArgs& a, int32_t i, int32_t& len,
                                             int32_t& row, bool report) {
  return seq_units_raw(a, __ldg(a.context_lens + i),
                       a.seq_rows != nullptr ? __ldg(a.seq_rows + i) : i, len, row, report);
}

struct Span {
  int64_t W, q, rem;  // total units, units per CTA, CTAs with one extra unit
  int64_t r0, r1;     // this CTA's unit range
  int32_t seq;        // sequence holding unit r0
  int64_t prefix;     // units of sequences before `seq`, for one kv head
};

__device__ __forceinline__ int64_t span_begin(int64_t c, int64_t q, int64_t rem) {
  return c * q + (c < rem ? c : rem);
}

// CTA whose span holds unit u.
__device__ __forceinline__ int64_t span_owner(int64_t u, int64_t q, int64_t rem) {
  const int64_t head = (q + 1) * rem;
  return u < head ? u / (q + 1) : rem + (u - head) / q;
}

// Record slot of CTA c for the segment starting at unit U: slot 0 is the
// segment the span starts in, slot 1 the one it ends in.
__device__ __forceinline__ int64_t record_index(int64_t c, int64_t U, int64_t q, int64_t rem) {
  return c * 2 + (U <= span_begin(c, q, rem) ? 0 : 1);
}

// Block-wide exclusive scan helper storage.
struct ScanSmem {
  int64_t warp_tot[32];
  int64_t total;
  int32_t found_seq;
  int64_t found_prefix;
};

__device__ __forceinline__ int64_t warp_inclusive_scan(int64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// All threads of the CTA call this.  Computes W and this CTA's span, and (when
// find_start) finds the sequence holding the span's first unit.
__device__ __forceinline__ Span compute_span(const DecodeArgs& a, ScanSmem& sm,
                                             bool find_start = true) {
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = (nthr + 31) >> 5;
  const int64_t C = gridDim.x, c = blockIdx.x;
  const int32_t B = a.num_seqs;
  Span sp;

  // Pass 1: total units.  Only CTA 0 reports bad lengths, once.
  int64_t local = 0;
  for (int32_t i = tid; i < B; i += nthr) {
    int32_t len, row;
    local += seq_units(a, i, len, row, c == 0);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if (lane == 0) sm.warp_tot[warp] = local;
  if (tid == 0) sm.found_seq = -1;
  __syncthreads();
  if (tid == 0) {
    int64_t t = 0;
    for (int w = 0; w < nwarps; ++w) t += sm.warp_tot[w];
    sm.total = t;
  }
  __syncthreads();
  const int64_t Hkv = a.num_kv_heads;
  sp.W = sm.total * Hkv;
  sp.q = sp.W / C;
  sp.rem = sp.W % C;
  sp.r0 = span_begin(c, sp.q, sp.rem);
  sp.r1 = sp.r0 + sp.q + (c < sp.rem ? 1 : 0);
  sp.seq = -1;
  sp.prefix = 0;
  if (sp.r0 >= sp.r1 || !find_start) return sp;

  // Pass 2: chunked exclusive scan until the sequence holding r0 is found.
  int64_t carry = 0;
  for (int32_t base = 0; base < B; base += nthr) {
    const int32_t i = base + tid;
    int64_t nb = 0;
    if (i < B) {
      int32_t len, row;
      nb = seq_units(a, i, len, row, false);
    }
    int64_t incl = warp_inclusive_scan(nb);
    __syncthreads();  // warp_tot reuse
    if (lane == 31) sm.warp_tot[warp] = incl;
    __syncthreads();
    int64_t before = carry;
    for (int w = 0; w < warp; ++w) before += sm.warp_tot[w];
    const int64_t excl = before + incl - nb;
    if (nb > 0 && excl * Hkv <= sp.r0 && sp.r0 < (excl + nb) * Hkv) {
      sm.found_seq = i;
      sm.found_prefix = excl;
    }
    int64_t chunk_total = 0;
    for (int w = 0; w < nwarps; ++w) chunk_total += sm.warp_tot[w];
    __syncthreads();
    if (sm.found_seq >= 0) break;
    carry += chunk_total;
  }
  sp.seq = sm.found_seq;
  sp.prefix = sm.found_prefix;
  if (sp.seq < 0) sp.r1 = sp.r0;  // cannot happen when r0 < W; never walk from nowhere
  return sp;
}

// Describes the part of one segment that a CTA processes.
struct Portion {
  int32_t seq, kvh;
  int32_t whole;          // the CTA sees every unit of the segment
  int64_t seg_unit;       // U(s)
  int32_t nb;             // units of the segment
};

template <typename OutT>
__device__ __forceinline__ void store_out(OutT* p, float v);
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store_out<float>(float* p, float v) {
  *p = v;
}

// Combines the NW per-warp states deposited in shared memory (sO [NW][G][D],
// sM / sL [NW][G], maxima in base 2) and writes either the output rows or this
// CTA's partial record; the last CTA of a cut segment merges all records.
// Called by the NW*32 consumer threads (ctid = 0 .. NW*32-1) with barrier `bar`.
template <int NW, typename OutT>
__device__ void emit_portion(const DecodeArgs& a, const Span& sp, const Portion& po,
                             const float* sO, const float* sM, const float* sL, int ctid,
                             int32_t* s_flag, uint32_t bar) {
  constexpr int NT = NW * 32;
  const int G = a.groups, D = a.head_dim;
  const int head0 = po.kvh * G;
  OutT* out = static_cast<OutT*>(a.out) + static_cast<int64_t>(po.seq) * a.o_stride_seq +
              static_cast<int64_t>(head0) * D;
  float* rec = nullptr;
  if (!po.whole) {
    rec = a.partials + record_index(blockIdx.x, po.seg_unit, sp.q, sp.rem) * a.rec_stride;
  }
  for (int e = ctid; e < G * D; e += NT) {
    const int r = e / D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sM[w * G + r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = fast_exp2(sM[w * G + r] - M);
      L += sL[w * G + r] * f;
      O += sO[(w * G + r) * D + (e - r * D)] * f;
    }
    if (po.whole) {
      store_out<OutT>(out + e, O / L);
    } else {
      rec[e] = O;
      if (e - r * D == 0) {
        rec[G * D + r] = M;
        rec[G * D + G + r] = L;
      }
    }
  }
  if (po.whole) {
    named_barrier_sync(bar, NT);  // shared state may be reused after this
    return;
  }
  __threadfence();
  named_barrier_sync(bar, NT);
  const int64_t seg = static_cast<int64_t>(po.seq) * a.num_kv_heads + po.kvh;
  const int64_t c_first = span_owner(po.seg_unit, sp.q, sp.rem);
  const int64_t c_last = span_owner(po.seg_unit + po.nb - 1, sp.q, sp.rem);
  if (ctid == 0) {
    const int prev = atomicAdd(a.seg_counters + seg, 1);
    const bool last = prev == static_cast<int>(c_last - c_first);
    *s_flag = last ? 1 : 0;
    if (last) atomicExch(a.seg_counters + seg, 0);
  }
  named_barrier_sync(bar, NT);
  if (*s_flag) {
    __threadfence();
    for (int e = ctid; e < G * D; e += NT) {
      const int r = e / D;
      float M = -INFINITY;
      for (int64_t cc = c_first; cc <= c_last; ++cc) {
        const float* rr = a.partials + record_index(cc, po.seg_unit, sp.q, sp.rem) * a.rec_stride;
        M = fmaxf(M, __ldcg(rr + G * D + r));
      }
      float L = 0.f, O = 0.f;
      for (int64_t cc = c_first; cc <= c_last; ++cc) {
        const float* rr = a.partials + record_index(cc, po.seg_unit, sp.q, sp.rem) * a.rec_stride;
        const float f = fast_exp2(__ldcg(rr + G * D + r) - M);
        L += __ldcg(rr + G * D + G + r) * f;
        O += __ldcg(rr + e) * f;
      }
      store_out<OutT>(out + e, O / L);
    }
  }
  named_barrier_sync(bar, NT);
}

// ------------------------------------------------------------------ warp spans

// Sequence (and units before it, per kv head) holding each of NW target units.
struct WarpStarts {
  int32_t seq[8];
  int64_t prefix[8];
  // Raw length and table row of each warp's first sequence and of the one after.
  int32_t len[8], row[8], nlen[8], nrow[8];
};

// Like compute_span, then splits the CTA span into NW contiguous warp spans and
// locates the sequence holding each warp's first unit.  All threads call it.
template <int NW>
__device__ __forceinline__ Span compute_warp_spans(const DecodeArgs& a, ScanSmem& sm,
                                                   WarpStarts& ws) {
  static_assert(NW <= 8, "at most 8 warp spans");
  Span sp = compute_span(a, sm, false);  // warp 0's start is the CTA's start
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = (nthr + 31) >> 5;
  const int32_t B = a.num_seqs;
  const int64_t Hkv = a.num_kv_heads;
  if (tid < NW) ws.seq[tid] = -1;
  __syncthreads();
  if (sp.r0 >= sp.r1) return sp;
  int64_t carry = 0;
  for (int32_t base = 0; base < B; base += nthr) {
    const int32_t i = base + tid;
    int64_t nb = 0;
    if (i < B) {
      int32_t len, row;
      nb = seq_units(a, i, len, row, false);
    }
    int64_t incl = warp_inclusive_scan(nb);
    __syncthreads();
    if (lane == 31) sm.warp_tot[warp] = incl;
    __syncthreads();
    int64_t before = carry;
    for (int w = 0; w < warp; ++w) before += sm.warp_tot[w];
    const int64_t excl = before + incl - nb;
    if (nb > 0) {
#pragma unroll
      for (int k = 0; k < NW; ++k) {
        const int64_t target = sp.r0 + (sp.r1 - sp.r0) * k / NW;
        if (excl * Hkv <= target && target < (excl + nb) * Hkv) {
          ws.seq[k] = i;
          ws.prefix[k] = excl;
        }
      }
    }
    int64_t chunk_total = 0;
    for (int w = 0; w < nwarps; ++w) chunk_total += sm.warp_tot[w];
    carry += chunk_total;
    __syncthreads();
    // The last target is the largest; once it is found every target is.
    const int64_t last_target = sp.r0 + (sp.r1 - sp.r0) * (NW - 1) / NW;
    if (carry * Hkv > last_target) break;
  }
  if (tid < NW && ws.seq[tid] >= 0) {
    const int32_t i = ws.seq[tid];
    ws.len[tid] = __ldg(a.context_lens + i);
    ws.row[tid] = a.seq_rows != nullptr ? __ldg(a.seq_rows + i) : i;
    ws.nlen[tid] = i + 1 < B ? __ldg(a.context_lens + i + 1) : 0;
    ws.nrow[tid] = i + 1 < B ? (a.seq_rows != nullptr ? __ldg(a.seq_rows + i + 1) : i + 1) : 0;
  }
  __syncthreads();
  sp.seq = ws.seq[0];
  sp.prefix = ws.prefix[0];
  if (sp.seq < 0) sp.r1 = sp.r0;  // cannot happen when r0 < W; never walk from nowhere
  return sp;
}

// compute_warp_spans with one round of global loads and one block scan: each
// thread loads a run of consecutive sequences (their raw lengths and table rows
// also go to `scratch`, 2 * B int32 of shared memory that nothing else uses
// until this returns), one inclusive scan of the per-thread unit counts gives
// every thread its prefix and everyone the total, and each thread then looks for
// the warp start units among its own sequences.  All threads call it.
template <int NW>
__device__ __forceinline__ Span compute_warp_spans_smem(const DecodeArgs& a, ScanSmem& sm,
                                                        WarpStarts& ws, int32_t* scratch) {
  static_assert(NW <= 8, "at most 8 warp spans");
  const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = (nthr + 31) >> 5;
  const int64_t C = gridDim.x, c = blockIdx.x;
  const int32_t B = a.num_seqs;
  const int64_t Hkv = a.num_kv_heads;
  int32_t* lens = scratch;
  int32_t* rows = scratch + B;
  const int32_t per = (B + nthr - 1) / nthr;
  const int32_t i0 = tid * per;
  int64_t local = 0;
  for (int32_t k = 0; k < per; ++k) {
    const int32_t i = i0 + k;
    if (i >= B) break;
    const int32_t len = __ldg(a.context_lens + i);
    const int32_t row = a.seq_rows != nullptr ? __ldg(a.seq_rows + i) : i;
    lens[i] = len;
    rows[i] = row;
    int32_t l2, r2;
    local += seq_units_raw(a, len, row, l2, r2, c == 0);  // CTA 0 reports bad input once
  }
  const int64_t incl = warp_inclusive_scan(local);
  if (lane == 31) sm.warp_tot[warp] = incl;
  if (tid < NW) ws.seq[tid] = -1;
  __syncthreads();
  int64_t before = 0, total = 0;
  for (int w = 0; w < nwarps; ++w) {
    if (w < warp) before += sm.warp_tot[w];
    total += sm.warp_tot[w];
  }
  Span sp;
  sp.W = total * Hkv;
  sp.q = sp.W / C;
  sp.rem = sp.W % C;
  sp.r0 = span_begin(c, sp.q, sp.rem);
  sp.r1 = sp.r0 + sp.q + (c < sp.rem ? 1 : 0);
  sp.seq = -1;
  sp.prefix = 0;
  if (sp.r0 < sp.r1 && local > 0) {
    int64_t run = before + incl - local;  // units before this thread's first sequence
    for (int32_t k = 0; k < per; ++k) {
      const int32_t i = i0 + k;
      if (i >= B) break;
      int32_t len, row;
      const int64_t nb = seq_units_raw(a, lens[i], rows[i], len, row, false);
      if (nb > 0) {
#pragma unroll
        for (int t = 0; t < NW; ++t) {
          const int64_t target = sp.r0 + (sp.r1 - sp.r0) * t / NW;
          if (run * Hkv <= target && target < (run + nb) * Hkv) {
            ws.seq[t] = i;
            ws.prefix[t] = run;
            ws.len[t] = lens[i];
            ws.row[t] = rows[i];
            ws.nlen[t] = i + 1 < B ? lens[i + 1] : 0;
            ws.nrow[t] = i + 1 < B ? rows[i + 1] : 0;
          }
        }
      }
      run += nb;
    }
  }
  __syncthreads();  // the starts are visible
  if (sp.r0 >= sp.r1) return sp;
  sp.seq = ws.seq[0];
  sp.prefix = ws.prefix[0];
  if (sp.seq < 0) sp.r1 = sp.r0;  // cannot happen when r0 < W; never walk from nowhere
  return sp;
}

// First half of the cross-CTA merge of a cut segment, done by one warp: writes
// this CTA's record (O unnormalised, M, L for the G rows; o/m/l in shared memory,
// O row-major [G][D]) and counts the CTA in.  Returns true (on every lane) when
// this CTA was the last contributor, which then owes the segment's final merge.
__device__ __forceinline__ void warp_store_record(const DecodeArgs& a, const Span& sp,
                                                  int64_t seg_unit, const float* o, const float* m,
                                                  const float* l, int lane) {
  const int G = a.groups, D = a.head_dim;
  float* rec = a.partials + record_index(blockIdx.x, seg_unit, sp.q, sp.rem) * a.rec_stride;
  for (int e = lane; e < G * D; e += 32) rec[e] = o[e];
  for (int r = lane; r < G; r += 32) {
    rec[G * D + r] = m[r];
    rec[G * D + G + r] = l[r];
  }
}

// warp_store_record for at most ROWS rows of DIM elements (compile-time bounds,
// so the copies issue back to back).
template <int ROWS, int DIM>
__device__ __forceinline__ void warp_store_record_fixed(const DecodeArgs& a, const Span& sp,
                                                        int64_t seg_unit, const float* o,
                                                        const float* m, const float* l,
                                                        int lane) {
  const int G = a.groups;
  float* rec = a.partials + record_index(blockIdx.x, seg_unit, sp.q, sp.rem) * a.rec_stride;
#pragma unroll
  for (int j = 0; j < ROWS * DIM / 32; ++j) {
    const int e = lane + 32 * j;
    if (e < G * DIM) rec[e] = o[e];
  }
  if (lane < G) {
    rec[G * DIM + lane] = m[lane];
    rec[G * DIM + G + lane] = l[lane];
  }
}

__device__ __forceinline__ bool warp_write_record(const DecodeArgs& a, const Span& sp,
                                                  int32_t seq, int32_t kvh, int64_t seg_unit,
                                                  int32_t nb, const float* o, const float* m,
                                                  const float* l, int lane) {
  warp_store_record(a, sp, seg_unit, o, m, l, lane);
  __threadfence();
  __syncwarp();
  const int64_t segi = static_cast<int64_t>(seq) * a.num_kv_heads + kvh;
  const int64_t c_first = span_owner(seg_unit, sp.q, sp.rem);
  const int64_t c_last = span_owner(seg_unit + nb - 1, sp.q, sp.rem);
  int last = 0;
  if (lane == 0) {
    const int prev = atomicAdd(a.seg_counters + segi, 1);
    last = prev == static_cast<int>(c_last - c_first);
    if (last) atomicExch(a.seg_counters + segi, 0);
  }
  return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// Second half: every thread of the CTA merges the n = c_last - c_first + 1
// records of a segment and writes its output rows.  `scratch` is shared memory
// for 2 * n * G + 2 * G floats.  Row weights are computed once per record, then
// the O rows stream in as float4 loads that do not depend on one another.
// Must be called by all threads of the CTA (it synchronises them).
template <typename OutT>
__device__ void cta_merge_records(const DecodeArgs& a, const Span& sp, int32_t seq, int32_t kvh,
                                  int64_t seg_unit, int32_t nb, float* scratch) {
  const int G = a.groups, D = a.head_dim;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int64_t c_first = span_owner(seg_unit, sp.q, sp.rem);
  const int n = static_cast<int>(span_owner(seg_unit + nb - 1, sp.q, sp.rem) - c_first + 1);
  float* wm = scratch;          // [n][G]: record maxima, then weights
  float* wl = scratch + n * G;  // [n][G]: record sums
  float* rowM = wl + n * G;     // [G]
  float* rowInvL = rowM + G;    // [G]
  auto record = [&](int c) {
    return a.partials + record_index(c_first + c, seg_unit, sp.q, sp.rem) * a.rec_stride;
  };
  // Up to kBatch records per round: their loads are independent and issue back
  // to back.  The first round of each thread's first element group goes out
  // with the maxima and sums below, so n <= kBatch costs one L2 round trip.
  constexpr int kBatch = 8;
  const int E4 = G * D / 4;
  float4 v[kBatch];
  if (tid < E4) {
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (u < n) v[u] = __ldcg(reinterpret_cast<const float4*>(record(u)) + tid);
    }
  }
  for (int idx = tid; idx < n * G; idx += nthr) {
    const int c = idx / G, r = idx - c * G;
    const float* rr = record(c);
    wm[idx] = __ldcg(rr + G * D + r);
    wl[idx] = __ldcg(rr + G * D + G + r);
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int c = 0; c < n; ++c) M = fmaxf(M, wm[c * G + tid]);
    rowM[tid] = M;
  }
  __syncthreads();
  for (int idx = tid; idx < n * G; idx += nthr) wm[idx] = fast_exp2(wm[idx] - rowM[idx % G]);
  __syncthreads();
  if (tid < G) {
    float L = 0.f;
    for (int c = 0; c < n; ++c) L += wl[c * G + tid] * wm[c * G + tid];
    rowInvL[tid] = 1.f / L;
  }
  __syncthreads();
  OutT* out = static_cast<OutT*>(a.out) + static_cast<int64_t>(seq) * a.o_stride_seq +
              static_cast<int64_t>(kvh) * G * D;
  for (int e4 = tid; e4 < E4; e4 += nthr) {
    const int r = (e4 * 4) / D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < n; c0 += kBatch) {
      if (e4 != tid || c0 != 0) {  // else: prefetched above
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (c0 + u < n) v[u] = __ldcg(reinterpret_cast<const float4*>(record(c0 + u)) + e4);
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (c0 + u < n) {
          const float w = wm[(c0 + u) * G + r];
          acc.x += w * v[u].x;
          acc.y += w * v[u].y;
          acc.z += w * v[u].z;
          acc.w += w * v[u].w;
        }
      }
    }
    const float inv = rowInvL[r];
    store_out<OutT>(out + 4 * e4 + 0, acc.x * inv);
    store_out<OutT>(out + 4 * e4 + 1, acc.y * inv);
    store_out<OutT>(out + 4 * e4 + 2, acc.z * inv);
    store_out<OutT>(out + 4 * e4 + 3, acc.w * inv);
  }
  __syncthreads();  // scratch may be reused
}

// Host-side launchers (defined in decode_mma.cu / decode_simt.cu).
int launch_decode_mma(const DecodeArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      int grid, cudaStream_t stream);
int decode_mma_ctas_per_sm(int head_dim, int groups);
int launch_decode_simt(const DecodeArgs& a, int dtype_is_bf16, int grid, cudaStream_t stream);
int decode_simt_ctas_per_sm(int head_dim, int groups, int dtype_is_bf16);

}  // namespace bsb
