// Tensor-core split-K decode attention for bf16 KV pools, block_size 16,
// head_dim 64 or 128, up to 16 query heads per kv head.
//
// One persistent CTA per (SM x occupancy) slot.  Warp 4 is the producer: it
// walks the CTA's span of KV blocks (see decode.cuh), looks each block up in the
// block table and issues one TMA box per block half (16 tokens x 64 dims,
// 128-byte swizzle) for K and for V into a ring of NSTAGE stages, plus a bulk copy
// of the query rows of the GQA group at the start of every segment.  Warps 0-3 are
// consumers: warp w owns block w of each 4-block tile and runs
//     S = Q K^T   (m16n8k16, rows = the group's query heads padded to 16)
//     online softmax on the fragments (quad shuffles, base-2)
//     O += P V    (P re-used from the S accumulators as the A operand)
// so each KV byte is read from HBM once for all query heads of its group (the
// reference op re-reads it once per query head, csrc/paged_attention.cpp:92-103).
#include "decode.cuh"

namespace bsb {
namespace {

constexpr int kNCW = 4;     // consumer warps == KV blocks per tile
constexpr int kBS = 16;     // tokens per block (fast path only)
constexpr int kThreads = (kNCW + 1) * 32;

enum : int32_t { kFirst = 1, kLast = 2, kWhole = 4 };

struct TileMeta {
  int32_t seq;   // -1: no more work
  int32_t kvh;
  int32_t blk0;  // index of the tile's first block within the sequence
  int32_t nblk;  // blocks in this tile
  int32_t len;   // context length of the sequence
  int32_t flags;
  int32_t nb;    // units of the segment
  int32_t pad;
  int64_t seg_unit;
};

template <int D, bool G16>
struct Cfg {
  static constexpr int HALVES = D / 64;
  static constexpr int BLOCK_BYTES = kBS * D * 2;        // one block of one kv head
  static constexpr int TILE_BYTES = kNCW * BLOCK_BYTES;  // K (or V) part of a stage
  static constexpr int Q_BYTES = 16 * D * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES + Q_BYTES;  // multiple of 1024
  static constexpr int NSTAGE = (D == 64) ? 5 : 3;
  static constexpr int GROWS = G16 ? 16 : 8;
  static constexpr int MERGE_FLOATS = kNCW * GROWS * D + 2 * kNCW * GROWS;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + NSTAGE * STAGE_BYTES + MERGE_FLOATS * 4;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must stay 1024-byte aligned");
};

template <int D, bool G16>
__global__ void __launch_bounds__(kThreads)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  using C = Cfg<D, G16>;
  constexpr int NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[NSTAGE];
  __shared__ uint64_t empty_bar[NSTAGE];
  __shared__ TileMeta meta[NSTAGE];
  __shared__ ScanSmem scan;
  __shared__ int32_t s_flag;

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* sO = reinterpret_cast<float*>(smem + NSTAGE * C::STAGE_BYTES);
  float* sM = sO + kNCW * C::GROWS * D;
  float* sL = sM + kNCW * C::GROWS;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kNCW);
    }
    fence_barrier_init();
  }
  if (warp == kNCW && lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  const Span sp = compute_span(a, scan);  // contains __syncthreads (orders the inits)
  if (sp.r0 >= sp.r1) return;

  const int G = a.groups;
  const int64_t Hkv = a.num_kv_heads;

  if (warp == kNCW) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    int32_t i = sp.seq;
    int64_t prefix = sp.prefix;
    int32_t len, row;
    int32_t nb = seq_units(a, i, len, row, false);
    int64_t rel = sp.r0 - prefix * Hkv;
    int32_t h = static_cast<int32_t>(rel / nb);
    int32_t off = static_cast<int32_t>(rel % nb);
    int64_t u = sp.r0;
    bool ok = true;
    while (u < sp.r1 && ok) {
      const int64_t left = sp.r1 - u;
      const int32_t take = (nb - off < left) ? (nb - off) : static_cast<int32_t>(left);
      const bool whole = (off == 0 && take == nb);
      const int64_t seg_unit = prefix * Hkv + static_cast<int64_t>(h) * nb;
      const int32_t* table = a.block_tables + static_cast<int64_t>(row) * a.bt_stride;
      for (int32_t t0 = off; t0 < off + take && ok; t0 += kNCW) {
        const int32_t nblk = min(kNCW, off + take - t0);
        int32_t blk = 0;
        bool valid = false;
        if (lane < nblk) {
          blk = __ldg(table + t0 + lane);
          valid = blk >= 0 && blk < a.num_blocks;
          if (!valid) set_status(a.status, kStatusBadBlock);
        }
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
        const bool first = (t0 == off);
        if (lane == 0) {
          ok = mbar_wait(&empty_bar[stage], phase ^ 1u);
          if (ok) {
            TileMeta& m = meta[stage];
            m.seq = i;
            m.kvh = h;
            m.blk0 = t0;
            m.nblk = nblk;
            m.len = len;
            m.flags = (first ? kFirst : 0) | ((t0 + kNCW >= off + take) ? kLast : 0) |
                      (whole ? kWhole : 0);
            m.nb = nb;
            m.seg_unit = seg_unit;
            const uint32_t bytes =
                __popc(vmask) * 2u * C::BLOCK_BYTES + (first ? G * D * 2u : 0u);
            mbar_arrive_expect_tx(&full_bar[stage], bytes);
          } else {
            set_status(a.status, kStatusWaitTimeout);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        uint8_t* st = smem + stage * C::STAGE_BYTES;
        if (valid) {
          // Row of the block in the [Hkv * NB * bs, D] view; the host checks that
          // Hkv * NB * bs fits in int32.
          const int32_t y = (h * a.num_blocks + blk) * kBS;
#pragma unroll
          for (int hf = 0; hf < C::HALVES; ++hf) {
            tma_load_2d_hint(st + (lane * C::HALVES + hf) * 2048, &kmap, &full_bar[stage], hf * 64,
                             y, policy);
            tma_load_2d_hint(st + C::TILE_BYTES + (lane * C::HALVES + hf) * 2048, &vmap,
                             &full_bar[stage], hf * 64, y, policy);
          }
        }
        if (first && lane == 0) {
          const __nv_bfloat16* qsrc = static_cast<const __nv_bfloat16*>(a.q) +
                                      static_cast<int64_t>(i) * a.q_stride_seq +
                                      static_cast<int64_t>(h) * G * D;
          bulk_load(st + 2 * C::TILE_BYTES, qsrc, G * D * 2u, &full_bar[stage]);
        }
        if (++stage == NSTAGE) {
          stage = 0;
          phase ^= 1u;
        }
      }
      u += take;
      off = 0;
      if (++h == Hkv) {
        h = 0;
        prefix += nb;
        do {
          ++i;
          nb = (i < a.num_seqs) ? seq_units(a, i, len, row, false) : 1;
        } while (nb == 0);
      }
    }
    // End-of-work marker (also sent after a timeout so consumers stop).
    if (lane == 0) {
      if (mbar_wait(&empty_bar[stage], phase ^ 1u)) {
        meta[stage].seq = -1;
        mbar_arrive(&full_bar[stage]);
      } else {
        set_status(a.status, kStatusWaitTimeout);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  constexpr int KSTEPS = D / 16;
  constexpr int NTILES = D / 8;
  uint32_t qa[KSTEPS][4];
  float o[NTILES][4];
  float m2[2], lsum[2];
  int stage = 0;
  uint32_t phase = 0;
  const float scale = a.scale;

  while (true) {
    if (!mbar_wait(&full_bar[stage], phase)) {
      set_status(a.status, kStatusWaitTimeout);
      break;
    }
    const TileMeta mt = meta[stage];
    if (mt.seq < 0) break;
    const uint8_t* st = smem + stage * C::STAGE_BYTES;
    if (mt.flags & kFirst) {
      m2[0] = m2[1] = -INFINITY;
      lsum[0] = lsum[1] = 0.f;
#pragma unroll
      for (int n = 0; n < NTILES; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      const uint32_t* sq = reinterpret_cast<const uint32_t*>(st + 2 * C::TILE_BYTES);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        // Row r, dims (16kk + 2t, +1) -> 32-bit word (r*D + 16kk + 2t) / 2.
        const int w0 = (g * D + 16 * kk + 2 * t) >> 1;
        const int w1 = ((g + 8) * D + 16 * kk + 2 * t) >> 1;
        qa[kk][0] = (g < G) ? sq[w0] : 0u;
        qa[kk][1] = (g + 8 < G) ? sq[w1] : 0u;
        qa[kk][2] = (g < G) ? sq[w0 + 4] : 0u;
        qa[kk][3] = (g + 8 < G) ? sq[w1 + 4] : 0u;
      }
    }
    if (warp < mt.nblk) {
      const int tok0 = (mt.blk0 + warp) * kBS;
      const int valid = min(kBS, mt.len - tok0);
      const uint32_t kbase = smem_u32(st) + warp * C::HALVES * 2048;
      const uint32_t vbase = kbase + C::TILE_BYTES;
      float s[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      {
        const int r = ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const int hf = kk >> 2;
          const int chunk = ((kk & 3) << 1) + ((lane >> 3) & 1);
          const uint32_t addr = kbase + hf * 2048 + r * 128 + ((chunk ^ (r & 7)) << 4);
          uint32_t b00, b01, b10, b11;
          ldmatrix_x4(addr, b00, b01, b10, b11);
          mma_bf16_16816(s[0], qa[kk], b00, b01);
          mma_bf16_16816(s[1], qa[kk], b10, b11);
        }
      }
      // Scores with the reference's rounding points; masked tokens -> -inf.
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = 8 * j + 2 * t + (e & 1);
          float v = round_bf16(round_bf16(s[j][e]) * scale) * kLog2e;
          v = (tok < valid) ? v : -INFINITY;
          s[j][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      }
      float corr[2];
      uint32_t pa[4];
#pragma unroll
      for (int hr = 0; hr < (G16 ? 2 : 1); ++hr) {
        float m = mx[hr];
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const float mnew = fmaxf(m2[hr], m);
        corr[hr] = fast_exp2(m2[hr] - mnew);
        m2[hr] = mnew;
        float ps = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float p0 = fast_exp2(s[j][2 * hr] - mnew);
          const float p1 = fast_exp2(s[j][2 * hr + 1] - mnew);
          s[j][2 * hr] = p0;
          s[j][2 * hr + 1] = p1;
          ps += p0 + p1;
        }
        lsum[hr] = lsum[hr] * corr[hr] + ps;
      }
      if (!G16) corr[1] = 1.f;
      pa[0] = pack_bf16x2(s[0][0], s[0][1]);
      pa[1] = G16 ? pack_bf16x2(s[0][2], s[0][3]) : 0u;
      pa[2] = pack_bf16x2(s[1][0], s[1][1]);
      pa[3] = G16 ? pack_bf16x2(s[1][2], s[1][3]) : 0u;
#pragma unroll
      for (int n = 0; n < NTILES; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        if (G16) {
          o[n][2] *= corr[1];
          o[n][3] *= corr[1];
        }
      }
      {
        const int r = (((lane >> 3) & 1) << 3) + (lane & 7);
        // Tokens held by this thread in the V fragments: 2t, 2t+1 (regs 0/2) and
        // 2t+8, 2t+9 (regs 1/3); zero the ones past the context (they may hold
        // stale or NaN data, and 0 * NaN would poison the sum).
        uint32_t keep_lo = 0xffffffffu, keep_hi = 0xffffffffu;
        if (valid < kBS) {
          keep_lo = ((2 * t < valid) ? 0x0000ffffu : 0u) | ((2 * t + 1 < valid) ? 0xffff0000u : 0u);
          keep_hi = ((2 * t + 8 < valid) ? 0x0000ffffu : 0u) |
                    ((2 * t + 9 < valid) ? 0xffff0000u : 0u);
        }
#pragma unroll
        for (int pp = 0; pp < D / 16; ++pp) {
          const int hf = pp >> 2;
          const int chunk = ((pp & 3) << 1) + (lane >> 4);
          const uint32_t addr = vbase + hf * 2048 + r * 128 + ((chunk ^ (r & 7)) << 4);
          uint32_t v0, v1, v2, v3;
          ldmatrix_x4_trans(addr, v0, v1, v2, v3);
          mma_bf16_16816(o[2 * pp], pa, v0 & keep_lo, v1 & keep_hi);
          mma_bf16_16816(o[2 * pp + 1], pa, v2 & keep_lo, v3 & keep_hi);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);
    if (++stage == NSTAGE) {
      stage = 0;
      phase ^= 1u;
    }

    if (mt.flags & kLast) {
      // Deposit this warp's state and merge the four warps.
#pragma unroll
      for (int hr = 0; hr < (G16 ? 2 : 1); ++hr) {
        float l = lsum[hr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int r = g + 8 * hr;
        if (r < G) {
          if (t == 0) {
            sM[warp * G + r] = m2[hr];
            sL[warp * G + r] = l;
          }
#pragma unroll
          for (int n = 0; n < NTILES; ++n) {
            float* dst = sO + (warp * G + r) * D + 8 * n + 2 * t;
            dst[0] = o[n][2 * hr];
            dst[1] = o[n][2 * hr + 1];
          }
        }
      }
      named_barrier_sync(1, kNCW * 32);
      Portion po;
      po.seq = mt.seq;
      po.kvh = mt.kvh;
      po.whole = (mt.flags & kWhole) ? 1 : 0;
      po.seg_unit = mt.seg_unit;
      po.nb = mt.nb;
      emit_portion<kNCW, __nv_bfloat16>(a, sp, po, sO, sM, sL, tid, &s_flag, 1);
    }
  }
}

template <int D, bool G16>
int launch_one(const DecodeArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int grid,
               cudaStream_t stream) {
  using C = Cfg<D, G16>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<D, G16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  decode_mma_kernel<D, G16><<<grid, kThreads, C::SMEM_BYTES, stream>>>(kmap, vmap, a);
  return static_cast<int>(cudaGetLastError());
}

template <int D, bool G16>
int occupancy_one() {
  using C = Cfg<D, G16>;
  cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<D, G16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return -static_cast<int>(e);
  int n = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mma_kernel<D, G16>, kThreads,
                                                    C::SMEM_BYTES);
  if (e != cudaSuccess) return -static_cast<int>(e);
  return n;
}

}  // namespace

int launch_decode_mma(const DecodeArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      int grid, cudaStream_t stream) {
  const bool g16 = a.groups > 8;
  if (a.head_dim == 64)
    return g16 ? launch_one<64, true>(a, kmap, vmap, grid, stream)
               : launch_one<64, false>(a, kmap, vmap, grid, stream);
  return g16 ? launch_one<128, true>(a, kmap, vmap, grid, stream)
             : launch_one<128, false>(a, kmap, vmap, grid, stream);
}

int decode_mma_ctas_per_sm(int head_dim, int groups) {
  const bool g16 = groups > 8;
  if (head_dim == 64) return g16 ? occupancy_one<64, true>() : occupancy_one<64, false>();
  return g16 ? occupancy_one<128, true>() : occupancy_one<128, false>();
}

}  // namespace bsb
