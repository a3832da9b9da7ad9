// Tensor-core split-K decode attention for bf16 KV pools, block_size 16,
// head_dim 64 or 128, up to 16 query heads per kv head.
//
// Every warp is an independent stream-K worker.  The CTA's span of KV blocks
// (decode.cuh) is cut into W contiguous warp spans; a warp walks its span one
// block at a time through its own ring of S shared-memory stages.  Its lane 0
// looks the block up in the block table (32 entries per coalesced load) and
// issues one TMA box per 64-dim half of the block for K and for V (16 tokens x
// 128 bytes, 128-byte swizzle), plus a bulk copy of the GQA group's query rows at
// the start of each segment; each stage completes on the warp's own mbarrier.
// Many short independent pipelines per SM keep far more DRAM requests moving than
// a few deep ones, because a pipeline drains in order.
//
// Per block the warp runs
//     S = Q K^T   (mma.sync m16n8k16; rows = the group's query heads padded to 16)
//     online softmax on the fragments (quad shuffles, base 2)
//     O += P V    (P reused from the S accumulators as the A operand)
// so each KV byte leaves HBM once for all query heads of its group; the
// reference op reads it once per query head (csrc/paged_attention.cpp:92-103).
// A segment whose blocks all lie in the warp's span is written straight from
// registers.  Cut segments go to per-warp slots in shared memory; after one CTA
// barrier the warp holding the end of each chain merges it and writes the output
// or, for a segment that crosses CTAs, the CTA's partial record (decode.cuh).
#include "decode.cuh"

namespace bsb {
namespace {

constexpr int kBS = 16;  // tokens per block (fast path only)

enum : int32_t { kFirst = 1, kLast = 2, kWhole = 4, kSlot1 = 8 };

struct TileMeta {
  int32_t seq;
  int32_t kvh;
  int32_t blk;  // block index within the sequence
  int32_t len;  // context length of the sequence
  int32_t flags;
  int32_t nb;   // units of the segment
  int64_t seg_unit;
};

template <int D, bool G16>
struct Cfg {
  static constexpr int W = 4;                  // warps per CTA
  // Stages per warp: two at either head_dim.  Deeper rings only lengthen the
  // DRAM queues (12 warps x 2 stages x 4 KiB per SM already cover bandwidth x
  // latency); measured at d64: 2 stages 1.6-2.5% faster than 3, 4 slower.
  static constexpr int S = 2;
  static constexpr int MIN_CTAS = (D == 64) ? 3 : 2;  // resident CTAs per SM
  // Registers per thread: MIN_CTAS CTAs leave room on the SM for a small CTA of
  // the kernel just ahead (it runs on during the programmatic launch), so no
  // decode CTA waits for it to exit.
  static constexpr int MAX_REGS = (D == 64) ? 160 : 232;
  static constexpr int HALVES = D / 64;
  static constexpr int GROWS = G16 ? 16 : 8;
  static constexpr int BLOCK_BYTES = kBS * D * 2;  // one block of one kv head
  static constexpr int Q_BYTES = GROWS * D * 2;
  static constexpr int STAGE_BYTES = 2 * BLOCK_BYTES + Q_BYTES;  // K | V | Q
  static constexpr int SLOT_FLOATS = GROWS * D + 2 * GROWS;
  // Slot 0 (a warp's first, cut portion) has its own storage; slot 1 (its last
  // portion) is written after the warp's final block and reuses its stages.
  static constexpr int SLOT0_BYTES = ((SLOT_FLOATS * 4 + 1023) / 1024) * 1024;
  static constexpr int SMEM_BYTES = 1024 + W * S * STAGE_BYTES + W * SLOT0_BYTES;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(SLOT_FLOATS * 4 <= S * STAGE_BYTES, "slot 1 must fit in the stages");
};

template <int D, bool G16>
__global__ void __maxnreg__((Cfg<D, G16>::MAX_REGS))
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  using C = Cfg<D, G16>;
  constexpr int W = C::W, S = C::S;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[W][S];
  __shared__ TileMeta meta[W][S];
  __shared__ ScanSmem scan;
  __shared__ WarpStarts starts;
  __shared__ int32_t slot_seq[W][2], slot_kvh[W][2], slot_nb[W][2];
  __shared__ int64_t slot_unit[W][2];
  // Segments whose last record this CTA wrote: merged by the whole CTA.
  __shared__ int32_t fin_count;
  __shared__ MergeTask task;  // the cut segment this CTA finishes (tasks mode)
  __shared__ int32_t fin_seq[2 * W], fin_kvh[2 * W], fin_nb[2 * W];
  __shared__ int64_t fin_unit[2 * W];

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto stages_of = [&](int w) { return smem + w * S * C::STAGE_BYTES; };
  auto slot_of = [&](int w, int k) {
    return reinterpret_cast<float*>(k == 0 ? smem + W * S * C::STAGE_BYTES + w * C::SLOT0_BYTES
                                           : stages_of(w));
  };
  uint8_t* wst = stages_of(warp);

  if (tid == 0) {
    for (int w = 0; w < W; ++w)
      for (int s = 0; s < S; ++s) mbar_init(&full_bar[w][s], 1);
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  if (tid < W * 2) slot_seq[tid / 2][tid % 2] = -1;
  if (tid == 0) {
    fin_count = 0;
    task.valid = 0;
  }
  pdl_trigger();  // the merge pass may launch now; it waits for this grid
  // lens_ready: the work split overlaps the kernel just ahead; after_append:
  // so do the first loads of blocks that kernel cannot have written.
  const bool early_loads = a.lens_ready && a.after_append;
  if (!a.lens_ready) pdl_wait();
  // The stages are free until the first copy: they hold the lengths and rows
  // for the span scan when they fit (one round of global loads).
  constexpr int kScratchInts = W * S * C::STAGE_BYTES / 4;
  const Span sp =
      2 * a.num_seqs <= kScratchInts
          ? compute_warp_spans_smem<W>(a, scan, starts, reinterpret_cast<int32_t*>(smem))
          : compute_warp_spans<W>(a, scan, starts);  // both sync the inits
  if (a.lens_ready && !early_loads) pdl_wait();  // query, pools from here on
  if (sp.r0 >= sp.r1) {
    if (a.tasks != nullptr && tid == 0) a.tasks[blockIdx.x].valid = 0;
    return;
  }

  const int G = a.groups;
  const int64_t Hkv = a.num_kv_heads;
  const int64_t spanw = sp.r1 - sp.r0;
  const int64_t wr0 = sp.r0 + spanw * warp / W;
  const int64_t wr1 = sp.r0 + spanw * (warp + 1) / W;
  const int32_t ntiles = static_cast<int32_t>(wr1 - wr0);

  // ---------------------------------------------------------------- issue cursor
  // All lanes keep identical copies; lane 0 writes the stage metadata and
  // issues the copies.
  const uint64_t policy = l2_policy_evict_first();
  int32_t ci = starts.seq[warp];
  int64_t cprefix = starts.prefix[warp];
  int32_t clen = 0, crow = 0, cnb = 0, ch = 0, cb = 0;
  int32_t nxt_len = 0, nxt_row = 0;
  int32_t win_row = -1, win0 = 0, win_val = 0;
  // The window that follows the current one, loaded when the current one is
  // (its latency then hides behind the blocks the current window still holds).
  int32_t pre_row = -1, pre0 = 0, pre_val = 0;
  int64_t cu = wr0;
  if (ntiles > 0) {
    cnb = units_of(a, starts.len[warp], starts.row[warp], clen, crow);
    const int64_t rel = wr0 - cprefix * Hkv;
    ch = static_cast<int32_t>(rel / cnb);
    cb = static_cast<int32_t>(rel % cnb);
    nxt_len = starts.nlen[warp];
    nxt_row = starts.nrow[warp];
  }

  // Stages holding a copy that was started and not yet waited for (bit s).
  uint32_t armed = 0;
  // The probe hook leaves this warp's stages unarmed (see DecodeArgs).
  const bool probe = a.probe_unarmed != 0 && blockIdx.x == 0 && warp == 0;
  // `dry`: metadata only, no copy (the walk after a wait gave up).
  // Lane i's entry of the 32-entry window of table row `row` starting at entry
  // `e0` (0 past the row's usable entries).
  auto window = [&](int32_t row, int32_t e0) -> int32_t {
    const int32_t* table = a.block_tables + static_cast<int64_t>(row) * a.bt_stride;
    return (e0 + lane < a.max_blocks) ? __ldg(table + e0 + lane) : 0;
  };
  auto issue = [&](int stage, bool dry) {
    // The window caches up to 32 entries of one table row, filled to the row's
    // width rather than this sequence's block count: sequences that share a row
    // (the tokens of a prefill chunk) have different lengths and reuse it.
    if (win_row != crow || cb < win0 || cb >= win0 + 32) {
      if (pre_row == crow && cb >= pre0 && cb < pre0 + 32) {
        win_row = pre_row;
        win0 = pre0;
        win_val = pre_val;
      } else {
        win_row = crow;
        win0 = cb;
        win_val = window(crow, cb);
      }
      // Prefetch the window the cursor needs next: the rest of this segment,
      // else this sequence's other kv heads (the same row from entry 0), else
      // the next sequence's row.
      int32_t next_row = -1, next0 = 0;
      if (win0 + 32 < cnb) {
        next_row = crow;
        next0 = win0 + 32;
      } else if (ch + 1 < a.num_kv_heads) {
        next_row = crow;
      } else if (ci + 1 < a.num_seqs && nxt_row >= 0 && nxt_row < a.bt_rows) {
        next_row = nxt_row;
      }
      if (next_row >= 0 && !(next_row == win_row && next0 == win0)) {
        pre_row = next_row;
        pre0 = next0;
        pre_val = window(next_row, next0);
      }
    }
    const int32_t blk = __shfl_sync(0xffffffffu, win_val, cb - win0);
    const bool valid = blk >= 0 && blk < a.num_blocks;
    const int64_t seg_unit = cprefix * Hkv + static_cast<int64_t>(ch) * cnb;
    const bool first = (cu == wr0) || (cb == 0);
    const bool last = (cu == wr1 - 1) || (cb == cnb - 1);
    const bool whole = seg_unit >= wr0 && seg_unit + cnb <= wr1;
    if (lane == 0) {
      if (!valid && !dry) set_status(a.status, kStatusBadBlock);
      TileMeta& m = meta[warp][stage];
      m.seq = ci;
      m.kvh = ch;
      m.blk = cb;
      m.len = clen;
      m.flags = (first ? kFirst : 0) | (last ? kLast : 0) | (whole ? kWhole : 0) |
                (seg_unit > wr0 ? kSlot1 : 0);
      m.nb = cnb;
      m.seg_unit = seg_unit;
    }
    if (lane == 0 && !dry && !probe) {
      uint8_t* st = wst + stage * C::STAGE_BYTES;
      const uint32_t bytes = (valid ? 2u * C::BLOCK_BYTES : 0u) + (first ? G * D * 2u : 0u);
      mbar_arrive_expect_tx(&full_bar[warp][stage], bytes);
      if (valid) {
        // Row of the block in the [Hkv * NB * bs, D] view; the host checks that
        // Hkv * NB * bs fits in int32.
        const int32_t y = (ch * a.num_blocks + blk) * kBS;
#pragma unroll
        for (int hf = 0; hf < C::HALVES; ++hf) {
          tma_load_2d_hint(st + hf * 2048, &kmap, &full_bar[warp][stage], hf * 64, y, policy);
          tma_load_2d_hint(st + C::BLOCK_BYTES + hf * 2048, &vmap, &full_bar[warp][stage],
                           hf * 64, y, policy);
        }
      }
      if (first) {
        const __nv_bfloat16* qsrc = static_cast<const __nv_bfloat16*>(a.q) +
                                    static_cast<int64_t>(ci) * a.q_stride_seq +
                                    static_cast<int64_t>(ch) * G * D;
        bulk_load(st + 2 * C::BLOCK_BYTES, qsrc, G * D * 2u, &full_bar[warp][stage]);
      }
    }
    if (!dry && !probe) armed |= 1u << stage;
    // Advance to the next unit.
    ++cu;
    if (++cb == cnb) {
      cb = 0;
      if (++ch == Hkv) {
        ch = 0;
        cprefix += cnb;
        ++ci;
        cnb = (ci < a.num_seqs) ? units_of(a, nxt_len, nxt_row, clen, crow) : 1;
        while (cnb == 0) {  // empty or invalid sequences own no units
          ++ci;
          cnb = (ci < a.num_seqs) ? seq_units(a, ci, clen, crow, false) : 1;
        }
        if (ci + 1 < a.num_seqs) {
          nxt_len = __ldg(a.context_lens + ci + 1);
          nxt_row = a.seq_rows != nullptr ? __ldg(a.seq_rows + ci + 1) : ci + 1;
        }
      }
    }
  };

  int issued = 0;
  if (early_loads) {
    // Stages up to (not including) the first block that ends a segment: the
    // append ahead may still be writing that one.
    for (; issued < S && issued < ntiles && cb != cnb - 1; ++issued) issue(issued, false);
    pdl_wait();
  }
  for (; issued < S && issued < ntiles; ++issued) issue(issued, false);

  // ---------------------------------------------------------------- compute
  const int g = lane >> 2, t = lane & 3;
  constexpr int KSTEPS = D / 16;
  constexpr int NTILES = D / 8;
  uint32_t qa[KSTEPS][4];
  float o[NTILES][4];
  float m2[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
  const float scale = a.scale;
  const uint64_t limit = a.wait_limit_ns != 0 ? a.wait_limit_ns : kWaitLimitNs;
  // After a wait gave up the warp walks the rest of its span without data: it
  // still parks (empty) portions, so the CTA merge and the per-segment counters
  // of the launch see every portion they expect and end in their usual state.
  bool dry = false;

  for (int32_t it = 0; it < ntiles; ++it) {
    const int stage = it % S;
    const uint32_t phase = (it / S) & 1;
    // Warp-uniform outcome: a lone lane leaving here would strand the others
    // at the warp-collective ldmatrix / mma.sync below.
    if (!dry && !__all_sync(0xffffffffu, mbar_wait(&full_bar[warp][stage], phase, limit))) {
      if (lane == 0) set_status(a.status, kStatusWaitTimeout);
      // Wait (with the full limit) for the copies this warp started: none may
      // still be writing its stages when they are reused or the CTA exits.
      if (lane == 0) {
        for (int32_t j = it; j < it + S && j < ntiles; ++j) {
          if (armed & (1u << (j % S))) mbar_wait(&full_bar[warp][j % S], (j / S) & 1);
        }
      }
      armed = 0;
      dry = true;
      __syncwarp();
    }
    armed &= ~(1u << stage);
    const TileMeta mt = meta[warp][stage];
    const uint8_t* st = wst + stage * C::STAGE_BYTES;
    if (mt.flags & kFirst) {
      m2[0] = m2[1] = -INFINITY;
      lsum[0] = lsum[1] = 0.f;
#pragma unroll
      for (int n = 0; n < NTILES; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    }
    if (!dry && (mt.flags & kFirst)) {
      const uint32_t* sq = reinterpret_cast<const uint32_t*>(st + 2 * C::BLOCK_BYTES);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        // Row r, dims (16kk + 2t, +1) -> 32-bit word (r*D + 16kk + 2t) / 2.
        const int w0 = (g * D + 16 * kk + 2 * t) >> 1;
        const int w1 = ((g + 8) * D + 16 * kk + 2 * t) >> 1;
        qa[kk][0] = (g < G) ? sq[w0] : 0u;
        qa[kk][1] = (G16 && g + 8 < G) ? sq[w1] : 0u;
        qa[kk][2] = (g < G) ? sq[w0 + 4] : 0u;
        qa[kk][3] = (G16 && g + 8 < G) ? sq[w1 + 4] : 0u;
      }
    }
    if (!dry) {
      const int tok0 = mt.blk * kBS;
      const int valid = min(kBS, mt.len - tok0);
      const uint32_t kbase = smem_u32(st);
      const uint32_t vbase = kbase + C::BLOCK_BYTES;
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
      float corr[2] = {1.f, 1.f};
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
      uint32_t pa[4];
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
    // The stage has been read: refill it with the block S positions ahead.
    __syncwarp();
    if (it + S < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(stage, dry);
    }

    if (mt.flags & kLast) {
      float lrow[2];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float l = lsum[hr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        lrow[hr] = l;
      }
      if (mt.flags & kWhole) {
        // The whole segment is in this warp: normalised output from registers.
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) +
                             static_cast<int64_t>(mt.seq) * a.o_stride_seq +
                             static_cast<int64_t>(mt.kvh) * G * D;
#pragma unroll
        for (int hr = 0; hr < (G16 ? 2 : 1); ++hr) {
          const int r = g + 8 * hr;
          if (r < G) {
            const float inv = 1.f / lrow[hr];
#pragma unroll
            for (int n = 0; n < NTILES; ++n) {
              *reinterpret_cast<uint32_t*>(out + r * D + 8 * n + 2 * t) =
                  pack_bf16x2(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
            }
          }
        }
      } else {
        // A cut portion: park it in slot 0 (first portion) or slot 1 (last).
        const int k = (mt.flags & kSlot1) ? 1 : 0;
        float* slot = slot_of(warp, k);
#pragma unroll
        for (int hr = 0; hr < (G16 ? 2 : 1); ++hr) {
          const int r = g + 8 * hr;
          if (r < G) {
#pragma unroll
            for (int n = 0; n < NTILES; ++n) {
              slot[r * D + 8 * n + 2 * t] = o[n][2 * hr];
              slot[r * D + 8 * n + 2 * t + 1] = o[n][2 * hr + 1];
            }
            if (t == 0) {
              slot[G * D + r] = m2[hr];
              slot[G * D + G + r] = lrow[hr];
            }
          }
        }
        if (lane == 0) {
          slot_seq[warp][k] = mt.seq;
          slot_kvh[warp][k] = mt.kvh;
          slot_nb[warp][k] = mt.nb;
          slot_unit[warp][k] = mt.seg_unit;
        }
      }
    }
  }

  // ---------------------------------------------------------------- CTA merge
  // A segment cut between warps is a chain: the last portion of the warp where
  // it starts, the only portion of warps inside it, the first portion of the
  // warp where it ends.  The chain's tail (no later non-empty warp continues the
  // segment) folds the earlier slots into its own and finishes the segment.
  __syncthreads();
  auto warp_empty = [&](int w) {
    return sp.r0 + spanw * (w + 1) / W == sp.r0 + spanw * w / W;
  };
  auto holds = [&](int w, int k, int32_t seq, int32_t kvh) {
    return slot_seq[w][k] == seq && slot_kvh[w][k] == kvh;
  };
  for (int k = 0; k < 2; ++k) {
    const int32_t seq = slot_seq[warp][k];
    if (seq < 0) continue;
    const int32_t kvh = slot_kvh[warp][k];
    bool tail = true;
    if (k == 1 || slot_seq[warp][1] < 0) {
      for (int w2 = warp + 1; w2 < W; ++w2) {
        if (warp_empty(w2)) continue;
        tail = !holds(w2, 0, seq, kvh);
        break;
      }
    }
    if (!tail) continue;
    float* mine = slot_of(warp, k);
    for (int w2 = warp - 1; w2 >= 0; --w2) {
      if (warp_empty(w2)) continue;
      const int k2 = holds(w2, 1, seq, kvh) ? 1 : (holds(w2, 0, seq, kvh) ? 0 : -1);
      if (k2 < 0) break;
      const float* other = slot_of(w2, k2);
      // Row factors once (lane r < G), then one FMA pair per element; a row
      // spans D >= 64 elements, so elements e = lane + 32j share row (32j) / D.
      float fa = 0.f, fb = 0.f;
      if (lane < G) {
        const float ma = mine[G * D + lane], mb = other[G * D + lane];
        const float M = fmaxf(ma, mb);
        fa = fast_exp2(ma - M);
        fb = fast_exp2(mb - M);
        mine[G * D + G + lane] = mine[G * D + G + lane] * fa + other[G * D + G + lane] * fb;
        mine[G * D + lane] = M;
      }
      // Compile-time bounds (rows padded to GROWS): the loads of all elements
      // issue back to back instead of one dependent step at a time.
#pragma unroll
      for (int j = 0; j < C::GROWS * D / 32; ++j) {
        const int r = (32 * j) / D;
        const float a0 = __shfl_sync(0xffffffffu, fa, r);
        const float b0 = __shfl_sync(0xffffffffu, fb, r);
        const int e = lane + 32 * j;
        if (r < G) mine[e] = mine[e] * a0 + other[e] * b0;
      }
      __syncwarp();
      if (k2 == 1) break;  // the chain starts in that warp
    }
    const int64_t seg_unit = slot_unit[warp][k];
    const int32_t nb = slot_nb[warp][k];
    if (seg_unit >= sp.r0 && seg_unit + nb <= sp.r1) {
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) +
                           static_cast<int64_t>(seq) * a.o_stride_seq +
                           static_cast<int64_t>(kvh) * G * D;
      const float inv_l = lane < G ? 1.f / mine[G * D + G + lane] : 0.f;
#pragma unroll
      for (int j = 0; j < C::GROWS * D / 32; ++j) {
        const int r = (32 * j) / D;
        const float inv = __shfl_sync(0xffffffffu, inv_l, r);
        const int e = lane + 32 * j;
        if (r < G) out[e] = __float2bfloat16_rn(mine[e] * inv);
      }
    } else if (a.tasks != nullptr) {
      // Cut across CTAs: leave this CTA's record; the segment is merged after
      // the kernel, listed by the CTA that holds its last unit.
      warp_store_record_fixed<C::GROWS, D>(a, sp, seg_unit, mine, mine + G * D,
                                           mine + G * D + G, lane);
      if (lane == 0 && seg_unit < sp.r0 && seg_unit + nb <= sp.r1) {
        task.seg_unit = seg_unit;
        task.q = sp.q;
        task.rem = sp.rem;
        task.seq = seq;
        task.kvh = kvh;
        task.nb = nb;
        task.valid = 1;
      }
    } else if (warp_write_record(a, sp, seq, kvh, seg_unit, nb, mine, mine + G * D,
                                 mine + G * D + G, lane)) {
      if (lane == 0) {
        const int idx = atomicAdd(&fin_count, 1);
        fin_seq[idx] = seq;
        fin_kvh[idx] = kvh;
        fin_nb[idx] = nb;
        fin_unit[idx] = seg_unit;
      }
    }
  }
  // Segments crossing CTAs for which this CTA came last: merge with all threads.
  // The stages and slots are free now and serve as scratch.
  __syncthreads();
  if (a.tasks != nullptr) {
    if (tid == 0) a.tasks[blockIdx.x] = task;
    return;
  }
  const int nfin = fin_count;
  for (int f = 0; f < nfin; ++f) {
    cta_merge_records<__nv_bfloat16>(a, sp, fin_seq[f], fin_kvh[f], fin_unit[f], fin_nb[f],
                                     reinterpret_cast<float*>(smem));
  }
}

template <int D, bool G16>
int launch_one(const DecodeArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap, int grid,
               cudaStream_t stream) {
  using C = Cfg<D, G16>;
  static unsigned long long configured = 0;  // one bit per device
  cudaError_t e = once_per_device(&configured, [] {
    return cudaFuncSetAttribute(decode_mma_kernel<D, G16>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::W * 32);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, decode_mma_kernel<D, G16>, kmap, vmap, a));
}

// Merges, after the decode kernel, the cut segments its CTAs listed: one CTA
// per decode CTA, all threads on the records of one segment.
// Three CTAs per SM: as many as the decode kernel's grid holds, all in one wave.
__global__ void __launch_bounds__(128, 3) decode_merge_kernel(const DecodeArgs a) {
  extern __shared__ float merge_scratch[];
  pdl_wait();
  const MergeTask t = a.tasks[blockIdx.x];
  if (!t.valid) return;
  Span sp{};
  sp.q = t.q;
  sp.rem = t.rem;
  cta_merge_records<__nv_bfloat16>(a, sp, t.seq, t.kvh, t.seg_unit, t.nb, merge_scratch);
}

template <int D, bool G16>
int occupancy_one() {
  using C = Cfg<D, G16>;
  cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<D, G16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return -static_cast<int>(e);
  int n = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mma_kernel<D, G16>, C::W * 32,
                                                    C::SMEM_BYTES);
  if (e != cudaSuccess) return -static_cast<int>(e);
  return n;
}

}  // namespace

int launch_decode_mma(const DecodeArgs& a, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      int grid, cudaStream_t stream) {
  const bool g16 = a.groups > 8;
  int rc;
  if (a.head_dim == 64)
    rc = g16 ? launch_one<64, true>(a, kmap, vmap, grid, stream)
             : launch_one<64, false>(a, kmap, vmap, grid, stream);
  else
    rc = g16 ? launch_one<128, true>(a, kmap, vmap, grid, stream)
             : launch_one<128, false>(a, kmap, vmap, grid, stream);
  if (rc != 0 || a.tasks == nullptr) return rc;
  // Merge pass: at most `grid` records per segment.
  const int smem = static_cast<int>((2 * static_cast<int64_t>(grid) * a.groups + 2 * a.groups) *
                                    sizeof(float));
  // The attribute is per device: set it on the current one whenever the
  // size grows past what that device was given.
  static int configured_smem[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev >= 64 || smem > configured_smem[dev]) {
    e = cudaFuncSetAttribute(decode_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 64) configured_smem[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, decode_merge_kernel, a));
}

int decode_mma_ctas_per_sm(int head_dim, int groups) {
  const bool g16 = groups > 8;
  if (head_dim == 64) return g16 ? occupancy_one<64, true>() : occupancy_one<64, false>();
  return g16 ? occupancy_one<128, true>() : occupancy_one<128, false>();
}

}  // namespace bsb
