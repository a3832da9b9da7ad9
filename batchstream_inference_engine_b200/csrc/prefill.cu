// Chunked-prefill paged attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), bf16, head_dim 64, block_size 16.
//
// A prefill chunk of n query tokens follows P cached tokens of its sequence;
// query token i (position P + i) attends to keys 0 .. P + i, causal within the
// chunk and full over the cached part — the reference's _read_blocks + attend
// with _causal_mask (src/server/torch_model.py:39-64, 165-167, 295-297).
//
// One CTA per (chunk, query head, 128-token query tile, piece of its key
// range; pieces only for batches with fewer query tiles that can hold tokens
// than SMs, merged by prefill_merge_kernel).  A CTA's time is its chain of key tiles, so when the
// grid is more than one wave of resident CTAs a one-CTA plan kernel runs first
// and ranks the work by key tiles: the longest chains start in the first wave
// instead of whenever their index comes up.  Three roles, one warp each for
// the first two:
//   * loader (warp 5): the query tile as one TMA box of a [T, H, D] tensor map,
//     then the sequence's K and V through the block table into a 4-stage K ring
//     and a 3-stage V ring (64 keys = 4 blocks per stage, one TMA box per block).
//     The loads are latency-bound (the pool is mostly read from L2), so the
//     rings are as deep as two CTAs per SM allow.  A K stage is
//     refilled once the S product that read it has completed, a V stage once
//     its P V product has; K runs two tiles ahead of V, which gives either load
//     about three softmax periods to land.  Block-table entries come from a
//     32-entry register window fetched one window ahead;
//   * MMA issuer (warp 4), from one thread:
//       S  = Q K^T   tcgen05.mma kind::f16, M=128 N=64 K=64  -> TMEM, 2 buffers
//       O += P V     tcgen05.mma kind::f16, M=128 N=64 K=64  -> TMEM
//     in steps of PV(j), S(j+2) and ONE commit: the tensor core computes the
//     scores two tiles ahead while the softmax warps work on tile j+1.  Each
//     tcgen05 instruction takes the issuing thread tens of nanoseconds, so a
//     step waits for all its operands first and signals every consumer (the
//     softmax, the loader's K and V stages) through that single commit;
//   * softmax (warps 0-3) own the 128 query
// rows (TMEM lane = row): they read their row of S (tcgen05.ld), apply the
// reference's rounding points (bf16(bf16(q.k) * scale); the second rounding is
// exact and skipped when the scale is a power of two) through packed
// conversions, mask only on tiles that reach past a row's position or the
// context, run an online softmax in base 2 that rescales O in TMEM only when a
// row maximum grows by more than 2^8, and write P (bf16) into one of two
// shared-memory buffers for the P V product.
//
// Waits are bounded (a status bit instead of a hang) and their outcome is made
// warp-uniform before any warp-collective tcgen05 instruction; before TMEM is
// freed the MMA warp drains every MMA and the loader every TMA load it started,
// also on the error path.  V rows of keys no row of the tile can see are zeroed before the P V
// product, so stale or NaN shared-memory and pool contents never reach the result.
#include "prefill.cuh"

namespace bsb {

namespace {

constexpr int kRows = 128;   // query rows per CTA (TMEM lanes)
constexpr int kKeys = 64;    // keys per KV tile (4 blocks)
constexpr int kD = 64;
constexpr int kKStages = 4;  // K ring depth
constexpr int kVStages = 3;  // V ring depth
constexpr int kSteps = 4;    // MMA step barriers (>= kKStages, >= kVStages + 1)
static_assert(kSteps >= kKStages && kSteps >= kVStages + 1 && kSteps >= 3,
              "a step waiter could fall a whole ring of step barriers behind");
constexpr int kThreads = 192;  // warps 0-3 softmax, warp 4 MMA issuer, warp 5 loader
constexpr int kTileBytes = kKeys * kD * 2;  // 8 KiB: K or V of one tile
constexpr int kQBytes = kRows * kD * 2;     // 16 KiB
constexpr int kPBytes = kRows * kKeys * 2;  // 16 KiB per P buffer
constexpr int kSmemBytes =
    1024 + kQBytes + (kKStages + kVStages) * kTileBytes + 2 * kPBytes;
constexpr uint32_t kTmemCols = 256;  // S0 [0, 64), S1 [64, 128), O [128, 192)
constexpr uint32_t kTmemO = 128;
constexpr float kLog2eP = 1.4426950408889634f;
constexpr float kRescaleSlack = 8.f;  // rescale O when a row max grows by > 2^8
// Merge pass: query rows per CTA, eight threads per row.
constexpr int kMergeRowsPerCta = 32;
constexpr int kMergeThreads = kMergeRowsPerCta * 8;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // sm100 shared-memory matrix descriptor: start, leading and stride byte
  // offsets in 16-byte units, version 1, 128-byte swizzle.
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of kind::f16: bf16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
}

__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31]));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 3-D tiled load (query tile): coordinates (dim, head, token).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Lane-wise maximum of two packed bf16 pairs.
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Byte offset of element (r, c) in a [rows][64] bf16 tile with 128-byte swizzle.
__device__ __forceinline__ uint32_t swz128(int r, int c) {
  return r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2;
}

// What one CTA computes: chunk r, head h, the query tile at t0 and piece sp of
// its key range (record item * splits + sp), with the chunk's first token,
// query tokens, context length and block-table row.
struct Work {
  int item, r, h, t0, sp;
  int tok0, n, ctx, row_tab;
};

// Work of CTA b without a plan: tiles with the most keys first (the last
// query tile of every chunk, then the one before, ...), heads inside, splits
// innermost.  Also numbers the merge kernel's items (b = item * splits).
__device__ __forceinline__ void item_work(const PrefillArgs& a, int b, Work& w) {
  w.sp = b % a.splits;
  w.item = b / a.splits;
  const int H = a.num_heads;
  w.h = w.item % H;
  const int rt = w.item / H;  // 0 .. num_rows * qtiles - 1
  const int t = a.qtiles - 1 - rt / a.num_rows;
  w.r = rt % a.num_rows;
  w.t0 = t * kRows;
  w.tok0 = __ldcg(a.cu_q + w.r);
  w.n = __ldcg(a.cu_q + w.r + 1) - w.tok0;
  w.ctx = __ldcg(a.context_lens + w.r);
  w.row_tab = a.seq_rows != nullptr ? __ldcg(a.seq_rows + w.r) : w.r;
}

// Work of CTA b: entry b / H of the plan (head b % H), or the plan-less
// numbering.  False for CTAs past the plan's entries.
__device__ __forceinline__ bool cta_work(const PrefillArgs& a, int b, Work& w) {
  if (a.plan == nullptr) {
    item_work(a, b, w);
    return true;
  }
  const int H = a.num_heads;
  const int d = b / H;  // < rows * qtiles * splits: inside the plan
  // Coherent loads: the plan kernel just ahead writes these while this grid,
  // launched early, is already resident (no read-only cache path for them).
  const int4 head = __ldcg(a.plan);
  const int4 x = __ldcg(a.plan + 1 + 2 * d);
  const int4 y = __ldcg(a.plan + 2 + 2 * d);
  if (d >= head.x) return false;
  w.h = b % H;
  w.sp = x.x % a.splits;
  const int rt = x.x / a.splits;
  w.item = rt * H + w.h;
  w.r = rt % a.num_rows;
  w.t0 = (a.qtiles - 1 - rt / a.num_rows) * kRows;
  w.tok0 = x.y;
  w.n = x.z;
  w.ctx = x.w;
  w.row_tab = y.x;
  return true;
}

// Work of CTA b when it ranks the (row, query tile) pairs itself: the plan
// kernel's order for a batch without splits (one entry per pair, most key tiles
// first, ties by index), computed by every CTA in shared memory that nothing
// uses yet instead of by a launch ahead that the CTA would wait for.  All
// threads call it.
__device__ __forceinline__ void cta_work_ranked(const PrefillArgs& a, int b, Work& w,
                                                uint8_t* scratch) {
  static_assert(kMaxCtaRankedRts <= kThreads, "one pair per thread");
  static_assert(kMaxCtaRankedRts * 20 + 4 <= kQBytes, "the scratch lies in the query tile");
  int4* s_row = reinterpret_cast<int4*>(scratch);
  int32_t* s_size = reinterpret_cast<int32_t*>(scratch + kMaxCtaRankedRts * 16);
  int32_t* s_pick = s_size + kMaxCtaRankedRts;
  const int tid = threadIdx.x;
  const int R = a.num_rows, Q = a.qtiles, H = a.num_heads;
  const int n_rt = R * Q;  // <= kMaxCtaRankedRts (host); the grid is n_rt * H
  int size = 0;
  if (tid < n_rt) {
    const int rt = tid, r = rt % R, t0 = (Q - 1 - rt / R) * kRows;
    const int tok0 = __ldcg(a.cu_q + r);
    const int n = __ldcg(a.cu_q + r + 1) - tok0;
    const int ctx = __ldcg(a.context_lens + r);
    const int row_tab = a.seq_rows != nullptr ? __ldcg(a.seq_rows + r) : r;
    s_row[rt] = make_int4(tok0, n, ctx, row_tab);
    // Rows the kernel rejects or skips count as no work (they are checked below).
    if (n > 0 && t0 < n && ctx >= n && ctx <= a.max_blocks * 16) {
      const long long kv_end = min(static_cast<long long>(ctx),
                                   static_cast<long long>(ctx - n) + t0 + kRows);
      size = static_cast<int>((kv_end + kKeys - 1) / kKeys);
    }
    s_size[rt] = size;
  }
  __syncthreads();
  if (tid < n_rt) {
    int rank = 0;
#pragma unroll 8
    for (int f = 0; f < n_rt; ++f) {
      const int g = s_size[f];
      rank += (g > size || (g == size && f < tid)) ? 1 : 0;
    }
    if (rank == b / H) *s_pick = tid;  // the ranks are a permutation of 0 .. n_rt - 1
  }
  __syncthreads();
  const int rt = *s_pick;
  const int4 row = s_row[rt];
  w.h = b % H;
  w.sp = 0;
  w.item = rt * H + w.h;
  w.r = rt % R;
  w.t0 = (Q - 1 - rt / R) * kRows;
  w.tok0 = row.x;
  w.n = row.y;
  w.ctx = row.z;
  w.row_tab = row.w;
  __syncthreads();  // the scratch is the query tile's shared memory
}

__global__ void __launch_bounds__(kThreads, 2)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // MMA step u issues P V(u - 2) (u >= 2), then S(u) (u < ntiles), and makes
  // one commit, to step_done[u % kSteps]: "S(j) is in TMEM", "K stage of S(j)
  // is free", "P V(t) is done" and "V stage of P V(t) is free" are all waits on
  // the step that holds the product (a commit completes once every MMA issued
  // before it has).  Every waiter checks a step less than kSteps steps behind
  // the newest one that can complete, so a parity wait is never ambiguous.
  __shared__ uint64_t q_full, k_full[kKStages], v_full[kVStages], step_done[kSteps], p_full[2],
      mma_done;
  __shared__ uint32_t tmem_base;

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  // K ring, then V ring, then the two P buffers.
  auto sK = [&](int st) { return smem + kQBytes + st * kTileBytes; };
  auto sV = [&](int st) { return smem + kQBytes + (kKStages + st) * kTileBytes; };
  auto sP = [&](int b) {
    return smem + kQBytes + (kKStages + kVStages) * kTileBytes + b * kPBytes;
  };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();

  Work wk;
  if (a.rank_in_cta) {
    cta_work_ranked(a, blockIdx.x, wk, smem);
  } else if (!cta_work(a, blockIdx.x, wk)) {
    return;
  }
  const int item = wk.item, h = wk.h, t0 = wk.t0, sp = wk.sp, tok0 = wk.tok0, n = wk.n;
  if (t0 == 0 && h == 0 && tid == 0 && n > a.qtiles * kRows) set_status(a.status, kStatusBadLength);
  if (t0 >= n) return;
  const int ctx = wk.ctx;
  const int prior = ctx - n;
  const int row_tab = wk.row_tab;
  if (n <= 0 || prior < 0 || row_tab < 0 || row_tab >= a.bt_rows ||
      ctx > a.max_blocks * 16) {
    if (tid == 0) set_status(a.status, row_tab < 0 || row_tab >= a.bt_rows ? kStatusBadRow
                                                                           : kStatusBadLength);
    return;
  }
  const int kv_end = min(ctx, prior + t0 + kRows);  // keys the tile's last row can see
  const int all_tiles = (kv_end + kKeys - 1) / kKeys;
  // This CTA's key tiles [j_lo, j_lo + ntiles) of the query tile's range.
  const int nsplit = prefill_tile_splits(all_tiles, a.splits);
  if (sp >= nsplit) return;
  const int j_lo = sp * all_tiles / nsplit;
  const int ntiles = (sp + 1) * all_tiles / nsplit - j_lo;
  const int kvh = h / a.groups;
  const int32_t* table = a.block_tables + static_cast<int64_t>(row_tab) * a.bt_stride;

  if (tid == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kKStages; ++s) mbar_init(&k_full[s], 1);
    for (int s = 0; s < kVStages; ++s) mbar_init(&v_full[s], 1);
    for (int s = 0; s < kSteps; ++s) mbar_init(&step_done[s], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&p_full[b], kRows);
    mbar_init(&mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  constexpr uint32_t kIdescS = umma_idesc(128, kKeys, 0, 0);
  constexpr uint32_t kIdescO = umma_idesc(128, kD, 0, 1);
  // A wait's outcome is the same for the whole warp (and the warp converged)
  // before any warp-collective instruction follows it.
  auto wait_all = [&](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
  };
  auto wait_step = [&](int u) { return wait_all(&step_done[u % kSteps], (u / kSteps) & 1); };

  if (warp == 5) {
    // ---------------------------------------------------------------- loader
    // Table window: lane i holds entry 32 w + i of window w (0 past the row).
    auto fetch = [&](int w) {
      const int e = w * 32 + lane;
      return (e < a.max_blocks && e * 16 < kv_end) ? __ldg(table + e) : 0;
    };
    int win = (j_lo * 4) / 32;
    int32_t win_cur = fetch(win), win_next = fetch(win + 1);
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, kQBytes);
      tma_load_3d(sQ, &qmap, &q_full, 0, h, tok0 + t0);
    }
    // Block of tile t held by lane (lanes 0-3), -1 when absent.  Tiles are
    // asked for in increasing order, V lagging K by two.
    auto block_of = [&](int t, int32_t wv) {
      const int b = t * 4 + (lane & 3);
      int32_t blk = __shfl_sync(0xffffffffu, wv, (t * 4) % 32 + (lane & 3));
      if (lane >= 4 || b * 16 >= kv_end) return -1;
      if (blk < 0 || blk >= a.num_blocks) {
        set_status(a.status, kStatusBadBlock);
        return -1;
      }
      return blk;
    };
    // One ring's tile t: expect its bytes on `full`, one box per block.
    auto load = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* full, int32_t blk) {
      const uint32_t valid = __ballot_sync(0xffffffffu, blk >= 0) & 0xfu;
      if (lane == 0) mbar_arrive_expect_tx(full, __popc(valid) * 2048u);
      __syncwarp();
      if (blk >= 0) tma_load_2d(dst + lane * 2048, map, full, 0, (kvh * a.num_blocks + blk) * 16);
    };
    bool ok = true;
    int k_loads = 0, v_loads = 0;
    int32_t hold_even = -1, hold_odd = -1;  // V's blocks lag K's by two tiles
    for (int i = 0; i < ntiles + 2 && ok; ++i) {
      // V(i - 2)'s blocks, taken before K(i) (same parity) replaces them.
      const int32_t vblk = (i & 1) ? hold_odd : hold_even;
      if (i < ntiles) {
        const int st = i % kKStages;
        if (i >= kKStages) {
          // K stage st is free once S of tile i - kKStages has read it (step
          // i - kKStages; step i cannot complete before K(i) lands).
          ok = wait_step(i - kKStages);
          if (!ok) break;
        }
        if (((j_lo + i) * 4) / 32 != win) {
          win_cur = win_next;
          ++win;
          win_next = fetch(win + 1);
        }
        const int32_t blk = block_of(j_lo + i, win_cur);
        load(&kmap, sK(st), &k_full[st], blk);
        k_loads = i + 1;
        if (i & 1) hold_odd = blk; else hold_even = blk;
      }
      const int t = i - 2;
      if (t >= 0 && t < ntiles) {
        const int st = t % kVStages;
        if (t >= kVStages) {
          // V stage st is free once P V of tile t - kVStages has read it (step
          // t - kVStages + 2; that step + kSteps needs V(t + 1), not loaded yet).
          ok = wait_step(t - kVStages + 2);
          if (!ok) break;
        }
        load(&vmap, sV(st), &v_full[st], vblk);
        v_loads = t + 1;
      }
    }
    // Drain: the loads of the last stages still hold their newest phase.
    bool drained = wait_all(&q_full, 0);
    for (int t = max(0, k_loads - kKStages); t < k_loads; ++t) {
      drained = wait_all(&k_full[t % kKStages], (t / kKStages) & 1) && drained;
    }
    for (int t = max(0, v_loads - kVStages); t < v_loads; ++t) {
      drained = wait_all(&v_full[t % kVStages], (t / kVStages) & 1) && drained;
    }
    if ((!ok || !drained) && lane == 0) set_status(a.status, kStatusWaitTimeout);
  } else if (warp == 4) {
    // ---------------------------------------------------------------- MMA issuer
    // Shared-memory descriptors of every operand, built once: a stage, buffer
    // or 16-wide K slice only moves the start address, whose field is the
    // address / 16 in the low 14 bits (every address here stays below 2^18),
    // so each MMA's descriptors are one add away from these.
    const uint64_t desc_q = umma_desc(smem_u32(sQ), 16, 1024);
    const uint64_t desc_k = umma_desc(smem_u32(sK(0)), 16, 1024);
    const uint64_t desc_v = umma_desc(smem_u32(sV(0)), 8192, 1024);
    const uint64_t desc_p = umma_desc(smem_u32(sP(0)), 16, 1024);
    constexpr uint64_t kStageStep = kTileBytes >> 4, kPStep = kPBytes >> 4;
    bool ok = wait_all(&q_full, 0);
    for (int u = 0; u < ntiles + 2 && ok; ++u) {
      // Step u: P V(j = u - 2) once softmax(j) has written P(j) (which also
      // frees S buffer j & 1), then S(u) into that buffer, then one commit.
      // The waits come first, so the step's MMAs issue back to back.
      const int j = u - 2;
      if (j >= 0) {
        ok = wait_all(&p_full[j & 1], (j >> 1) & 1) &&
             wait_all(&v_full[j % kVStages], (j / kVStages) & 1);
      }
      if (ok && u < ntiles) ok = wait_all(&k_full[u % kKStages], (u / kKStages) & 1);
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        if (j >= 0) {
          const uint64_t p0 = desc_p + (j & 1) * kPStep;
          const uint64_t v0 = desc_v + (j % kVStages) * kStageStep;
#pragma unroll
          for (int k = 0; k < kKeys / 16; ++k) {
            // P: 32 bytes per 16-key slice; V: 2048 bytes (16 key rows).
            umma_f16(tmem + kTmemO, p0 + 2 * k, v0 + 128 * k, kIdescO, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        if (u < ntiles) {
          const uint32_t d = tmem + (u & 1) * kKeys;
          const uint64_t k0 = desc_k + (u % kKStages) * kStageStep;
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {
            // Q and K: 32 bytes per 16-dim slice.
            umma_f16(d, desc_q + 2 * k, k0 + 2 * k, kIdescS, k > 0 ? 1u : 0u);
          }
        }
        umma_commit(&step_done[u % kSteps]);
      }
      __syncwarp();
    }
    // Drain: no MMA may still use TMEM once the CTA frees it.  The commit
    // tracks every MMA issued above.
    if (lane == 0) umma_commit(&mma_done);
    __syncwarp();
    const bool drained = wait_all(&mma_done, 0);
    if ((!ok || !drained) && lane == 0) set_status(a.status, kStatusWaitTimeout);
  } else {
    // ---------------------------------------------------------------- softmax
    const int row = tid;  // TMEM lane and query row
    const int qpos = prior + t0 + row;  // position of this row's token
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    // z = score * scale * log2(e); rows keep m (max z used for P) and l.
    const float zscale = (a.exact_scale ? a.scale : 1.f) * kLog2eP;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = wait_step(j);  // S(j) is in TMEM
      if (!ok) break;
      tc_fence_after();
      // Scores rounded to bf16 (the reference's first rounding), kept as packed
      // pairs: lane bits [15:0] hold key 2i, [31:16] key 2i + 1.
      uint32_t sp[kKeys / 2];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(tmem + lane_base + (j & 1) * kKeys, v0);
        tmem_ld32(tmem + lane_base + (j & 1) * kKeys + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          sp[i] = pack_bf16x2(__uint_as_float(v0[2 * i]), __uint_as_float(v0[2 * i + 1]));
          sp[16 + i] = pack_bf16x2(__uint_as_float(v1[2 * i]), __uint_as_float(v1[2 * i + 1]));
        }
      }
      if (!a.exact_scale) {
#pragma unroll
        for (int i = 0; i < kKeys / 2; ++i) {
          sp[i] = pack_bf16x2(__uint_as_float(sp[i] << 16) * a.scale,
                              __uint_as_float(sp[i] & 0xFFFF0000u) * a.scale);
        }
      }
      const int key0 = (j_lo + j) * kKeys;
      // Tiles wholly at or before the first row's position need no mask;
      // masked keys become bf16 -inf.
      if (key0 + kKeys - 1 > prior + t0) {
#pragma unroll
        for (int i = 0; i < kKeys / 2; ++i) {
          const int k0 = key0 + 2 * i;
          const bool lo = k0 <= qpos && k0 < ctx, hi = k0 + 1 <= qpos && k0 + 1 < ctx;
          sp[i] = (lo ? (sp[i] & 0xFFFFu) : 0xFF80u) | (hi ? (sp[i] & 0xFFFF0000u) : 0xFF800000u);
        }
      }
      uint32_t mp[4] = {sp[0], sp[1], sp[2], sp[3]};
#pragma unroll
      for (int i = 4; i < kKeys / 2; ++i) mp[i & 3] = max_bf16x2(mp[i & 3], sp[i]);
      const uint32_t m2 = max_bf16x2(max_bf16x2(mp[0], mp[1]), max_bf16x2(mp[2], mp[3]));
      const float m_tile = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xFFFF0000u));
      const float m_tile_z = m_tile * zscale;
      // Key 0 is visible to every row, so m_used is finite from the first tile
      // on when the range starts at key 0; a later range's first tiles may hide
      // every key from some rows (m_used -inf until one shows, P 0 meanwhile).
      const bool grow = m_tile_z > m_used + kRescaleSlack;
      if (j == 0) {
        m_used = m_tile_z;
      } else if (__any_sync(0xffffffffu, grow)) {
        // tcgen05.ld/st are warp-collective: the warp rescales if any row
        // grew past the slack (factor 1 for the others).
        ok = wait_step(j + 1);  // P V of the previous tile is done
        if (!ok) break;
        tc_fence_after();
        const float m_new = grow ? m_tile_z : m_used;
        const float corr = grow ? fast_exp2(m_used - m_new) : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < kD; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + kTmemO + lane_base + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __float_as_uint(__uint_as_float(v[c]) * corr);
          tmem_st32(tmem + kTmemO + lane_base + c0, v);
        }
        tmem_wait_st();
        l_run *= corr;
        m_used = m_new;
      }
      // P = 2^(z - m_used) <= 2^8, packed to bf16 into P buffer j & 1 (free:
      // the step of S(j) also holds the P V of tile j - 2 that read it).
      // Sums kept in 8 partials (key index mod 8), two per packed register.
      float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
      const float m_base = m_used == -INFINITY ? 0.f : m_used;  // no -inf - -inf
      const float2 zs = make_float2(zscale, zscale), mm = make_float2(-m_base, -m_base);
      uint8_t* prow = sP(j & 1);
#pragma unroll
      for (int ch = 0; ch < kKeys / 8; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t u = sp[ch * 4 + e];
          const float2 z = __ffma2_rn(make_float2(__uint_as_float(u << 16),
                                                  __uint_as_float(u & 0xFFFF0000u)), zs, mm);
          const float2 pe = make_float2(fast_exp2(z.x), fast_exp2(z.y));
          ps[e] = __fadd2_rn(ps[e], pe);
          w[e] = pack_bf16x2(pe.x, pe.y);
        }
        *reinterpret_cast<uint4*>(prow + swz128(row, ch * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
      // Keys no row of this CTA sees (past the context, or past the last row's
      // position): their V rows hold stale pool data or never-loaded shared
      // memory, possibly NaN, which would poison 0 * V in the tensor core.
      if (j == ntiles - 1 && row < kKeys && key0 + kKeys > kv_end) {
        // The V tile must have landed before its tail rows are overwritten.
        ok = wait_all(&v_full[j % kVStages], (j / kVStages) & 1);
        if (!ok) break;
      }
      if (row < kKeys && key0 + row >= kv_end) {
        uint4 z = make_uint4(0u, 0u, 0u, 0u);
        uint8_t* vrow = sV(j % kVStages) + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vrow + c * 16) = z;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    if (ok) ok = wait_step(ntiles + 1);  // the last P V is done
    if (ok && nsplit > 1) {
      tc_fence_after();
      // One record per CTA: unnormalised O, then (max, sum) of the row.
      const int64_t rec = static_cast<int64_t>(item) * a.splits + sp;
      float* orow = a.part_o + (rec * kRows + row) * kD;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + kTmemO + lane_base + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          *reinterpret_cast<float4*>(orow + c0 + c) =
              make_float4(__uint_as_float(v[c]), __uint_as_float(v[c + 1]),
                          __uint_as_float(v[c + 2]), __uint_as_float(v[c + 3]));
        }
      }
      *reinterpret_cast<float2*>(a.part_ml + (rec * kRows + row) * 2) = make_float2(m_used, l_run);
    } else if (ok) {
      tc_fence_after();
      // Every lane reads its TMEM row (warp-collective); rows past the chunk
      // are not stored.
      const bool store = t0 + row < n;
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) +
                           static_cast<int64_t>(tok0 + t0 + (store ? row : 0)) * a.o_stride_tok +
                           static_cast<int64_t>(h) * kD;
      const float inv = 1.f / l_run;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + kTmemO + lane_base + c0, v);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[c]) * inv, __uint_as_float(v[c + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[c + 2]) * inv, __uint_as_float(v[c + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[c + 4]) * inv, __uint_as_float(v[c + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[c + 6]) * inv, __uint_as_float(v[c + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c0 + c) = w;
          }
        }
      }
    } else if (tid == 0) {
      set_status(a.status, kStatusWaitTimeout);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// Merges the split records of the work items, kMergeRowsPerCta query rows of
// one item per CTA and eight threads per row (eight columns each), so that a
// thread's loads are all independent: one round trip for the (max, sum) pairs
// of its row, one for its columns of every record.  out = sum_s 2^(m_s - M) O_s /
// sum_s 2^(m_s - M) l_s in bf16, summed in split order.  Items whose key range
// was not split were written by the prefill kernel itself.
__global__ void __launch_bounds__(kMergeThreads) prefill_merge_kernel(const PrefillArgs a) {
  pdl_wait();
  constexpr int kCtasPerItem = kRows / kMergeRowsPerCta;
  Work wk;
  item_work(a, (blockIdx.x / kCtasPerItem) * a.splits, wk);
  const int item = wk.item, h = wk.h, t0 = wk.t0, tok0 = wk.tok0, n = wk.n;
  const int row = (blockIdx.x % kCtasPerItem) * kMergeRowsPerCta + threadIdx.x / 8;
  const int c = (threadIdx.x % 8) * 8;
  if (t0 >= n || t0 + row >= n) return;
  const int ctx = wk.ctx;
  const int prior = ctx - n;
  const int row_tab = wk.row_tab;
  if (prior < 0 || row_tab < 0 || row_tab >= a.bt_rows || ctx > a.max_blocks * 16) return;
  const int kv_end = min(ctx, prior + t0 + kRows);
  const int nsplit = prefill_tile_splits((kv_end + kKeys - 1) / kKeys, a.splits);
  if (nsplit <= 1) return;
  const int64_t rec0 = static_cast<int64_t>(item) * a.splits;
  float2 ml[kMaxPrefillSplits];
  float4 x[kMaxPrefillSplits], y[kMaxPrefillSplits];
#pragma unroll
  for (int s = 0; s < kMaxPrefillSplits; ++s) {
    ml[s] = make_float2(-INFINITY, 0.f);
    x[s] = y[s] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s < nsplit) {
      const int64_t r = (rec0 + s) * kRows + row;
      ml[s] = *reinterpret_cast<const float2*>(a.part_ml + r * 2);
      const float* o = a.part_o + r * kD + c;
      x[s] = *reinterpret_cast<const float4*>(o);
      y[s] = *reinterpret_cast<const float4*>(o + 4);
    }
  }
  float M = -INFINITY;
#pragma unroll
  for (int s = 0; s < kMaxPrefillSplits; ++s) M = fmaxf(M, ml[s].x);
  float w[kMaxPrefillSplits];
  float L = 0.f;
#pragma unroll
  for (int s = 0; s < kMaxPrefillSplits; ++s) {
    // A range none of whose keys this row sees has max -inf: weight 0, and its
    // O (all zero) does not enter the sum.
    const float f = ml[s].x == -INFINITY ? 0.f : fast_exp2(ml[s].x - M);
    L += f * ml[s].y;
    w[s] = f;
  }
  const float inv = 1.f / L;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < kMaxPrefillSplits; ++s) {
    if (w[s] == 0.f) continue;  // also every s >= nsplit
    acc[0] += w[s] * x[s].x; acc[1] += w[s] * x[s].y; acc[2] += w[s] * x[s].z;
    acc[3] += w[s] * x[s].w; acc[4] += w[s] * y[s].x; acc[5] += w[s] * y[s].y;
    acc[6] += w[s] * y[s].z; acc[7] += w[s] * y[s].w;
  }
  uint4 out;
  out.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  out.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  out.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  out.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) +
                       static_cast<int64_t>(tok0 + t0 + row) * a.o_stride_tok +
                       static_cast<int64_t>(h) * kD + c;
  *reinterpret_cast<uint4*>(dst) = out;
}


// Ranks the prefill work, one CTA: every (row, query tile) rt has
//   tiles(rt) = ceil(min(ctx, prior + t0 + 128) / 64)
// key tiles per head, cut into pieces as the kernel cuts them; the pieces are
// ranked by size, largest first (ties by index), so that launched in that
// order the longest chains start first.
constexpr int kPlanThreads = kMaxPlanEntries;

__global__ void __launch_bounds__(kPlanThreads) prefill_plan_kernel(const PrefillArgs a) {
  // Per rt (at most half the entries: the host keeps rt * 2 within them): the
  // row's first token, query tokens, context and block-table row.
  __shared__ int4 s_row[kMaxPlanEntries / 2];
  __shared__ int32_t s_size[kMaxPlanEntries];  // per slot rt * splits + piece, -1 unused
  pdl_trigger();  // the prefill CTAs may take their SMs and wait for the plan
  pdl_wait();     // cu_q and context_lens come from the kernels just ahead
  const int tid = threadIdx.x;
  const int R = a.num_rows, Q = a.qtiles, S = a.splits;
  const int n_slot = R * Q * S;  // <= kMaxPlanEntries (host)

  // Slot rt * S + p holds piece p of rt while p < pieces(rt); a row without
  // work keeps one entry, so the kernel still checks it.
  int size = -1;
  if (tid < n_slot) {
    const int rt = tid / S, p = tid % S;
    const int r = rt % R, t0 = (Q - 1 - rt / R) * kRows;
    const int tok0 = __ldcg(a.cu_q + r);
    const int n = __ldcg(a.cu_q + r + 1) - tok0;
    const int ctx = __ldcg(a.context_lens + r);
    if (p == 0) {
      const int row_tab = a.seq_rows != nullptr ? __ldcg(a.seq_rows + r) : r;
      s_row[rt] = make_int4(tok0, n, ctx, row_tab);
    }
    int tiles = 0;
    // Rows the prefill kernel rejects or skips count as no work.
    if (n > 0 && t0 < n && ctx >= n && ctx <= a.max_blocks * 16) {
      const long long kv_end = min(static_cast<long long>(ctx),
                                   static_cast<long long>(ctx - n) + t0 + kRows);
      tiles = static_cast<int>((kv_end + kKeys - 1) / kKeys);
    }
    const int k = prefill_tile_splits(tiles, S);
    if (p < k) size = (p + 1) * tiles / k - p * tiles / k;
    s_size[tid] = size;
  }
  const int entries = __syncthreads_count(size >= 0);
  if (tid == 0) a.plan[0] = make_int4(entries, 0, 0, 0);
  if (size >= 0) {
    int rank = 0;
#pragma unroll 8
    for (int f = 0; f < n_slot; ++f) {
      const int g = s_size[f];
      rank += (g > size || (g == size && f < tid)) ? 1 : 0;
    }
    const int4 row = s_row[tid / S];
    a.plan[1 + 2 * rank] = make_int4(tid, row.x, row.y, row.z);
    a.plan[2 + 2 * rank] = make_int4(row.w, 0, 0, 0);
  }
}

}  // namespace

int prefill_smem_bytes() { return kSmemBytes; }

int launch_prefill_merge(const PrefillArgs& a, int64_t items, cudaStream_t stream) {
  const int64_t grid = items * (kRows / kMergeRowsPerCta);
  if (grid > 0x7fffffff) return static_cast<int>(cudaErrorInvalidConfiguration);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kMergeThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, prefill_merge_kernel, a));
}

namespace {

int configure_prefill() {
  static unsigned long long configured = 0;  // one bit per device
  return static_cast<int>(once_per_device(&configured, [] {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    // All of the unified L1 as shared memory: two CTAs per SM.
    return cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                100);
  }));
}

}  // namespace

// Prefill CTAs resident on one SM: as many as its shared memory holds with the
// whole unified L1 carved out as shared memory (the launch asks for that; the
// occupancy calculator assumes the default carve-out and reports one), at most
// two by TMEM (kTmemCols of 512 columns each) and by the launch bounds.
int prefill_ctas_per_sm() {
  static int ctas = 0;
  if (ctas == 0) {
    int dev = 0, smem_sm = 0, reserved = 0;
    cudaFuncAttributes fa{};
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) !=
            cudaSuccess ||
        cudaFuncGetAttributes(&fa, prefill_kernel) != cudaSuccess) {
      return 1;
    }
    const int per_cta = kSmemBytes + static_cast<int>(fa.sharedSizeBytes) + reserved;
    const int by_smem = smem_sm / per_cta;
    const int by_tmem = 512 / static_cast<int>(kTmemCols);
    ctas = by_smem < by_tmem ? by_smem : by_tmem;
    if (ctas < 1) ctas = 1;
  }
  return ctas;
}

int launch_prefill_plan(const PrefillArgs& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kPlanThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, prefill_plan_kernel, a));
}

int launch_prefill_tc(const PrefillArgs& a, const CUtensorMap& qmap, const CUtensorMap& kmap,
                      const CUtensorMap& vmap, int grid, cudaStream_t stream) {
  if (int e = configure_prefill()) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, prefill_kernel, qmap, kmap, vmap, a));
}

}  // namespace bsb
