// Chunked-prefill paged attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), bf16, head_dim 64, block_size 16.
//
// A prefill chunk of n query tokens follows P cached tokens of its sequence;
// query token i (position P + i) attends to keys 0 .. P + i, causal within the
// chunk and full over the cached part — the reference's _read_blocks + attend
// with _causal_mask (src/server/torch_model.py:39-64, 165-167, 295-297).
//
// One CTA per (chunk, query head, 128-token query tile).  Warp 4 is the issuer:
// it loads the query tile with one TMA box of a [T, H, D] tensor map (128 tokens
// x 64 dims, 128-byte swizzle), streams the sequence's K and V 16-token blocks
// through the block table into a two-stage ring (one TMA box per block), and
// from one thread issues
//     S  = Q K^T   tcgen05.mma kind::f16, M=128 N=128 K=64, S in TMEM (128 cols)
//     O += P V     tcgen05.mma kind::f16, M=128 N=64 K=128, O in TMEM (64 cols)
// with operands read straight from swizzled shared memory (K-major Q, K and P;
// V as an MN-major operand).  Warps 0-3 own the 128 query rows (TMEM lane = row):
// they read their row of S with tcgen05.ld, apply the reference's rounding
// points (bf16(bf16(q.k) * scale)), the causal and length masks and an online
// softmax in base 2 with no cross-thread reductions, rescale O in TMEM when a
// row maximum grows, and write P (bf16) into shared memory for the next MMA.
//
// Waits are bounded (a status bit instead of a hang) and their outcome is made
// warp-uniform before any warp-collective tcgen05 instruction; before TMEM is
// freed the issuer drains every MMA and TMA load it started, also on the error
// path.  V rows of keys no row of the tile can see are zeroed before the P V
// product, so stale or NaN shared-memory and pool contents never reach the result.
#include "prefill.cuh"

namespace bsb {

namespace {

constexpr int kRows = 128;   // query rows per CTA (TMEM lanes)
constexpr int kKeys = 128;   // keys per KV tile
constexpr int kD = 64;
constexpr int kThreads = 160;  // warps 0-3 softmax, warp 4 issuer
constexpr int kTileBytes = kKeys * kD * 2;  // 16 KiB (K or V of one tile)
constexpr int kQBytes = kRows * kD * 2;
constexpr int kPBytes = kRows * kKeys * 2;  // two [128][64] regions
constexpr int kSmemBytes = 1024 + kQBytes + 2 * 2 * kTileBytes + kPBytes;
constexpr uint32_t kTmemCols = 256;  // S: [0, 128), O: [128, 192)
constexpr float kLog2eP = 1.4426950408889634f;

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

// Byte offset of element (r, c) in a [rows][64] bf16 tile with 128-byte swizzle.
__device__ __forceinline__ uint32_t swz128(int r, int c) {
  return r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full, kv_full[2], s_full, p_full, o_full, mma_done;
  __shared__ uint32_t tmem_base;

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  // Stage st holds K at sK(st) and V right after it.
  auto sK = [&](int st) { return smem + kQBytes + st * 2 * kTileBytes; };
  auto sV = [&](int st) { return smem + kQBytes + st * 2 * kTileBytes + kTileBytes; };
  uint8_t* sP = smem + kQBytes + 4 * kTileBytes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();

  const int H = a.num_heads;
  const int r = blockIdx.x / (H * a.qtiles);
  const int h = (blockIdx.x / a.qtiles) % H;
  const int t0 = (blockIdx.x % a.qtiles) * kRows;
  const int tok0 = __ldg(a.cu_q + r);
  const int n = __ldg(a.cu_q + r + 1) - tok0;
  if (t0 == 0 && tid == 0 && n > a.qtiles * kRows) set_status(a.status, kStatusBadLength);
  if (t0 >= n) return;
  const int ctx = __ldg(a.context_lens + r);
  const int prior = ctx - n;
  const int row_tab = a.seq_rows != nullptr ? __ldg(a.seq_rows + r) : r;
  if (n <= 0 || prior < 0 || row_tab < 0 || row_tab >= a.bt_rows ||
      ctx > a.max_blocks * 16) {
    if (tid == 0) set_status(a.status, row_tab < 0 || row_tab >= a.bt_rows ? kStatusBadRow
                                                                           : kStatusBadLength);
    return;
  }
  const int kv_end = min(ctx, prior + t0 + kRows);  // keys the tile's last row can see
  const int ntiles = (kv_end + kKeys - 1) / kKeys;
  const int kvh = h / a.groups;
  const int32_t* table = a.block_tables + static_cast<int64_t>(row_tab) * a.bt_stride;

  if (tid == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    mbar_init(&s_full, 1);
    mbar_init(&p_full, kRows);
    mbar_init(&o_full, 1);
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
  const uint32_t tS = tmem_base;
  const uint32_t tO = tmem_base + 128;

  constexpr uint32_t kIdescS = umma_idesc(128, 128, 0, 0);
  constexpr uint32_t kIdescO = umma_idesc(128, 64, 0, 1);

  if (warp == 4) {
    // ---------------------------------------------------------------- issuer
    // Loads one KV tile: lanes 0-7 look up their block, lane 0 issues.
    auto load_kv = [&](int j, int st) {
      const int b = j * 8 + (lane & 7);
      int32_t blk = -1;
      if (lane < 8 && b * 16 < kv_end) {
        blk = __ldg(table + b);
        if (blk < 0 || blk >= a.num_blocks) {
          set_status(a.status, kStatusBadBlock);
          blk = -1;
        }
      }
      const uint32_t valid = __ballot_sync(0xffffffffu, blk >= 0) & 0xffu;
      if (lane == 0) mbar_arrive_expect_tx(&kv_full[st], __popc(valid) * 2u * 2048u);
      __syncwarp();
      if (lane < 8 && blk >= 0) {
        const int32_t y = (kvh * a.num_blocks + blk) * 16;
        tma_load_2d(sK(st) + lane * 2048, &kmap, &kv_full[st], 0, y);
        tma_load_2d(sV(st) + lane * 2048, &vmap, &kv_full[st], 0, y);
      }
    };
    auto issue_s = [&](int st) {
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          umma_f16(tS, umma_desc(smem_u32(sQ) + 32 * k, 16, 1024),
                   umma_desc(smem_u32(sK(st)) + 32 * k, 16, 1024), kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full);
      }
      __syncwarp();
    };
    // A wait's outcome is the same for the whole warp (and the warp converged)
    // before any warp-collective instruction follows it.
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
    };
    int loads = 0;  // KV tiles whose loads were issued
    int ready = 0;  // KV tiles whose loads were seen complete
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, kQBytes);
      tma_load_3d(sQ, &qmap, &q_full, 0, h, tok0 + t0);
    }
    load_kv(0, 0);
    loads = 1;
    if (ntiles > 1) {
      load_kv(1, 1);
      loads = 2;
    }
    const bool q_ready = wait_all(&q_full, 0);
    bool ok = q_ready && wait_all(&kv_full[0], 0);
    if (ok) {
      ready = 1;
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < ntiles && ok; ++j) {
      ok = wait_all(&p_full, j & 1);
      if (!ok) break;
      tc_fence_after();
      const int st = j & 1;
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          umma_f16(tO, umma_desc(smem_u32(sP) + (k >> 2) * 16384 + 32 * (k & 3), 16, 1024),
                   umma_desc(smem_u32(sV(st)) + 2048 * k, 16384, 1024), kIdescO,
                   (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&o_full);
      }
      __syncwarp();
      if (j + 1 < ntiles) {
        ok = wait_all(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1);
        if (!ok) break;
        ready = j + 2;
        issue_s((j + 1) & 1);
      }
      if (j + 2 < ntiles) {
        // Stage j & 1 is free once the P V product of tile j has read it.
        ok = wait_all(&o_full, j & 1);
        if (!ok) break;
        load_kv(j + 2, st);
        loads = j + 3;
      }
    }
    // Drain: no MMA may still use TMEM and no TMA load may still write shared
    // memory once the CTA frees them.  The commit tracks every MMA issued above.
    if (lane == 0) umma_commit(&mma_done);
    __syncwarp();
    bool drained = wait_all(&mma_done, 0);
    if (!q_ready) drained = wait_all(&q_full, 0) && drained;
    for (int t = ready; t < loads; ++t) drained = wait_all(&kv_full[t & 1], (t >> 1) & 1) && drained;
    if ((!ok || !drained) && lane == 0) set_status(a.status, kStatusWaitTimeout);
  } else {
    // ---------------------------------------------------------------- softmax
    const int row = tid;  // TMEM lane and query row
    const int qpos = prior + t0 + row;  // position of this row's token
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
    };
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = wait_all(&s_full, j & 1);
      if (!ok) break;
      tc_fence_after();
      float s[kKeys];
#pragma unroll
      for (int c0 = 0; c0 < kKeys; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tS + lane_base + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) s[c0 + c] = __uint_as_float(v[c]);
      }
      float m_tile = -INFINITY;
      const int key0 = j * kKeys;
#pragma unroll
      for (int c = 0; c < kKeys; ++c) {
        const int key = key0 + c;
        float x = round_bf16(round_bf16(s[c]) * a.scale) * kLog2eP;
        x = (key <= qpos && key < ctx) ? x : -INFINITY;
        s[c] = x;
        m_tile = fmaxf(m_tile, x);
      }
      // Key 0 is visible to every row, so m_new is finite from tile 0 on.
      const float m_new = fmaxf(m_run, m_tile);
      const float corr = m_new > m_run ? fast_exp2(m_run - m_new) : 1.f;
      if (j > 0) {
        ok = wait_all(&o_full, (j - 1) & 1);  // P V of the previous tile is done
        if (!ok) break;
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: the warp rescales if any row grew
        // (factor 1 for the others).
        if (__any_sync(0xffffffffu, m_new > m_run)) {
#pragma unroll
          for (int c0 = 0; c0 < kD; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(tO + lane_base + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] = __float_as_uint(__uint_as_float(v[c]) * corr);
            tmem_st32(tO + lane_base + c0, v);
          }
          tmem_wait_st();
        }
      }
      m_run = m_new;
      float psum = 0.f;
      uint8_t* prow = sP;
#pragma unroll
      for (int ch = 0; ch < kKeys / 8; ++ch) {  // 16-byte chunks of the P row
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = fast_exp2(s[ch * 8 + e] - m_new);
          psum += p[e];
        }
        uint4 w;
        w.x = pack_bf16x2(p[0], p[1]);
        w.y = pack_bf16x2(p[2], p[3]);
        w.z = pack_bf16x2(p[4], p[5]);
        w.w = pack_bf16x2(p[6], p[7]);
        const int col = (ch & 7) * 8;
        *reinterpret_cast<uint4*>(prow + (ch >> 3) * 16384 + swz128(row, col)) = w;
      }
      l_run = l_run * corr + psum;
      // Keys no row of this CTA sees (past the context, or past the last row's
      // position): their V rows hold stale pool data or never-loaded shared
      // memory, possibly NaN, which would poison 0 * V in the tensor core.
      if (key0 + row >= kv_end) {
        uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(sV(j & 1) + row * 128 + c * 16) = z;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full);
    }
    if (ok) ok = wait_all(&o_full, (ntiles - 1) & 1);
    if (ok) {
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
        tmem_ld32(tO + lane_base + c0, v);
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tS),
                 "r"(kTmemCols));
  }
}

}  // namespace

int prefill_smem_bytes() { return kSmemBytes; }

int launch_prefill_tc(const PrefillArgs& a, const CUtensorMap& qmap, const CUtensorMap& kmap,
                      const CUtensorMap& vmap, int grid, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
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
