// SIMT split-K decode attention: every dtype (bf16 or fp32 pools) and shape the
// tensor-core kernel does not cover (any block size, head_dim <= 256, up to 16
// query heads per kv head).  It is the path for the fp32 pool of the engine and
// for the small shapes of the reference's unit tests.
//
// Same stream-K span and merge as the tensor-core kernel (decode.cuh).  Inside a
// span each of the 4 warps takes groups of 32 consecutive tokens; lane j owns
// token j of its group for the scores (full-length dot products against the query
// rows held in shared memory), the group's softmax statistics come from warp
// reductions, and the weighted V sum is spread over lanes by head dimension.
#include "decode.cuh"

namespace bsb {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Score of one token for the reference rounding of its dtype.
template <typename T>
__device__ __forceinline__ float finish_score(float dot, float scale);
template <>
__device__ __forceinline__ float finish_score<float>(float dot, float scale) {
  return dot * scale;
}
template <>
__device__ __forceinline__ float finish_score<__nv_bfloat16>(float dot, float scale) {
  return round_bf16(round_bf16(dot) * scale);
}

// The probability that weights V: bf16 pools round it, as the reference does.
template <typename T>
__device__ __forceinline__ float weight_of(float p);
template <>
__device__ __forceinline__ float weight_of<float>(float p) {
  return p;
}
template <>
__device__ __forceinline__ float weight_of<__nv_bfloat16>(float p) {
  return round_bf16(p);
}

// DPL: head dims per lane (ceil(D / 32)); GM: register rows for query heads.
template <typename T, int DPL, int GM>
__global__ void __launch_bounds__(kThreads) decode_simt_kernel(const DecodeArgs a) {
  __shared__ ScanSmem scan;
  __shared__ int32_t s_flag;
  extern __shared__ float dsm[];  // sQ [G*D] | sO [warps*G*D] | sM [warps*G] | sL [warps*G]

  pdl_wait();
  const Span sp = compute_span(a, scan);
  if (sp.r0 >= sp.r1) return;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.groups, D = a.head_dim, bs = a.block_size;
  float* sQ = dsm;
  float* sO = sQ + G * D;
  float* sM = sO + kWarps * G * D;
  float* sL = sM + kWarps * G;
  const int64_t Hkv = a.num_kv_heads;
  const int64_t head_stride = static_cast<int64_t>(a.num_blocks) * bs * D;  // per kv head
  const T* kpool = static_cast<const T*>(a.k_pool);
  const T* vpool = static_cast<const T*>(a.v_pool);

  int32_t i = sp.seq;
  int64_t prefix = sp.prefix;
  int32_t len, row;
  int32_t nb = seq_units(a, i, len, row, false);
  const int64_t rel = sp.r0 - prefix * Hkv;
  int32_t h = static_cast<int32_t>(rel / nb);
  int32_t off = static_cast<int32_t>(rel % nb);
  int64_t u = sp.r0;

  while (u < sp.r1) {
    const int64_t left = sp.r1 - u;
    const int32_t take = (nb - off < left) ? (nb - off) : static_cast<int32_t>(left);
    Portion po;
    po.seq = i;
    po.kvh = h;
    po.whole = (off == 0 && take == nb) ? 1 : 0;
    po.seg_unit = prefix * Hkv + static_cast<int64_t>(h) * nb;
    po.nb = nb;

    // Query rows of the group -> shared memory (fp32).
    const T* qrow = static_cast<const T*>(a.q) + static_cast<int64_t>(i) * a.q_stride_seq +
                    static_cast<int64_t>(h) * G * D;
    for (int e = tid; e < G * D; e += kThreads) sQ[e] = to_f<T>(qrow[e]);
    __syncthreads();

    const int32_t* table = a.block_tables + static_cast<int64_t>(row) * a.bt_stride;
    const T* kh = kpool + h * head_stride;
    const T* vh = vpool + h * head_stride;
    const int tok_begin = off * bs;
    const int tok_end = min(len, (off + take) * bs);

    float m[GM], l[GM], o[GM][DPL];
#pragma unroll
    for (int r = 0; r < GM; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[r][k] = 0.f;
    }

    for (int base = tok_begin + warp * 32; base < tok_end; base += kWarps * 32) {
      const int tok = base + lane;
      const bool live = tok < tok_end;
      int64_t rowoff = 0;
      if (live) {
        const int32_t blk = __ldg(table + tok / bs);
        if (blk >= 0 && blk < a.num_blocks) {
          rowoff = (static_cast<int64_t>(blk) * bs + tok % bs) * D;
        } else {
          set_status(a.status, kStatusBadBlock);
        }
      }
      // Scores of this lane's token for every head of the group.
      float s[GM];
#pragma unroll
      for (int r = 0; r < GM; ++r) s[r] = 0.f;
      if (live) {
        const T* krow = kh + rowoff;
        for (int d = 0; d < D; ++d) {
          const float kv = to_f<T>(krow[d]);
#pragma unroll
          for (int r = 0; r < GM; ++r) {
            if (r < G) s[r] = fmaf(sQ[r * D + d], kv, s[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < GM; ++r) {
        if (r >= G) continue;
        const float v = live ? finish_score<T>(s[r], a.scale) * kLog2e : -INFINITY;
        float mx = v;
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
        const float mnew = fmaxf(m[r], mx);
        const float corr = fast_exp2(m[r] - mnew);
        m[r] = mnew;
        const float p = fast_exp2(v - mnew);
        l[r] = l[r] * corr + p;  // lane-local partial sum
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[r][k] *= corr;
        s[r] = p;
      }
      // Weighted V rows: token j's probability is broadcast from lane j.
      const int ntok = min(32, tok_end - base);
      for (int j = 0; j < ntok; ++j) {
        const int64_t vo = __shfl_sync(0xffffffffu, rowoff, j);
        const T* vrow = vh + vo;
        float vv[DPL];
#pragma unroll
        for (int k = 0; k < DPL; ++k) {
          const int d = lane + 32 * k;
          vv[k] = (d < D) ? to_f<T>(vrow[d]) : 0.f;
        }
#pragma unroll
        for (int r = 0; r < GM; ++r) {
          if (r >= G) continue;
          const float w = weight_of<T>(__shfl_sync(0xffffffffu, s[r], j));
#pragma unroll
          for (int k = 0; k < DPL; ++k) o[r][k] = fmaf(w, vv[k], o[r][k]);
        }
      }
    }
    // Deposit per-warp state: layout [warp][r][d] with d = lane + 32k.
#pragma unroll
    for (int r = 0; r < GM; ++r) {
      if (r >= G) continue;
      float lr = l[r];
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) lr += __shfl_xor_sync(0xffffffffu, lr, o2);
      if (lane == 0) {
        sM[warp * G + r] = m[r];
        sL[warp * G + r] = lr;
      }
#pragma unroll
      for (int k = 0; k < DPL; ++k) {
        const int d = lane + 32 * k;
        if (d < D) sO[(warp * G + r) * D + d] = o[r][k];
      }
    }
    named_barrier_sync(1, kThreads);
    emit_portion<kWarps, T>(a, sp, po, sO, sM, sL, tid, &s_flag, 1);

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
}

using KernelFn = void (*)(const DecodeArgs);

template <typename T, int GM>
KernelFn pick_g(int head_dim) {
  const int dpl = (head_dim + 31) / 32;
  if (dpl <= 1) return decode_simt_kernel<T, 1, GM>;
  if (dpl <= 2) return decode_simt_kernel<T, 2, GM>;
  if (dpl <= 4) return decode_simt_kernel<T, 4, GM>;
  return decode_simt_kernel<T, 8, GM>;
}

KernelFn pick(int head_dim, int groups, int bf16) {
  if (bf16) return groups <= 8 ? pick_g<__nv_bfloat16, 8>(head_dim) : pick_g<__nv_bfloat16, 16>(head_dim);
  return groups <= 8 ? pick_g<float, 8>(head_dim) : pick_g<float, 16>(head_dim);
}

size_t smem_bytes(int head_dim, int groups) {
  return static_cast<size_t>(5 * groups * head_dim + 2 * kWarps * groups) * sizeof(float);
}

int prepare(KernelFn fn, size_t smem) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

}  // namespace

int launch_decode_simt(const DecodeArgs& a, int dtype_is_bf16, int grid, cudaStream_t stream) {
  KernelFn fn = pick(a.head_dim, a.groups, dtype_is_bf16);
  const size_t smem = smem_bytes(a.head_dim, a.groups);
  if (int e = prepare(fn, smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, fn, a));
}

int decode_simt_ctas_per_sm(int head_dim, int groups, int dtype_is_bf16) {
  KernelFn fn = pick(head_dim, groups, dtype_is_bf16);
  const size_t smem = smem_bytes(head_dim, groups);
  if (int e = prepare(fn, smem)) return -e;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem);
  if (e != cudaSuccess) return -static_cast<int>(e);
  return n;
}

}  // namespace bsb
