// Fused elementwise steps of the model around the attention path.  Each
// replaces a chain of small framework ops of the reference's TorchModel
// (src/server/torch_model.py) with one launch, keeping its rounding points:
//
//   rms_norm    (:283-287)  weight * (s_f32 * rsqrt(mean(s_f32^2) + eps)).to(T)
//               with s = T(x + add), the residual add before it (:272, :281),
//               optionally over gathered rows (the embedding lookup, :234,
//               or the last token of each sequence, :228)
//   rope_append (:262-264, :190-192, :149-153 / 289-292)
//               q' = T(T(q * cos) + T(rotate_half(q) * sin)), the same for k;
//               q' to the attention input, k' and v into their pool slots
//   silu_mul    (:278-281)  T(T(silu(gate)) * up)
//   argmax_rows (backend/paged.py:95-99) greedy token of each logits row
//
// T is the model dtype (bf16, or fp32 where the roundings vanish); cos/sin are
// the bf16-rounded rotary tables gathered by position.  All are bandwidth-bound
// and tiny per step; their value is the launches they remove.
#include "common.cuh"

namespace bsb {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ T st(float x);
template <>
__device__ __forceinline__ float st<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 st<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
// The value a T-typed framework op would produce: rounded to T.
template <typename T>
__device__ __forceinline__ float rt(float x);
template <>
__device__ __forceinline__ float rt<float>(float x) { return x; }
template <>
__device__ __forceinline__ float rt<__nv_bfloat16>(float x) { return round_bf16(x); }

// Rounds 8 values to T as separate T-typed ops would (packed conversions for
// bf16).
template <typename T>
__device__ __forceinline__ void round8(float (&v)[8]);
template <>
__device__ __forceinline__ void round8<float>(float (&)[8]) {}
template <>
__device__ __forceinline__ void round8<__nv_bfloat16>(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; j += 2) round_bf16x2(v[j], v[j + 1]);
}

// One warp per output row r, reading source row i = index ? index[r] : r:
// s = T(x[i] + add[i]) (s = x[i] without add), sum_out[r] = s, out[r] =
// RMSNorm(s).  sum_out may be x itself (the residual stream updated in place:
// every element is read and written by the same lane) when index is null.
// VEC: 8 elements per access (hidden and every row stride a multiple of 8,
// 16-byte aligned rows).
constexpr int kNormRowsPerCta = 4;
// Rows up to kNormChunks x 256 elements (8 per lane and chunk) stay in registers.
constexpr int kNormChunks = 4;

template <typename T, bool VEC>
__global__ void __launch_bounds__(32 * kNormRowsPerCta)
    rms_norm_kernel(const T* x, int64_t x_stride, const T* __restrict__ add, int64_t add_stride,
                    const int32_t* __restrict__ index, int32_t x_rows, const T* __restrict__ w,
                    int32_t rows, int32_t hidden, float eps, T* __restrict__ out,
                    int64_t out_stride, T* sum_out, int64_t sum_stride, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int32_t r = blockIdx.x * kNormRowsPerCta + (threadIdx.x >> 5);
  if (r >= rows) return;
  int64_t src = r;
  if (index != nullptr) {
    src = index[r];
    if (src < 0 || src >= x_rows) {
      if (lane == 0) set_status(status, kStatusBadIndex);
      return;
    }
  }
  const T* row = x + src * x_stride;
  const T* arow = add != nullptr ? add + src * add_stride : nullptr;
  T* srow = sum_out != nullptr ? sum_out + static_cast<int64_t>(r) * sum_stride : nullptr;
  T* orow = out + static_cast<int64_t>(r) * out_stride;
  float ss = 0.f;
  if constexpr (VEC) {
    if (hidden <= kNormChunks * 256) {
      // The whole row in registers, every load issued before the first use
      // (one round trip instead of one per chunk and pass); same arithmetic
      // in the same order as the loops below.
      float v[kNormChunks][8], a[kNormChunks][8], wt[kNormChunks][8];
#pragma unroll
      for (int k = 0; k < kNormChunks; ++k) {
        const int32_t i = lane * 8 + k * 256;
        if (i < hidden) {
          load8(row + i, v[k]);
          if (arow != nullptr) load8(arow + i, a[k]);
          load8(w + i, wt[k]);
        }
      }
#pragma unroll
      for (int k = 0; k < kNormChunks; ++k) {
        const int32_t i = lane * 8 + k * 256;
        if (i < hidden) {
          if (arow != nullptr) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[k][j] = __fadd_rn(v[k][j], a[k][j]);
            round8<T>(v[k]);
          }
          if (srow != nullptr) store8(srow + i, v[k]);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss = fmaf(v[k][j], v[k][j], ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(ss / static_cast<float>(hidden) + eps);
#pragma unroll
      for (int k = 0; k < kNormChunks; ++k) {
        const int32_t i = lane * 8 + k * 256;
        if (i < hidden) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[k][j] = __fmul_rn(v[k][j], inv);
          round8<T>(v[k]);  // normalized.to(T)
#pragma unroll
          for (int j = 0; j < 8; ++j) v[k][j] = __fmul_rn(wt[k][j], v[k][j]);
          store8(orow + i, v[k]);
        }
      }
      return;
    }
    for (int32_t i = lane * 8; i < hidden; i += 256) {
      float v[8];
      load8(row + i, v);
      if (arow != nullptr) {
        float a[8];
        load8(arow + i, a);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], a[j]);
        round8<T>(v);
      }
      if (srow != nullptr) store8(srow + i, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    }
  } else {
    for (int32_t i = lane; i < hidden; i += 32) {
      float v = ld<T>(row + i);
      if (arow != nullptr) v = rt<T>(__fadd_rn(v, ld<T>(arow + i)));
      if (srow != nullptr) srow[i] = st<T>(v);
      ss = fmaf(v, v, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(hidden) + eps);
  // Second pass over this lane's own elements of s (re-read, or recomputed).
  if constexpr (VEC) {
    for (int32_t i = lane * 8; i < hidden; i += 256) {
      float v[8], wt[8];
      if (srow != nullptr) {
        load8(srow + i, v);
      } else {
        load8(row + i, v);
        if (arow != nullptr) {
          float a[8];
          load8(arow + i, a);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], a[j]);
          round8<T>(v);
        }
      }
      load8(w + i, wt);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(v[j], inv);
      round8<T>(v);  // normalized.to(T)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(wt[j], v[j]);
      store8(orow + i, v);
    }
  } else {
    for (int32_t i = lane; i < hidden; i += 32) {
      float v = srow != nullptr ? ld<T>(srow + i) : ld<T>(row + i);
      if (srow == nullptr && arow != nullptr) v = rt<T>(__fadd_rn(v, ld<T>(arow + i)));
      const float normalized = rt<T>(__fmul_rn(v, inv));
      orow[i] = st<T>(__fmul_rn(ld<T>(w + i), normalized));
    }
  }
}

// One thread per (token, head, dim pair d, d + D/2) of q and k; v is copied.
// qkv rows: [H*D | Hkv*D | Hkv*D].  A negative slot skips the pool write (a
// padding row); a slot past the pool or a position outside [0, num_pos) skips
// the access and sets a status bit.  Grid: x over a token's pairs, y over
// tokens.
template <typename T, typename Tpool>
__global__ void __launch_bounds__(128)
    rope_append_kernel(const T* __restrict__ qkv, int64_t qkv_stride,
                       const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                       int32_t num_pos, const int32_t* __restrict__ pos,
                       const int32_t* __restrict__ slots, int32_t ntok, int32_t H, int32_t Hkv,
                       int32_t D, T* __restrict__ q_out, Tpool* __restrict__ k_pool,
                       Tpool* __restrict__ v_pool, int64_t pool_slots, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int32_t half = D >> 1;
  const int32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= (H + 2 * Hkv) * half) return;
  const int32_t hh = r / half, d = r - hh * half;  // head in [0, H + 2 Hkv)
  for (int32_t t = blockIdx.y; t < ntok; t += gridDim.y) {
    const T* row = qkv + t * qkv_stride + hh * D;
    const float a = ld<T>(row + d), b = ld<T>(row + d + half);
    const int32_t slot = hh >= H ? slots[t] : -1;
    if (slot >= pool_slots) {
      if (d == 0) set_status(status, kStatusBadSlot);
      continue;
    }
    if (hh >= H + Hkv) {  // v: copied into its slot
      if (slot >= 0) {
        Tpool* dst = v_pool + (static_cast<int64_t>(hh - H - Hkv) * pool_slots + slot) * D;
        dst[d] = st<Tpool>(a);
        dst[d + half] = st<Tpool>(b);
      }
      continue;
    }
    const int32_t p = pos[t];
    if (p < 0 || p >= num_pos) {
      if (d == 0 && hh == 0) set_status(status, kStatusBadPosition);
      continue;
    }
    const float c0 = ld<T>(cos_t + static_cast<int64_t>(p) * D + d);
    const float c1 = ld<T>(cos_t + static_cast<int64_t>(p) * D + d + half);
    const float s0 = ld<T>(sin_t + static_cast<int64_t>(p) * D + d);
    const float s1 = ld<T>(sin_t + static_cast<int64_t>(p) * D + d + half);
    // rotate_half(x) = cat(-x2, x1): element d takes -b, element d + half takes a.
    const float lo = rt<T>(__fadd_rn(rt<T>(__fmul_rn(a, c0)), rt<T>(__fmul_rn(-b, s0))));
    const float hi = rt<T>(__fadd_rn(rt<T>(__fmul_rn(b, c1)), rt<T>(__fmul_rn(a, s1))));
    if (hh < H) {
      T* dst = q_out + (static_cast<int64_t>(t) * H + hh) * D;
      dst[d] = st<T>(lo);
      dst[d + half] = st<T>(hi);
    } else if (slot >= 0) {
      Tpool* dst = k_pool + (static_cast<int64_t>(hh - H) * pool_slots + slot) * D;
      dst[d] = st<Tpool>(lo);
      dst[d + half] = st<Tpool>(hi);
    }
  }
}

// rope_append_kernel for bf16 rows and pools with 16-byte accesses: one thread
// per (token, head, 8-dim chunk of the head's first half), which also rotates
// the partner dims half a head away; the per-element arithmetic is the scalar
// kernel's.  Needs D a multiple of 16 and every row 16-byte aligned.
__global__ void __launch_bounds__(128)
    rope_append_vec_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride,
                           const __nv_bfloat16* __restrict__ cos_t,
                           const __nv_bfloat16* __restrict__ sin_t, int32_t num_pos,
                           const int32_t* __restrict__ pos, const int32_t* __restrict__ slots,
                           int32_t ntok, int32_t H, int32_t Hkv, int32_t D,
                           __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_pool,
                           __nv_bfloat16* __restrict__ v_pool, int64_t pool_slots,
                           uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int32_t half = D >> 1, chunks = half >> 3;
  const int32_t per_tok = (H + 2 * Hkv) * chunks;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(ntok) * per_tok) return;
  const int32_t t = static_cast<int32_t>(idx / per_tok);
  const int32_t rem = static_cast<int32_t>(idx - static_cast<int64_t>(t) * per_tok);
  const int32_t hh = rem / chunks, d = (rem - hh * chunks) * 8;
  const __nv_bfloat16* row = qkv + t * qkv_stride + hh * D;
  float a[8], b[8];
  load8(row + d, a);
  load8(row + d + half, b);
  const int32_t slot = hh >= H ? slots[t] : -1;
  if (slot >= pool_slots) {
    if (d == 0) set_status(status, kStatusBadSlot);
    return;
  }
  if (hh >= H + Hkv) {  // v: copied into its slot
    if (slot >= 0) {
      __nv_bfloat16* dst = v_pool + (static_cast<int64_t>(hh - H - Hkv) * pool_slots + slot) * D;
      store8(dst + d, a);
      store8(dst + d + half, b);
    }
    return;
  }
  const int32_t p = pos[t];
  if (p < 0 || p >= num_pos) {
    if (d == 0 && hh == 0) set_status(status, kStatusBadPosition);
    return;
  }
  float c0[8], c1[8], s0[8], s1[8];
  const int64_t prow = static_cast<int64_t>(p) * D;
  load8(cos_t + prow + d, c0);
  load8(cos_t + prow + d + half, c1);
  load8(sin_t + prow + d, s0);
  load8(sin_t + prow + d + half, s1);
  float lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    lo[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(a[j], c0[j])),
                                 round_bf16(__fmul_rn(-b[j], s0[j]))));
    hi[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(b[j], c1[j])),
                                 round_bf16(__fmul_rn(a[j], s1[j]))));
  }
  __nv_bfloat16* dst = nullptr;
  if (hh < H) {
    dst = q_out + (static_cast<int64_t>(t) * H + hh) * D;
  } else if (slot >= 0) {
    dst = k_pool + (static_cast<int64_t>(hh - H) * pool_slots + slot) * D;
  }
  if (dst != nullptr) {
    store8(dst + d, lo);
    store8(dst + d + half, hi);
  }
}

// Rows [gate | up] -> silu(gate) * up.  Grid: x over a row's elements (8 per
// thread when VEC: intermediate and the row stride multiples of 8, 16-byte
// aligned rows), y over tokens.
template <typename T, bool VEC>
__global__ void __launch_bounds__(128)
    silu_mul_kernel(const T* __restrict__ gate_up, int64_t stride, int32_t ntok, int32_t inter,
                    T* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * (VEC ? 8 : 1);
  if (c >= inter) return;
  for (int32_t t = blockIdx.y; t < ntok; t += gridDim.y) {
    const T* g = gate_up + t * stride + c;
    T* o = out + static_cast<int64_t>(t) * inter + c;
    if constexpr (VEC) {
      float gv[8], uv[8];
      load8(g, gv);
      load8(g + inter, uv);
#pragma unroll
      for (int j = 0; j < 8; ++j) gv[j] = __fdiv_rn(gv[j], __fadd_rn(1.0f, expf(-gv[j])));
      round8<T>(gv);  // silu(gate) in T
#pragma unroll
      for (int j = 0; j < 8; ++j) gv[j] = __fmul_rn(gv[j], uv[j]);
      store8(o, gv);
    } else {
      const float gs = ld<T>(g), u = ld<T>(g + inter);
      const float s = rt<T>(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))));
      *o = st<T>(__fmul_rn(s, u));
    }
  }
}

// Greedy argmax of each row (the first index of the maximum; a NaN counts as
// larger than any number, as torch.argmax has it): one CTA per row, 8 elements
// per 16-byte load when VEC, then a warp and a block reduction of (value, index).
constexpr int kArgmaxThreads = 512;

__device__ __forceinline__ bool argmax_better(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;  // NaN wins over numbers
  if (!vn && v != bv) return v > bv;
  return i < bi;  // equal (or both NaN): the first index
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_rows_kernel(const T* __restrict__ x, int64_t stride, int64_t cols,
                       int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const T* row = x + static_cast<int64_t>(blockIdx.x) * stride;
  float best = -INFINITY;
  int64_t bi = cols;  // past every index: loses all ties
  if constexpr (VEC) {
    for (int64_t c = threadIdx.x * 8; c < cols; c += kArgmaxThreads * 8) {
      float v[8];
      load8(row + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (argmax_better(v[j], c + j, best, bi)) {
          best = v[j];
          bi = c + j;
        }
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += kArgmaxThreads) {
      const float v = ld<T>(row + c);
      if (argmax_better(v, c, best, bi)) {
        best = v;
        bi = c;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float wv[kArgmaxThreads / 32];
  __shared__ int64_t wi[kArgmaxThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    wv[warp] = best;
    wi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w) {
      if (argmax_better(wv[w], wi[w], best, bi)) {
        best = wv[w];
        bi = wi[w];
      }
    }
    out[blockIdx.x] = static_cast<int32_t>(bi);
  }
}

cudaLaunchConfig_t cfg_of(dim3 grid, int threads, cudaStream_t stream,
                          cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

constexpr int32_t kMaxGridY = 65535;

}  // namespace

int launch_rms_norm(const void* x, int64_t x_stride, const void* add, int64_t add_stride,
                    const int32_t* index, int32_t x_rows, const void* w, int32_t rows,
                    int32_t hidden, float eps, void* out, int64_t out_stride, void* sum_out,
                    int64_t sum_stride, bool bf16, bool vec, uint32_t* status,
                    cudaStream_t stream) {
  if (rows == 0) return 0;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3((rows + kNormRowsPerCta - 1) / kNormRowsPerCta),
                                  32 * kNormRowsPerCta, stream, attr);
#define BS_RMS(T, V)                                                                            \
  return static_cast<int>(cudaLaunchKernelEx(                                                   \
      &cfg, rms_norm_kernel<T, V>, static_cast<const T*>(x), x_stride,                          \
      static_cast<const T*>(add), add_stride, index, x_rows, static_cast<const T*>(w), rows,    \
      hidden, eps, static_cast<T*>(out), out_stride, static_cast<T*>(sum_out), sum_stride,      \
      status))
  if (bf16) {
    if (vec) BS_RMS(__nv_bfloat16, true);
    BS_RMS(__nv_bfloat16, false);
  }
  if (vec) BS_RMS(float, true);
  BS_RMS(float, false);
#undef BS_RMS
}

int launch_rope_append(const void* qkv, int64_t qkv_stride, const void* cos_t, const void* sin_t,
                       int32_t num_pos, const int32_t* pos, const int32_t* slots, int32_t ntok,
                       int32_t H, int32_t Hkv, int32_t D, void* q_out, void* k_pool,
                       void* v_pool, int64_t pool_slots, bool bf16, bool pool_bf16, int sms,
                       uint32_t* status, cudaStream_t stream) {
  (void)sms;
  if (ntok == 0) return 0;
  const int32_t pairs = (H + 2 * Hkv) * (D / 2);
  cudaLaunchAttribute attr[1];
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (bf16 && pool_bf16 && D % 16 == 0 && qkv_stride % 8 == 0 && a16(qkv) && a16(cos_t) &&
      a16(sin_t) && a16(q_out) && a16(k_pool) && a16(v_pool)) {
    const int64_t threads = static_cast<int64_t>(ntok) * (H + 2 * Hkv) * (D / 16);
    cudaLaunchConfig_t cfg = cfg_of(dim3(static_cast<unsigned>((threads + 127) / 128)), 128,
                                    stream, attr);
    return static_cast<int>(cudaLaunchKernelEx(
        &cfg, rope_append_vec_kernel, static_cast<const __nv_bfloat16*>(qkv), qkv_stride,
        static_cast<const __nv_bfloat16*>(cos_t), static_cast<const __nv_bfloat16*>(sin_t),
        num_pos, pos, slots, ntok, H, Hkv, D, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(k_pool), static_cast<__nv_bfloat16*>(v_pool), pool_slots,
        status));
  }
  cudaLaunchConfig_t cfg =
      cfg_of(dim3((pairs + 127) / 128, ntok < kMaxGridY ? ntok : kMaxGridY), 128, stream, attr);
#define BS_ROPE(T, TP)                                                                          \
  return static_cast<int>(cudaLaunchKernelEx(                                                   \
      &cfg, rope_append_kernel<T, TP>, static_cast<const T*>(qkv), qkv_stride,                  \
      static_cast<const T*>(cos_t), static_cast<const T*>(sin_t), num_pos, pos, slots, ntok, H, \
      Hkv, D, static_cast<T*>(q_out), static_cast<TP*>(k_pool), static_cast<TP*>(v_pool),      \
      pool_slots, status))
  if (bf16 && pool_bf16) BS_ROPE(__nv_bfloat16, __nv_bfloat16);
  if (bf16) BS_ROPE(__nv_bfloat16, float);
  if (pool_bf16) BS_ROPE(float, __nv_bfloat16);
  BS_ROPE(float, float);
#undef BS_ROPE
}

int launch_silu_mul(const void* gate_up, int64_t stride, int32_t ntok, int32_t inter, void* out,
                    bool bf16, bool vec, int sms, cudaStream_t stream) {
  (void)sms;
  if (ntok == 0) return 0;
  const int32_t per_thread = vec ? 8 : 1;
  const int32_t threads = (inter + per_thread - 1) / per_thread;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      cfg_of(dim3((threads + 127) / 128, ntok < kMaxGridY ? ntok : kMaxGridY), 128, stream, attr);
#define BS_SILU(T, V)                                                                           \
  return static_cast<int>(cudaLaunchKernelEx(&cfg, silu_mul_kernel<T, V>,                       \
                                             static_cast<const T*>(gate_up), stride, ntok, inter, \
                                             static_cast<T*>(out)))
  if (bf16) {
    if (vec) BS_SILU(__nv_bfloat16, true);
    BS_SILU(__nv_bfloat16, false);
  }
  if (vec) BS_SILU(float, true);
  BS_SILU(float, false);
#undef BS_SILU
}

int launch_argmax_rows(const void* x, int64_t stride, int32_t rows, int64_t cols, void* out,
                       bool bf16, bool vec, cudaStream_t stream) {
  if (rows == 0) return 0;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(rows), kArgmaxThreads, stream, attr);
#define BS_ARGMAX(T, V)                                                                         \
  return static_cast<int>(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<T, V>,                    \
                                             static_cast<const T*>(x), stride, cols,            \
                                             static_cast<int32_t*>(out)))
  if (bf16) {
    if (vec) BS_ARGMAX(__nv_bfloat16, true);
    BS_ARGMAX(__nv_bfloat16, false);
  }
  if (vec) BS_ARGMAX(float, true);
  BS_ARGMAX(float, false);
#undef BS_ARGMAX
}

}  // namespace bsb
