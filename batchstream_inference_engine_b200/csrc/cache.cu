// Paged-KV bookkeeping kernels: the per-step metadata builder and the K/V slot
// write.
//
// Metadata.  The reference assembles every step on the host: positions per
// sequence (src/server/torch_model.py:234-236), the flat-batch slices (:239) and,
// per token, (block, offset) = BlockAllocator.locate (src/server/block_allocator.py:28-30),
// which PagedKVCache.append turns into one indexed store per token (torch_model.py:149-153).
// Here the block tables live on the device and one launch derives, for a ragged
// batch of R rows with n_new[r] new tokens each:
//     cu_q[r]      = sum_{j<r} n_new[j]                     (R + 1 entries)
//     positions[t] = start_pos[r] + (t - cu_q[r])
//     slots[t]     = table[row][pos / bs] * bs + pos % bs    (locate, flattened)
//     context[r]   = start_pos[r] + n_new[r]
// bit-exact with the reference allocator's locate().
//
// Decode append (one new token per row) fuses both for decode steps.
//
// Slot write.  k/v rows [T, Hkv, D] (any token stride) land at
// pool[h, slot / bs, slot % bs, :] with 16-byte vector loads and stores; an fp32
// input into a bf16 pool is rounded to nearest-even, as torch's indexed
// assignment into a bf16 tensor does.  Negative slots are padding and skipped.
#include "common.cuh"

namespace bsb {
namespace {

cudaLaunchConfig_t pdl_config(int grid, int threads, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  return cfg;
}

// Programmatic stream serialization: the kernel may launch before the previous
// one on the stream finishes; it calls pdl_wait() before reading any input.
void pdl_attr(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
}

constexpr int kMetaThreads = 256;
constexpr int kMaxMetaRows = 8192;

__global__ void __launch_bounds__(kMetaThreads)
    step_metadata_kernel(const int32_t* __restrict__ seq_rows, const int32_t* __restrict__ start_pos,
                         const int32_t* __restrict__ n_new, int32_t R,
                         const int32_t* __restrict__ block_tables, int64_t bt_stride,
                         int32_t bt_rows, int32_t max_blocks, int32_t block_size,
                         int32_t num_blocks, int32_t T, int32_t* __restrict__ cu_q,
                         int32_t* __restrict__ positions, int32_t* __restrict__ slots,
                         int32_t* __restrict__ context_lens, uint32_t* status) {
  __shared__ int32_t cu[kMaxMetaRows + 1];
  __shared__ int32_t warp_tot[kMetaThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();
  pdl_wait();

  // Block-wide exclusive scan of n_new in chunks of kMetaThreads.
  int32_t carry = 0;
  for (int32_t base = 0; base < R; base += kMetaThreads) {
    const int32_t r = base + tid;
    const int32_t v = (r < R) ? max(0, n_new[r]) : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int32_t before = carry, total = 0;
    for (int w = 0; w < kMetaThreads / 32; ++w) {
      if (w < warp) before += warp_tot[w];
      total += warp_tot[w];
    }
    if (r < R) cu[r] = before + incl - v;
    __syncthreads();
    carry += total;
  }
  if (tid == 0) cu[R] = carry;
  __syncthreads();

  if (blockIdx.x == 0) {
    for (int32_t r = tid; r <= R; r += kMetaThreads) cu_q[r] = cu[r];
    for (int32_t r = tid; r < R; r += kMetaThreads) {
      context_lens[r] = start_pos[r] < 0 ? 0 : start_pos[r] + max(0, n_new[r]);
    }
  }

  const int32_t t = blockIdx.x * kMetaThreads + tid;
  if (t >= T) return;
  if (t >= cu[R]) {  // more tokens requested than rows provide
    positions[t] = 0;
    slots[t] = -1;
    return;
  }
  // Last row r with cu[r] <= t (rows with n_new == 0 are skipped by '<=').
  int32_t lo = 0, hi = R - 1;
  while (lo < hi) {
    const int32_t mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int32_t r = lo;
  if (start_pos[r] < 0) {  // padding row: its tokens read and write nothing
    positions[t] = 0;
    slots[t] = -1;
    return;
  }
  const int32_t pos = start_pos[r] + (t - cu[r]);
  positions[t] = pos;
  const int32_t row = seq_rows != nullptr ? seq_rows[r] : r;
  const int32_t bi = pos / block_size;
  if (row < 0 || row >= bt_rows || pos < 0 || bi >= max_blocks) {
    set_status(status, row < 0 || row >= bt_rows ? kStatusBadRow : kStatusBadLength);
    slots[t] = -1;
    return;
  }
  const int32_t blk = block_tables[static_cast<int64_t>(row) * bt_stride + bi];
  if (blk < 0 || blk >= num_blocks) {
    set_status(status, kStatusBadBlock);
    slots[t] = -1;
    return;
  }
  slots[t] = blk * block_size + pos % block_size;
}

// bf16 -> bf16 keeps the raw bits (no float round trip needed, but it is exact).
template <typename Tin, typename Tpool>
__global__ void __launch_bounds__(256)
    slot_write_vec_kernel(const Tin* __restrict__ k, const Tin* __restrict__ v, int64_t k_stride,
                          int64_t v_stride, const int32_t* __restrict__ slots, int32_t T,
                          int32_t Hkv, int32_t D, Tpool* __restrict__ k_pool,
                          Tpool* __restrict__ v_pool, int64_t pool_slots, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int32_t vecs = D >> 3;
  const int64_t per_tensor = static_cast<int64_t>(T) * Hkv * vecs;
  const int64_t total = 2 * per_tensor;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const bool is_v = idx >= per_tensor;
    const int64_t e = is_v ? idx - per_tensor : idx;
    const int32_t j = static_cast<int32_t>(e % vecs);
    const int64_t th = e / vecs;
    const int32_t h = static_cast<int32_t>(th % Hkv);
    const int32_t t = static_cast<int32_t>(th / Hkv);
    const int32_t slot = __ldg(slots + t);
    if (slot < 0) continue;
    if (slot >= pool_slots) {
      set_status(status, kStatusBadSlot);
      continue;
    }
    const Tin* src = (is_v ? v + t * v_stride : k + t * k_stride) + h * D + 8 * j;
    Tpool* dst = (is_v ? v_pool : k_pool) + (h * pool_slots + slot) * D + 8 * j;
    float x[8];
    load8(src, x);
    store8(dst, x);
  }
}

template <typename T>
__device__ __forceinline__ float as_float(T x);
template <>
__device__ __forceinline__ float as_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ float as_float<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// One element per thread, for head sizes that are not a multiple of 8.
template <typename Tin, typename Tpool>
__global__ void __launch_bounds__(256)
    slot_write_scalar_kernel(const Tin* __restrict__ k, const Tin* __restrict__ v, int64_t k_stride,
                             int64_t v_stride, const int32_t* __restrict__ slots, int32_t T,
                             int32_t Hkv, int32_t D, Tpool* __restrict__ k_pool,
                             Tpool* __restrict__ v_pool, int64_t pool_slots, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int64_t per_tensor = static_cast<int64_t>(T) * Hkv * D;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       idx < 2 * per_tensor; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const bool is_v = idx >= per_tensor;
    const int64_t e = is_v ? idx - per_tensor : idx;
    const int32_t d = static_cast<int32_t>(e % D);
    const int64_t th = e / D;
    const int32_t h = static_cast<int32_t>(th % Hkv);
    const int32_t t = static_cast<int32_t>(th / Hkv);
    const int32_t slot = __ldg(slots + t);
    if (slot < 0) continue;
    if (slot >= pool_slots) {
      set_status(status, kStatusBadSlot);
      continue;
    }
    const Tin* src = (is_v ? v + t * v_stride : k + t * k_stride) + h * D + d;
    Tpool* dst = (is_v ? v_pool : k_pool) + (h * pool_slots + slot) * D + d;
    *dst = from_float<Tpool>(as_float<Tin>(*src));
  }
}

// Decode append: one new token per row (a pure decode step).  One warp per
// row: lane 0 locates the token's slot through the row's block table
// (BlockAllocator.locate, src/server/block_allocator.py:28-30) and writes
// context_lens[r] = start_pos[r] + 1 and slots[r]; the warp then copies the
// row's K and V [Hkv, D] into the pool (PagedKVCache.append,
// src/server/torch_model.py:149-153) with 16-byte accesses when VEC.  It
// replaces the metadata + slot-write pair for decode steps and lets the next
// kernel launch at once.
template <typename Tin, typename Tpool, bool VEC>
__global__ void __launch_bounds__(64)
    decode_append_kernel(const int32_t* __restrict__ seq_rows, const int32_t* __restrict__ start_pos,
                         int32_t R, const int32_t* __restrict__ block_tables, int64_t bt_stride,
                         int32_t bt_rows, int32_t max_blocks, int32_t block_size,
                         int32_t num_blocks, const Tin* __restrict__ k, const Tin* __restrict__ v,
                         int64_t k_stride, int64_t v_stride, int32_t Hkv, int32_t D,
                         Tpool* __restrict__ k_pool, Tpool* __restrict__ v_pool,
                         int64_t pool_slots, int32_t* __restrict__ context_lens,
                         int32_t* __restrict__ slots, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  int32_t slot = -1;
  if (lane == 0) {
    const int32_t pos = start_pos[r];
    const int32_t row = seq_rows != nullptr ? seq_rows[r] : r;
    const int32_t bi = pos / block_size;
    if (pos < 0) {
      // Padding row: nothing written, context length 0.
    } else if (row < 0 || row >= bt_rows || bi >= max_blocks) {
      set_status(status, row < 0 || row >= bt_rows ? kStatusBadRow : kStatusBadLength);
    } else {
      const int32_t blk = block_tables[static_cast<int64_t>(row) * bt_stride + bi];
      if (blk < 0 || blk >= num_blocks) {
        set_status(status, kStatusBadBlock);
      } else {
        slot = blk * block_size + pos % block_size;
      }
    }
    context_lens[r] = pos < 0 ? 0 : pos + 1;
    slots[r] = slot;
  }
  slot = __shfl_sync(0xffffffffu, slot, 0);
  if (slot < 0 || k == nullptr) return;  // padding row, or locate-only call
  const int32_t per = VEC ? Hkv * (D >> 3) : Hkv * D;  // vectors (or elements) per tensor
  for (int32_t i = lane; i < 2 * per; i += 32) {
    const bool is_v = i >= per;
    const int32_t e = is_v ? i - per : i;
    const int32_t h = e / (VEC ? (D >> 3) : D);
    const int32_t c = (e % (VEC ? (D >> 3) : D)) * (VEC ? 8 : 1);
    const Tin* src = (is_v ? v + r * v_stride : k + r * k_stride) + h * D + c;
    Tpool* dst = (is_v ? v_pool : k_pool) + (h * pool_slots + slot) * D + c;
    if (VEC) {
      float x[8];
      load8(src, x);
      store8(dst, x);
    } else {
      *dst = from_float<Tpool>(as_float<Tin>(*src));
    }
  }
}

template <typename Tin, typename Tpool>
int launch_decode_append_t(const int32_t* seq_rows, const int32_t* start_pos, int32_t R,
                           const int32_t* bt, int64_t bt_stride, int32_t bt_rows,
                           int32_t max_blocks, int32_t bs, int32_t nb, const void* k,
                           const void* v, int64_t ks, int64_t vs, int32_t Hkv, int32_t D, void* kp,
                           void* vp, int64_t pool_slots, bool vec, int32_t* ctx, int32_t* slots,
                           uint32_t* status, cudaStream_t stream) {
  if (R == 0) return 0;
  // Two rows (warps) per CTA: small CTAs fit beside the decode CTAs that launch
  // behind this kernel, so none of those waits for a slot.
  cudaLaunchConfig_t cfg = pdl_config((R + 1) / 2, 64, stream);
  cudaLaunchAttribute attr[1];
  pdl_attr(cfg, attr);
  auto kernel = vec ? decode_append_kernel<Tin, Tpool, true> : decode_append_kernel<Tin, Tpool, false>;
  return static_cast<int>(cudaLaunchKernelEx(
      &cfg, kernel, seq_rows, start_pos, R, bt, bt_stride, bt_rows, max_blocks, bs, nb,
      static_cast<const Tin*>(k), static_cast<const Tin*>(v), ks, vs, Hkv, D,
      static_cast<Tpool*>(kp), static_cast<Tpool*>(vp), pool_slots, ctx, slots, status));
}

template <typename Tin, typename Tpool>
int launch_slot_write_t(const void* k, const void* v, int64_t ks, int64_t vs, const int32_t* slots,
                        int32_t T, int32_t Hkv, int32_t D, void* kp, void* vp, int64_t pool_slots,
                        bool vec, int sms, uint32_t* status, cudaStream_t stream) {
  const int64_t work = 2ll * T * Hkv * (vec ? D / 8 : D);
  if (work == 0) return 0;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = pdl_config(static_cast<int>(blocks), 256, stream);
  cudaLaunchAttribute attr[1];
  pdl_attr(cfg, attr);
  auto kernel = vec ? slot_write_vec_kernel<Tin, Tpool> : slot_write_scalar_kernel<Tin, Tpool>;
  return static_cast<int>(cudaLaunchKernelEx(
      &cfg, kernel, static_cast<const Tin*>(k), static_cast<const Tin*>(v), ks, vs, slots, T, Hkv,
      D, static_cast<Tpool*>(kp), static_cast<Tpool*>(vp), pool_slots, status));
}

}  // namespace

int max_metadata_rows() { return kMaxMetaRows; }

int launch_step_metadata(const int32_t* seq_rows, const int32_t* start_pos, const int32_t* n_new,
                         int32_t R, const int32_t* block_tables, int64_t bt_stride,
                         int32_t bt_rows, int32_t max_blocks, int32_t block_size,
                         int32_t num_blocks, int32_t T, int32_t* cu_q, int32_t* positions,
                         int32_t* slots, int32_t* context_lens, uint32_t* status,
                         cudaStream_t stream) {
  const int grid = T > 0 ? (T + kMetaThreads - 1) / kMetaThreads : 1;
  cudaLaunchConfig_t cfg = pdl_config(grid, kMetaThreads, stream);
  cudaLaunchAttribute attr[1];
  pdl_attr(cfg, attr);
  return static_cast<int>(cudaLaunchKernelEx(
      &cfg, step_metadata_kernel, seq_rows, start_pos, n_new, R, block_tables, bt_stride, bt_rows,
      max_blocks, block_size, num_blocks, T, cu_q, positions, slots, context_lens, status));
}

int launch_decode_append(const int32_t* seq_rows, const int32_t* start_pos, int32_t R,
                         const int32_t* block_tables, int64_t bt_stride, int32_t bt_rows,
                         int32_t max_blocks, int32_t block_size, int32_t num_blocks,
                         const void* k, const void* v, int64_t k_stride, int64_t v_stride,
                         int in_bf16, int32_t Hkv, int32_t D, void* k_pool, void* v_pool,
                         int pool_bf16, int64_t pool_slots, bool vec, int32_t* context_lens,
                         int32_t* slots, uint32_t* status, cudaStream_t stream) {
#define BS_APPEND(TI, TP)                                                                      \
  return launch_decode_append_t<TI, TP>(seq_rows, start_pos, R, block_tables, bt_stride,       \
                                        bt_rows, max_blocks, block_size, num_blocks, k, v,     \
                                        k_stride, v_stride, Hkv, D, k_pool, v_pool, pool_slots, \
                                        vec, context_lens, slots, status, stream)
  if (in_bf16 && pool_bf16) BS_APPEND(__nv_bfloat16, __nv_bfloat16);
  if (in_bf16) BS_APPEND(__nv_bfloat16, float);
  if (pool_bf16) BS_APPEND(float, __nv_bfloat16);
  BS_APPEND(float, float);
#undef BS_APPEND
}

// in_bf16 / pool_bf16: element types of the k/v rows and of the pool.
int launch_slot_write(const void* k, const void* v, int64_t k_stride, int64_t v_stride,
                      int in_bf16, const int32_t* slots, int32_t T, int32_t Hkv, int32_t D,
                      void* k_pool, void* v_pool, int pool_bf16, int64_t pool_slots, bool vec,
                      int sms, uint32_t* status, cudaStream_t stream) {
  if (in_bf16 && pool_bf16)
    return launch_slot_write_t<__nv_bfloat16, __nv_bfloat16>(k, v, k_stride, v_stride, slots, T,
                                                            Hkv, D, k_pool, v_pool, pool_slots,
                                                            vec, sms, status, stream);
  if (in_bf16)
    return launch_slot_write_t<__nv_bfloat16, float>(k, v, k_stride, v_stride, slots, T, Hkv, D,
                                                     k_pool, v_pool, pool_slots, vec, sms, status,
                                                     stream);
  if (pool_bf16)
    return launch_slot_write_t<float, __nv_bfloat16>(k, v, k_stride, v_stride, slots, T, Hkv, D,
                                                     k_pool, v_pool, pool_slots, vec, sms, status,
                                                     stream);
  return launch_slot_write_t<float, float>(k, v, k_stride, v_stride, slots, T, Hkv, D, k_pool,
                                           v_pool, pool_slots, vec, sms, status, stream);
}

}  // namespace bsb

namespace bsb {
namespace {

__global__ void __launch_bounds__(256)
    expand_rows_kernel(const int32_t* __restrict__ cu_q, const int32_t* __restrict__ context_lens,
                       const int32_t* __restrict__ seq_rows, int32_t R, int32_t T,
                       int32_t* __restrict__ token_lens, int32_t* __restrict__ token_rows) {
  pdl_trigger();
  pdl_wait();
  const int32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  // Last row r with cu_q[r] <= t.
  int32_t lo = 0, hi = R - 1;
  while (lo < hi) {
    const int32_t mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_q + mid) <= t) lo = mid; else hi = mid - 1;
  }
  const int32_t begin = __ldg(cu_q + lo), end = __ldg(cu_q + lo + 1);
  if (t >= end) {  // past the last chunk: a query with no context (reported by decode)
    token_lens[t] = 0;
    token_rows[t] = 0;
    return;
  }
  const int32_t prior = __ldg(context_lens + lo) - (end - begin);
  token_lens[t] = prior + (t - begin) + 1;
  token_rows[t] = seq_rows != nullptr ? __ldg(seq_rows + lo) : lo;
}

}  // namespace

int launch_expand_rows(const int32_t* cu_q, const int32_t* context_lens, const int32_t* seq_rows,
                       int32_t R, int32_t T, int32_t* token_lens, int32_t* token_rows,
                       cudaStream_t stream) {
  if (T <= 0) return 0;
  cudaLaunchConfig_t cfg = pdl_config((T + 255) / 256, 256, stream);
  cudaLaunchAttribute attr[1];
  pdl_attr(cfg, attr);
  return static_cast<int>(cudaLaunchKernelEx(&cfg, expand_rows_kernel, cu_q, context_lens,
                                             seq_rows, R, T, token_lens, token_rows));
}

}  // namespace bsb
