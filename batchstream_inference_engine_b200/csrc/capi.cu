// C ABI of the paged-attention path (declared in include/batchstream_b200.h).
//
// Host-side validation mirrors the reference op's check_inputs
// (csrc/paged_attention.cpp:22-44): every malformed input is an error code plus a
// message, never a crash and never a device fault.  Kernel launches go on the
// caller's stream; nothing here allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/batchstream_b200.h"
#include "decode.cuh"
#include "prefill.cuh"

namespace bsb {
int max_metadata_rows();
int launch_step_metadata(const int32_t* seq_rows, const int32_t* start_pos, const int32_t* n_new,
                         int32_t R, const int32_t* block_tables, int64_t bt_stride,
                         int32_t bt_rows, int32_t max_blocks, int32_t block_size,
                         int32_t num_blocks, int32_t T, int32_t* cu_q, int32_t* positions,
                         int32_t* slots, int32_t* context_lens, uint32_t* status,
                         cudaStream_t stream);
int launch_rms_norm(const void* x, int64_t x_stride, const void* add, int64_t add_stride,
                    const int32_t* index, int32_t x_rows, const void* w, int32_t rows,
                    int32_t hidden, float eps, void* out, int64_t out_stride, void* sum_out,
                    int64_t sum_stride, bool bf16, bool vec, uint32_t* status,
                    cudaStream_t stream);
int launch_rope_append(const void* qkv, int64_t qkv_stride, const void* cos_t, const void* sin_t,
                       int32_t num_pos, const int32_t* pos, const int32_t* slots, int32_t ntok,
                       int32_t H, int32_t Hkv, int32_t D, void* q_out, void* k_pool,
                       void* v_pool, int64_t pool_slots, bool bf16, bool pool_bf16, int sms,
                       uint32_t* status, cudaStream_t stream);
int launch_silu_mul(const void* gate_up, int64_t stride, int32_t ntok, int32_t inter, void* out,
                    bool bf16, bool vec, int sms, cudaStream_t stream);
int launch_argmax_rows(const void* x, int64_t stride, int32_t rows, int64_t cols, void* out,
                       bool bf16, bool vec, cudaStream_t stream);
int launch_decode_append(const int32_t* seq_rows, const int32_t* start_pos, int32_t R,
                         const int32_t* block_tables, int64_t bt_stride, int32_t bt_rows,
                         int32_t max_blocks, int32_t block_size, int32_t num_blocks,
                         const void* k, const void* v, int64_t k_stride, int64_t v_stride,
                         int in_bf16, int32_t Hkv, int32_t D, void* k_pool, void* v_pool,
                         int pool_bf16, int64_t pool_slots, bool vec, int32_t* context_lens,
                         int32_t* slots, uint32_t* status, cudaStream_t stream);
int launch_slot_write(const void* k, const void* v, int64_t k_stride, int64_t v_stride,
                      int in_bf16, const int32_t* slots, int32_t T, int32_t Hkv, int32_t D,
                      void* k_pool, void* v_pool, int pool_bf16, int64_t pool_slots, bool vec,
                      int sms, uint32_t* status, cudaStream_t stream);
}  // namespace bsb

namespace {

thread_local std::string g_error;

// Kernels this library has enqueued (or recorded into a stream capture) in
// this process; read by bs_kernel_launches().
std::atomic<uint64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add(static_cast<uint64_t>(n)); }

// Settings of bs_set_wait_probe, read at each decode launch (test use only).
std::atomic<uint64_t> g_wait_limit_ns{0};
std::atomic<int32_t> g_probe_unarmed{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define BS_CHECK(cond, ...)                      \
  do {                                           \
    if (!(cond)) return fail(BS_ERR_INVALID, __VA_ARGS__); \
  } while (0)

constexpr int64_t kMaxHeadDim = 256;
constexpr int64_t kMaxGroups = 16;
constexpr int64_t kInt32Max = 2147483647ll;

struct DeviceInfo {
  int sms = 0;
  int occ_mma[2][2] = {{0, 0}, {0, 0}};  // [d128][g16]
  int occ_simt[2][2][2] = {};           // [bf16][d>64 bucket][g16] (coarse cache)
};

std::mutex g_mu;
std::vector<DeviceInfo> g_devices;

int current_device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mu);
  if (static_cast<int>(g_devices.size()) <= dev) g_devices.resize(dev + 1);
  DeviceInfo& d = g_devices[dev];
  if (d.sms == 0) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    d.sms = sms;
  }
  *out = &d;
  return BS_OK;
}

bool use_mma_path(int32_t dtype, int64_t block_size, int64_t head_dim, int64_t groups) {
  return dtype == BS_BF16 && block_size == 16 && (head_dim == 64 || head_dim == 128) &&
         groups <= kMaxGroups;
}

// Persistent grid size for the chosen decode kernel on the current device.
int decode_grid(bool mma, int32_t dtype, int64_t head_dim, int64_t groups, int* grid) {
  DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    int* slot = mma ? &d->occ_mma[head_dim == 128][groups > 8]
                    : &d->occ_simt[dtype == BS_BF16][head_dim > 64][groups > 8];
    if (*slot == 0) {
      const int n = mma ? bsb::decode_mma_ctas_per_sm(static_cast<int>(head_dim),
                                                      static_cast<int>(groups))
                        : bsb::decode_simt_ctas_per_sm(static_cast<int>(head_dim),
                                                       static_cast<int>(groups),
                                                       dtype == BS_BF16);
      if (n <= 0) {
        return fail(BS_ERR_CUDA, "occupancy query for the decode kernel failed (%d)", n);
      }
      *slot = n;
    }
    occ = *slot;
  }
  *grid = d->sms * occ;
  return BS_OK;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

int32_t record_stride(int64_t groups, int64_t head_dim) {
  return static_cast<int32_t>(round_up(groups * head_dim + 2 * groups, 4));
}

// Workspace layout: [status 256 B][segment counters, fixed capacity][staging
// ints][partial records].  The counter region has the same offset and size for
// every call, whatever its batch, so no call's staging or records ever land on
// another call's counters: the kernels leave every counter at zero, and a
// workspace that was zero-filled once stays valid for any sequence of calls.
constexpr int64_t kMaxSegments = 1 << 16;

struct WsLayout {
  int64_t tasks;  // [grid] merge tasks of the tensor-core decode
  int64_t counters, staging, partials, total;
};

WsLayout ws_layout(int64_t segments, int64_t staging_ints, int64_t grid, int64_t rec_stride) {
  (void)segments;  // bounded by kMaxSegments, checked by the callers
  WsLayout w;
  w.counters = 256;
  w.staging = w.counters + kMaxSegments * 4;
  w.partials = w.staging + round_up(staging_ints * 4, 256);
  w.tasks = w.partials + round_up(2 * grid * rec_stride * 4, 256);
  w.total = w.tasks + round_up(grid * static_cast<int64_t>(sizeof(bsb::MergeTask)), 256);
  return w;
}

// Split-KV factor of the tensor-core prefill: up to one CTA per SM for the
// query tiles that can hold tokens (at most ceil(num_tokens / 128) + num_rows
// per head; the other tiles of a padded launch exit at once).  A second CTA on
// an SM adds less than a first, and every piece costs a CTA's set-up and a
// merge, so only batches with fewer such tiles than SMs are split.
int prefill_splits(int64_t num_rows, int64_t qtiles, int64_t num_tokens, int64_t heads, int sms) {
  const int64_t items =
      std::min(num_rows * qtiles, (num_tokens + 127) / 128 + num_rows) * heads;
  if (items <= 0) return 1;
  const int64_t want = (static_cast<int64_t>(sms) + items - 1) / items;
  return static_cast<int>(std::min<int64_t>(std::max<int64_t>(want, 1), bsb::kMaxPrefillSplits));
}

// Rows x query tiles whose work the plan kernel ranks (0: no plan): only when
// the query tiles that hold tokens — at most ceil(num_tokens / 128) + num_rows
// of the rows x ceil(max_query_len / 128) launched, the rest exit at once —
// are more than one wave of resident CTAs (inside one wave the order does not
// matter), and for plans one CTA ranks (rts * max(splits, 2) entries at most).
int64_t prefill_plan_rts(int64_t num_rows, int64_t qtiles, int64_t num_tokens, int64_t heads,
                         int splits, int sms) {
  const int64_t rts = num_rows * qtiles;
  const int64_t busy = std::min(rts, (num_tokens + 127) / 128 + num_rows);
  const int64_t slots = static_cast<int64_t>(sms) * bsb::prefill_ctas_per_sm();
  if (rts <= 0 || busy * heads * splits <= slots ||
      rts * std::max(splits, 2) > bsb::kMaxPlanEntries) {
    return 0;
  }
  return rts;
}

// Workspace of the tensor-core prefill: the split records (splits > 1) start
// where the decode's scratch does, past the status word and the segment
// counters (which stay zero between calls); the plan follows them.
int64_t prefill_split_offset() { return ws_layout(0, 0, 0, 0).staging; }
int64_t prefill_records_bytes(int64_t items, int splits) {
  return splits > 1 ? items * splits * (bsb::kPrefillRecordO + bsb::kPrefillRecordML) * 4 : 0;
}
int64_t prefill_ws_bytes(int64_t items, int splits, int64_t plan_entries) {
  int64_t b = prefill_split_offset() + prefill_records_bytes(items, splits);
  if (plan_entries > 0) b += (1 + 2 * plan_entries) * 16;
  return b;
}

// ------------------------------------------------------------------ tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) cached = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (cached == nullptr) {
    return fail(BS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (%s)", cudaGetErrorString(err));
  }
  *fn = cached;
  return BS_OK;
}

// [rows, head_dim] bf16 view of one pool, boxes of 16 rows x 64 columns,
// 128-byte swizzle (the layout the decode kernel's ldmatrix addressing expects).
int encode_pool_map(CUtensorMap* map, const void* base, int64_t rows, int64_t head_dim) {
  EncodeTiledFn fn = nullptr;
  if (int rc = get_encode_fn(&fn)) return rc;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(head_dim * 2)};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return BS_OK;
}

// [T, H, 64] bf16 query view in boxes of (64 dims, 1 head, 128 tokens) with
// 128-byte swizzle: one box is the query tile of one head for the prefill kernel.
int encode_query_map(CUtensorMap* map, const void* base, int64_t tokens, int64_t heads) {
  EncodeTiledFn fn = nullptr;
  if (int rc = get_encode_fn(&fn)) return rc;
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {64 * 2, static_cast<cuuint64_t>(heads * 64 * 2)};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BS_ERR_CUDA, "cuTensorMapEncodeTiled (query) failed (%d)", static_cast<int>(r));
  return BS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The pointer must be device (or managed) memory of the current device, so that
// a host tensor passed by mistake is an error instead of a device fault.
int require_device(const void* p, const char* what) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(e, what);
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
    return fail(BS_ERR_INVALID, "%s must be CUDA device memory", what);
  }
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev) {
    return fail(BS_ERR_INVALID, "%s is on device %d but the current device is %d", what,
                attr.device, dev);
  }
  return BS_OK;
}

bool is_contiguous(int32_t ndim, const int64_t* shape, const int64_t* strides) {
  int64_t expect = 1;
  for (int32_t d = ndim - 1; d >= 0; --d) {
    if (shape[d] != 1 && strides[d] != expect) return false;
    expect *= shape[d];
  }
  return true;
}

// Shared launch of the decode kernels once everything is validated.
// Encoded pool maps of the last few pools seen by this thread (a model's layers
// reuse the same views every step, so encoding once per view is enough).
struct MapCacheEntry {
  const void* base = nullptr;
  int64_t rows = 0, head_dim = 0;
  CUtensorMap map;
};

int cached_pool_map(CUtensorMap* out, const void* base, int64_t rows, int64_t head_dim) {
  constexpr int kEntries = 128;
  thread_local MapCacheEntry cache[kEntries];
  thread_local int next = 0;
  for (int i = 0; i < kEntries; ++i) {
    const MapCacheEntry& e = cache[i];
    if (e.base == base && e.rows == rows && e.head_dim == head_dim) {
      *out = e.map;
      return BS_OK;
    }
  }
  MapCacheEntry& e = cache[next];
  if (int rc = encode_pool_map(&e.map, base, rows, head_dim)) {
    e.base = nullptr;
    return rc;
  }
  e.base = base;
  e.rows = rows;
  e.head_dim = head_dim;
  next = (next + 1) % kEntries;
  *out = e.map;
  return BS_OK;
}

int launch_decode(bsb::DecodeArgs& a, int32_t dtype, int grid, cudaStream_t stream,
                  bsb::MergeTask* tasks) {
  const bool mma = use_mma_path(dtype, a.block_size, a.head_dim, a.groups);
  a.tasks = mma ? tasks : nullptr;
  bsb::apply_wait_probe(a);
  int rc;
  if (mma) {
    CUtensorMap kmap, vmap;
    const int64_t rows = static_cast<int64_t>(a.num_kv_heads) * a.num_blocks * a.block_size;
    if ((rc = cached_pool_map(&kmap, a.k_pool, rows, a.head_dim))) return rc;
    if ((rc = cached_pool_map(&vmap, a.v_pool, rows, a.head_dim))) return rc;
    rc = bsb::launch_decode_mma(a, kmap, vmap, grid, stream);
  } else {
    rc = bsb::launch_decode_simt(a, dtype == BS_BF16, grid, stream);
  }
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "decode kernel launch");
  count_launches(a.tasks != nullptr ? 2 : 1);  // the merge pass runs with tasks
  return BS_OK;
}

int dtype_size(int32_t dtype) { return dtype == BS_BF16 ? 2 : 4; }

}  // namespace

extern "C" {

const char* bs_last_error(void) { return g_error.c_str(); }

const char* bs_version(void) { return "batchstream_b200 0.1 (sm_100a)"; }

uint64_t bs_kernel_launches(void) { return g_launches.load(); }

int bs_paged_attention_workspace_bytes(int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                       int64_t block_table_len, int32_t dtype,
                                       int64_t block_size, uint64_t* bytes_out) {
  BS_CHECK(bytes_out != nullptr, "bytes_out is null");
  BS_CHECK(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "heads must equal kv_heads * groups");
  const int64_t groups = num_heads / num_kv_heads;
  int grid = 0;
  if (int rc = decode_grid(use_mma_path(dtype, block_size, head_dim, groups), dtype, head_dim,
                           groups, &grid))
    return rc;
  const WsLayout w = ws_layout(num_kv_heads, 1 + block_table_len, grid,
                               record_stride(groups, head_dim));
  *bytes_out = static_cast<uint64_t>(w.total);
  return BS_OK;
}

int bs_paged_attention_check(int32_t query_dtype, int32_t query_ndim, const int64_t* query_shape,
                             const int64_t* query_strides, int32_t keys_dtype, int32_t keys_ndim,
                             const int64_t* keys_shape, const int64_t* keys_strides,
                             int32_t values_dtype, int32_t values_ndim,
                             const int64_t* values_shape, const int64_t* values_strides,
                             const int64_t* block_table, int64_t block_table_len, int64_t length,
                             int64_t block_size, int64_t groups) {
  // The reference's checks, in its order (csrc/paged_attention.cpp:25-43).
  BS_CHECK((query_dtype == BS_BF16 || query_dtype == BS_F32) && keys_dtype == query_dtype &&
               values_dtype == query_dtype,
           "query, keys and values must all be bfloat16 or all float32");
  BS_CHECK(query_ndim == 2, "query must have shape (heads, head_dim)");
  BS_CHECK(keys_ndim == 4, "keys must have shape (kv_heads, blocks, block_size, head_dim)");
  bool same = values_ndim == keys_ndim;
  for (int d = 0; same && d < 4; ++d) same = keys_shape[d] == values_shape[d];
  BS_CHECK(same, "keys and values must have the same shape");
  BS_CHECK(is_contiguous(4, keys_shape, keys_strides) &&
               is_contiguous(4, values_shape, values_strides),
           "keys and values must be contiguous");
  BS_CHECK(block_size > 0 && block_size == keys_shape[2], "block_size does not match keys");
  BS_CHECK(query_shape[1] == keys_shape[3], "query and keys disagree on head_dim");
  BS_CHECK(groups > 0 && query_shape[0] == keys_shape[0] * groups,
           "heads must equal kv_heads * groups");
  BS_CHECK(length > 0, "length must be positive");
  const int64_t blocks_needed = (length + block_size - 1) / block_size;
  BS_CHECK(block_table != nullptr || blocks_needed == 0, "block table is null");
  BS_CHECK(block_table_len >= blocks_needed, "block table is too short for length");
  const int64_t num_blocks = keys_shape[1];
  for (int64_t i = 0; i < blocks_needed; ++i) {
    BS_CHECK(block_table[i] >= 0 && block_table[i] < num_blocks, "block table entry out of range");
  }
  (void)query_strides;
  return BS_OK;
}

int bs_paged_attention(const void* query, int32_t query_dtype, int32_t query_ndim,
                       const int64_t* query_shape, const int64_t* query_strides,
                       const void* keys, int32_t keys_dtype, int32_t keys_ndim,
                       const int64_t* keys_shape, const int64_t* keys_strides,
                       const void* values, int32_t values_dtype, int32_t values_ndim,
                       const int64_t* values_shape, const int64_t* values_strides,
                       const int64_t* block_table, int64_t block_table_len, int64_t length,
                       int64_t block_size, int64_t groups, double scaling, void* output,
                       void* workspace, uint64_t workspace_bytes, void* stream) {
  // The reference's checks, in its order (csrc/paged_attention.cpp:25-43).
  if (int rc = bs_paged_attention_check(query_dtype, query_ndim, query_shape, query_strides,
                                        keys_dtype, keys_ndim, keys_shape, keys_strides,
                                        values_dtype, values_ndim, values_shape, values_strides,
                                        block_table, block_table_len, length, block_size,
                                        groups)) {
    return rc;
  }
  const int64_t blocks_needed = (length + block_size - 1) / block_size;
  const int64_t num_blocks = keys_shape[1];
  // This library's own requirements.
  const int64_t heads = query_shape[0], head_dim = query_shape[1], kv_heads = keys_shape[0];
  BS_CHECK(is_contiguous(2, query_shape, query_strides),
           "query must be contiguous (the binding copies it first)");
  if (head_dim > kMaxHeadDim || groups > kMaxGroups || kv_heads > kMaxSegments) {
    return fail(BS_ERR_UNSUPPORTED, "head_dim <= %lld and groups <= %lld are supported",
                static_cast<long long>(kMaxHeadDim), static_cast<long long>(kMaxGroups));
  }
  if (kv_heads * num_blocks * block_size > kInt32Max) {
    return fail(BS_ERR_UNSUPPORTED, "pool has more than 2^31 rows");
  }
  BS_CHECK(query != nullptr && keys != nullptr && values != nullptr && output != nullptr,
           "null tensor pointer");
  if (int rc = require_device(query, "query")) return rc;
  if (int rc = require_device(keys, "keys")) return rc;
  if (int rc = require_device(values, "values")) return rc;
  if (int rc = require_device(output, "output")) return rc;

  int grid_max = 0;
  const bool mma = use_mma_path(query_dtype, block_size, head_dim, groups);
  if (int rc = decode_grid(mma, query_dtype, head_dim, groups, &grid_max)) return rc;
  const WsLayout w = ws_layout(kv_heads, 1 + blocks_needed, grid_max,
                               record_stride(groups, head_dim));
  if (workspace == nullptr || workspace_bytes < static_cast<uint64_t>(w.total)) {
    return fail(BS_ERR_WORKSPACE, "workspace of %llu bytes is smaller than the %lld needed",
                static_cast<unsigned long long>(workspace_bytes), static_cast<long long>(w.total));
  }
  if (mma && (!aligned16(query) || !aligned16(keys) || !aligned16(values))) {
    return fail(BS_ERR_INVALID, "query, keys and values must be 16-byte aligned");
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Stage [length, table...] as int32 into the workspace.
  std::vector<int32_t> staged(static_cast<size_t>(1 + blocks_needed));
  staged[0] = static_cast<int32_t>(length);
  for (int64_t i = 0; i < blocks_needed; ++i) staged[1 + i] = static_cast<int32_t>(block_table[i]);
  int32_t* dev_staged = reinterpret_cast<int32_t*>(ws + w.staging);
  cudaError_t e = cudaMemcpyAsync(dev_staged, staged.data(), staged.size() * sizeof(int32_t),
                                  cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "staging the block table");

  bsb::DecodeArgs a{};
  a.q = query;
  a.q_stride_seq = heads * head_dim;
  a.out = output;
  a.o_stride_seq = heads * head_dim;
  a.k_pool = keys;
  a.v_pool = values;
  a.block_tables = dev_staged + 1;
  a.bt_stride = blocks_needed;
  a.bt_rows = 1;
  a.seq_rows = nullptr;
  a.context_lens = dev_staged;
  a.num_seqs = 1;
  a.num_heads = static_cast<int32_t>(heads);
  a.num_kv_heads = static_cast<int32_t>(kv_heads);
  a.groups = static_cast<int32_t>(groups);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.block_size = static_cast<int32_t>(block_size);
  a.num_blocks = static_cast<int32_t>(num_blocks);
  a.max_blocks = static_cast<int32_t>(blocks_needed);
  a.scale = static_cast<float>(scaling);
  a.partials = reinterpret_cast<float*>(ws + w.partials);
  a.rec_stride = record_stride(groups, head_dim);
  a.seg_counters = reinterpret_cast<int32_t*>(ws + w.counters);
  a.status = reinterpret_cast<uint32_t*>(ws);
  // A few blocks per CTA keeps the cross-CTA merge short for one sequence.
  const int64_t units = kv_heads * blocks_needed;
  int64_t grid = (units + 7) / 8;
  if (grid < 1) grid = 1;
  if (grid > grid_max) grid = grid_max;
  return launch_decode(a, query_dtype, static_cast<int>(grid), st,
                       reinterpret_cast<bsb::MergeTask*>(ws + w.tasks));
}

int bs_paged_attention_batched_workspace_bytes(int64_t num_seqs, int64_t num_heads,
                                               int64_t num_kv_heads, int64_t head_dim,
                                               int64_t block_size, int32_t dtype,
                                               uint64_t* bytes_out) {
  BS_CHECK(bytes_out != nullptr, "bytes_out is null");
  BS_CHECK(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "heads must equal kv_heads * groups");
  const int64_t groups = num_heads / num_kv_heads;
  int grid = 0;
  if (int rc = decode_grid(use_mma_path(dtype, block_size, head_dim, groups), dtype, head_dim,
                           groups, &grid))
    return rc;
  const WsLayout w = ws_layout(num_seqs * num_kv_heads, 0, grid, record_stride(groups, head_dim));
  *bytes_out = static_cast<uint64_t>(w.total);
  return BS_OK;
}

int bs_paged_attention_batched(const void* query, int64_t query_seq_stride, const void* key_pool,
                               const void* value_pool, const int32_t* block_tables,
                               int64_t table_stride, int64_t table_rows, const int32_t* seq_rows,
                               const int32_t* context_lens, int64_t num_seqs, int64_t num_heads,
                               int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                               int64_t num_blocks, int64_t max_blocks_per_seq, int32_t dtype,
                               double scaling, int64_t units_hint, int32_t flags, void* output,
                               int64_t output_seq_stride, void* workspace,
                               uint64_t workspace_bytes, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK((flags & ~(BS_LENS_READY | BS_AFTER_APPEND)) == 0, "unknown flags");
  BS_CHECK(!(flags & BS_AFTER_APPEND) || (flags & BS_LENS_READY),
           "BS_AFTER_APPEND needs BS_LENS_READY");
  BS_CHECK(num_seqs >= 0, "num_seqs must be non-negative");
  BS_CHECK(num_kv_heads > 0 && num_heads > 0 && num_heads % num_kv_heads == 0,
           "heads must equal kv_heads * groups");
  BS_CHECK(head_dim > 0 && block_size > 0 && num_blocks > 0, "sizes must be positive");
  BS_CHECK(max_blocks_per_seq > 0 && max_blocks_per_seq <= table_stride,
           "max_blocks_per_seq must be in [1, table_stride]");
  BS_CHECK(table_rows > 0 && table_rows <= kInt32Max, "table_rows out of range");
  BS_CHECK(query_seq_stride >= num_heads * head_dim && output_seq_stride >= num_heads * head_dim,
           "sequence strides must cover heads * head_dim");
  const int64_t groups = num_heads / num_kv_heads;
  if (head_dim > kMaxHeadDim || groups > kMaxGroups) {
    return fail(BS_ERR_UNSUPPORTED, "head_dim <= %lld and groups <= %lld are supported",
                static_cast<long long>(kMaxHeadDim), static_cast<long long>(kMaxGroups));
  }
  if (num_kv_heads * num_blocks * block_size > kInt32Max ||
      max_blocks_per_seq * block_size > kInt32Max || num_seqs > kInt32Max) {
    return fail(BS_ERR_UNSUPPORTED, "pool or table larger than 2^31 rows");
  }
  if (num_seqs * num_kv_heads > kMaxSegments) {
    return fail(BS_ERR_UNSUPPORTED, "num_seqs * num_kv_heads must be at most %lld",
                static_cast<long long>(kMaxSegments));
  }
  if (num_seqs == 0) return BS_OK;
  BS_CHECK(query && key_pool && value_pool && block_tables && context_lens && output,
           "null pointer argument");
  const bool mma = use_mma_path(dtype, block_size, head_dim, groups);
  if (mma) {
    BS_CHECK(aligned16(query) && aligned16(key_pool) && aligned16(value_pool) &&
                 (query_seq_stride * 2) % 16 == 0,
             "query, pools and query rows must be 16-byte aligned");
  }
  int grid_max = 0;
  if (int rc = decode_grid(mma, dtype, head_dim, groups, &grid_max)) return rc;
  const WsLayout w =
      ws_layout(num_seqs * num_kv_heads, 0, grid_max, record_stride(groups, head_dim));
  if (workspace == nullptr || workspace_bytes < static_cast<uint64_t>(w.total)) {
    return fail(BS_ERR_WORKSPACE, "workspace of %llu bytes is smaller than the %lld needed",
                static_cast<unsigned long long>(workspace_bytes), static_cast<long long>(w.total));
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  bsb::DecodeArgs a{};
  a.q = query;
  a.q_stride_seq = query_seq_stride;
  a.out = output;
  a.o_stride_seq = output_seq_stride;
  a.k_pool = key_pool;
  a.v_pool = value_pool;
  a.block_tables = block_tables;
  a.bt_stride = table_stride;
  a.bt_rows = static_cast<int32_t>(table_rows);
  a.seq_rows = seq_rows;
  a.context_lens = context_lens;
  a.num_seqs = static_cast<int32_t>(num_seqs);
  a.num_heads = static_cast<int32_t>(num_heads);
  a.num_kv_heads = static_cast<int32_t>(num_kv_heads);
  a.groups = static_cast<int32_t>(groups);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.block_size = static_cast<int32_t>(block_size);
  a.num_blocks = static_cast<int32_t>(num_blocks);
  a.max_blocks = static_cast<int32_t>(max_blocks_per_seq);
  a.scale = static_cast<float>(scaling);
  a.partials = reinterpret_cast<float*>(ws + w.partials);
  a.rec_stride = record_stride(groups, head_dim);
  a.seg_counters = reinterpret_cast<int32_t*>(ws + w.counters);
  a.status = reinterpret_cast<uint32_t*>(ws);
  a.lens_ready = (flags & BS_LENS_READY) ? 1 : 0;
  a.after_append = (flags & BS_AFTER_APPEND) ? 1 : 0;
  int64_t grid = grid_max;
  if (units_hint > 0) {
    const int64_t want = (units_hint + 3) / 4;
    if (want < grid) grid = want;
  }
  return launch_decode(a, dtype, static_cast<int>(grid), static_cast<cudaStream_t>(stream),
                       reinterpret_cast<bsb::MergeTask*>(ws + w.tasks));
}

int bs_prefill_attention_workspace_bytes(int64_t num_tokens, int64_t num_rows,
                                         int64_t max_query_len, int64_t num_heads,
                                         int64_t num_kv_heads, int64_t head_dim,
                                         int64_t block_size, int32_t dtype, uint64_t* bytes_out) {
  BS_CHECK(bytes_out != nullptr, "bytes_out is null");
  BS_CHECK(num_tokens >= 0 && num_rows >= 0 && max_query_len >= 0, "counts must be non-negative");
  BS_CHECK(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "heads must equal kv_heads * groups");
  const int64_t groups = num_heads / num_kv_heads;
  int grid = 0;
  if (int rc = decode_grid(use_mma_path(dtype, block_size, head_dim, groups), dtype, head_dim,
                           groups, &grid))
    return rc;
  // The per-token path stages token lengths and rows, then runs the decode.
  const WsLayout w = ws_layout(num_tokens * num_kv_heads, 2 * num_tokens, grid,
                               record_stride(groups, head_dim));
  int64_t need = w.total;
  // The tensor-core path: split-KV records after the decode's counters.
  DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  const int64_t qtiles = (max_query_len + 127) / 128;
  const int64_t items = num_rows * num_heads * qtiles;
  const int splits = prefill_splits(num_rows, qtiles, num_tokens, num_heads, d->sms);
  const int64_t rts = prefill_plan_rts(num_rows, qtiles, num_tokens, num_heads, splits, d->sms);
  need = std::max(need, prefill_ws_bytes(items, splits, rts * splits));
  *bytes_out = static_cast<uint64_t>(need);
  return BS_OK;
}

int bs_prefill_attention(const void* query, int64_t query_token_stride, const int32_t* cu_q,
                         int64_t num_rows, int64_t num_tokens, int64_t max_query_len,
                         const int32_t* context_lens, const int32_t* seq_rows,
                         const void* key_pool, const void* value_pool,
                         const int32_t* block_tables, int64_t table_stride, int64_t table_rows,
                         int64_t max_blocks_per_seq, int64_t num_heads, int64_t num_kv_heads,
                         int64_t head_dim, int64_t block_size, int64_t num_blocks, int32_t dtype,
                         double scaling, int32_t flags, void* output, int64_t output_token_stride,
                         void* workspace, uint64_t workspace_bytes, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK((flags & ~BS_PREFILL_PER_TOKEN) == 0, "unknown flags");
  BS_CHECK(num_rows >= 0 && num_tokens >= 0 && num_tokens <= kInt32Max, "bad row or token count");
  BS_CHECK(num_kv_heads > 0 && num_heads > 0 && num_heads % num_kv_heads == 0,
           "heads must equal kv_heads * groups");
  BS_CHECK(head_dim > 0 && block_size > 0 && num_blocks > 0, "sizes must be positive");
  BS_CHECK(max_blocks_per_seq > 0 && max_blocks_per_seq <= table_stride,
           "max_blocks_per_seq must be in [1, table_stride]");
  BS_CHECK(table_rows > 0 && table_rows <= kInt32Max, "table_rows out of range");
  BS_CHECK(query_token_stride >= num_heads * head_dim && output_token_stride >= num_heads * head_dim,
           "token strides must cover heads * head_dim");
  const int64_t groups = num_heads / num_kv_heads;
  if (head_dim > kMaxHeadDim || groups > kMaxGroups) {
    return fail(BS_ERR_UNSUPPORTED, "head_dim <= %lld and groups <= %lld are supported",
                static_cast<long long>(kMaxHeadDim), static_cast<long long>(kMaxGroups));
  }
  if (num_kv_heads * num_blocks * block_size > kInt32Max ||
      max_blocks_per_seq * block_size > kInt32Max) {
    return fail(BS_ERR_UNSUPPORTED, "pool or table larger than 2^31 rows");
  }
  if (num_tokens * num_kv_heads > kMaxSegments) {
    return fail(BS_ERR_UNSUPPORTED, "num_tokens * num_kv_heads must be at most %lld",
                static_cast<long long>(kMaxSegments));
  }
  if (num_rows == 0 || num_tokens == 0) return BS_OK;
  BS_CHECK(query && cu_q && context_lens && key_pool && value_pool && block_tables && output,
           "null pointer argument");
  BS_CHECK(max_query_len > 0, "max_query_len must be positive");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  BS_CHECK(ws != nullptr, "workspace is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The tensor-core path folds the scale into the running maximum: it needs a
  // positive scale (other scales take the per-token path).
  const bool fast = !(flags & BS_PREFILL_PER_TOKEN) && dtype == BS_BF16 && head_dim == 64 &&
                    scaling > 0.0 && block_size == 16 && query_token_stride == num_heads * head_dim &&
                    aligned16(query) && aligned16(key_pool) && aligned16(value_pool) &&
                    (output_token_stride * 2) % 16 == 0 && aligned16(output);
  if (fast) {
    CUtensorMap qmap, kmap, vmap;
    const int64_t rows = num_kv_heads * num_blocks * block_size;
    int rc;
    if ((rc = encode_query_map(&qmap, query, num_tokens, num_heads))) return rc;
    if ((rc = cached_pool_map(&kmap, key_pool, rows, head_dim))) return rc;
    if ((rc = cached_pool_map(&vmap, value_pool, rows, head_dim))) return rc;
    bsb::PrefillArgs p{};
    p.q = query;
    p.out = output;
    p.o_stride_tok = output_token_stride;
    p.cu_q = cu_q;
    p.context_lens = context_lens;
    p.seq_rows = seq_rows;
    p.block_tables = block_tables;
    p.bt_stride = table_stride;
    p.bt_rows = static_cast<int32_t>(table_rows);
    p.max_blocks = static_cast<int32_t>(max_blocks_per_seq);
    p.num_rows = static_cast<int32_t>(num_rows);
    p.num_heads = static_cast<int32_t>(num_heads);
    p.num_kv_heads = static_cast<int32_t>(num_kv_heads);
    p.groups = static_cast<int32_t>(groups);
    p.num_blocks = static_cast<int32_t>(num_blocks);
    p.qtiles = static_cast<int32_t>((max_query_len + 127) / 128);
    p.scale = static_cast<float>(scaling);
    {
      int e = 0;
      p.exact_scale = std::frexp(static_cast<double>(p.scale), &e) == 0.5 ? 1 : 0;
    }
    p.status = reinterpret_cast<uint32_t*>(ws);
    const int64_t items = num_rows * num_heads * p.qtiles;
    DeviceInfo* d = nullptr;
    if ((rc = current_device_info(&d))) return rc;
    // Split and plan as far as the workspace holds them.
    const int64_t wsb = static_cast<int64_t>(workspace_bytes);
    p.splits = prefill_splits(num_rows, p.qtiles, num_tokens, num_heads, d->sms);
    if (wsb < prefill_ws_bytes(items, p.splits, 0)) p.splits = 1;
    int64_t rts =
        prefill_plan_rts(num_rows, p.qtiles, num_tokens, num_heads, p.splits, d->sms);
    // A batch with few enough (row, query tile) pairs ranks them in every CTA:
    // no plan launch to wait for, and no plan in the workspace.
    p.rank_in_cta = rts > 0 && p.splits == 1 && rts <= bsb::kMaxCtaRankedRts ? 1 : 0;
    if (p.rank_in_cta || wsb < prefill_ws_bytes(items, p.splits, rts * p.splits)) rts = 0;
    float* records = reinterpret_cast<float*>(ws + prefill_split_offset());
    p.part_o = records;
    p.part_ml = records + items * p.splits * bsb::kPrefillRecordO;
    p.plan = rts > 0 ? reinterpret_cast<int4*>(ws + prefill_split_offset() +
                                               prefill_records_bytes(items, p.splits))
                     : nullptr;
    const int64_t grid = items * p.splits;
    if (grid > kInt32Max) return fail(BS_ERR_UNSUPPORTED, "too many query tiles");
    if (p.plan != nullptr) {
      rc = bsb::launch_prefill_plan(p, st);
      if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "prefill plan launch");
      count_launches(1);
    }
    rc = bsb::launch_prefill_tc(p, qmap, kmap, vmap, static_cast<int>(grid), st);
    if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "prefill kernel launch");
    count_launches(1);
    if (p.splits > 1) {
      rc = bsb::launch_prefill_merge(p, items, st);
      if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "prefill merge launch");
      count_launches(1);
    }
    return BS_OK;
  }
  // Per-token path: token i of a chunk is a decode query over its causal length.
  int grid_max = 0;
  const bool mma = use_mma_path(dtype, block_size, head_dim, groups);
  if (int rc = decode_grid(mma, dtype, head_dim, groups, &grid_max)) return rc;
  const WsLayout w = ws_layout(num_tokens * num_kv_heads, 2 * num_tokens, grid_max,
                               record_stride(groups, head_dim));
  if (workspace_bytes < static_cast<uint64_t>(w.total)) {
    return fail(BS_ERR_WORKSPACE, "workspace of %llu bytes is smaller than the %lld needed",
                static_cast<unsigned long long>(workspace_bytes), static_cast<long long>(w.total));
  }
  if (mma) {
    BS_CHECK(aligned16(query) && aligned16(key_pool) && aligned16(value_pool) &&
                 (query_token_stride * 2) % 16 == 0,
             "query, pools and query rows must be 16-byte aligned");
  }
  int32_t* token_lens = reinterpret_cast<int32_t*>(ws + w.staging);
  int32_t* token_rows = token_lens + num_tokens;
  int rc = bsb::launch_expand_rows(cu_q, context_lens, seq_rows, static_cast<int32_t>(num_rows),
                                   static_cast<int32_t>(num_tokens), token_lens, token_rows, st);
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "prefill row expansion");
  count_launches(1);
  bsb::DecodeArgs a{};
  a.q = query;
  a.q_stride_seq = query_token_stride;
  a.out = output;
  a.o_stride_seq = output_token_stride;
  a.k_pool = key_pool;
  a.v_pool = value_pool;
  a.block_tables = block_tables;
  a.bt_stride = table_stride;
  a.bt_rows = static_cast<int32_t>(table_rows);
  a.seq_rows = token_rows;
  a.context_lens = token_lens;
  a.num_seqs = static_cast<int32_t>(num_tokens);
  a.num_heads = static_cast<int32_t>(num_heads);
  a.num_kv_heads = static_cast<int32_t>(num_kv_heads);
  a.groups = static_cast<int32_t>(groups);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.block_size = static_cast<int32_t>(block_size);
  a.num_blocks = static_cast<int32_t>(num_blocks);
  a.max_blocks = static_cast<int32_t>(max_blocks_per_seq);
  a.scale = static_cast<float>(scaling);
  a.partials = reinterpret_cast<float*>(ws + w.partials);
  a.rec_stride = record_stride(groups, head_dim);
  a.seg_counters = reinterpret_cast<int32_t*>(ws + w.counters);
  a.status = reinterpret_cast<uint32_t*>(ws);
  a.lens_ready = 0;
  return launch_decode(a, dtype, grid_max, st, reinterpret_cast<bsb::MergeTask*>(ws + w.tasks));
}

int bs_decode_append(const int32_t* seq_rows, const int32_t* start_pos, int64_t num_rows,
                     const int32_t* block_tables, int64_t table_stride, int64_t table_rows,
                     int64_t max_blocks_per_seq, const void* key, const void* value,
                     int64_t key_row_stride, int64_t value_row_stride, int32_t input_dtype,
                     void* key_pool, void* value_pool, int32_t pool_dtype, int64_t num_kv_heads,
                     int64_t num_blocks, int64_t block_size, int64_t head_dim,
                     int32_t* context_lens, int32_t* slot_mapping, uint32_t* status,
                     void* stream) {
  BS_CHECK(input_dtype == BS_BF16 || input_dtype == BS_F32, "input dtype must be bf16 or fp32");
  BS_CHECK(pool_dtype == BS_BF16 || pool_dtype == BS_F32, "pool dtype must be bf16 or fp32");
  BS_CHECK(num_rows >= 0 && num_rows <= kInt32Max, "num_rows out of range");
  BS_CHECK(num_kv_heads > 0 && num_blocks > 0 && block_size > 0 && head_dim > 0,
           "sizes must be positive");
  BS_CHECK(max_blocks_per_seq > 0 && max_blocks_per_seq <= table_stride,
           "max_blocks_per_seq must be in [1, table_stride]");
  BS_CHECK(table_rows > 0 && table_rows <= kInt32Max, "table_rows out of range");
  BS_CHECK(key_row_stride >= num_kv_heads * head_dim && value_row_stride >= num_kv_heads * head_dim,
           "row strides must cover kv_heads * head_dim");
  if (num_kv_heads * num_blocks * block_size > kInt32Max * 64ll ||
      num_blocks * block_size > kInt32Max) {
    return fail(BS_ERR_UNSUPPORTED, "pool too large");
  }
  if (num_rows == 0) return BS_OK;
  BS_CHECK((key == nullptr) == (value == nullptr), "key and value must both be given or both NULL");
  BS_CHECK(start_pos && block_tables && key_pool && value_pool && context_lens && slot_mapping,
           "null pointer argument");
  const int in_sz = dtype_size(input_dtype), pool_sz = dtype_size(pool_dtype);
  const bool vec = head_dim % 8 == 0 && aligned16(key) && aligned16(value) &&
                   aligned16(key_pool) && aligned16(value_pool) &&
                   (key_row_stride * in_sz) % 16 == 0 && (value_row_stride * in_sz) % 16 == 0 &&
                   (head_dim * pool_sz) % 16 == 0;
  const int rc = bsb::launch_decode_append(
      seq_rows, start_pos, static_cast<int32_t>(num_rows), block_tables, table_stride,
      static_cast<int32_t>(table_rows), static_cast<int32_t>(max_blocks_per_seq),
      static_cast<int32_t>(block_size), static_cast<int32_t>(num_blocks), key, value,
      key_row_stride, value_row_stride, input_dtype == BS_BF16, static_cast<int32_t>(num_kv_heads),
      static_cast<int32_t>(head_dim), key_pool, value_pool, pool_dtype == BS_BF16,
      num_blocks * block_size, vec, context_lens, slot_mapping, status,
      static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "decode append launch");
  count_launches(1);
  return BS_OK;
}

int bs_rms_norm(const void* x, int64_t x_row_stride, int64_t x_rows, const void* add,
                int64_t add_row_stride, const int32_t* row_index, const void* weight, int64_t rows,
                int64_t hidden, double eps, int32_t dtype, void* out, int64_t out_row_stride,
                void* sum_out, int64_t sum_row_stride, uint32_t* status, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK(rows >= 0 && rows <= kInt32Max && hidden > 0 && hidden <= kInt32Max,
           "rows or hidden out of range");
  BS_CHECK(x_rows >= 0 && x_rows <= kInt32Max, "x_rows out of range");
  BS_CHECK(row_index != nullptr || rows <= x_rows, "rows beyond x without a row index");
  BS_CHECK(x_row_stride >= hidden && out_row_stride >= hidden, "row strides must cover hidden");
  BS_CHECK(add == nullptr || add_row_stride >= hidden, "add row stride must cover hidden");
  BS_CHECK(sum_out == nullptr || sum_row_stride >= hidden, "sum row stride must cover hidden");
  BS_CHECK(row_index == nullptr || sum_out != x, "sum_out may alias x only without a row index");
  if (rows == 0) return BS_OK;
  BS_CHECK(x && weight && out, "null pointer argument");
  const bool vec = hidden % 8 == 0 && x_row_stride % 8 == 0 && out_row_stride % 8 == 0 &&
                   (add == nullptr || add_row_stride % 8 == 0) &&
                   (sum_out == nullptr || sum_row_stride % 8 == 0) && aligned16(x) &&
                   aligned16(add) && aligned16(weight) && aligned16(out) && aligned16(sum_out);
  const int rc = bsb::launch_rms_norm(
      x, x_row_stride, add, add_row_stride, row_index, static_cast<int32_t>(x_rows), weight,
      static_cast<int32_t>(rows), static_cast<int32_t>(hidden), static_cast<float>(eps), out,
      out_row_stride, sum_out, sum_row_stride, dtype == BS_BF16, vec, status,
      static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "rms_norm launch");
  count_launches(1);
  return BS_OK;
}

int bs_rope_append(const void* qkv, int64_t qkv_row_stride, int32_t dtype, const void* cos_table,
                   const void* sin_table, int64_t num_positions, const int32_t* positions,
                   const int32_t* slot_mapping, int64_t num_tokens, int64_t num_heads,
                   int64_t num_kv_heads, int64_t head_dim, void* query_out, void* key_pool,
                   void* value_pool, int32_t pool_dtype, int64_t num_blocks, int64_t block_size,
                   uint32_t* status, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK(pool_dtype == BS_BF16 || pool_dtype == BS_F32, "pool dtype must be bf16 or fp32");
  BS_CHECK(num_tokens >= 0 && num_tokens <= kInt32Max, "num_tokens out of range");
  BS_CHECK(num_heads > 0 && num_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0,
           "heads must be positive and head_dim even");
  BS_CHECK(qkv_row_stride >= (num_heads + 2 * num_kv_heads) * head_dim,
           "qkv rows must hold q, k and v");
  BS_CHECK(num_blocks > 0 && block_size > 0, "sizes must be positive");
  BS_CHECK(num_positions > 0 && num_positions <= kInt32Max, "num_positions out of range");
  if (num_kv_heads * num_blocks * block_size > kInt32Max * 64ll) {
    return fail(BS_ERR_UNSUPPORTED, "pool too large");
  }
  if (num_tokens == 0) return BS_OK;
  BS_CHECK(qkv && cos_table && sin_table && positions && slot_mapping && query_out && key_pool &&
               value_pool,
           "null pointer argument");
  DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  const int rc = bsb::launch_rope_append(
      qkv, qkv_row_stride, cos_table, sin_table, static_cast<int32_t>(num_positions), positions,
      slot_mapping, static_cast<int32_t>(num_tokens), static_cast<int32_t>(num_heads),
      static_cast<int32_t>(num_kv_heads), static_cast<int32_t>(head_dim), query_out, key_pool,
      value_pool, num_blocks * block_size, dtype == BS_BF16, pool_dtype == BS_BF16, d->sms,
      status, static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "rope_append launch");
  count_launches(1);
  return BS_OK;
}

int bs_silu_mul(const void* gate_up, int64_t row_stride, int64_t num_tokens, int64_t intermediate,
                int32_t dtype, void* out, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK(num_tokens >= 0 && num_tokens <= kInt32Max && intermediate > 0 &&
               intermediate <= kInt32Max,
           "sizes out of range");
  BS_CHECK(row_stride >= 2 * intermediate, "rows must hold gate and up");
  if (num_tokens == 0) return BS_OK;
  BS_CHECK(gate_up && out, "null pointer argument");
  DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  const bool vec = intermediate % 8 == 0 && row_stride % 8 == 0 && aligned16(gate_up) &&
                   aligned16(out);
  const int rc = bsb::launch_silu_mul(gate_up, row_stride, static_cast<int32_t>(num_tokens),
                                      static_cast<int32_t>(intermediate), out, dtype == BS_BF16,
                                      vec, d->sms, static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "silu_mul launch");
  count_launches(1);
  return BS_OK;
}

int bs_argmax_rows(const void* logits, int64_t row_stride, int64_t rows, int64_t cols,
                   int32_t dtype, int32_t* out, void* stream) {
  BS_CHECK(dtype == BS_BF16 || dtype == BS_F32, "dtype must be bfloat16 or float32");
  BS_CHECK(rows >= 0 && rows <= kInt32Max && cols > 0 && cols <= kInt32Max,
           "rows or cols out of range");
  BS_CHECK(row_stride >= cols, "row stride must cover cols");
  if (rows == 0) return BS_OK;
  BS_CHECK(logits && out, "null pointer argument");
  const bool vec = cols % 8 == 0 && row_stride % 8 == 0 && aligned16(logits);
  const int rc = bsb::launch_argmax_rows(logits, row_stride, static_cast<int32_t>(rows), cols, out,
                                         dtype == BS_BF16, vec, static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "argmax launch");
  count_launches(1);
  return BS_OK;
}

int bs_reshape_and_cache(const void* key, const void* value, int64_t key_token_stride,
                         int64_t value_token_stride, int32_t input_dtype,
                         const int32_t* slot_mapping, int64_t num_tokens, void* key_pool,
                         void* value_pool, int32_t pool_dtype, int64_t num_kv_heads,
                         int64_t num_blocks, int64_t block_size, int64_t head_dim,
                         uint32_t* status, void* stream) {
  BS_CHECK(input_dtype == BS_BF16 || input_dtype == BS_F32, "input dtype must be bf16 or fp32");
  BS_CHECK(pool_dtype == BS_BF16 || pool_dtype == BS_F32, "pool dtype must be bf16 or fp32");
  BS_CHECK(num_tokens >= 0 && num_tokens <= kInt32Max, "num_tokens out of range");
  BS_CHECK(num_kv_heads > 0 && num_blocks > 0 && block_size > 0 && head_dim > 0,
           "sizes must be positive");
  BS_CHECK(key_token_stride >= num_kv_heads * head_dim &&
               value_token_stride >= num_kv_heads * head_dim,
           "token strides must cover kv_heads * head_dim");
  const int64_t pool_slots = num_blocks * block_size;
  if (num_kv_heads * pool_slots > kInt32Max * 64ll) {
    return fail(BS_ERR_UNSUPPORTED, "pool too large");
  }
  if (num_tokens == 0) return BS_OK;
  BS_CHECK(key && value && slot_mapping && key_pool && value_pool, "null pointer argument");
  const int in_sz = dtype_size(input_dtype), pool_sz = dtype_size(pool_dtype);
  const bool vec = head_dim % 8 == 0 && aligned16(key) && aligned16(value) &&
                   aligned16(key_pool) && aligned16(value_pool) &&
                   (key_token_stride * in_sz) % 16 == 0 && (value_token_stride * in_sz) % 16 == 0 &&
                   (head_dim * pool_sz) % 16 == 0;
  DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  const int rc = bsb::launch_slot_write(
      key, value, key_token_stride, value_token_stride, input_dtype == BS_BF16, slot_mapping,
      static_cast<int32_t>(num_tokens), static_cast<int32_t>(num_kv_heads),
      static_cast<int32_t>(head_dim), key_pool, value_pool, pool_dtype == BS_BF16, pool_slots, vec,
      d->sms, status, static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "slot write launch");
  count_launches(1);
  return BS_OK;
}

int bs_step_metadata(const int32_t* seq_rows, const int32_t* start_pos, const int32_t* n_new,
                     int64_t num_rows, const int32_t* block_tables, int64_t table_stride,
                     int64_t table_rows, int64_t max_blocks_per_seq, int64_t block_size,
                     int64_t num_blocks, int64_t num_tokens, int32_t* cu_q, int32_t* positions,
                     int32_t* slot_mapping, int32_t* context_lens, uint32_t* status,
                     void* stream) {
  BS_CHECK(num_rows >= 0 && num_rows <= bsb::max_metadata_rows(), "num_rows must be in [0, %d]",
           bsb::max_metadata_rows());
  BS_CHECK(num_tokens >= 0 && num_tokens <= kInt32Max, "num_tokens out of range");
  BS_CHECK(block_size > 0 && num_blocks > 0 && num_blocks * block_size <= kInt32Max,
           "pool slots must fit in int32");
  BS_CHECK(max_blocks_per_seq > 0 && max_blocks_per_seq <= table_stride,
           "max_blocks_per_seq must be in [1, table_stride]");
  BS_CHECK(table_rows > 0 && table_rows <= kInt32Max, "table_rows out of range");
  if (num_rows == 0) return BS_OK;
  BS_CHECK(start_pos && n_new && block_tables && cu_q && context_lens, "null pointer argument");
  BS_CHECK(num_tokens == 0 || (positions && slot_mapping), "null pointer argument");
  const int rc = bsb::launch_step_metadata(
      seq_rows, start_pos, n_new, static_cast<int32_t>(num_rows), block_tables, table_stride,
      static_cast<int32_t>(table_rows), static_cast<int32_t>(max_blocks_per_seq),
      static_cast<int32_t>(block_size), static_cast<int32_t>(num_blocks),
      static_cast<int32_t>(num_tokens), cu_q, positions, slot_mapping, context_lens, status,
      static_cast<cudaStream_t>(stream));
  if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "metadata kernel launch");
  count_launches(1);
  return BS_OK;
}

int bs_take_status(void* workspace, void* stream, uint32_t* status_out) {
  BS_CHECK(workspace != nullptr, "workspace is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t bits = 0;
  cudaError_t e = cudaMemcpyAsync(&bits, workspace, sizeof(bits), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && bits != 0) e = cudaMemsetAsync(workspace, 0, sizeof(bits), st);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  if (status_out != nullptr) *status_out = bits;
  if (bits == 0) return BS_OK;
  std::string msg = "device reported:";
  if (bits & BS_STATUS_BAD_BLOCK) msg += " block table entry out of range;";
  if (bits & BS_STATUS_BAD_LENGTH) msg += " context length out of range;";
  if (bits & BS_STATUS_WAIT_TIMEOUT) msg += " pipeline wait timed out;";
  if (bits & BS_STATUS_BAD_SLOT) msg += " slot outside the pool;";
  if (bits & BS_STATUS_BAD_ROW) msg += " sequence row outside the block tables;";
  if (bits & BS_STATUS_BAD_POSITION) msg += " position outside the rotary tables;";
  if (bits & BS_STATUS_BAD_INDEX) msg += " gathered row index out of range;";
  g_error = msg;
  return BS_ERR_DEVICE;
}

int bs_reset_workspace(void* workspace, void* stream) {
  BS_CHECK(workspace != nullptr, "workspace is null");
  const cudaError_t e = cudaMemsetAsync(workspace, 0,
                                        static_cast<size_t>(ws_layout(0, 0, 0, 0).staging),
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "clearing the workspace counters");
  return BS_OK;
}

int bs_set_wait_probe(int32_t unarmed, uint64_t wait_limit_ns) {
  g_wait_limit_ns.store(wait_limit_ns);
  g_probe_unarmed.store(unarmed != 0 ? 1 : 0);
  return BS_OK;
}

}  // extern "C"

namespace bsb {
// Lets other translation units of the library report through bs_last_error().
void set_last_error(const char* message) { g_error = message; }

void apply_wait_probe(DecodeArgs& a) {
  a.wait_limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  a.probe_unarmed = g_probe_unarmed.load(std::memory_order_relaxed);
}

// The decode grid and kernel choice of the workspace entry points, shared with
// the allocation-free one (noalloc.cu) so the two cannot drift apart.
bool decode_uses_mma(int32_t dtype, int64_t block_size, int64_t head_dim, int64_t groups) {
  return use_mma_path(dtype, block_size, head_dim, groups);
}
int decode_grid_for(bool mma, int32_t dtype, int64_t head_dim, int64_t groups, int* grid) {
  return decode_grid(mma, dtype, head_dim, groups, grid);
}
int32_t decode_record_stride(int64_t groups, int64_t head_dim) {
  return record_stride(groups, head_dim);
}
void add_kernel_launches(int n) { count_launches(n); }
}  // namespace bsb
