// Batched decode attention that allocates nothing.
//
// The regular batched entry point (bs_paged_attention_batched) needs a scratch
// workspace that the caller allocates.  Some callers cannot do that at the point
// where they run attention: a host that has already handed the whole device to a
// fixed-size memory pool, an embedding whose only allocator is not reachable
// from the code calling us (a plain C or FFI host without torch), or a context
// where allocation is forbidden because a device allocation could block or
// fail unpredictably (a real-time step, a callback).  For them this file keeps
// the decode's scratch in one statically sized device array that exists once per
// GPU as soon as the library's kernels are loaded on it, and is never freed
// before the process exits.
//
// Limits: at most kMaxSegments (sequence, kv head) pairs per call (bigger calls
// are rejected with an error message) and kScratchBytes of scratch in total
// (status word, segment counters, two partial records per CTA: a shape whose
// records for the regular grid do not fit runs on fewer CTAs).  Every call uses the same array, so calls that overlap on the GPU
// (two streams, two threads) race and must be serialised by the caller.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/batchstream_b200.h"
#include "decode.cuh"

namespace bsb {
// capi.cu: messages, launch count and the workspace entry points' choice of
// kernel and grid, which this entry point shares.
void set_last_error(const char* message);
void add_kernel_launches(int n);
bool decode_uses_mma(int32_t dtype, int64_t block_size, int64_t head_dim, int64_t groups);
int decode_grid_for(bool mma, int32_t dtype, int64_t head_dim, int64_t groups, int* grid);
int32_t decode_record_stride(int64_t groups, int64_t head_dim);
}  // namespace bsb

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
constexpr int64_t kMaxSegments = 16384;            // num_seqs * num_kv_heads per call
constexpr size_t kStatusBytes = 256;
constexpr size_t kCounterBytes = size_t(kMaxSegments) * 4;
constexpr size_t kRecordsOffset = kStatusBytes + kCounterBytes;

// The scratch itself.  In host code this name only stands for the symbol; the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// Messages go to the same per-thread slot as every other entry point, so
// bs_last_error() reports them.
int noalloc_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  bsb::set_last_error(buf);
  return code;
}

struct DeviceScratch {
  uint8_t* base = nullptr;  // device address of g_noalloc_scratch on that GPU
};

std::mutex g_mu;
std::vector<DeviceScratch> g_dev;

// One-time set-up on the current device: find the array's device address and
// zero the status word and the counters (every finished call leaves the
// counters at zero again).  Done by the first call on each GPU.
int scratch_for_current_device(DeviceScratch** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(BS_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_mu);
  if (static_cast<int>(g_dev.size()) <= dev) g_dev.resize(dev + 1);
  DeviceScratch& d = g_dev[dev];
  if (d.base == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      return noalloc_fail(BS_ERR_CUDA, "cudaGetSymbolAddress of the scratch array: %s",
                          cudaGetErrorString(e));
    }
    e = cudaMemset(p, 0, kRecordsOffset);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      return noalloc_fail(BS_ERR_CUDA, "clearing the scratch array: %s", cudaGetErrorString(e));
    }
    d.base = static_cast<uint8_t*>(p);
  }
  *out = &d;
  return BS_OK;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows, head_dim] bf16 view of a pool in 16 x 64 boxes with 128-byte swizzle,
// the layout the tensor-core decode kernel reads.
int pool_map(CUtensorMap* map, const void* base, int64_t rows, int64_t head_dim) {
  static EncodeFn encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      encode = reinterpret_cast<EncodeFn>(p);
    }
  });
  if (encode == nullptr) return noalloc_fail(BS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(head_dim * 2)};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t elem[2] = {1, 1};
  const CUresult r =
      encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return noalloc_fail(BS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", r);
  return BS_OK;
}

bool is_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int bs_paged_attention_batched_noalloc(
    const void* query, int64_t query_seq_stride, const void* key_pool, const void* value_pool,
    const int32_t* block_tables, int64_t table_stride, int64_t table_rows,
    const int32_t* seq_rows, const int32_t* context_lens, int64_t num_seqs, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t block_size, int64_t num_blocks,
    int64_t max_blocks_per_seq, int32_t dtype, double scaling, void* output,
    int64_t output_seq_stride, uint32_t* device_status, void* stream) {
  const int64_t i32max = 2147483647ll;
  if (dtype != BS_BF16 && dtype != BS_F32) {
    return noalloc_fail(BS_ERR_INVALID, "dtype must be bfloat16 or float32");
  }
  if (num_seqs < 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0) {
    return noalloc_fail(BS_ERR_INVALID, "heads must equal kv_heads * groups, num_seqs >= 0");
  }
  if (head_dim <= 0 || block_size <= 0 || num_blocks <= 0 || table_rows <= 0 ||
      max_blocks_per_seq <= 0 || max_blocks_per_seq > table_stride || table_rows > i32max) {
    return noalloc_fail(BS_ERR_INVALID, "sizes must be positive and fit the block table");
  }
  if (query_seq_stride < num_heads * head_dim || output_seq_stride < num_heads * head_dim) {
    return noalloc_fail(BS_ERR_INVALID, "sequence strides must cover heads * head_dim");
  }
  const int64_t groups = num_heads / num_kv_heads;
  if (head_dim > 256 || groups > 16) {
    return noalloc_fail(BS_ERR_UNSUPPORTED, "head_dim <= 256 and groups <= 16 are supported");
  }
  if (num_kv_heads * num_blocks * block_size > i32max ||
      max_blocks_per_seq * block_size > i32max) {
    return noalloc_fail(BS_ERR_UNSUPPORTED, "pool or table larger than 2^31 rows");
  }
  if (num_seqs * num_kv_heads > kMaxSegments) {
    return noalloc_fail(BS_ERR_UNSUPPORTED,
                        "num_seqs * num_kv_heads = %lld exceeds the %lld (sequence, kv head) "
                        "pairs the allocation-free entry point supports",
                        static_cast<long long>(num_seqs * num_kv_heads),
                        static_cast<long long>(kMaxSegments));
  }
  if (device_status == nullptr) {
    // The array's own status word has no reader: without the caller's word a
    // kernel-side problem would go unreported.
    return noalloc_fail(BS_ERR_INVALID, "device_status must point to a device word");
  }
  if (num_seqs == 0) return BS_OK;
  if (!query || !key_pool || !value_pool || !block_tables || !context_lens || !output) {
    return noalloc_fail(BS_ERR_INVALID, "null pointer argument");
  }
  const bool mma = bsb::decode_uses_mma(dtype, block_size, head_dim, groups);
  if (mma && (!is_aligned16(query) || !is_aligned16(key_pool) || !is_aligned16(value_pool) ||
              (query_seq_stride * 2) % 16 != 0)) {
    return noalloc_fail(BS_ERR_INVALID, "query, pools and query rows must be 16-byte aligned");
  }

  DeviceScratch* d = nullptr;
  if (int rc = scratch_for_current_device(&d)) return rc;
  // The same kernel and persistent grid as bs_paged_attention_batched.
  int grid = 0;
  if (int rc = bsb::decode_grid_for(mma, dtype, head_dim, groups, &grid)) return rc;
  const int64_t rec_stride = bsb::decode_record_stride(groups, head_dim);
  // Two partial records per CTA.  Where the persistent grid's records do not
  // fit the array, fewer CTAs run (the split points move; the answer does not).
  const size_t per_cta = size_t(2) * rec_stride * sizeof(float);
  const int64_t fit = static_cast<int64_t>((kScratchBytes - kRecordsOffset) / per_cta);
  if (fit < 1) {
    return noalloc_fail(BS_ERR_UNSUPPORTED,
                        "this shape needs %zu bytes of scratch per CTA; the allocation-free entry "
                        "point holds %zu",
                        kRecordsOffset + per_cta, kScratchBytes);
  }
  if (grid > fit) grid = static_cast<int>(fit);

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
  a.partials = reinterpret_cast<float*>(d->base + kRecordsOffset);
  a.rec_stride = static_cast<int32_t>(rec_stride);
  a.seg_counters = reinterpret_cast<int32_t*>(d->base + kStatusBytes);
  a.status = device_status;
  a.lens_ready = 0;
  bsb::apply_wait_probe(a);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (mma) {
    CUtensorMap kmap, vmap;
    const int64_t rows = num_kv_heads * num_blocks * block_size;
    if ((rc = pool_map(&kmap, key_pool, rows, head_dim))) return rc;
    if ((rc = pool_map(&vmap, value_pool, rows, head_dim))) return rc;
    rc = bsb::launch_decode_mma(a, kmap, vmap, grid, st);
  } else {
    rc = bsb::launch_decode_simt(a, dtype == BS_BF16, grid, st);
  }
  if (rc != 0) {
    return noalloc_fail(BS_ERR_CUDA, "decode kernel launch: %s",
                        cudaGetErrorString(static_cast<cudaError_t>(rc)));
  }
  bsb::add_kernel_launches(1);
  return BS_OK;
}
