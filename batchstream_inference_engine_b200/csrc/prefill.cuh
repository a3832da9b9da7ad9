// Chunked-prefill attention: arguments shared by the tensor-core kernel
// (prefill.cu) and the C ABI (capi.cu).
#pragma once

#include "common.cuh"

namespace bsb {

struct PrefillArgs {
  const void* q;  // [T, H, D] bf16, heads of a token contiguous
  void* out;      // [T, H, D] bf16 (token stride o_stride_tok elements)
  int64_t o_stride_tok;
  const int32_t* cu_q;          // [R + 1] token offsets of the chunks
  const int32_t* context_lens;  // [R] cached tokens after the chunk (prior + n)
  const int32_t* seq_rows;      // [R] block-table row (may be null: row r)
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t bt_rows, max_blocks;
  int32_t num_rows, num_heads, num_kv_heads, groups, num_blocks, qtiles;
  float scale;
  // Non-zero when scale is a power of two: bf16(bf16(q.k) * scale) then equals
  // bf16(q.k) * scale exactly and the second rounding is skipped.
  int32_t exact_scale;
  uint32_t* status;
  // Split-KV: each query tile's key tiles are cut into up to `splits` ranges
  // of at least kMinSplitTiles tiles, one CTA each; with more than one, every
  // CTA writes its unnormalised O [128][64] (part_o) and per-row (max, sum)
  // (part_ml, max in base-2 units) for prefill_merge_kernel, else the output.
  int32_t splits;
  float* part_o;
  float* part_ml;
  // Work order (may be null), written by prefill_plan_kernel just ahead of the
  // prefill kernel: plan[0] = {entries E, 0, 0, 0}; entry d, run by CTAs
  // d * H .. d * H + H - 1 (one per query head), is
  //   plan[1 + 2d] = {rt * splits + piece, first token, query tokens, context}
  //   plan[2 + 2d] = {block-table row, 0, 0, 0}
  // with rt the (row, query tile) index of the plan-less numbering.  Entries are
  // ranked by key tiles, most first: when the grid is more than one wave of
  // resident CTAs, the longest ranges then start in the first.
  int4* plan;
  // Non-zero (with plan null and splits 1, for at most kMaxCtaRankedRts rows x
  // query tiles): every CTA ranks the (row, query tile) pairs itself, in the
  // plan kernel's order, and takes entry b / H; no plan launch ahead.
  int32_t rank_in_cta;
};

// Rows x query tiles a prefill CTA ranks itself (one per thread).
constexpr int kMaxCtaRankedRts = 192;

constexpr int kMinSplitTiles = 4;
constexpr int kMaxPrefillSplits = 4;
// Largest plan ranked in one CTA (entries = rows x query tiles x splits).
constexpr int kMaxPlanEntries = 1024;

// Ranges a query tile with `ntiles` key tiles is cut into.
__host__ __device__ __forceinline__ int prefill_tile_splits(int ntiles, int splits) {
  const int by_size = (ntiles + kMinSplitTiles - 1) / kMinSplitTiles;
  return by_size < splits ? (by_size > 0 ? by_size : 1) : splits;
}

int prefill_smem_bytes();
// Record floats per split CTA (O rows, then (max, sum) per row).
constexpr int64_t kPrefillRecordO = 128 * 64;
constexpr int64_t kPrefillRecordML = 128 * 2;
int launch_prefill_merge(const PrefillArgs& a, int64_t items, cudaStream_t stream);
int launch_prefill_plan(const PrefillArgs& a, cudaStream_t stream);
int prefill_ctas_per_sm();
int launch_prefill_tc(const PrefillArgs& a, const CUtensorMap& qmap, const CUtensorMap& kmap,
                      const CUtensorMap& vmap, int grid, cudaStream_t stream);

// Per-token decode view of prefill chunks: token t of chunk r becomes a query
// with context length (ctx[r] - n[r]) + i + 1 over block-table row rows[r].
int launch_expand_rows(const int32_t* cu_q, const int32_t* context_lens, const int32_t* seq_rows,
                       int32_t R, int32_t T, int32_t* token_lens, int32_t* token_rows,
                       cudaStream_t stream);

}  // namespace bsb
