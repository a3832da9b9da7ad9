/*
 * batchstream_b200 — C ABI of the B200 paged-attention path of the BatchStream
 * inference engine.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed
 * as `void*`, returns BS_OK (0) or an error code, and never throws.  On error,
 * bs_last_error() returns a message for the calling thread; a binding raises it
 * as the reference's RuntimeError.  Nothing here allocates device memory: a call
 * that needs scratch space takes a caller-provided `workspace` whose size comes
 * from the matching *_workspace_bytes() query.  A workspace must be zero-filled
 * once, when it is first allocated: its first 256 KiB + 256 bytes hold the
 * status word and per-segment counters, which every call leaves at zero again;
 * the rest is scratch.  Any sequence of calls (any batch size, single-sequence
 * and batched) may share one workspace, one call at a time.
 *
 * Layouts (row-major, elements):
 *   query     [num_seqs, num_heads, head_dim], heads of a sequence contiguous
 *   key/value pool of one layer [num_kv_heads, num_blocks, block_size, head_dim],
 *             contiguous — the reference's PagedKVPool layer view
 *             (src/server/torch_model.py:120-122)
 *   block tables  int32 [rows, table_stride]; context lengths int32 [num_seqs]
 *
 * Device-side problems (a table entry out of range, a bad length or slot) never
 * fault: the kernels skip the access and set a bit in the status word at byte 0 of
 * the workspace; bs_take_status() reads and clears it.
 */
#ifndef BATCHSTREAM_B200_H_
#define BATCHSTREAM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum bs_dtype { BS_BF16 = 0, BS_F32 = 1 };

enum bs_error {
  BS_OK = 0,
  BS_ERR_INVALID = 1,     /* malformed input: the reference's TORCH_CHECK cases */
  BS_ERR_UNSUPPORTED = 2, /* valid but outside this library's limits */
  BS_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  BS_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  BS_ERR_DEVICE = 5       /* a kernel reported a status bit (bs_take_status) */
};

/* Status bits reported by kernels (see bs_take_status). */
#define BS_STATUS_BAD_BLOCK 0x1u
#define BS_STATUS_BAD_LENGTH 0x2u
#define BS_STATUS_WAIT_TIMEOUT 0x4u
#define BS_STATUS_BAD_SLOT 0x8u
#define BS_STATUS_BAD_ROW 0x10u
#define BS_STATUS_BAD_POSITION 0x20u
#define BS_STATUS_BAD_INDEX 0x40u

/* Message of the last failing call on this thread ("" if none). */
const char* bs_last_error(void);

/*
 * Kernels this library has launched in this process (each successful entry
 * adds the kernels it enqueued, e.g. 2 for a tensor-core decode with its merge
 * pass).  A launch recorded into a CUDA graph counts once at capture.
 */
uint64_t bs_kernel_launches(void);

/* Library version string. */
const char* bs_version(void);

/*
 * Single-sequence decode attention, the drop-in for the reference op
 *   paged_attention(query, keys, values, block_table, length, block_size,
 *                   groups, scaling) -> Tensor[heads, head_dim]
 * (csrc/paged_attention.cpp:76-105, bound at :109-111; Python twin
 * src/server/torch_model.py:67-80).  Shapes and strides are passed so that the
 * same sixteen input checks run here (paged_attention.cpp:22-44); the query must
 * already be contiguous (the reference copies it, paged_attention.cpp:81).
 * Unlike the reference, float32 is accepted when query, keys and values are all
 * float32.  `block_table` is host memory (the reference's list[int]); the table
 * is validated on the host and staged through the workspace.  `output` is
 * [heads, head_dim] contiguous in the query dtype.
 */
int bs_paged_attention(const void* query, int32_t query_dtype, int32_t query_ndim,
                       const int64_t* query_shape, const int64_t* query_strides,
                       const void* keys, int32_t keys_dtype, int32_t keys_ndim,
                       const int64_t* keys_shape, const int64_t* keys_strides,
                       const void* values, int32_t values_dtype, int32_t values_ndim,
                       const int64_t* values_shape, const int64_t* values_strides,
                       const int64_t* block_table, int64_t block_table_len, int64_t length,
                       int64_t block_size, int64_t groups, double scaling, void* output,
                       void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * The sixteen input checks of bs_paged_attention alone (the reference's
 * check_inputs, csrc/paged_attention.cpp:22-44), touching no memory but the
 * shape, stride and table arrays: BS_OK or BS_ERR_INVALID with the message
 * bs_paged_attention would give.  A binding that receives the reference's host
 * tensors validates them with this before staging them on the device.
 */
int bs_paged_attention_check(int32_t query_dtype, int32_t query_ndim, const int64_t* query_shape,
                             const int64_t* query_strides, int32_t keys_dtype, int32_t keys_ndim,
                             const int64_t* keys_shape, const int64_t* keys_strides,
                             int32_t values_dtype, int32_t values_ndim,
                             const int64_t* values_shape, const int64_t* values_strides,
                             const int64_t* block_table, int64_t block_table_len, int64_t length,
                             int64_t block_size, int64_t groups);

/* Workspace bytes bs_paged_attention needs for this shape (current device). */
int bs_paged_attention_workspace_bytes(int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                       int64_t block_table_len, int32_t dtype,
                                       int64_t block_size, uint64_t* bytes_out);

/*
 * Batched ragged decode attention: one new token per sequence, all sequences of
 * a step in one launch.  Replaces the per-sequence loop of op calls in
 * TorchModel._attention (src/server/torch_model.py:268-270 -> PagedKVCache.attend
 * :155-164).  Sequence b attends over context_lens[b] tokens whose blocks are
 * block_tables[seq_rows ? seq_rows[b] : b][0 .. ceil(len / block_size)).
 * context_lens[b] == 0 marks a padding row (fixed-size batches, CUDA graphs):
 * nothing is read for it and its output row is not written; a negative length,
 * one past the table row or a bad row sets a status bit.
 * `units_hint` is the total number of (kv head, block) pairs of the batch if the
 * caller knows it, else 0; it only sizes the grid.  `flags` may hold
 * BS_LENS_READY: context_lens, block_tables and seq_rows were final before the
 * kernel launched just ahead of this call on the stream, so the kernel's span
 * search may overlap that kernel (query and pools are always read after it).
 */
#define BS_LENS_READY 0x1
/* With BS_LENS_READY: the kernel launched just ahead wrote nothing this call
 * reads except, at most, each sequence's last pool block (a decode append or
 * slot write of the step's new token), so every other block and the query
 * may be read before it finishes. */
#define BS_AFTER_APPEND 0x2
int bs_paged_attention_batched(const void* query, int64_t query_seq_stride, const void* key_pool,
                               const void* value_pool, const int32_t* block_tables,
                               int64_t table_stride, int64_t table_rows, const int32_t* seq_rows,
                               const int32_t* context_lens, int64_t num_seqs, int64_t num_heads,
                               int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                               int64_t num_blocks, int64_t max_blocks_per_seq, int32_t dtype,
                               double scaling, int64_t units_hint, int32_t flags, void* output,
                               int64_t output_seq_stride, void* workspace,
                               uint64_t workspace_bytes, void* stream);

/*
 * Allocation-free form of bs_paged_attention_batched.  It has no counterpart in
 * the reference (whose op allocates its scratch on the host heap); it exists for
 * callers that cannot allocate device memory where they run attention — a host
 * whose device memory already belongs to a fixed pool, an FFI caller without an
 * allocator of its own, a step that must not block on an allocation.  Its
 * scratch is one static device array of 8 MiB per GPU, present from the moment
 * the library's kernels load on that GPU until the process exits.  Limit: at
 * most 16384 (sequence, kv head) pairs per call; a larger call fails with
 * BS_ERR_UNSUPPORTED and a message.  Shapes whose partial records for the
 * regular grid would not fit the array run on fewer CTAs.  The first call on
 * each GPU finds the array's device address and clears it (synchronising that
 * GPU once), so make that first call before capturing a stream.  All calls share
 * the array: calls that overlap on the GPU race, so serialise them.  Kernel-side
 * problems (bad table entry, length or row, a wait that gave up) are OR-ed into
 * *device_status, a device word the caller zeroes and reads; it must not be
 * NULL (BS_ERR_INVALID), since nothing else would report them.
 */
int bs_paged_attention_batched_noalloc(const void* query, int64_t query_seq_stride,
                                       const void* key_pool, const void* value_pool,
                                       const int32_t* block_tables, int64_t table_stride,
                                       int64_t table_rows, const int32_t* seq_rows,
                                       const int32_t* context_lens, int64_t num_seqs,
                                       int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                       int64_t block_size, int64_t num_blocks,
                                       int64_t max_blocks_per_seq, int32_t dtype, double scaling,
                                       void* output, int64_t output_seq_stride,
                                       uint32_t* device_status, void* stream);

int bs_paged_attention_batched_workspace_bytes(int64_t num_seqs, int64_t num_heads,
                                               int64_t num_kv_heads, int64_t head_dim,
                                               int64_t block_size, int32_t dtype,
                                               uint64_t* bytes_out);

/*
 * Chunked-prefill attention for a ragged batch of prompt chunks, the batched
 * form of PagedKVCache.attend's multi-token branch (_read_blocks + attend with
 * _causal_mask, src/server/torch_model.py:39-64, 165-167, 295-297).  Chunk r has
 * query tokens cu_q[r] .. cu_q[r+1] (rows of `query` [num_tokens, num_heads,
 * head_dim]); its sequence holds context_lens[r] tokens after the chunk was
 * written to the pool (the chunk's own K/V included), so query token i attends
 * to keys 0 .. context_lens[r] - n + i.  bf16 with head_dim 64 and block size 16
 * runs on the tcgen05 tensor cores (one CTA per chunk, head and 128-token tile;
 * `max_query_len` bounds n); every other case, or BS_PREFILL_PER_TOKEN, runs
 * each query token as a decode query over its own causal length.
 */
#define BS_PREFILL_PER_TOKEN 0x2
int bs_prefill_attention(const void* query, int64_t query_token_stride, const int32_t* cu_q,
                         int64_t num_rows, int64_t num_tokens, int64_t max_query_len,
                         const int32_t* context_lens, const int32_t* seq_rows,
                         const void* key_pool, const void* value_pool,
                         const int32_t* block_tables, int64_t table_stride, int64_t table_rows,
                         int64_t max_blocks_per_seq, int64_t num_heads, int64_t num_kv_heads,
                         int64_t head_dim, int64_t block_size, int64_t num_blocks, int32_t dtype,
                         double scaling, int32_t flags, void* output, int64_t output_token_stride,
                         void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Workspace for bs_prefill_attention over num_tokens tokens in num_rows chunks
 * of at most max_query_len tokens.  On the tensor-core path a small batch of
 * chunks (fewer query tiles than SMs, counting the at most
 * ceil(num_tokens / 128) + num_rows per head that can hold tokens) splits
 * each tile's key range over up to 4 CTAs whose partial results a second
 * kernel merges, and a batch of more than one wave of CTAs is ranked first
 * (query tiles with the most keys start first): inside every CTA for up to 192
 * (chunk, query tile) pairs, by a planning kernel launched ahead for more.  The split records and the plan
 * live in this workspace; a smaller one only turns them off.
 */
int bs_prefill_attention_workspace_bytes(int64_t num_tokens, int64_t num_rows,
                                         int64_t max_query_len, int64_t num_heads,
                                         int64_t num_kv_heads, int64_t head_dim,
                                         int64_t block_size, int32_t dtype, uint64_t* bytes_out);

/*
 * K/V slot write: key/value rows [num_tokens, num_kv_heads, head_dim] (token
 * stride in elements, heads contiguous) go to pool[h, slot / bs, slot % bs, :].
 * Replaces PagedKVCache.append's per-token indexed stores
 * (src/server/torch_model.py:149-153 with BlockAllocator.locate,
 * src/server/block_allocator.py:28-30).  A negative slot is skipped.  `status`
 * is a device uint32 word (may be NULL) that gets BS_STATUS_BAD_SLOT for a slot
 * beyond the pool.
 */
int bs_reshape_and_cache(const void* key, const void* value, int64_t key_token_stride,
                         int64_t value_token_stride, int32_t input_dtype,
                         const int32_t* slot_mapping, int64_t num_tokens, void* key_pool,
                         void* value_pool, int32_t pool_dtype, int64_t num_kv_heads,
                         int64_t num_blocks, int64_t block_size, int64_t head_dim,
                         uint32_t* status, void* stream);

/*
 * One decode step's K/V append: row r (block-table row seq_rows[r], or r when
 * null) gains one token at position start_pos[r].  Locates its slot through
 * the block table (BlockAllocator.locate, src/server/block_allocator.py:28-30),
 * writes key[r] / value[r] ([num_kv_heads, head_dim], row strides in elements)
 * into pool[h, slot / bs, slot % bs] (PagedKVCache.append,
 * src/server/torch_model.py:149-153), and writes context_lens[r] =
 * start_pos[r] + 1 and slot_mapping[r].  The fused form of bs_step_metadata +
 * bs_reshape_and_cache for steps in which every row decodes one token; a
 * table entry outside the pool or a bad row sets a status bit and skips the row.
 * A row with start_pos < 0 is padding (fixed-size batches, CUDA graphs):
 * nothing is written, context_lens = 0 and slot_mapping = -1.  With key and
 * value both NULL only context_lens and slot_mapping are written (the slots
 * for a later bs_rope_append, which then writes the rows).
 */
int bs_decode_append(const int32_t* seq_rows, const int32_t* start_pos, int64_t num_rows,
                     const int32_t* block_tables, int64_t table_stride, int64_t table_rows,
                     int64_t max_blocks_per_seq, const void* key, const void* value,
                     int64_t key_row_stride, int64_t value_row_stride, int32_t input_dtype,
                     void* key_pool, void* value_pool, int32_t pool_dtype, int64_t num_kv_heads,
                     int64_t num_blocks, int64_t block_size, int64_t head_dim,
                     int32_t* context_lens, int32_t* slot_mapping, uint32_t* status,
                     void* stream);

/*
 * Step metadata on the device for a ragged batch of `num_rows` rows with
 * n_new[r] new tokens after start_pos[r] cached ones (the reference builds these
 * on the host in TorchModel._hidden_states, src/server/torch_model.py:231-241,
 * and per token through BlockAllocator.locate).  Writes cu_q[num_rows + 1],
 * positions[num_tokens], slot_mapping[num_tokens] and
 * context_lens[num_rows] = start_pos + n_new.  num_tokens is normally
 * sum(n_new); tokens past the last row, and the tokens of a padding row
 * (start_pos < 0, context length 0), get position 0 and slot -1, so a
 * fixed-size (graph-captured) step can carry padding.
 */
int bs_step_metadata(const int32_t* seq_rows, const int32_t* start_pos, const int32_t* n_new,
                     int64_t num_rows, const int32_t* block_tables, int64_t table_stride,
                     int64_t table_rows, int64_t max_blocks_per_seq, int64_t block_size,
                     int64_t num_blocks, int64_t num_tokens, int32_t* cu_q, int32_t* positions,
                     int32_t* slot_mapping, int32_t* context_lens, uint32_t* status,
                     void* stream);

/*
 * Fused model steps around the attention path, used by the engine's model
 * step (each replaces a chain of framework ops of the reference TorchModel,
 * src/server/torch_model.py, with its rounding points; dtype is the model's):
 *  - bs_rms_norm:    per output row r with source row i = row_index[r] (or r):
 *                    s = (x[i] + add[i]).to(dtype) (s = x[i] when add is NULL),
 *                    sum_out[r] = s (when not NULL), and
 *                    out[r] = weight * (s_f32 * rsqrt(mean(s_f32^2) + eps)).to(dtype)
 *                    (:283-287, with the residual add of :272/:281 before it).
 *                    sum_out may be x itself only without row_index; an index
 *                    outside [0, x_rows) skips the row and sets
 *                    BS_STATUS_BAD_INDEX in *status.
 *  - bs_rope_append: rows of qkv = [q heads | k heads | v heads] after the
 *                    projection; q and k rotated with cos/sin tables [pos, D]
 *                    (rotate_half RoPE, :190-192, :262-264), q written to
 *                    query_out [T, H, D], k and v to the pools
 *                    [kv_heads, num_blocks, block_size, D] at slot_mapping
 *                    (slots < 0 skipped) — PagedKVCache.append (:149-153).
 *                    Tables hold num_positions rows; a position outside them
 *                    or a slot past the pool skips the access and sets
 *                    BS_STATUS_BAD_POSITION / BS_STATUS_BAD_SLOT in *status.
 *  - bs_silu_mul:    out[t, i] = silu(gate[t, i]) * up[t, i], rows [gate | up]
 *                    (:278-281).
 */
int bs_rms_norm(const void* x, int64_t x_row_stride, int64_t x_rows, const void* add,
                int64_t add_row_stride, const int32_t* row_index, const void* weight, int64_t rows,
                int64_t hidden, double eps, int32_t dtype, void* out, int64_t out_row_stride,
                void* sum_out, int64_t sum_row_stride, uint32_t* status, void* stream);
int bs_rope_append(const void* qkv, int64_t qkv_row_stride, int32_t dtype, const void* cos_table,
                   const void* sin_table, int64_t num_positions, const int32_t* positions,
                   const int32_t* slot_mapping, int64_t num_tokens, int64_t num_heads,
                   int64_t num_kv_heads, int64_t head_dim, void* query_out, void* key_pool,
                   void* value_pool, int32_t pool_dtype, int64_t num_blocks, int64_t block_size,
                   uint32_t* status, void* stream);
int bs_silu_mul(const void* gate_up, int64_t row_stride, int64_t num_tokens, int64_t intermediate,
                int32_t dtype, void* out, void* stream);
/*
 * Greedy token of each logits row (backend/paged.py:95-99, on the device):
 * out[r] = the first index of the row's maximum, a NaN counting as the maximum
 * (torch.argmax's rule), over `cols` entries.
 */
int bs_argmax_rows(const void* logits, int64_t row_stride, int64_t rows, int64_t cols,
                   int32_t dtype, int32_t* out, void* stream);

/*
 * Waits for `stream`, then reads and clears the status word at the start of a
 * workspace.  Returns BS_ERR_DEVICE (with a message naming the bits) when any
 * bit was set, BS_OK otherwise; *status_out gets the bits.
 */
int bs_take_status(void* workspace, void* stream, uint32_t* status_out);

/*
 * Zero-fills the status word and the per-segment counters of a workspace (its
 * first 256 KiB + 256 bytes) on `stream`.  A launch that reported a problem
 * (any status bit) may have stopped short of the work that returns the
 * counters to zero; call this after such a launch before the workspace is used
 * again.  No counterpart in the reference, whose op keeps no state between
 * calls.
 */
int bs_reset_workspace(void* workspace, void* stream);

/*
 * Test hook of the bounded-wait error path; no counterpart in the reference.
 * Sets, for every later decode launch of this process, the limit of each
 * pipeline wait of the tensor-core decode kernel (0 restores the default of
 * about 2 s) and, when `unarmed` is non-zero, makes one warp of that kernel wait
 * on stages that nothing fills, so the wait runs out with no copy in flight: the
 * launch then sets BS_STATUS_WAIT_TIMEOUT and finishes without faulting.  Never
 * set outside tests.
 */
int bs_set_wait_probe(int32_t unarmed, uint64_t wait_limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* BATCHSTREAM_B200_H_ */
