/* C ABI of the B200 (sm_100a) paged-KV attention path of a looped
 * (recurrent-depth) transformer.
 *
 * Every entry point takes plain device pointers, element counts and element
 * strides (in elements, not bytes), launches on the given CUDA stream and
 * returns immediately: no host synchronisation, no allocation, so each call
 * can be captured into a CUDA graph. Scratch memory (split-KV partials) is
 * passed in by the caller; its size comes from the matching *_bytes query.
 *
 * Return value: RLT_OK (0), a negative RLT_E* code for an invalid argument
 * (nothing was launched), or a positive cudaError_t from the launch.
 *
 * Data layouts follow the reference engine (vllm_rlt):
 *   KV pool      [num_blocks, num_layers, page, num_kv_heads, head_dim]
 *                (vllm_rlt/core/kv_cache_manager.py:132-134); attention takes
 *                the layer view [num_blocks, page, num_kv_heads, head_dim]
 *                whose block stride is num_layers*page*num_kv_heads*head_dim.
 *   block tables int32 [rows, width], padded with -1 (or 0 in static buffers).
 *   lengths      int32 [rows], 0 for padding rows.
 *   q / out      [rows, num_q_heads, head_dim].
 * The last (head_dim) dimension of q, out, K and V must be contiguous.
 *
 * status (optional, may be NULL): an int32 device word that kernels OR error
 * bits into when metadata points outside the pool (RLT_STATUS_*). The bad
 * page/row is skipped instead of being dereferenced.
 */
#ifndef RLT_B200_H_
#define RLT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element type codes */
#define RLT_F32 0
#define RLT_F16 1
#define RLT_BF16 2

/* return codes */
#define RLT_OK 0
#define RLT_E_DTYPE -1
#define RLT_E_HEAD_DIM -2
#define RLT_E_HEADS -3
#define RLT_E_WORKSPACE -4
#define RLT_E_SHAPE -5
#define RLT_E_ALIGN -6
#define RLT_E_DEVICE -7
#define RLT_E_SCRATCH -8

/* status bits */
#define RLT_STATUS_BAD_LENGTH 1
#define RLT_STATUS_BAD_BLOCK 2
#define RLT_STATUS_BAD_OFFSET 4
#define RLT_STATUS_BAD_SLOT 8
#define RLT_STATUS_BAD_SEQUENCE 16
#define RLT_STATUS_TIMEOUT 32 /* a bounded wait inside a tensor-core kernel gave up */
#define RLT_STATUS_LAYOUT 64  /* a tensor-core kernel found its shared memory misaligned */

/* Library version (major*10000 + minor*100 + patch). */
int rlt_version(void);

/* Bytes of scratch rlt_paged_decode needs for this launch shape: int
 * metadata -- one merge counter per (row, query head), the rows + 1 work
 * schedule and a claim counter, all rebuilt on the stream by every call --
 * and fp32 split-KV partials (acc, running max, normaliser) for every row,
 * query head and split (a row of n tokens takes min(ceil(n/256), 128)
 * splits). 0 when no row can need more than one split. */
size_t rlt_paged_decode_workspace_bytes(int32_t num_rows, int32_t num_q_heads, int32_t head_dim,
                                        int32_t page_size, int32_t table_width);

/* Depth-aware paged decode attention: one query token per row, each row with
 * its own block table (the row's depth plane already selected by the caller),
 * GQA, fp32 softmax/accumulation, output in the input dtype.
 *   out[r, h] = softmax(q[r, h] . K[r, :len_r, h/g]^T * scale) V[r, :len_r, h/g]
 * with K[r, t] = key_cache[block_tables[r, t / page], t % page]; len_r = 0
 * rows produce zeros.
 * Replaces: vllm_rlt/kernels/triton_attention.py:100-125 (paged_attention,
 * Triton kernel :13-97), the FA4 decode call at
 * vllm_rlt/kernels/flash_attention.py:98-130, and the oracle
 * vllm_rlt/kernels/paged_attention.py:12-36 (torch_paged_attention). */
int rlt_paged_decode(const void* q, const void* key_cache, const void* value_cache,
                     const int32_t* block_tables, const int32_t* context_lengths, void* out,
                     void* workspace, size_t workspace_bytes, int32_t* status, int32_t dtype,
                     int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t page_size, int32_t table_width,
                     int64_t num_blocks, int64_t q_row_stride, int64_t q_head_stride,
                     int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride,
                     int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride,
                     int64_t table_row_stride, int64_t out_row_stride, int64_t out_head_stride,
                     float scale, void* stream);

/* rlt_paged_decode that also writes, per row and query head, the base-2
 * log-sum-exp of the scaled scores, lse[row * Hq + h] = max + log2(sum) in
 * units of scale * log2(e) (-inf for an empty row), so that attention over
 * disjoint token ranges can be merged exactly. lse must not be NULL. The
 * reference's torch path computes the same quantity inside its softmax
 * (vllm_rlt/kernels/paged_attention.py:12-36) without returning it. */
int rlt_paged_decode_lse(const void* q, const void* key_cache, const void* value_cache,
                         const int32_t* block_tables, const int32_t* context_lengths, void* out,
                         void* workspace, size_t workspace_bytes, int32_t* status, int32_t dtype,
                         int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t page_size, int32_t table_width,
                         int64_t num_blocks, int64_t q_row_stride, int64_t q_head_stride,
                         int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride,
                         int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride,
                         int64_t table_row_stride, int64_t out_row_stride,
                         int64_t out_head_stride, float scale, float* lse, void* stream);

/* Bytes of scratch rlt_paged_prefill needs: per-token (table row, causal
 * length) pairs plus the split-KV partials of the CUDA-core path. */
size_t rlt_paged_prefill_workspace_bytes(int32_t num_tokens, int32_t num_q_heads,
                                         int32_t head_dim, int32_t page_size,
                                         int32_t table_width);

/* Packed chunked-prefill paged causal attention with bottom-right alignment:
 * sequence s owns query tokens cu_seqlens_q[s] .. cu_seqlens_q[s+1]-1 and
 * keys 0 .. context_lengths[s]-1 through block_tables[s]; query i of the
 * chunk (0-based) sees keys up to context_lengths[s] - qlen_s + i.
 * The chunk's own K/V are already written to the pool (no gathering).
 * max_seqlen_q is accepted for interface parity and never shapes a launch.
 * Replaces: vllm_rlt/kernels/flash_attention.py:66-96
 * (FlashPagedAttention.prefill, FA4 flash_attn_varlen_func with page_table,
 * seqused_k, causal=True), called from vllm_rlt/core/kv_cache_manager.py:570-579. */
int rlt_paged_prefill(const void* q, const void* key_cache, const void* value_cache,
                      const int32_t* block_tables, const int32_t* context_lengths,
                      const int32_t* cu_seqlens_q, void* out, void* workspace,
                      size_t workspace_bytes, int32_t* status, int32_t dtype, int32_t num_tokens,
                      int32_t num_seqs, int32_t max_seqlen_q, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                      int32_t table_width, int64_t num_blocks, int64_t q_row_stride,
                      int64_t q_head_stride, int64_t k_block_stride, int64_t k_token_stride,
                      int64_t k_head_stride, int64_t v_block_stride, int64_t v_token_stride,
                      int64_t v_head_stride, int64_t table_row_stride, int64_t out_row_stride,
                      int64_t out_head_stride, float scale, void* stream);

/* 1 if rlt_paged_prefill runs this dtype/head_dim/page on the tcgen05
 * tensor-core kernel (bf16/fp16, head_dim 128, page in {8..128}; all
 * pointers and strides 16-byte aligned), 0 if on the CUDA-core path (fp32,
 * other head_dims or pages). No counterpart in the reference, whose FA4
 * wheel makes the same choice internally. */
int rlt_paged_prefill_uses_tensor_cores(int32_t dtype, int32_t head_dim, int32_t page_size);

/* Diagnostics: choose the tensor-core prefill kernel for the process (6 =
 * the default: 5 with bf16 P split into a hi + lo pair in the query tiles
 * whose rows attend fewer than 512 keys; 7 = 5 with P split everywhere; 8 =
 * 6 with 64-key steps and two S buffers per query tile (pages of 8 to 64
 * tokens); 5 = warp-specialised two-tile kernel with P in TMEM whose softmax
 * warpgroups hold a row's 128 scores in registers (setmaxnreg); 4 = P in
 * TMEM, each row's softmax split over two warps by key-column half; 3 = P in
 * TMEM, one warp per 32 rows reading S twice; 2 = as 3 with P in shared
 * memory; 1 = single-tile kernel); returns the previous choice (any other
 * value only queries). No counterpart in the reference. */
int rlt_prefill_tc_select(int32_t version);

/* Decode attention that reads K/V pages shared by several rows once
 * (prefix caching: vllm_rlt/core/kv_cache_manager.py:211-251 hands the
 * same physical prompt pages to many requests). Same result as
 * rlt_paged_decode (softmax(q K^T * scale) V over each row's context,
 * vllm_rlt/kernels/paged_attention.py:12-36) for the rows the plan covers;
 * the plan is built on the host (vllm_rlt_b200.plan_shared_prefix):
 *   chunks[c*5 + 0..4] = table row, token begin, token end, member begin,
 *     member count; the chunk's tokens are read once through that table row
 *     and attended by every member row; member count * (Hq / Hkv) <= 32;
 *   members[member begin + i] = row id (num_members entries in all);
 *     member_slots[...] = the partial slot of that (row, chunk);
 *     row_slots[r] .. row_slots[r + 1] = row r's slots.
 * All plan arrays are device int32. The chunks cover only the shared
 * prefixes: on entry `out` must hold each row's attention over its own tokens
 * after the prefix and `suffix_lse` [rows, Hq] its base-2 log-sum-exp, as
 * rlt_paged_decode_lse leaves them when run on the per-row suffix tables
 * (each row's table shifted past its shared pages); the prefix partials are
 * merged into `out` in place. Workspace: fp32 partials, size
 * rlt_paged_decode_shared_workspace_bytes(num_slots, Hq, D). head_dim 64 or
 * 128; K/V pointers and strides 16-byte aligned. Two kernel launches (chunk
 * partials, merge); asynchronous, no allocation. The reference has no
 * counterpart: its decode reads shared pages once per row. */
size_t rlt_paged_decode_shared_workspace_bytes(int32_t num_slots, int32_t num_q_heads,
                                               int32_t head_dim);
int rlt_paged_decode_shared(const void* q, const void* key_cache, const void* value_cache,
                            const int32_t* block_tables, const int32_t* chunks,
                            const int32_t* members, const int32_t* member_slots,
                            const int32_t* row_slots, const float* suffix_lse, void* out,
                            void* workspace, size_t workspace_bytes, int32_t* status,
                            int32_t dtype,
                            int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                            int32_t head_dim, int32_t page_size, int32_t table_width,
                            int64_t num_blocks, int32_t num_chunks, int32_t num_slots,
                            int32_t num_members, int64_t q_row_stride, int64_t q_head_stride,
                            int64_t k_block_stride,
                            int64_t k_token_stride, int64_t k_head_stride,
                            int64_t v_block_stride, int64_t v_token_stride,
                            int64_t v_head_stride, int64_t table_row_stride,
                            int64_t out_row_stride, int64_t out_head_stride, float scale,
                            void* stream);

/* rlt_paged_decode_shared with its two launches selectable: phases = 1 runs
 * only the prefix-chunk partials (they need neither `out` nor `suffix_lse`,
 * so they may run on another stream while rlt_paged_decode_lse computes the
 * suffixes), 2 only their merge into `out`, 3 both (= rlt_paged_decode_shared).
 * Same arguments otherwise. No counterpart in the reference. */
int rlt_paged_decode_shared_phases(const void* q, const void* key_cache, const void* value_cache,
                                   const int32_t* block_tables, const int32_t* chunks,
                                   const int32_t* members, const int32_t* member_slots,
                                   const int32_t* row_slots, const float* suffix_lse, void* out,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   int32_t dtype, int32_t num_rows, int32_t num_q_heads,
                                   int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                   int32_t table_width, int64_t num_blocks, int32_t num_chunks,
                                   int32_t num_slots, int32_t num_members, int64_t q_row_stride,
                                   int64_t q_head_stride, int64_t k_block_stride,
                                   int64_t k_token_stride, int64_t k_head_stride,
                                   int64_t v_block_stride, int64_t v_token_stride,
                                   int64_t v_head_stride, int64_t table_row_stride,
                                   int64_t out_row_stride, int64_t out_head_stride, float scale,
                                   int32_t phases, void* stream);

/* Per-call suffix metadata of the shared-prefix decode, built on the device
 * from the call's own block tables and context lengths, so a plan made once
 * for a batch stays valid while its rows grow (decode steps, CUDA-graph
 * replays): suffix_tables[r] = block_tables[r] shifted past prefix_pages[r]
 * pages and padded with -1 (row stride table_width), suffix_lengths[r] =
 * context_lengths[r] - prefix_pages[r] * page_size. A row whose context no
 * longer covers its shared pages gets an empty suffix and raises status bit 1
 * (its plan is stale). One launch. No counterpart in the reference. */
int rlt_shared_prefix_suffix(const int32_t* block_tables, const int32_t* context_lengths,
                             const int32_t* prefix_pages, int32_t* suffix_tables,
                             int32_t* suffix_lengths, int32_t* status, int32_t num_rows,
                             int32_t table_width, int32_t page_size, int64_t table_row_stride,
                             void* stream);

/* How the 16-bit shared-prefix chunk kernel stages K/V: 2 (default) = tiled
 * TMA loads of whole pages into 128-byte-swizzled shared memory where the
 * page size is 8, 16, 32 or 64 tokens (cp.async otherwise); 1 = cp.async from
 * the page table always. Returns the previous choice (any other value only
 * queries). Results agree within rounding (bit-identical for page-aligned
 * chunk starts). No counterpart in the reference. */
int rlt_shared_prefix_select(int32_t staging);

/* Size of the static split-KV scratch of rlt_paged_decode_noalloc (bytes). */
#define RLT_NOALLOC_SCRATCH_BYTES (16u << 20)

/* rlt_paged_decode for callers that cannot allocate device memory when they
 * run attention (a runtime that reserves all device memory for its own pool,
 * a host that forbids driver allocations after start-up, or code where an
 * allocation would synchronise the device). Same inputs, outputs and results
 * as rlt_paged_decode; there is no workspace argument: the split-KV scratch is
 * a 16 MiB (RLT_NOALLOC_SCRATCH_BYTES) device array inside the library that
 * every GPU using this entry point holds until the process exits. It calls no
 * cudaMalloc/cudaFree or other allocating routine.
 *  - The first call on a device looks up that device's copy of the array
 *    (with the device current), and under lazy module loading it is also the
 *    moment the driver places the array: make that first call at start-up,
 *    before any stream capture on the device. The looked-up address is kept
 *    for the life of the process, so the device must not be reset
 *    (cudaDeviceReset) while the library is in use.
 *  - Returns RLT_E_SCRATCH, launching nothing, when a launch that splits rows
 *    (the 16-byte-vector path: head_dim 32/64/128/256 with 16-byte aligned
 *    strides) needs more split partials than the array holds, i.e. when
 *    rlt_paged_decode_workspace_bytes(num_rows, num_q_heads, head_dim,
 *    page_size, table_width) > RLT_NOALLOC_SCRATCH_BYTES. Other shapes run
 *    without splits and use none of the array, at any size.
 *  - All calls share the array; calls that overlap on the GPU race on it, so
 *    serialise them (one stream, or events between streams).
 * This entry point has no counterpart in the reference, which always
 * allocates its outputs and scratch through torch. */
int rlt_paged_decode_noalloc(const void* q, const void* key_cache, const void* value_cache,
                             const int32_t* block_tables, const int32_t* context_lengths,
                             void* out, int32_t* status, int32_t dtype, int32_t num_rows,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             int32_t page_size, int32_t table_width, int64_t num_blocks,
                             int64_t q_row_stride, int64_t q_head_stride, int64_t k_block_stride,
                             int64_t k_token_stride, int64_t k_head_stride,
                             int64_t v_block_stride, int64_t v_token_stride,
                             int64_t v_head_stride, int64_t table_row_stride,
                             int64_t out_row_stride, int64_t out_head_stride, float scale,
                             void* stream);

/* KV page write into the depth plane (reshape_and_cache):
 *   key_cache[write_blocks[i], layer, write_offsets[i]] = k[i]   (i < num_rows)
 *   value_cache[...]                                    = v[i]
 * Bit-exact copy. Pool strides are those of the 5-D pool.
 * Replaces: vllm_rlt/core/kv_cache_manager.py:531-532 (_write_prepared) and
 * the graph-captured copy at vllm_rlt/worker/cuda_graph.py:16-19. */
int rlt_kv_write(const void* k, const void* v, void* key_cache, void* value_cache,
                 const int64_t* write_blocks, const int64_t* write_offsets, int32_t* status,
                 int32_t dtype, int32_t num_rows, int32_t num_kv_heads, int32_t head_dim,
                 int32_t layer, int32_t page_size, int64_t num_blocks, int64_t k_row_stride,
                 int64_t k_head_stride, int64_t v_row_stride, int64_t v_head_stride,
                 int64_t cache_block_stride, int64_t cache_layer_stride,
                 int64_t cache_token_stride, int64_t cache_head_stride, void* stream);

/* LAST-EXITED exit copy: for each descriptor row (slot, depth, pos) copy the
 * token's K and V of every layer from plane `depth` into every deeper plane
 * (depth, planes), through the resident tables[slot, plane, width].
 * descriptor may be a mapped (UVA) pinned host pointer. Bit-exact.
 * Replaces: vllm_rlt/kernels/routing.py:79-109 (finalize_kernel, launched at
 * vllm_rlt/worker/model_runner.py:543-557) and the eager copies of
 * vllm_rlt/core/kv_cache_manager.py:601-611 (finalize_token). */
int rlt_finalize(const int64_t* descriptor, const int32_t* tables, void* key_cache,
                 void* value_cache, int32_t* status, int32_t dtype, int32_t num_rows,
                 int32_t num_slots, int32_t width, int32_t planes, int32_t page_size,
                 int32_t num_layers, int32_t channels, int64_t num_blocks,
                 int64_t block_stride, int64_t layer_stride, int64_t token_stride, void* stream);

/* Depth/page resolution of one routing bank: descriptor rows (slot, depth,
 * pos) -> slots, positions, lengths = pos + 1 (0 for rows >= n), write block /
 * offset, and the row's depth-plane table copied into out_tables[row, :out_width]
 * (row stride `width`). Rows in [n, size) are padding.
 * Replaces: vllm_rlt/kernels/routing.py:7-41 (metadata_kernel, launched at
 * vllm_rlt/worker/async_state.py:181-197). */
int rlt_metadata(const int64_t* descriptor, const int32_t* tables, int64_t* slots,
                 int64_t* positions, int32_t* lengths, int64_t* blocks, int64_t* offsets,
                 int32_t* out_tables, int32_t* status, int32_t n, int32_t size, int32_t width,
                 int32_t page_size, int32_t planes, int32_t out_width, int32_t num_slots,
                 void* stream);

/* Copy a (mapped pinned or device) int64 metadata bank to device int64 and
 * int32 copies. Replaces: vllm_rlt/kernels/prefill_metadata.py:7-12
 * (stage_prefill, launched at vllm_rlt/worker/prefill_metadata.py:53-55). */
int rlt_stage_prefill(const int64_t* source, int64_t* target, int32_t* target32, int64_t n,
                      void* stream);

/* Per packed-prefill token: block = tables[seq * width + pos / page],
 * offset = pos % page. Replaces: vllm_rlt/kernels/prefill_metadata.py:15-32
 * (expand_prefill, launched at vllm_rlt/worker/prefill_metadata.py:75-86). */
int rlt_expand_prefill(const int64_t* positions, const int64_t* sequences, const int32_t* tables,
                       int64_t* blocks, int64_t* offsets, int32_t* status, int64_t n,
                       int32_t width, int32_t page_size, int64_t num_table_entries,
                       void* stream);

/* Resident-slot gather: out[row, :] = pool[slots[row], :] for row < n, zeros
 * for n <= row < size. elem_bytes in {1, 2, 4, 8}; strides in elements.
 * Replaces: vllm_rlt/kernels/routing.py:44-59 (gather_kernel, launched at
 * vllm_rlt/worker/async_state.py:215-224). */
int rlt_gather(const void* pool, const int64_t* slots, void* out, int32_t n, int32_t size,
               int32_t width, int32_t elem_bytes, int64_t in_stride, int64_t out_stride,
               void* stream);

/* Resident-slot scatter: pool[slots[row], :] = values[row, :] for row < n.
 * Replaces: vllm_rlt/kernels/routing.py:62-76 (scatter_kernel, launched at
 * vllm_rlt/worker/async_state.py:226-234). */
int rlt_scatter(const void* values, const int64_t* slots, void* pool, int32_t n, int32_t width,
                int32_t elem_bytes, int64_t in_stride, int64_t out_stride, void* stream);

/* ---- fused per-layer glue of the recurrent core (calling context) ---- */

/* RMSNorm over rows of `hidden` elements with the reference's rounding:
 * y = weight * to_dtype(x * rsqrt(mean(x^2) + eps)) in fp32; if residual is
 * not NULL, out = residual + y (rounded to the dtype). hidden <= 4096.
 * Replaces: vllm_rlt/models/ouro.py:33-36 (OuroRMSNorm.forward) and the
 * residual adds of the decoder layer at :143-147. */
int rlt_rms_norm(const void* x, const void* weight, const void* residual, void* out,
                 int32_t dtype, int32_t rows, int32_t hidden, float eps, int64_t x_stride,
                 int64_t residual_stride, int64_t out_stride, void* stream);

/* rlt_rms_norm followed by a second RMSNorm of its output in one launch:
 * out = [residual +] weight * norm(x); out2 = weight2 * norm(out), out2
 * computed from out's rounded values, bit-identical to two rlt_rms_norm
 * calls. The decoder layer's residual stream feeds one norm into the next:
 * post-attention norm + residual -> MLP input norm, and post-MLP norm +
 * residual -> the next layer's input norm (or the final norm). Needs 16-byte
 * aligned rows (RLT_E_ALIGN otherwise); hidden <= 4096.
 * Replaces: vllm_rlt/models/ouro.py:118-125 and :143-147 (two norm calls). */
int rlt_rms_norm2(const void* x, const void* weight, const void* residual, void* out,
                  const void* weight2, void* out2, int32_t dtype, int32_t rows, int32_t hidden,
                  float eps, int64_t x_stride, int64_t residual_stride, int64_t out_stride,
                  int64_t out2_stride, void* stream);

/* RoPE on q and k straight out of the fused qkv projection, k written (with
 * v) into the KV page of its depth plane:
 *   angles = pos * inv_freq (fp32); cos/sin rounded to the dtype;
 *   x' = x * cos + rotate_half(x) * sin (each op rounded to the dtype);
 *   q_out[r] = q'; key_cache[blocks[r], layer, offsets[r]] = k'; value_cache[..] = v.
 * qkv rows hold [heads*D | kv_heads*D | kv_heads*D]; D <= 512. Bit-identical
 * to the unfused torch expression followed by rlt_kv_write.
 * Replaces: vllm_rlt/models/ouro.py:61-75 and :104-110 plus the page write of
 * vllm_rlt/core/kv_cache_manager.py:531-532. */
int rlt_rope_write_kv(const void* qkv, const int64_t* positions, const float* inv_freq,
                      void* q_out, void* key_cache, void* value_cache,
                      const int64_t* write_blocks, const int64_t* write_offsets, int32_t* status,
                      int32_t dtype, int32_t rows, int32_t heads, int32_t kv_heads,
                      int32_t head_dim, int32_t layer, int32_t page_size, int64_t num_blocks,
                      int64_t qkv_stride, int64_t q_row_stride, int64_t q_head_stride,
                      int64_t cache_block_stride, int64_t cache_layer_stride,
                      int64_t cache_token_stride, int64_t cache_head_stride, void* stream);

/* SwiGLU: out = silu(gate) * up with gate_up rows [gate | up] (each op rounded
 * to the dtype). Replaces: vllm_rlt/models/ouro.py:122-123. */
int rlt_silu_mul(const void* gate_up, void* out, int32_t dtype, int32_t rows,
                 int32_t intermediate, int64_t in_stride, int64_t out_stride, void* stream);

/* KV page transport for prefill/decode disaggregation: copy byte segments
 * segments[i*3 + 0..2] = {source address, destination address, bytes}
 * (device int64 array; addresses and sizes multiples of 16 bytes) on the
 * stream's device. A destination on another GPU must be mapped in this
 * process (rlt_enable_peer_access, or a CUDA-IPC mapping of the other
 * process's pool); it is written with plain stores over NVLink.
 * max_segment_bytes bounds the largest segment (it sizes the launch).
 * Misaligned segments are skipped and raise RLT_STATUS_BAD_OFFSET.
 * Replaces: the NIXL WRITE of vllm_rlt/pd/transport.py:114-133, whose
 * segments come from kv_segments / partition_segments (:18-72). */
int rlt_copy_segments(const int64_t* segments, int32_t num_segments, int64_t max_segment_bytes,
                      int32_t* status, void* stream);

/* Enable access from the current device to peer_device's memory (no-op if
 * already enabled or if peer_device is the current device); RLT_E_DEVICE
 * when the pair cannot use peer access. */
int rlt_enable_peer_access(int32_t peer_device);

#ifdef __cplusplus
}
#endif

#endif /* RLT_B200_H_ */
