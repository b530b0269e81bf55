/*
 * qwen36_paged_kv.h -- C ABI of the B200 (sm_100a) paged KV-cache hot path.
 *
 * This header is the drop-in boundary between the host runtime (Python through ctypes, or any
 * other FFI) and the CUDA kernels in libqwen36_paged_kv.so. Every entry point takes plain device
 * pointers, integer sizes and element strides, returns an int status (PKV_OK == 0), never
 * allocates or frees device memory, and launches asynchronously on the stream it is given
 * (a cudaStream_t passed as void*; NULL is the legacy default stream). On failure the message of
 * the calling thread's last error is available through pkv_last_error().
 *
 * Layout vocabulary used below:
 *   page     -- one physical block of `block_size` token slots of one layer's pool.
 *   pool     -- per layer, a key pool and a value pool. The native layout is
 *               (num_pages, num_kv_heads, block_size, head_dim), head_dim contiguous; any layout
 *               whose head_dim is contiguous is addressable through (stride_page, stride_head,
 *               stride_slot), given in ELEMENTS.
 *   slot     -- page * block_size + offset_in_page (the position a token is written to).
 *   table    -- per request, logical block -> physical page (int32 or int64, row-major
 *               (batch, max_blocks), unused entries may hold -1).
 *
 * Device-side faults are never raised with a trap: kernels that meet a page id or slot outside
 * the pool skip the access, write zeros where an output was due, and OR a PKV_DEVERR_* bit into
 * the caller's int32 error word (`error_flag`, may be NULL), which the host reads when it wants.
 */
#ifndef QWEN36_PAGED_KV_H
#define QWEN36_PAGED_KV_H

#include <stdint.h>

#if defined(__GNUC__)
#define PKV_API __attribute__((visibility("default")))
#else
#define PKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element and index types -------------------------------------------------------------- */
#define PKV_DTYPE_F32 0
#define PKV_DTYPE_F16 1
#define PKV_DTYPE_BF16 2

#define PKV_INDEX_I32 0
#define PKV_INDEX_I64 1

/* ---- host status codes --------------------------------------------------------------------- */
#define PKV_OK 0
#define PKV_ERR_INVALID_ARGUMENT 1
#define PKV_ERR_UNSUPPORTED 2
#define PKV_ERR_CUDA 3
#define PKV_ERR_WORKSPACE_TOO_SMALL 4

/* ---- device error bits (ORed into *error_flag) ---------------------------------------------- */
#define PKV_DEVERR_PAGE_OUT_OF_RANGE 1
#define PKV_DEVERR_SLOT_OUT_OF_RANGE 2
#define PKV_DEVERR_WAIT_TIMEOUT 4
#define PKV_DEVERR_TABLE_TOO_SHORT 8
#define PKV_DEVERR_BAD_SEQUENCE_LENGTH 16

/* ---- library ------------------------------------------------------------------------------- */

/* Message of the last failing call made by this thread ("" when none). No reference counterpart;
 * the reference reports errors as TORCH_CHECK exceptions (src/csrc/fp8_linear_cuda.cu:1199-1240). */
PKV_API const char* pkv_last_error(void);

/* ABI version of this header (bumped on any signature change). */
PKV_API int pkv_abi_version(void);

/* Per-entry-point call counters since load or the last reset, written to out[0..n). Index order:
 * 0 append, 1 copy_pages, 2 gather, 3 decode (tensor-core path), 4 decode (generic path),
 * 5 decode splits merged, 6 reference single decode, 7 reference batched decode, 8 prefill,
 * 9 lse_merge, 10 qk_norm_rope_append, 11 kv_append_fp8, 12 decode over fp8 pools, 13 gated_o_proj. Replaces the native counters exported by fp8_native_stats
 * (src/csrc/fp8_linear_cuda.cu:1151-1189). Returns the number of counters available. */
PKV_API int pkv_stats(int64_t* out, int n);
PKV_API void pkv_reset_stats(void);

/* ---- a1: slot-mapped K/V append -------------------------------------------------------------
 * Replaces FullAttentionCache.append_blocks (src/decode_state.py:271-293) and the per-row append
 * loop of the batched decode (src/tp_runtime.py:2481-2483): token i of `key`/`value`
 * (shape (num_tokens, num_kv_heads, head_dim), head_dim contiguous) is copied bit for bit into
 * slot slot_mapping[i] of every KV head of the pools. Negative slots are skipped (padding tokens);
 * slots >= num_pages*block_size are skipped and flagged PKV_DEVERR_SLOT_OUT_OF_RANGE. */
PKV_API int pkv_kv_append(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                  const void* value, int64_t value_stride_token, int64_t value_stride_head,
                  const int64_t* slot_mapping, int64_t num_tokens,
                  void* key_pool, void* value_pool,
                  int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                  int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                  int dtype, int32_t* error_flag, void* stream);

/* The same append for ONE request addressed by its block table instead of a slot list -- what
 * FullAttentionCache.append_blocks (src/decode_state.py:271-293) does per call, in one launch with no
 * host-built slots: token i goes to logical position start + i, i.e. slot
 * block_table[(start + i) / block_size] * block_size + (start + i) % block_size, with block_table an
 * int64 device array of table_len entries. Positions past the table are rejected on the host; a table
 * entry outside the pool skips that token and sets PKV_DEVERR_PAGE_OUT_OF_RANGE. */
PKV_API int pkv_kv_append_positions(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                  const void* value, int64_t value_stride_token, int64_t value_stride_head,
                  const int64_t* block_table, int64_t table_len, int64_t start, int64_t num_tokens,
                  void* key_pool, void* value_pool,
                  int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                  int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                  int dtype, int32_t* error_flag, void* stream);

/* ---- a1/a2: decode-step slot mapping from the device block tables ----------------------------
 * For one new token per request: slot_mapping[b] = block_tables[b][L / block_size] * block_size
 * + L % block_size with L = seq_lens[b] (the slot FullAttentionCache.append_blocks writes to,
 * src/decode_state.py:278-284), then, when `advance` is nonzero, seq_lens[b] = L + 1. Requests whose
 * seq_lens[b] < 0 get slot -1 (skipped by the append); a table entry outside the table or the pool
 * gives slot -1 and PKV_DEVERR_TABLE_TOO_SHORT / PKV_DEVERR_PAGE_OUT_OF_RANGE. One launch replaces
 * the reference's per-step host table rebuild (src/decode_state.py:305-312, 545-603). */
PKV_API int pkv_decode_slot_mapping(const void* block_tables, int64_t table_stride, int64_t max_blocks,
                            void* seq_lens, int index_dtype, int64_t batch, int64_t block_size,
                            int64_t num_pages, int64_t* slot_mapping, int advance,
                            int32_t* error_flag, void* stream);
/* The same for num_layers layers whose pools are stacked (layer l = pages [l * num_pages, (l + 1) *
 * num_pages) of one pool): slot_mapping (num_layers, batch) gets slot + l * num_pages * block_size, so
 * one pkv_kv_append over the stacked pools appends every layer's new token. */
PKV_API int pkv_decode_slot_mapping_layers(const void* block_tables, int64_t table_stride, int64_t max_blocks,
                            void* seq_lens, int index_dtype, int64_t batch, int64_t block_size,
                            int64_t num_pages, int64_t num_layers, int64_t* slot_mapping, int advance,
                            int32_t* error_flag, void* stream);

/* ---- a2/a3: block-table gather (as_tensors / batch_kv_tensors semantics) ---------------------
 * Replaces FullAttentionCache.as_tensors / _gather_blocks (src/decode_state.py:295-303, 395-404)
 * and batch_kv_tensors (src/decode_state.py:501-542): writes the logical-order K and V of every
 * request into dense outputs (batch, num_kv_heads, max_len, head_dim) with the given output
 * strides, zero-filling positions >= seq_lens[b]. Debug / oracle use; the attention kernels walk
 * the tables directly and never materialise this. */
PKV_API int pkv_gather_kv(const void* key_pool, const void* value_pool,
                  int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                  int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                  const void* block_tables, int64_t table_stride, int64_t max_blocks,
                  const void* seq_lens, int index_dtype, int64_t batch, int64_t max_len,
                  void* key_out, void* value_out,
                  int64_t out_stride_batch, int64_t out_stride_head, int64_t out_stride_token,
                  int dtype, int32_t* error_flag, void* stream);

/* ---- a10: page copy / compaction --------------------------------------------------------------
 * No reference counterpart beyond the growth copy grown[:, :, :old] = old
 * (src/decode_state.py:66-67): for every pair i and every layer, page src_pages[i] of both pools
 * is copied bit for bit to page dst_pages[i]. A page is `chunks_per_page` contiguous chunks of
 * `chunk_bytes`, chunk c of page p starting at p*page_stride_bytes + c*chunk_stride_bytes (one chunk
 * for the native layout; one chunk per (batch, head) for the reference layout (B,H,P,bs,D)).
 * Layers are `layer_stride_bytes` apart in both pools. Requires that no page is both a source and
 * a destination in the same call (the compaction planner guarantees it); pairs with an id outside
 * [0, num_pages) are skipped and flagged. Either pool pointer may be NULL. */
PKV_API int pkv_copy_pages(void* key_pool, void* value_pool,
                   int64_t num_layers, int64_t layer_stride_bytes,
                   int64_t num_pages, int64_t page_stride_bytes,
                   int64_t chunks_per_page, int64_t chunk_stride_bytes, int64_t chunk_bytes,
                   const int32_t* src_pages, const int32_t* dst_pages, int64_t num_pairs,
                   int32_t* error_flag, void* stream);

/* ---- a4/a5/a6: GQA paged decode attention with split-KV and log-sum-exp merge ----------------
 * Replaces paged_attention_decode(_batched) (src/csrc/fp8_linear_cuda.cu:862-1059, 1192-1365) over
 * ONE shared pool: out[b, h] = softmax(scale * q[b,h] . K[b]^T) V[b] over the seq_lens[b] tokens of
 * request b, query head h reading KV head h / (num_q_heads / num_kv_heads) (no repeated-head
 * storage). query/output are (batch, num_q_heads, head_dim) with the given strides and head_dim
 * contiguous; block_tables/seq_lens use index_dtype. Rows with seq_lens[b] <= 0 produce zeros.
 * fp16/bf16 pools with head_dim in {64,128,256}, block_size % 16 == 0, a native-compatible layout
 * and <= 8 query heads per KV head take the TMA + tensor-core path; everything else (fp32, other
 * shapes) the generic CUDA-core path. Both accumulate in fp32.
 * Work is split so that every resident warp streams an equal share of the 16-token tiles;
 * `pages_per_split` > 0 instead gives each warp (split) about that many pages. Split partials,
 * merge counters and the generic path's plan live in `workspace` (size from
 * pkv_paged_decode_workspace_size, 256-byte aligned), which must be zero-filled before its first
 * use; every completed call leaves its counters at zero again, so one workspace serves any number
 * of stream-ordered calls (calls that share a workspace must not run concurrently). The merge of
 * the splits is fused: the last split of each (request, KV head) to finish merges them. */
PKV_API int64_t pkv_paged_decode_workspace_size(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                        int64_t head_dim, int64_t max_blocks, int64_t block_size,
                                        int64_t pages_per_split);

PKV_API int pkv_paged_decode(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                     const void* key_pool, const void* value_pool,
                     int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                     int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                     const void* block_tables, int64_t table_stride, int64_t max_blocks,
                     const void* seq_lens, int index_dtype,
                     int64_t batch, int64_t num_q_heads, float scale, int64_t pages_per_split,
                     void* workspace, int64_t workspace_bytes,
                     void* output, int64_t o_stride_batch, int64_t o_stride_head,
                     int dtype, int32_t* error_flag, void* stream);

#define PKV_DECODE_STATIC_SCRATCH_BYTES (32ll << 20)
/* Paged decode for callers that cannot allocate device memory. No counterpart in the reference.
 * Some callers can't allocate: a serving runtime that reserved nearly all HBM for its KV page pools
 * up front and forbids later allocations, or a host reached through an FFI (cgo, JNI) that passes
 * raw pointers of buffers it already owns and has no device allocator to call. Same arguments and
 * results as pkv_paged_decode without the workspace: the scratch lives in a library-owned device
 * array of PKV_DECODE_STATIC_SCRATCH_BYTES per GPU, held on every GPU that loads the library until
 * exit. Calls needing more scratch than that (pkv_paged_decode_workspace_size) are rejected with
 * PKV_ERR_INVALID_ARGUMENT; every argument is checked before anything is enqueued. Every call on a
 * GPU shares the array, so calls that overlap on the GPU race; stream-ordered calls are fine. The
 * first call on each device looks up the array's device address, so make that first call before
 * any stream capture; the address is cached for the process, so do not call it after a device reset
 * (cudaDeviceReset) in the same process. Allocates nothing. */
PKV_API int pkv_paged_decode_static_scratch(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                     const void* key_pool, const void* value_pool,
                     int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                     int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                     const void* block_tables, int64_t table_stride, int64_t max_blocks,
                     const void* seq_lens, int index_dtype,
                     int64_t batch, int64_t num_q_heads, float scale, int64_t pages_per_split,
                     void* output, int64_t o_stride_batch, int64_t o_stride_head,
                     int dtype, int32_t* error_flag, void* stream);

/* Standalone log-sum-exp merge of S partial attention results (no reference counterpart):
 * partial_out (S, rows, head_dim) fp32 normalised per part, partial_lse (S, rows) fp32 natural-log
 * LSE (-inf for an empty part) -> out (rows, head_dim) in `dtype` with out_stride_row, and
 * optionally out_lse (rows) fp32. */
PKV_API int pkv_lse_merge(const float* partial_out, const float* partial_lse, int64_t num_parts, int64_t rows,
                  int64_t head_dim, void* out, int64_t out_stride_row, float* out_lse, int dtype,
                  void* stream);

/* ---- reference-layout compatibility entry points --------------------------------------------
 * Same arguments and semantics as the reference's pybind functions, for callers that still hold
 * the reference's repeated-head per-request pools (batch, heads, blocks, block_size, head_dim).
 * pkv_paged_attention_decode replaces paged_attention_decode (src/csrc/fp8_linear_cuda.cu:1192-1266,
 * src/fp8_cuda.py:217-232): one int64 block_table shared by all batch rows, `sequence_length`
 * tokens, query/output (batch, heads, 1, head_dim) contiguous, scale 1/sqrt(head_dim).
 * pkv_paged_attention_decode_batched replaces paged_attention_decode_batched
 * (src/csrc/fp8_linear_cuda.cu:1269-1365, src/fp8_cuda.py:235-250): key/value_block_ptrs and
 * physical_block_counts are DEVICE arrays of `batch` entries (each pool (1, heads, P_b, bs, D)),
 * block_tables int64 (batch, max_blocks), sequence_lengths int64 device (batch,); rows with
 * sequence length <= 0 produce zeros. Unlike the reference, fp16 and bf16 are accepted too. */
PKV_API int pkv_paged_attention_decode(const void* query, const int64_t* block_table, int64_t table_len,
                               const void* key_blocks, const void* value_blocks,
                               int64_t batch, int64_t heads, int64_t physical_blocks,
                               int64_t block_size, int64_t head_dim, int64_t sequence_length,
                               void* output, int dtype, int32_t* error_flag, void* stream);

PKV_API int pkv_paged_attention_decode_batched(const void* query, const int64_t* block_tables,
                                       int64_t max_blocks, const void* const* key_block_ptrs,
                                       const void* const* value_block_ptrs,
                                       const int64_t* physical_block_counts,
                                       const int64_t* sequence_lengths, int64_t batch,
                                       int64_t heads, int64_t block_size, int64_t head_dim,
                                       void* output, int dtype, int32_t* error_flag, void* stream);

/* The batched decode over a LIST of per-request pools in the native layout: what
 * paged_attention_decode_batched (src/csrc/fp8_linear_cuda.cu:1269-1365, src/fp8_cuda.py:235-250) does
 * for caches that each own a private pool, here (pool_pages[b], num_kv_heads, block_size, head_dim)
 * with head_dim contiguous and no repeated heads. key/value_pool_ptrs and pool_pages are DEVICE arrays
 * of `batch` entries; block_tables int64 (batch, max_blocks), -1 padded; seq_lens int64 device (batch);
 * query/output (batch, num_q_heads, head_dim) with element strides; query head h reads KV head
 * h / (num_q_heads / num_kv_heads). Rows with seq_lens[b] <= 0 produce zeros; a page id outside its
 * request's pool is skipped and flagged. CUDA cores, one CTA per (request, KV head), fp32 accumulation. */
PKV_API int pkv_paged_decode_request_pools(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                     const void* const* key_pool_ptrs, const void* const* value_pool_ptrs,
                     const int64_t* pool_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                     const int64_t* block_tables, int64_t max_blocks, const int64_t* seq_lens,
                     int64_t batch, int64_t num_q_heads, float scale,
                     void* output, int64_t o_stride_batch, int64_t o_stride_head,
                     int dtype, int32_t* error_flag, void* stream);

/* ---- a11: chunked-prefill paged causal attention ---------------------------------------------
 * Replaces the dense prefill fallback (src/tp_runtime.py:597-610, causal mask :716-721,
 * src/reference_ops.py:353-359): request b owns query tokens [cu_q[b], cu_q[b+1]) of `query`
 * (total_q, num_q_heads, head_dim) at absolute positions seq_lens[b] - q_len_b + i, and attends
 * causally over the first (position + 1) tokens of its pages (prefix pages and the chunk's own,
 * already appended). cu_q is int32 (batch + 1); tables/seq_lens use index_dtype. Tensor cores for
 * fp16/bf16, head_dim in {64, 128, 256}, num_q_heads / num_kv_heads in {1, 2, 4, 8, 16},
 * block_size % 16 == 0, native-compatible pool layout, 16-byte aligned rows and scale > 0; CUDA
 * cores for every other case (fp32 included). Probabilities stay fp32-accurate. */
PKV_API int pkv_paged_prefill(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                      const int32_t* cu_q, int64_t total_q, int64_t max_q_len,
                      const void* key_pool, const void* value_pool,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      const void* block_tables, int64_t table_stride, int64_t max_blocks,
                      const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, void* output, int64_t o_stride_token, int64_t o_stride_head,
                      int dtype, int32_t* error_flag, void* stream);

/* Flags of pkv_paged_prefill_ex. */
#define PKV_PREFILL_ROUND_PROBS 1 /* P may be rounded once to the compute dtype before P.V -- the
                                     reference's probs.to(query.dtype) (src/tp_runtime.py:723) --
                                     instead of being carried fp32-accurate (bf16: half the P.V
                                     tensor-core work) */

/* pkv_paged_prefill with `flags` (PKV_PREFILL_*). No separate reference counterpart: flags = 0 is
 * pkv_paged_prefill; PKV_PREFILL_ROUND_PROBS reproduces the reference's probability rounding. */
PKV_API int pkv_paged_prefill_ex(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                      const int32_t* cu_q, int64_t total_q, int64_t max_q_len,
                      const void* key_pool, const void* value_pool,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      const void* block_tables, int64_t table_stride, int64_t max_blocks,
                      const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, void* output, int64_t o_stride_token, int64_t o_stride_head,
                      int dtype, int flags, int32_t* error_flag, void* stream);

/* ---- f1: fused q/k RMSNorm + partial rotary embedding + K/V append -------------------------
 * Replaces the per-layer norm / RoPE / repeat / append sequence in front of attention
 * (src/tp_runtime.py:510-525, batched decode :2461-2483; rms_norm src/reference_ops.py:166-169,
 * rotary_embeddings :203-212, apply_rotary_pos_emb :215-224, append_blocks
 * src/decode_state.py:271-293) with one launch. For token t at position p = positions[t] +
 * position_offset (positions use index_dtype):
 *   q_out[t, h]          = rope(rms_norm(query[t, h], q_weight), p)     h < num_q_heads
 *   key_pool[slot_t, h]  = rope(rms_norm(key[t, h], k_weight), p)       h < num_kv_heads
 *   value_pool[slot_t, h] = value[t, h]
 * rms_norm(x, w) = x * (1 / sqrt(mean(x^2) + eps)) * (1 + w) in fp32, rounded to dtype; rope acts on
 * the first rotary_dim elements: rnd(rnd(x * cos) + rnd(rotate_half(x) * sin)) with cos/sin read
 * from `cos_sin` row p ((max_position, 2 * rotary_dim) in dtype, cos then sin, as
 * rotary_embeddings builds them); rnd rounds to dtype. Only the pool's KV heads are stored (no
 * repetition): a tensor-parallel rank passes key/value offset to its first KV head. q_weight /
 * k_weight are (head_dim) in dtype. head_dim in {64, 128, 256, 512, 1024}; rotary_dim a multiple of
 * head_dim / 16. Slots < 0 are skipped; slots past the pool set PKV_DEVERR_SLOT_OUT_OF_RANGE and
 * positions outside [0, max_position) set PKV_DEVERR_BAD_SEQUENCE_LENGTH (that token is not
 * written). */
PKV_API int pkv_qk_norm_rope_append(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                      const void* key, int64_t k_stride_token, int64_t k_stride_head,
                      const void* value, int64_t v_stride_token, int64_t v_stride_head,
                      const void* q_weight, const void* k_weight, float eps,
                      const void* cos_sin, int64_t max_position, int64_t rotary_dim,
                      const void* positions, int64_t position_offset, int index_dtype,
                      const int64_t* slot_mapping,
                      void* key_pool, void* value_pool,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      void* q_out, int64_t qo_stride_token, int64_t qo_stride_head,
                      int64_t num_tokens, int64_t num_q_heads, int dtype, int32_t* error_flag, void* stream);

/* ---- f4: FP8 (e4m3) KV pages ------------------------------------------------------------------
 * A new page format (no reference counterpart; the reference's e4m3 decoding table is
 * src/csrc/fp8_linear_cuda.cu:64-97): K and V pools hold e4m3 bytes (uint8, shape (pages, kv heads,
 * block_size, head_dim)), and each (slot, KV head) row has an fp32 dequantisation scale in a scale pool
 * of shape (pages, kv heads, block_size) with slot stride 1 (scale_stride_page / _head in floats).
 * Row value = e4m3 code value * scale. */

/* Quantising append: like pkv_kv_append, from fp32/fp16/bf16 rows of `dtype`. Per row:
 * amax = max |x|, scale = amax / 448, code = e4m3 of x * (448 / amax), round to nearest even,
 * saturating (rows of zeros: scale 0, codes 0). head_dim in {64, 128, 256, 512, 1024}. */
PKV_API int pkv_kv_append_fp8(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                      const void* value, int64_t value_stride_token, int64_t value_stride_head,
                      const int64_t* slot_mapping, int64_t num_tokens,
                      void* key_pool, void* value_pool, float* key_scales, float* value_scales,
                      int64_t scale_stride_page, int64_t scale_stride_head,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      int dtype, int32_t* error_flag, void* stream);

/* pkv_paged_decode over fp8 pools: same arguments and workspace (pkv_paged_decode_workspace_size),
 * plus the scale pools; `dtype` is the query/output type (fp16 or bf16). The attention is exact over
 * the dequantised cache (fp32 accumulation; the query is used in fp16). Tensor cores only:
 * head_dim 128 or 256, block_size % 16 == 0, at most 8 query heads per KV head (else
 * PKV_ERR_UNSUPPORTED). */
/* pkv_paged_decode / pkv_paged_decode_fp8 plus an `int flags` argument before error_flag.
 * PKV_DECODE_CHAINED launches the tensor-core attention and its merge with programmatic stream
 * serialisation: each is made resident while the previous kernel of the stream drains and waits
 * (griddepcontrol.wait) before reading anything, so results never depend on the flag; it only hides
 * launch and scheduling latency between consecutive kernels of a step. Unknown bits are rejected;
 * pkv_paged_decode_fp8_ex accepts PKV_DECODE_CHAINED and PKV_DECODE_PREFETCH. */
#define PKV_DECODE_CHAINED 1
/* pkv_paged_decode_ex only: run the CUDA-core formulation (per-warp dot products and shuffles, no
 * tensor-core MMA, no TMA) even where the tensor-core path applies -- the comparison the choice of
 * the MMA formulation rests on. Same results within the attention tolerance. */
#define PKV_DECODE_CUDA_CORES 2
/* With PKV_DECODE_CHAINED (pkv_paged_decode_ex, pkv_paged_decode_fp8_ex): the caller guarantees that the kernel before this
 * call in the stream does not write the pools, tables or lengths this call reads (e.g. it is the previous
 * layer's decode or output stage). The tensor-core kernel then computes its work split and starts its
 * page loads before waiting for that kernel, so they overlap its end; the query, the output and the
 * workspace are still touched only after the wait. Same results. */
#define PKV_DECODE_PREFETCH 4
PKV_API int pkv_paged_decode_ex(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                      const void* key_pool, const void* value_pool,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      const void* block_tables, int64_t table_stride, int64_t max_blocks,
                      const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, int64_t pages_per_split, void* workspace, int64_t workspace_bytes,
                      void* output, int64_t o_stride_batch, int64_t o_stride_head,
                      int dtype, int flags, int32_t* error_flag, void* stream);
PKV_API int pkv_paged_decode_fp8_ex(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                      const void* key_pool, const void* value_pool,
                      const float* key_scales, const float* value_scales,
                      int64_t scale_stride_page, int64_t scale_stride_head,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      const void* block_tables, int64_t table_stride, int64_t max_blocks,
                      const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, int64_t pages_per_split, void* workspace, int64_t workspace_bytes,
                      void* output, int64_t o_stride_batch, int64_t o_stride_head,
                      int dtype, int flags, int32_t* error_flag, void* stream);

PKV_API int pkv_paged_decode_fp8(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                      const void* key_pool, const void* value_pool,
                      const float* key_scales, const float* value_scales,
                      int64_t scale_stride_page, int64_t scale_stride_head,
                      int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                      int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                      const void* block_tables, int64_t table_stride, int64_t max_blocks,
                      const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, int64_t pages_per_split, void* workspace, int64_t workspace_bytes,
                      void* output, int64_t o_stride_batch, int64_t o_stride_head,
                      int dtype, int32_t* error_flag, void* stream);

/* ---- attention output stage: gate, FP8 block-scaled o_proj, tensor-parallel all-reduce ----------------
 * Replaces _tp_full_attention_finish_from_heads (src/tp_runtime.py:672-695):
 *     out = all_reduce_sum((heads.transpose(1, 2).reshape(B, S, H*D) * sigmoid(gate))
 *                          @ dequantize_fp8_weight(W, scale_inv)^T).to(out dtype)
 * with the linear of src/reference_ops.py:436-506 (e4m3 weight, bf16 scale_inv per 128 x 128 block)
 * and the NCCL SUM of TpRuntime.all_reduce_sum (src/tp_runtime.py:288-298).
 *
 * heads: (batch, num_heads, seq_len, head_dim) of heads_dtype, head_dim contiguous, element strides;
 * gate: (batch, seq_len, num_heads * head_dim) of gate_dtype, last axis contiguous; the gated product
 * follows torch's rounding (sigmoid rounded to the gate's type, product to the promoted type) and is
 * then used by the tensor cores as f16. weight: this rank's row-parallel shard, e4m3 bytes (hidden,
 * num_heads * head_dim) with w_stride_row bytes between rows; scale_inv: bf16 (hidden / 128,
 * num_heads * head_dim / 128) with element strides. out: (batch * seq_len, hidden) of out_dtype,
 * o_stride_token elements between tokens. num_heads * head_dim and hidden multiples of 128,
 * head_dim a multiple of 8; 16-byte aligned rows. workspace: pkv_o_proj_workspace_size bytes
 * (256-byte aligned; no zeroing needed, each call clears its own sums).
 *
 * world > 1: comm_buffers[p] is rank p's exchange buffer of pkv_o_proj_comm_bytes bytes as mapped in
 * this process (comm_buffers[rank] is this rank's own, the others IPC mappings from
 * pkv_ipc_open), zero-filled before first use and shared by every call of the group with the same
 * world, capacity and hidden; every rank makes the same sequence of calls. Ranks push their rounded
 * partials into each other's buffers over NVLink as 8-byte words that carry the call's epoch next to
 * the data (so a word proves its own arrival: no flags, no fences) and a finishing kernel sums them
 * in rank order (fp32, one rounding to out_dtype -- for two ranks exactly NCCL's SUM). phases: 1 =
 * gate, project and push; 2 = wait for the peers and finish; 3 = both. A peer whose words do not
 * arrive within 2 s sets PKV_DEVERR_WAIT_TIMEOUT (those values then hold this rank's partial only). phases | PKV_OPROJ_CHAINED
 * launches the gating kernel with programmatic stream serialisation too, so that the whole stage is
 * resident while the kernel before it (a layer's decode) drains: it waits (griddepcontrol.wait)
 * before reading the heads, and the projection's weight loads, which read no earlier result, start
 * at once. Results never depend on the flag. */
#define PKV_OPROJ_CHAINED 4
PKV_API int64_t pkv_o_proj_workspace_size(int64_t num_tokens, int64_t k_local, int64_t hidden);
PKV_API int64_t pkv_o_proj_comm_bytes(int world, int64_t capacity_tokens, int64_t hidden, int out_dtype);
PKV_API int pkv_gated_o_proj(const void* heads, int64_t h_stride_batch, int64_t h_stride_head, int64_t h_stride_seq,
                      int heads_dtype, const void* gate, int64_t g_stride_batch, int64_t g_stride_seq,
                      int gate_dtype, int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim,
                      const void* weight, int64_t w_stride_row, const void* scale_inv, int64_t s_stride_row,
                      int64_t s_stride_col, int64_t hidden, void* out, int64_t o_stride_token, int out_dtype,
                      void* workspace, int64_t workspace_bytes, int rank, int world,
                      void* const* comm_buffers, int64_t comm_capacity_tokens, int phases,
                      int32_t* error_flag, void* stream);

/* Exchange buffers shared between the processes of a tensor-parallel group (CUDA IPC): the library
 * allocates (and zero-fills) them, since IPC handles name whole allocations. handle points to
 * pkv_ipc_handle_bytes() bytes. */
PKV_API int64_t pkv_ipc_handle_bytes(void);
PKV_API int pkv_ipc_alloc(int64_t bytes, void** ptr, void* handle);
PKV_API int pkv_ipc_open(const void* handle, void** ptr);
PKV_API int pkv_ipc_close(void* ptr);
PKV_API int pkv_ipc_free(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* QWEN36_PAGED_KV_H */
