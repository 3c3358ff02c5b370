/*
 * C ABI of the B200 (sm_100a) INT4 KV-cache library: libint4kv_b200.so.
 *
 * Conventions (the reference's, csrc/flash_decode_int4.cu:226-286):
 *   - plain device pointers, int sizes and a cudaStream_t; no torch types;
 *   - every launcher returns cudaErrorInvalidValue for bad sizes / null or
 *     misaligned pointers, otherwise the launch's cudaGetLastError();
 *   - launchers never allocate and keep no state between calls (safe on
 *     concurrent streams): scratch space is passed in by the caller. Two
 *     documented exceptions: int4kv_exchange_alloc allocates the peer-exchange
 *     buffer (its whole purpose), and int4kv_paged_decode_static_scratch uses a
 *     library-owned device array shared by every call on a device.
 *   - int4kv_stage_inputs is the one entry point that reads host memory (mapped
 *     pinned memory, passed by the caller).
 *
 * Numerical contract: quantizer bins, scales and zero-points are bit-identical
 * to the reference's NumPy oracle (src/quantize_int4_ref.py:51-75: IEEE float32,
 * round half to even). The library is built without fast-math.
 */
#ifndef INT4KV_B200_H_
#define INT4KV_B200_H_

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Largest batch the paged decode accepts (its per-CTA prefix table of pages per
 * sequence lives in shared memory). */
#define INT4KV_MAX_PAGED_BATCH 4096
#ifdef __cplusplus
static constexpr int kMaxPagedBatch = INT4KV_MAX_PAGED_BATCH;
#endif

/* Storage type of the value pool (v_pool) of the *_ex entry points. The
 * reference's vLLM shim stores values as float16 (src/vllm_integration.py:55);
 * the decode widens 16-bit values to float32 exactly on load. */
#define INT4KV_VALUES_F32 0
#define INT4KV_VALUES_F16 1
#define INT4KV_VALUES_BF16 2

/* Status bits a kernel ORs into the optional `status` word when it had to
 * defend itself against malformed device-resident metadata. */
#define INT4KV_STATUS_BAD_PAGE 1u      /* block-table entry outside [0, num_pages) */
#define INT4KV_STATUS_BAD_LENGTH 2u    /* length < 0, beyond its table row, or misaligned start */
#define INT4KV_STATUS_WAIT_TIMEOUT 4u  /* an async-copy wait hit its time limit */
#define INT4KV_STATUS_PEER_TIMEOUT 8u  /* a peer GPU's exchange flag did not arrive in time */

/* ---------------------------------------------------------------------------
 * Drop-in replacements for the reference's two C launchers.
 * ------------------------------------------------------------------------- */

/* Replaces cu_quantize_int4 (reference csrc/flash_decode_int4.cu:228-247).
 * kv[num_rows, num_channels] float32 row-major; ONE group = all rows; per
 * channel asymmetric INT4. Outputs one code per byte q_out[num_rows,
 * num_channels], scale_out/zp_out[num_channels]. Same signature and error
 * behaviour; rounding is half-to-even (the reference's oracle) rather than the
 * reference kernel's half-up. */
cudaError_t cu_quantize_int4(const float* kv, int num_rows, int num_channels, uint8_t* q_out,
                             float* scale_out, float* zp_out, cudaStream_t stream);

/* Replaces cu_flash_decode_int4 (reference csrc/flash_decode_int4.cu:249-284).
 * Every query in query[batch, num_heads, head_dim] attends over ONE shared
 * page stream: k_q[num_blocks, block_size, head_dim] uint8 (one code per byte),
 * k_scale/k_zp[num_blocks, head_dim], value[num_blocks, block_size, head_dim]
 * float32, block_lens[num_blocks] valid rows per page (clamped to
 * [0, block_size] on the device). head_dim in [1, 256]. No softmax scale.
 * One launch: query tiles x stream ranges, the ranges of a query tile merged
 * through distributed shared memory (no scratch); logits exact on the tensor
 * cores (integer codes x fixed-point digits of q * scale). */
cudaError_t cu_flash_decode_int4(const float* query, const uint8_t* k_q, const float* k_scale,
                                 const float* k_zp, const float* value, const int* block_lens,
                                 int batch_size, int num_heads, int head_dim, int num_blocks,
                                 int block_size, float* output, cudaStream_t stream);

/* Same contract and kernel as cu_flash_decode_int4 (kept for callers written
 * against an earlier form that took a split-KV workspace). cu_flash_decode_int4
 * already splits the page stream across the CTAs of a thread-block cluster and
 * merges the partial softmax states in distributed shared memory, so
 * int4kv_dense_decode_workspace_size reports 16 bytes and the workspace
 * argument is not used. */
cudaError_t int4kv_dense_decode_workspace_size(int batch_size, int num_heads, int head_dim,
                                               int num_blocks, int block_size, size_t* bytes);
cudaError_t int4kv_dense_decode(const float* query, const uint8_t* k_q, const float* k_scale,
                                const float* k_zp, const float* value, const int* block_lens,
                                int batch_size, int num_heads, int head_dim, int num_blocks,
                                int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Grouped quantizer (benchmark config 1): per-(group, head, channel) scale and
 * zero-point, two codes per byte. Replaces the per-block calls of
 * quantize_int4_ref + pack_int4 the reference makes in its vLLM shim
 * (src/vllm_integration.py:48-56) and benchmarks
 * (benchmarks/bench_three_backend.py:120-124).
 *   kv[num_tokens, num_heads, head_dim] float32 (16-byte aligned, head_dim % 4 == 0)
 *   packed_out[num_tokens, num_heads, head_dim/2]: channel 2i -> low nibble,
 *       2i+1 -> high nibble (src/int4_pack.py:27-29)
 *   scale_out/zp_out[ceil(num_tokens/group_tokens), num_heads, head_dim]
 * The last group may be partial and then uses only its own rows.
 * ------------------------------------------------------------------------- */
cudaError_t int4kv_quantize_grouped(const float* kv, int num_tokens, int num_heads, int head_dim,
                                    int group_tokens, uint8_t* packed_out, float* scale_out,
                                    float* zp_out, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Paged cache layout ("prepared cache"), shared by the writer and the decode:
 *   k_pool  uint8   [num_pages, num_kv_heads, page_tokens, head_dim/2]
 *   v_pool  float32 [num_pages, num_kv_heads, page_tokens, head_dim]
 *   sz_pool float32 [num_pages, num_kv_heads, 2, head_dim]   ([scale; zp] of the
 *           group whose first token lives in that page)
 *   block_table int32 [batch, max_pages]  logical page -> physical page
 *   seq_lens    int32 [batch]             tokens per sequence
 * Replaces the reference's host-side padding of page lists into a dense
 * layout (src/ops.py:293-308) and its dict-of-pages cache
 * (src/vllm_integration.py:42-60).
 * ------------------------------------------------------------------------- */

/* Quantize keys and scatter keys + values of `batch` sequences into the pools.
 * Rows of sequence b are k/v[tok_offsets[b] : tok_offsets[b+1], H, D];
 * they are written at absolute positions start_pos[b] + row (start_pos may be
 * NULL for 0; it must be a multiple of group_tokens). `max_rows_per_seq`
 * bounds tok_offsets[b+1]-tok_offsets[b]. v may be NULL (keys only).
 * group_tokens <= 128 and a multiple of page_tokens; head_dim % 4 == 0. */
cudaError_t int4kv_cache_write(const float* k, const float* v, const int32_t* tok_offsets,
                               const int32_t* start_pos, int batch, int max_rows_per_seq,
                               int num_heads, int head_dim, int group_tokens, int page_tokens,
                               const int32_t* block_table, int max_pages, int num_pages,
                               uint8_t* k_pool, float* v_pool, float* sz_pool, uint32_t* status,
                               cudaStream_t stream);

/* Fused INT4 paged flash-decode (split-KV over page runs, combine fused in
 * the same kernel). The workspace must be zero-filled before its first use;
 * every launch that completes leaves it zero-filled again (a launch that set
 * INT4KV_STATUS_WAIT_TIMEOUT does not: zero it again before reuse).
 * query/out [batch, num_q_heads, head_dim] float32; head_dim in {64,128,256};
 * page_tokens == 16; group_tokens a multiple of 16; num_q_heads a multiple G
 * of num_kv_heads (query head h reads kv head h / G: grouped-query attention).
 * Replaces the attention call of the reference's decode path
 * (src/ops.py:176-253 -> csrc/flash_decode_int4.cu:104-221) for distinct
 * per-(sequence, head) KV streams. `status` (nullable) collects
 * INT4KV_STATUS_* bits. `out` may also be the device pointer of mapped
 * pinned host memory (cudaHostAlloc with cudaHostAllocMapped): every output
 * row is stored once, with plain stores, so the result reaches the host
 * without a separate device-to-host copy. The kernel is launched with
 * programmatic stream serialization (programmatic dependent launch): its
 * CTAs may become resident while the previous kernel on `stream` still runs,
 * but each first waits for that kernel's completion and memory, so stream
 * order is kept; it lets its own successor be dispatched once its page loops
 * are done (a following decode or any kernel launched the same way). */
cudaError_t int4kv_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                               int head_dim, size_t* bytes);
cudaError_t int4kv_paged_decode(const float* query, const uint8_t* k_pool, const float* v_pool,
                                const float* sz_pool, const int32_t* block_table,
                                const int32_t* seq_lens, int batch, int num_q_heads,
                                int num_kv_heads, int head_dim, int page_tokens, int group_tokens,
                                int max_pages, int num_pages, float* out, void* workspace,
                                size_t workspace_bytes, uint32_t* status, cudaStream_t stream);

/* int4kv_paged_decode plus timing instrumentation: when non-NULL, ev_before
 * is recorded on `stream` right before the decode kernel and ev_after right
 * after it (the combine is fused into that kernel), so a caller can time the
 * kernel alone. The work done is identical. */
cudaError_t int4kv_paged_decode_profiled(const float* query, const uint8_t* k_pool,
                                         const float* v_pool, const float* sz_pool,
                                         const int32_t* block_table, const int32_t* seq_lens,
                                         int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                         int page_tokens, int group_tokens, int max_pages,
                                         int num_pages, float* out, void* workspace,
                                         size_t workspace_bytes, uint32_t* status,
                                         cudaStream_t stream, cudaEvent_t ev_before,
                                         cudaEvent_t ev_after);

/* int4kv_paged_decode_workspace_size / int4kv_paged_decode_profiled with the
 * value pool stored as `value_dtype` (INT4KV_VALUES_*): v_pool is then
 * [num_pages, num_kv_heads, page_tokens, head_dim] of that type. Halving the
 * value bytes halves most of the decode's HBM traffic. No counterpart in the
 * reference's kernels (float32 values only); its vLLM shim keeps float16. */
cudaError_t int4kv_paged_decode_workspace_size_ex(int batch, int num_q_heads, int num_kv_heads,
                                                  int head_dim, int value_dtype, size_t* bytes);
cudaError_t int4kv_paged_decode_ex(const float* query, const uint8_t* k_pool, const void* v_pool,
                                   int value_dtype, const float* sz_pool,
                                   const int32_t* block_table, const int32_t* seq_lens, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_tokens, int group_tokens, int max_pages, int num_pages,
                                   float* out, void* workspace, size_t workspace_bytes,
                                   uint32_t* status, cudaStream_t stream, cudaEvent_t ev_before,
                                   cudaEvent_t ev_after);

/* int4kv_cache_write with the values converted (round to nearest even) to
 * `value_dtype` as they are stored; v_pool as in int4kv_paged_decode_ex. */
cudaError_t int4kv_cache_write_ex(const float* k, const float* v, const int32_t* tok_offsets,
                                  const int32_t* start_pos, int batch, int max_rows_per_seq,
                                  int num_heads, int head_dim, int group_tokens, int page_tokens,
                                  const int32_t* block_table, int max_pages, int num_pages,
                                  uint8_t* k_pool, void* v_pool, int value_dtype, float* sz_pool,
                                  uint32_t* status, cudaStream_t stream);

/* Shared-stream decode over a list of blocks of a vLLM-style block cache,
 * read in place: every query of [batch_size, num_heads] attends to blocks
 * block_ids[0 .. num_listed) of the storage, in that order. Storage, indexed
 * by block id: k_packed uint8 [*, block_size, ceil(head_dim/2)] (two codes per
 * byte, low nibble = even dim), k_scale / k_zp float32 [*, head_dim] (one
 * group = the block), value [*, block_size, head_dim] of `value_dtype`,
 * block_lens int32 [*] valid rows per block; `num_blocks` blocks in all (a
 * listed id outside [0, num_blocks) is skipped, never read). Workspace as
 * int4kv_dense_decode_workspace_size(batch_size, num_heads, head_dim,
 * num_listed, block_size). Replaces the per-call host unpack + cast + gather
 * of the reference's shim (src/vllm_integration.py:62-78) with reads of the
 * stored bytes; same math as cu_flash_decode_int4. */
cudaError_t int4kv_block_decode(const float* query, const uint8_t* k_packed, const float* k_scale,
                                const float* k_zp, const void* value, int value_dtype,
                                const int32_t* block_lens, const int32_t* block_ids,
                                int num_listed, int num_blocks, int batch_size, int num_heads,
                                int head_dim, int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream);

/* Append one token to each of `batch` sequences (a decode step's KV write).
 * Sequence b's new token has absolute position positions[b]; its 128-token
 * group is still open and is quantized again over its valid rows only (the
 * reference's rule for a partial group, min/max over the rows it holds), so
 * after any number of appends the pools equal a bulk int4kv_cache_write of the
 * same tokens bit for bit. The float32 keys of each open group are kept in
 * k_stage [num_slots, group_tokens, num_heads * head_dim]: stage_slots[b]
 * names sequence b's slot, whose rows 0 .. positions[b] % group_tokens - 1
 * must hold the group's earlier keys (this call writes the new row there).
 * k_new / v_new [batch, num_heads, head_dim] float32 (v_new nullable); the
 * pages of the group must already be in block_table. No counterpart in the
 * reference (its shim writes whole blocks, src/vllm_integration.py:48-58). */
cudaError_t int4kv_cache_append(const float* k_new, const float* v_new, const int32_t* positions,
                                const int32_t* stage_slots, float* k_stage, int num_slots,
                                int batch, int num_heads, int head_dim, int group_tokens,
                                int page_tokens, const int32_t* block_table, int max_pages,
                                int num_pages, uint8_t* k_pool, void* v_pool, int value_dtype,
                                float* sz_pool, uint32_t* status, cudaStream_t stream);

/* Rotary position embedding of rows x[rows, num_heads, head_dim] at
 * positions[rows] into out (no overlap with x), with the arithmetic of
 * int4kv_cache_append_rope: the prefill's keys are rotated with it before
 * int4kv_cache_write. head_dim % 8 == 0; a position outside
 * [0, rope_positions) writes NaN and sets INT4KV_STATUS_BAD_LENGTH. */
cudaError_t int4kv_rope(const float* x, const int32_t* positions, int rows, int num_heads,
                        int head_dim, const float* rope_cos, const float* rope_sin,
                        int rope_positions, float* out, uint32_t* status, cudaStream_t stream);

/* The decode step's write with the rotary position embedding fused in (one
 * launch): the new key is rotated at its position before it is staged and
 * quantized (the cache holds post-RoPE keys, as the reference's model path
 * quantizes them: scripts/validate_llama.py:23-31), and the step's query
 * q_in [batch, num_q_heads, head_dim] is rotated at the same position into
 * q_out (q_in nullable). Rotation: Llama's rotate-half form
 * (transformers' apply_rotary_pos_emb), out_i = x_i c_i - x_{i+D/2} s_i below
 * D/2 and x_i c_i + x_{i-D/2} s_i above, float32 products and sum each rounded
 * (no contraction); rope_cos / rope_sin [rope_positions, head_dim / 2] float32
 * hold c, s per position (both NULL: no rotation). head_dim % 8 == 0 with a
 * table; a position >= rope_positions sets INT4KV_STATUS_BAD_LENGTH and the
 * sequence is skipped. Otherwise as int4kv_cache_append, which is this call
 * with no table and no query. */
cudaError_t int4kv_cache_append_rope(const float* k_new, const float* v_new,
                                     const int32_t* positions, const int32_t* stage_slots,
                                     float* k_stage, int num_slots, int batch, int num_heads,
                                     int head_dim, int group_tokens, int page_tokens,
                                     const int32_t* block_table, int max_pages, int num_pages,
                                     uint8_t* k_pool, void* v_pool, int value_dtype, float* sz_pool,
                                     const float* rope_cos, const float* rope_sin,
                                     int rope_positions, const float* q_in, float* q_out,
                                     int num_q_heads, uint32_t* status, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence split across GPUs (one long sequence, tokens partitioned into
 * 128-token-group-aligned ranges, one range per GPU). Each GPU decodes its
 * range into per-stream partial records, the records of all GPUs are gathered
 * (one collective, e.g. ncclAllGather), and int4kv_merge_partials combines
 * them. Record of one (sequence, head) stream, INT4KV_PARTIAL_RECORD_BYTES:
 *   [m float64][l float64][acc float32 x head_dim]
 * m = running max logit, l = sum of e^(logit - m), acc = sum of e^(logit - m) v
 * (unnormalized); an empty stream is m = -inf, l = 0, acc = 0. No counterpart
 * in the reference, whose kernel merges the same triple across the warps of
 * one CTA (csrc/flash_decode_int4.cu:199-220).
 * ------------------------------------------------------------------------- */
#define INT4KV_PARTIAL_RECORD_BYTES(head_dim) (16 + 4 * (head_dim))

/* int4kv_paged_decode, but writing partials [batch * num_kv_heads] records
 * (16-byte aligned) instead of normalized outputs. */
cudaError_t int4kv_paged_decode_partials(const float* query, const uint8_t* k_pool,
                                         const float* v_pool, const float* sz_pool,
                                         const int32_t* block_table, const int32_t* seq_lens,
                                         int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                         int page_tokens, int group_tokens, int max_pages,
                                         int num_pages, void* partials, void* workspace,
                                         size_t workspace_bytes, uint32_t* status,
                                         cudaStream_t stream);
/* The same with the value pool stored as `value_dtype` (INT4KV_VALUES_*);
 * workspace as int4kv_paged_decode_workspace_size_ex. */
cudaError_t int4kv_paged_decode_partials_ex(const float* query, const uint8_t* k_pool,
                                            const void* v_pool, int value_dtype,
                                            const float* sz_pool, const int32_t* block_table,
                                            const int32_t* seq_lens, int batch, int num_q_heads,
                                            int num_kv_heads, int head_dim, int page_tokens,
                                            int group_tokens, int max_pages, int num_pages,
                                            void* partials, void* workspace,
                                            size_t workspace_bytes, uint32_t* status,
                                            cudaStream_t stream);

/* Combine partials [num_parts][streams] records into out [streams, head_dim]
 * float32: out = sum_p acc_p e^(m_p - M) / max(sum_p l_p e^(m_p - M), 1e-10)
 * with M = max_p m_p, parts with m = -inf skipped (the reference's warp merge,
 * csrc/flash_decode_int4.cu:199-220), evaluated in float64. */
cudaError_t int4kv_merge_partials(const void* partials, int num_parts, int streams, int head_dim,
                                  float* out, cudaStream_t stream);

/* Fused exchange + merge over NVLink peer memory, in place of the gather and
 * int4kv_merge_partials: each GPU stores its partial records straight into
 * every GPU's exchange buffer, raises a per-chunk flag there (release, system
 * scope), waits for the other GPUs' flags of the same chunk (acquire; bounded
 * to 2 s, then INT4KV_STATUS_PEER_TIMEOUT is set in *status and the chunk's
 * outputs are NaN) and merges as int4kv_merge_partials does.
 * peer_bufs[r] = rank r's exchange buffer as mapped on this GPU (the own one
 * for r == rank; int4kv_ipc_open for the others), each
 * int4kv_exchange_bytes large, 128-byte aligned and zero-filled once before
 * the first call. Every rank calls it once per step with the same sizes; the
 * steps of one buffer set must be issued in the same order on every rank. */
#define INT4KV_EXCHANGE_MAX_RANKS 8
cudaError_t int4kv_exchange_bytes(int world, int streams, int head_dim, size_t* bytes);
cudaError_t int4kv_exchange_merge(const void* partials, void* const* peer_bufs, int world, int rank,
                                  int streams, int head_dim, float* out, uint32_t* status,
                                  cudaStream_t stream);

/* Exchange buffers and their CUDA IPC between the processes of one node:
 * int4kv_exchange_alloc makes a zero-filled allocation of its own on `device`
 * (synchronous); int4kv_ipc_handle writes INT4KV_IPC_HANDLE_BYTES opaque bytes
 * for such an allocation (the pointer must be the allocation's start: a
 * handle names a whole allocation); int4kv_ipc_open maps a peer's handle on
 * the current device (peer access enabled) and int4kv_ipc_close unmaps it. */
#define INT4KV_IPC_HANDLE_BYTES 64
cudaError_t int4kv_exchange_alloc(int device, size_t bytes, void** ptr);
cudaError_t int4kv_exchange_free(void* ptr);
cudaError_t int4kv_ipc_handle(const void* dev_ptr, void* handle);
cudaError_t int4kv_ipc_open(const void* handle, void** dev_ptr);
cudaError_t int4kv_ipc_close(void* dev_ptr);

/* The sequence split in ONE launch: the paged decode fused with the exchange
 * over NVLink peer memory. Every stream's GPU-local (m, l, acc) is stored
 * straight into every rank's exchange buffer the moment it is final (plain
 * stores through the peer mappings, then a per-stream flag with release
 * semantics at system scope); each warp, after all of its pushes, waits
 * (bounded, 2 s; then INT4KV_STATUS_PEER_TIMEOUT and NaN) for the other
 * ranks' flags of the streams it finished and merges the ranks' records into
 * out [batch, num_q_heads, head_dim] -- the full attention output, on every
 * rank. peer_bufs[r] = rank r's buffer as mapped on this GPU (the own one
 * for r == rank; int4kv_exchange_alloc + int4kv_ipc_open), each
 * int4kv_paged_decode_split_bytes large, 128-byte aligned, zero-filled once;
 * world <= INT4KV_EXCHANGE_MAX_RANKS. Every rank launches it once per step
 * with the same batch and heads. The workspace is that of
 * int4kv_paged_decode_workspace_size_ex. The grid is one resident wave, and
 * a warp only ever waits for other GPUs' pushes, all of which precede any
 * wait: launch it where no other kernel holds SMs of the GPU (a concurrent
 * kernel on every rank can keep some CTAs from starting while the resident
 * ones wait for them across GPUs; the step then ends in the bounded wait with
 * INT4KV_STATUS_PEER_TIMEOUT instead of hanging). After a timeout the ranks'
 * step counters differ: free and re-create the buffers before the next step. */
cudaError_t int4kv_paged_decode_split_bytes(int batch, int num_q_heads, int head_dim,
                                            size_t* bytes);
cudaError_t int4kv_paged_decode_split(const float* query, const uint8_t* k_pool,
                                      const void* v_pool, int value_dtype, const float* sz_pool,
                                      const int32_t* block_table, const int32_t* seq_lens,
                                      int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                      int page_tokens, int group_tokens, int max_pages,
                                      int num_pages, void* const* peer_bufs, int world, int rank,
                                      float* out, void* workspace, size_t workspace_bytes,
                                      uint32_t* status, cudaStream_t stream);

/* Scratch capacity of int4kv_paged_decode_static_scratch, per device: a
 * file-scope device array in the library, 8 MiB. That holds about 14,000
 * (sequence, query head) streams at head_dim 128; the exact limit depends on
 * the launch grid, because the scratch holds one record per resident warp as
 * well as one per stream -- *scratch_needed, or
 * int4kv_paged_decode_workspace_size, gives the exact bytes for a shape. */
#define INT4KV_STATIC_SCRATCH_BYTES (8u << 20)

/* int4kv_paged_decode without a workspace argument, for callers that cannot
 * allocate device memory on the decode path (a host runtime bound through
 * this C ABI with no device allocator of its own; a serving step whose device
 * memory is reserved up front, where cudaMalloc would fail or synchronize the
 * device). No counterpart in the reference: its launcher allocated nothing
 * because it had no split-KV scratch. Scratch is a fixed device array of
 * INT4KV_STATIC_SCRATCH_BYTES per device; a launch that would need more is
 * rejected with cudaErrorInvalidValue, and *scratch_needed (nullable) receives
 * the bytes it would need. Each call zeroes the scratch's counter region on
 * `stream` itself; nothing has to be zeroed by the caller. All calls on one
 * device share the scratch: calls that overlap in time race, so serialize
 * them. The first call on a device (and the first per head_dim and batch
 * size class) performs set-up -- it resolves the array's device address and
 * sets the kernel's shared-memory attribute -- and should precede any stream
 * capture. The array's device address is resolved once per device and kept
 * for the life of the process: cudaDeviceReset (or destroying the device's
 * primary context) after the first call is not supported. Value pools are
 * float32 only (the 16-bit pools of int4kv_paged_decode_ex are not accepted
 * here). Other arguments, checks and results as int4kv_paged_decode. */
cudaError_t int4kv_paged_decode_static_scratch(const float* query, const uint8_t* k_pool,
                                               const float* v_pool, const float* sz_pool,
                                               const int32_t* block_table,
                                               const int32_t* seq_lens, int batch,
                                               int num_q_heads, int num_kv_heads, int head_dim,
                                               int page_tokens, int group_tokens, int max_pages,
                                               int num_pages, float* out, uint32_t* status,
                                               size_t* scratch_needed, cudaStream_t stream);

/* Copy `bytes` from mapped pinned host memory (`src`: the device-usable
 * address of a cudaHostAlloc(..., cudaHostAllocMapped) buffer, from
 * cudaHostGetDevicePointer) into device memory `dst`, on `stream`, by SM
 * loads instead of the copy engine: a decode step's inputs (queries, block
 * table, lengths) are a few hundred KB at most, where the copy engine's fixed
 * cost dominates (135 KB: 17.1 us for a pinned cudaMemcpyAsync + a kernel
 * against 12.3 us for this kernel + the same kernel, between CUDA events on
 * B200). The loads bypass the device caches, so a host buffer rewritten
 * between calls is read afresh. Both pointers 16-byte aligned, `bytes` a
 * multiple of 16 (else cudaErrorInvalidValue, nothing launched). No
 * counterpart in the reference, whose CUDA path moves every input to the
 * device with a torch copy (src/ops.py:307). */
cudaError_t int4kv_stage_inputs(void* dst, const void* src, size_t bytes, cudaStream_t stream);

/* Library identification: returns a static string naming the build. */
const char* int4kv_build_info(void);

#ifdef __cplusplus
}
#endif

#endif /* INT4KV_B200_H_ */
