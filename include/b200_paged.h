/*
 * b200_paged.h — C ABI of the B200 (sm_100a) paged/packed attention hot path.
 *
 * The reference engine (pedrosilva-a11y/llm-engineering) runs this path in PyTorch:
 * it scatters new K/V rows into a flat slot pool, gathers every sequence's whole
 * history back, concatenates the histories and runs dense masked SDPA over them.
 * The entry points below replace those steps with hand-written CUDA kernels that
 * read the pool in place through block tables.
 *
 * Conventions
 *   - Every pointer is a device pointer unless its name ends in _host.
 *   - The KV pool has the reference layout (serving/engine/paged_kv_storage.py:56-74):
 *       key_cache, value_cache : [num_layers, num_slots, num_kv_heads, head_dim], contiguous,
 *       num_slots = num_blocks * block_size, slot = block_id * block_size + offset.
 *   - Token-major activations ([tokens, heads, head_dim]) are passed with explicit
 *     token and head strides in elements; head_dim is always contiguous.
 *   - dtype: B2P_BF16, B2P_F16 or B2P_F32 (storage and activation type; softmax and
 *     accumulation are always fp32).
 *   - stream is a cudaStream_t passed as void*. Kernels never allocate, never
 *     synchronise and launch on that stream only.
 *   - Return value: 0 on success, a negative B2P_E* code for a rejected argument or
 *     an unsupported shape (nothing is launched then), or B2P_ELAUNCH when the launch
 *     itself failed (cudaGetLastError; b2p_last_cuda_error() gives the code).
 *   - err_flag (optional, may be NULL): a device int32 that kernels OR bits into
 *     when they meet bad data they can only see on the device (slot id out of range,
 *     block id out of range, a bounded wait that ran out). The caller reads it
 *     whenever it chooses; nothing is ever written to memory outside the
 *     pool, the outputs and the workspace because of bad data.
 */
#ifndef B200_PAGED_H
#define B200_PAGED_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2P_API __attribute__((visibility("default")))
#else
#define B2P_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum b2p_dtype { B2P_BF16 = 0, B2P_F16 = 1, B2P_F32 = 2 };

enum b2p_status {
  B2P_OK = 0,
  B2P_EINVAL = -1,       /* null pointer, non-positive size, bad stride */
  B2P_EUNSUPPORTED = -2, /* shape or dtype this build has no kernel for   */
  B2P_ERANGE = -3,       /* layer index or size outside the pool          */
  B2P_EWORKSPACE = -4,   /* workspace smaller than the *_workspace_size() */
  B2P_ELAUNCH = -5,      /* cudaGetLastError() after the launch failed    */
  B2P_EDRIVER = -6       /* tensor-map encode or driver entry point failed */
};

/* Bits that kernels OR into *err_flag. */
enum b2p_device_error {
  B2P_DEV_SLOT_RANGE = 1,   /* slot id >= num_slots                      */
  B2P_DEV_BLOCK_RANGE = 2,  /* block id outside [0, num_slots/block_size) */
  B2P_DEV_WAIT_TIMEOUT = 4, /* a bounded mbarrier / flag wait gave up     */
  B2P_DEV_LENGTH = 8        /* a context/query length that does not fit  */
};

/* Library version (major*10000 + minor*100 + patch). */
B2P_API int b2p_version(void);

/* Last CUDA error code recorded by this library's launch checks (cudaError_t). */
B2P_API int b2p_last_cuda_error(void);

/* Human-readable text for a b2p_status. */
B2P_API const char* b2p_status_string(int status);

/*
 * bf16/f16 launches of kernel 2 (b2p_paged_decode / _append / _noalloc) or kernel 3
 * (b2p_paged_prefill) since the library was loaded that ran on the CUDA-core kernels
 * because the tensor-core kernel's preconditions were not met (block_size not a multiple
 * of 16, unsupported head_dim or GQA group, unaligned rows or strides). Such a call
 * still returns B2P_OK with correct results, but runs many times slower; fp32 calls,
 * which always take the CUDA-core kernels, are not counted. Returns -1 for another
 * kernel number. No counterpart in the reference (its PyTorch path has one route).
 */
B2P_API int64_t b2p_cuda_core_fallbacks(int kernel);

/*
 * Zero, on `stream`, the device-resident claim counters of b2p_paged_prefill on the
 * current device. Every prefill launch that runs to its end leaves its counters zeroed;
 * call this after a launch reported B2P_DEV_WAIT_TIMEOUT (its counters may then be left
 * set), with no prefill launch in flight. (The decode workspace is the caller's: zero it
 * with a memset in that case.) No counterpart in the reference.
 */
B2P_API int b2p_reset_scratch(void* stream);

/*
 * K1 — KV-cache write.
 * Replaces PagedKVStorage.scatter (serving/engine/paged_kv_storage.py:76-136), i.e. the
 * two index_copy_ calls at :135-136, for a whole packed batch in one launch: row t of
 * keys/values goes to slot slot_mapping[t] of layer layer_index.
 *   keys, values : [num_tokens, num_kv_heads, head_dim] with the given strides (elements)
 *   slot_mapping : int32 [num_tokens]; a negative entry means "no write" (padding);
 *                  an entry >= num_slots is skipped and sets B2P_DEV_SLOT_RANGE.
 * Rows are copied with 16-byte vector loads/stores when every address allows it.
 */
B2P_API int b2p_kv_write(const void* keys, int64_t k_tok_stride, int64_t k_head_stride,
                 const void* values, int64_t v_tok_stride, int64_t v_head_stride,
                 void* key_cache, void* value_cache, const int32_t* slot_mapping,
                 int64_t num_tokens, int64_t layer_index, int64_t num_layers,
                 int64_t num_slots, int num_kv_heads, int head_dim, int dtype,
                 int32_t* err_flag, void* stream);

/*
 * K2 — ragged GQA decode attention over the paged pool (one query token per sequence).
 * Replaces, for DECODE executions, HFBatchedPagedCache.update's gather + cat
 * (serving/engine/hf_batched_paged_cache.py:90-148), the dense mask
 * (serving/engine/attention_mask.py:9-120) and HF sdpa_attention_forward
 * (transformers/integrations/sdpa_attention.py:40-104) called at
 * transformers/models/qwen2/modeling_qwen2.py:227-240.
 *   q            : [num_seqs, num_q_heads, head_dim] (strides in elements)
 *   block_tables : int32 [num_seqs, block_table_stride]; row i lists sequence i's
 *                  physical blocks in logical order (BlockTable.blocks_for_request,
 *                  serving/engine/block.py:295-312)
 *   context_lens : int32 [num_seqs], the key length of each sequence (the new token's
 *                  K/V must already be in the pool, as after PagedKVCache's scatter)
 *   out          : [num_seqs, num_q_heads, head_dim] (strides in elements)
 *   workspace    : device scratch of b2p_paged_decode_workspace_size() bytes, zero-filled
 *                  once by the caller before its first use. It holds the split partial
 *                  records, then the count-in counters at an offset fixed by the launch
 *                  shape (heads, head_dim, dtype); every launch that completes leaves the
 *                  counters zero, so launches of one shape reuse it with any num_seqs up
 *                  to the size it was queried for. Zero it again before a launch of
 *                  another shape, and after a launch that set B2P_DEV_WAIT_TIMEOUT.
 * Scores are q.k * scale (scale = head_dim^-0.5 for Qwen2, modeling_qwen2.py:199).
 */
B2P_API size_t b2p_paged_decode_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                       int head_dim);

B2P_API int b2p_paged_decode(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                     const void* key_cache, const void* value_cache, int64_t layer_index,
                     int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                     int64_t block_table_stride, const int32_t* context_lens, int num_seqs,
                     int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                     float scale, void* out, int64_t out_tok_stride, int64_t out_head_stride,
                     void* workspace, size_t workspace_bytes, int dtype, int32_t* err_flag,
                     void* stream);

/*
 * K2 without caller-provided scratch. No counterpart in the reference (its PyTorch path
 * has no scratch to provide). Same arguments and results as b2p_paged_decode minus the
 * workspace: the split-K counters and partial records live in a 16 MiB array compiled
 * into this library (kept by every GPU that loads it until the process exits). Meant for
 * callers that cannot allocate device memory for the library, such as a runtime whose
 * device memory is all reserved by its own arena, or a binding from a language that has
 * no device allocator of its own.
 *   - The first call on a device looks up the array's device address (with that device
 *     current); make that first call before any stream capture.
 *   - Every call clears the counters on `stream` and reuses the same array, so calls whose
 *     work overlaps on the GPU (other streams, other threads) race: serialise them.
 *   - Checks every argument, and the scratch the chosen kernel needs against the array's
 *     size, before it queues anything: a call that returns an error (B2P_EWORKSPACE when
 *     the problem needs more than the array holds) has queued no work on `stream`.
 *   - Allocates nothing (no cudaMalloc / cudaFree).
 */
B2P_API int b2p_paged_decode_noalloc(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                                     const void* key_cache, const void* value_cache,
                                     int64_t layer_index, int64_t num_layers, int64_t num_slots,
                                     const int32_t* block_tables, int64_t block_table_stride,
                                     const int32_t* context_lens, int num_seqs, int num_q_heads,
                                     int num_kv_heads, int head_dim, int block_size, float scale,
                                     void* out, int64_t out_tok_stride, int64_t out_head_stride,
                                     int dtype, int32_t* err_flag, void* stream);

/*
 * K1 and K2 for the decode rows of a step in one launch: each sequence's newest K/V row
 * (the key at position context_lens[i] - 1) is stored into the pool at the slot its block
 * table gives for that position, and the sequence's query attends over its whole history,
 * that row included. Same result as b2p_kv_write over the step's decode rows with
 * slot_mapping[i] = block_tables[i][(ctx_i - 1) / block_size] * block_size
 * + (ctx_i - 1) % block_size (the decode write of PagedKVCache.update_and_gather,
 * serving/engine/paged_kv_cache.py:51-58) followed by b2p_paged_decode, without the second
 * launch or a second pass over the new rows.
 *   new_keys, new_values : [num_seqs, num_kv_heads, head_dim] (strides in elements); rows
 *                          16-byte aligned
 * All other arguments, the workspace and the results are those of b2p_paged_decode.
 */
B2P_API int b2p_paged_decode_append(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                                    const void* new_keys, int64_t k_tok_stride,
                                    int64_t k_head_stride, const void* new_values,
                                    int64_t v_tok_stride, int64_t v_head_stride, void* key_cache,
                                    void* value_cache, int64_t layer_index, int64_t num_layers,
                                    int64_t num_slots, const int32_t* block_tables,
                                    int64_t block_table_stride, const int32_t* context_lens,
                                    int num_seqs, int num_q_heads, int num_kv_heads, int head_dim,
                                    int block_size, float scale, void* out, int64_t out_tok_stride,
                                    int64_t out_head_stride, void* workspace,
                                    size_t workspace_bytes, int dtype, int32_t* err_flag,
                                    void* stream);

/*
 * K3 — packed variable-length causal attention (prefill and chunked prefill) over the
 * paged pool. Replaces, for PREFILL executions, the same reference steps as K2 plus the
 * causal tril blocks of build_attention_mask (serving/engine/attention_mask.py:37-45).
 * Sequence i owns query rows [cu_seqlens_q[i], cu_seqlens_q[i+1]) and has key length
 * context_lens[i] >= its query length; query row j of sequence i sits at logical
 * position context_lens[i] - q_len_i + j and attends keys 0..that position. When
 * q_len_i == context_lens[i] this is the reference's whole-history prefill.
 *   q   : [total_q, num_q_heads, head_dim]    out : same shape
 *   cu_seqlens_q holds absolute row offsets into q and need not start at 0, so a caller
 *   can run the trailing executions of a packed batch by passing views of its metadata.
 *   total_q = the number of rows of q and out (>= cu_seqlens_q[num_seqs]); it bounds the
 *   grid and the TMA view of q, so no device value is read back on the host.
 *   max_q_len = the longest query run (informational).
 * bf16/f16 with head_dim 64 or 128 and block_size % 16 == 0 run on tcgen05 tensor cores
 * (TMEM accumulators); other shapes and fp32 run on CUDA cores (counted by
 * b2p_cuda_core_fallbacks(3) for bf16/f16).
 * Each tensor-core launch takes one of 64 device-resident claim-counter slots, round
 * robin, and leaves it zeroed when it ends: at most 64 prefill launches may be in flight
 * on one device at a time (streams and threads together). A launch captured into a CUDA
 * graph keeps the slot it drew at capture, so replays of that graph must not overlap, on
 * the GPU, with other prefill launches (the 64th launch after it draws the same slot):
 * replay it on the stream the other prefill launches use.
 */
B2P_API int b2p_paged_prefill(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                      const void* key_cache, const void* value_cache, int64_t layer_index,
                      int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                      int64_t block_table_stride, const int32_t* cu_seqlens_q,
                      const int32_t* context_lens, int num_seqs, int64_t total_q,
                      int max_q_len, int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                      float scale, void* out, int64_t out_tok_stride, int64_t out_head_stride,
                      int dtype, int32_t* err_flag, void* stream);

/*
 * K4 — packed batch metadata on the GPU.
 * Replaces BatchLayout (serving/engine/batch_layout.py:40-81), the position half of
 * build_packed_inputs (serving/engine/packed_inputs.py:106-131), the per-token
 * slot_for_position loop of Engine._build_model_execution (serving/engine/engine.py:121-127,
 * serving/engine/block.py:370-405) and PagedKVCache's write-slot choice
 * (serving/engine/paged_kv_cache.py:51-58), from a per-step descriptor of B executions:
 *   query_lens[i]  : query tokens of execution i (prefill: current_length, decode: 1,
 *                    chunked prefill: the chunk length)
 *   context_lens[i]: key length of execution i (current_length)
 *   table_rows[i]  : row of execution i in the device block-table mirror
 *   block_mirror   : int32 [mirror_rows, mirror_stride]
 * Outputs (all device, caller-sized):
 *   cu_seqlens_q [B+1], cu_seqlens_k [B+1]           (int32)
 *   positions    [total_q]  int64 (HF position_ids)
 *   slot_mapping [total_q]  int32 (slots the new K/V rows of this step go to)
 *   logit_indices[B]        int64
 *   block_tables [B, max_blocks_per_seq] int32, padded with -1
 * total_q = sum(query_lens), known to the host that built the descriptor (it sizes the
 * grid). B is limited to 8192 executions per launch. The outputs are bit-exact with the reference's values for whole-history prefill and
 * decode.
 */
B2P_API int b2p_build_metadata(const int32_t* query_lens, const int32_t* context_lens,
                       const int32_t* table_rows, int num_execs,
                       const int32_t* block_mirror, int64_t mirror_stride,
                       int64_t mirror_rows, int block_size, int32_t* cu_seqlens_q,
                       int32_t* cu_seqlens_k, int64_t* positions, int32_t* slot_mapping,
                       int64_t* logit_indices, int32_t* block_tables,
                       int max_blocks_per_seq, int64_t total_q, int32_t* err_flag,
                       void* stream);

/* K6 — LM head fused with the greedy argmax. Replaces, for greedy rows, the LM head over
 * each execution's last row plus the argmax over its logits
 * (serving/engine/paged_model_runner.py:83-91, serving/engine/sampling.py:78-79):
 *   out_ids[r] = argmax_v round(hidden[r] . weight[v])   for r < rows
 * where round() is the rounding to the model dtype (the reference's LM head returns bf16 /
 * f16 logits and takes the argmax of those; equal values go to the lowest index, as torch's
 * argmax does). The (rows, vocab) logits are never written. hidden [rows, hidden_size] and
 * weight [vocab, hidden_size] are bf16 or f16 (dtype B2P_BF16 / B2P_F16), row-major with the
 * given row strides (elements), 16-byte aligned; hidden_size a multiple of 64 and rows a
 * multiple of 128 (pad the hidden rows; the ids of padding rows are computed and unused).
 * out_max (optional, nullable) receives the rounded maximum logit of each row.
 * NaN logits are passed over: a row whose logits are all NaN or -inf (as a NaN hidden row
 * gives) gets id 0 and maximum NaN, torch's id for it, so every id is a valid token; a row
 * with some NaN logits gets the largest of the others (torch would return the first NaN).
 * workspace: b2p_lm_head_argmax_workspace_size(rows) bytes, 8-byte aligned and zero before
 * the first launch; every launch that runs to its end leaves it zero again.
 * Returns B2P_EUNSUPPORTED for other dtypes or shapes (the caller keeps its logits path),
 * B2P_EWORKSPACE when the workspace is too small (nothing queued). No reference function
 * has this form: it fuses two reference steps.
 */
B2P_API size_t b2p_lm_head_argmax_workspace_size(int rows);
B2P_API int b2p_lm_head_argmax(const void* hidden, int64_t hidden_row_stride, const void* weight,
                               int64_t weight_row_stride, int rows, int64_t vocab,
                               int hidden_size, int dtype, int64_t* out_ids, float* out_max,
                               void* workspace, size_t workspace_bytes, int32_t* err_flag,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_PAGED_H */
