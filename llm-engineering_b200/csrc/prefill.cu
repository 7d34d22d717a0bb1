// K3 entry point: packed variable-length causal prefill / chunked prefill over the
// paged pool. bf16/f16 with head_dim 64 or 128, block sizes that are multiples of 16 and
// 16-byte aligned rows run on the tcgen05 kernel (prefill_tc.cu); fp32 and other shapes
// run on the CUDA-core kernel in attn_simt.cu. A bf16/f16 call that takes the CUDA-core
// kernel is counted (b2p_cuda_core_fallbacks(3)), since it runs many times slower.
#include "common.cuh"

int b2p_prefill_tc(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                   const void* key_cache, const void* value_cache, int64_t layer_index,
                   int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                   int64_t block_table_stride, const int32_t* cu_seqlens_q,
                   const int32_t* context_lens, int num_seqs, int64_t total_q, int num_q_heads,
                   int num_kv_heads, int head_dim, int block_size, float scale, void* out,
                   int64_t out_tok_stride, int64_t out_head_stride, int dtype, int32_t* err_flag,
                   void* stream);

int b2p_prefill_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                     const void* key_cache, const void* value_cache, int64_t layer_index,
                     int64_t num_slots, const int32_t* block_tables, int64_t block_table_stride,
                     const int32_t* cu_seqlens_q, const int32_t* context_lens, int num_seqs,
                     int64_t num_rows, int num_q_heads, int num_kv_heads, int head_dim,
                     int block_size, float scale, void* out, int64_t out_tok_stride,
                     int64_t out_head_stride, int dtype, int32_t* err_flag, void* stream);

extern "C" int b2p_paged_prefill(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                                 const void* key_cache, const void* value_cache,
                                 int64_t layer_index, int64_t num_layers, int64_t num_slots,
                                 const int32_t* block_tables, int64_t block_table_stride,
                                 const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                 int num_seqs, int64_t total_q, int max_q_len, int num_q_heads,
                                 int num_kv_heads, int head_dim, int block_size, float scale,
                                 void* out, int64_t out_tok_stride, int64_t out_head_stride,
                                 int dtype, int32_t* err_flag, void* stream) {
  if (num_seqs < 0 || total_q < 0 || max_q_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      head_dim <= 0 || block_size <= 0 || num_slots <= 0 || num_layers <= 0)
    return B2P_EINVAL;
  if (num_q_heads % num_kv_heads != 0 || num_slots % block_size != 0) return B2P_EINVAL;
  if (layer_index < 0 || layer_index >= num_layers) return B2P_ERANGE;
  if (num_seqs == 0 || total_q == 0) return B2P_OK;
  if (!q || !key_cache || !value_cache || !block_tables || !cu_seqlens_q || !context_lens || !out)
    return B2P_EINVAL;
  const int rc = b2p_prefill_tc(q, q_tok_stride, q_head_stride, key_cache, value_cache,
                               layer_index, num_layers, num_slots, block_tables,
                               block_table_stride, cu_seqlens_q, context_lens, num_seqs, total_q,
                               num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                               out_tok_stride, out_head_stride, dtype, err_flag, stream);
  if (rc != B2P_EUNSUPPORTED) return rc;
  if (dtype != B2P_F32) b2p_host::note_fallback(3);
  return b2p_prefill_simt(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                          num_slots, block_tables, block_table_stride, cu_seqlens_q,
                          context_lens, num_seqs, total_q, num_q_heads, num_kv_heads, head_dim,
                          block_size, scale, out, out_tok_stride, out_head_stride, dtype,
                          err_flag, stream);
}
