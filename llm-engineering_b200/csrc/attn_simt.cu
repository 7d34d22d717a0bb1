// CUDA-core paged attention for the shapes the tensor-core kernels do not take:
// fp32 storage (the reference's CPU configuration runs in fp32), head dims that are not
// a multiple of 64, block sizes that are not a multiple of 16, GQA groups above 16.
//
// One warp owns one (query row, query head). Keys are processed 32 at a time: lane j
// computes the full dot product of key (base + j) with the query (query in shared
// memory, read as a broadcast), the warp updates its online-softmax state, then each
// lane accumulates P.V for the head dims it owns (d = lane + 32k). Causality follows
// the reference's packed masks (serving/engine/attention_mask.py:37-45): query row j of a
// sequence with q_len queries and ctx keys sits at position ctx - q_len + j and sees keys
// 0..that position; a decode row (q_len = 1) sees its whole history.
#include "common.cuh"

namespace {

using namespace b2p;

constexpr int kWarps = 4;
constexpr int kMaxD = 256;

struct SimtParams {
  const uint8_t* q;
  int64_t q_tok, q_head;
  const uint8_t* k_cache;  // layer base
  const uint8_t* v_cache;
  int64_t row_elems;  // num_kv_heads * head_dim
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* cu_q;  // null: decode mode, row i is sequence i with q_len 1
  const int32_t* context_lens;
  int num_seqs;
  int num_q_heads, group, head_dim, block_size;
  int64_t num_blocks;
  float scale;
  uint8_t* out;
  int64_t o_tok, o_head;
  int32_t* err;
};

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) paged_attn_simt(const SimtParams p) {
  __shared__ float qs[kWarps][kMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Decode mode: row i is sequence i. Prefill mode: rows start at cu_q[0], which lets a
  // caller run a trailing slice of a packed batch with views of the metadata.
  const int64_t row = blockIdx.x + (p.cu_q == nullptr ? 0 : __ldg(p.cu_q));
  const int qh = blockIdx.y * kWarps + warp;
  if (qh >= p.num_q_heads) return;

  int seq;
  int q_len, q_idx;
  if (p.cu_q == nullptr) {
    seq = (int)row;
    q_len = 1;
    q_idx = 0;
  } else {
    int lo = 0, hi = p.num_seqs - 1;  // last seq with cu_q[seq] <= row
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(p.cu_q + mid) <= row) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    if (row >= __ldg(p.cu_q + p.num_seqs)) return;  // grid covers all rows of q
    q_len = __ldg(p.cu_q + seq + 1) - __ldg(p.cu_q + seq);
    q_idx = (int)(row - __ldg(p.cu_q + seq));
  }
  const int ctx = __ldg(p.context_lens + seq);
  const int pos = ctx - q_len + q_idx;  // logical position of this query
  const int kvh = qh / p.group;
  const int D = p.head_dim;

  const T* qrow = reinterpret_cast<const T*>(p.q) + row * p.q_tok + (int64_t)qh * p.q_head;
  for (int d = lane; d < D; d += 32) qs[warp][d] = to_f32<T>(qrow[d]);
  __syncwarp();

  T* orow = reinterpret_cast<T*>(p.out) + row * p.o_tok + (int64_t)qh * p.o_head;
  if (pos < 0 || q_len <= 0 || ctx <= 0) {
    if (lane == 0) set_device_error(p.err, B2P_DEV_LENGTH);
    for (int d = lane; d < D; d += 32) orow[d] = from_f32<T>(0.f);
    return;
  }

  float m = -INFINITY, l = 0.f;
  float acc[kMaxD / 32];
#pragma unroll
  for (int k = 0; k < kMaxD / 32; ++k) acc[k] = 0.f;
  const int32_t* bt = p.block_tables + (int64_t)seq * p.bt_stride;
  const int nkeys = pos + 1;
  for (int base = 0; base < nkeys; base += 32) {
    const int t = base + lane;
    float s = -INFINITY;
    int64_t slot = -1;
    if (t < nkeys) {
      const int64_t col = t / p.block_size;
      const int32_t blk = col < p.bt_stride ? __ldg(bt + col) : -1;
      if (blk < 0 || blk >= p.num_blocks) {
        set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
      } else {
        slot = (int64_t)blk * p.block_size + t % p.block_size;
        const T* krow = reinterpret_cast<const T*>(p.k_cache) + slot * p.row_elems + (int64_t)kvh * D;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(qs[warp][d], to_f32<T>(krow[d]), dot);
        s = dot * p.scale;
      }
    }
    float mx = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mn = fmaxf(m, mx);
    if (mn == -INFINITY) continue;  // every key of this chunk was invalid
    const float alpha = __expf(m - mn);
    const float pr = (s == -INFINITY) ? 0.f : __expf(s - mn);
    float ps = pr;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * alpha + ps;
    m = mn;
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) acc[k] *= alpha;
    const int cnt = min(32, nkeys - base);
    for (int j = 0; j < cnt; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pr, j);
      const int64_t sj = __shfl_sync(0xffffffffu, slot, j);
      if (sj < 0) continue;
      const T* vrow = reinterpret_cast<const T*>(p.v_cache) + sj * p.row_elems + (int64_t)kvh * D;
#pragma unroll
      for (int k = 0; k < kMaxD / 32; ++k) {
        const int d = lane + 32 * k;
        if (d < D) acc[k] = fmaf(pj, to_f32<T>(vrow[d]), acc[k]);
      }
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int k = 0; k < kMaxD / 32; ++k) {
    const int d = lane + 32 * k;
    if (d < D) orow[d] = from_f32<T>(acc[k] * inv);
  }
}

int launch_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* key_cache,
                const void* value_cache, int64_t layer_index, int64_t num_slots,
                const int32_t* block_tables, int64_t block_table_stride, const int32_t* cu_q,
                const int32_t* context_lens, int num_seqs, int64_t num_rows, int num_q_heads,
                int num_kv_heads, int head_dim, int block_size, float scale, void* out,
                int64_t out_tok_stride, int64_t out_head_stride, int dtype, int32_t* err_flag,
                void* stream) {
  if (head_dim > kMaxD) return B2P_EUNSUPPORTED;
  int es;
  switch (dtype) {
    case B2P_BF16:
    case B2P_F16:
      es = 2;
      break;
    case B2P_F32:
      es = 4;
      break;
    default:
      return B2P_EUNSUPPORTED;
  }
  if (num_rows == 0) return B2P_OK;
  if (num_rows > 0x7fffffffLL) return B2P_EUNSUPPORTED;
  SimtParams p;
  p.q = static_cast<const uint8_t*>(q);
  p.q_tok = q_tok_stride;
  p.q_head = q_head_stride;
  p.row_elems = (int64_t)num_kv_heads * head_dim;
  const int64_t layer_bytes = num_slots * p.row_elems * es;
  p.k_cache = static_cast<const uint8_t*>(key_cache) + layer_index * layer_bytes;
  p.v_cache = static_cast<const uint8_t*>(value_cache) + layer_index * layer_bytes;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.cu_q = cu_q;
  p.context_lens = context_lens;
  p.num_seqs = num_seqs;
  p.num_q_heads = num_q_heads;
  p.group = num_q_heads / num_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.num_blocks = num_slots / block_size;
  p.scale = scale;
  p.out = static_cast<uint8_t*>(out);
  p.o_tok = out_tok_stride;
  p.o_head = out_head_stride;
  p.err = err_flag;
  dim3 grid((unsigned)num_rows, (unsigned)((num_q_heads + kWarps - 1) / kWarps));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2P_BF16)
    paged_attn_simt<__nv_bfloat16><<<grid, kWarps * 32, 0, s>>>(p);
  else if (dtype == B2P_F16)
    paged_attn_simt<__half><<<grid, kWarps * 32, 0, s>>>(p);
  else
    paged_attn_simt<float><<<grid, kWarps * 32, 0, s>>>(p);
  return b2p_host::check_launch();
}

}  // namespace

// Decode through the CUDA-core kernel (row i = sequence i, one query each).
int b2p_decode_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                    const void* key_cache, const void* value_cache, int64_t layer_index,
                    int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                    int64_t block_table_stride, const int32_t* context_lens, int num_seqs,
                    int num_q_heads, int num_kv_heads, int head_dim, int block_size, float scale,
                    void* out, int64_t out_tok_stride, int64_t out_head_stride, int dtype,
                    int32_t* err_flag, void* stream) {
  (void)num_layers;
  return launch_simt(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                     num_slots, block_tables, block_table_stride, nullptr, context_lens, num_seqs,
                     num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                     out_tok_stride, out_head_stride, dtype, err_flag, stream);
}

// Packed causal prefill through the CUDA-core kernel; total rows = cu_q[num_seqs]
// must be passed by the caller as num_rows.
int b2p_prefill_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                     const void* key_cache, const void* value_cache, int64_t layer_index,
                     int64_t num_slots, const int32_t* block_tables, int64_t block_table_stride,
                     const int32_t* cu_seqlens_q, const int32_t* context_lens, int num_seqs,
                     int64_t num_rows, int num_q_heads, int num_kv_heads, int head_dim,
                     int block_size, float scale, void* out, int64_t out_tok_stride,
                     int64_t out_head_stride, int dtype, int32_t* err_flag, void* stream) {
  return launch_simt(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                     num_slots, block_tables, block_table_stride, cu_seqlens_q, context_lens,
                     num_seqs, num_rows, num_q_heads, num_kv_heads, head_dim, block_size, scale,
                     out, out_tok_stride, out_head_stride, dtype, err_flag, stream);
}
