// K1 — KV-cache write: scatter a packed batch's new K/V rows into pool slots.
//
// Reference behaviour (serving/engine/paged_kv_storage.py:76-136): for one layer,
// key_cache[layer].index_copy_(0, slots, keys) and the same for values, where keys is
// (num_tokens, num_kv_heads, head_dim). Here one launch writes the whole packed batch:
// each token's K row and V row (num_kv_heads * head_dim elements each) are moved as
// 16-byte vectors, one vector per thread, so a warp moves 512 contiguous bytes of the
// destination slot row per instruction. The work is pure HBM streaming:
// 2 * num_tokens * row_bytes read + the same written.
#include "common.cuh"

namespace {

using namespace b2p;

struct KvWriteParams {
  const uint8_t* k;
  const uint8_t* v;
  int64_t k_tok, k_head;  // strides in bytes
  int64_t v_tok, v_head;
  uint8_t* k_cache;  // base of the selected layer
  uint8_t* v_cache;
  const int32_t* slots;
  int64_t num_tokens;
  int64_t num_slots;
  int64_t row_bytes;   // num_kv_heads * head_dim * elem
  int64_t head_bytes;  // head_dim * elem
  int32_t* err;
};

// Vector path: every source head row and every destination row is 16-byte aligned.
// Work item = (token, 16-byte chunk of the K row or of the V row).
__global__ void __launch_bounds__(256) kv_write_vec16(KvWriteParams p) {
  const int64_t chunks_per_row = p.row_bytes >> 4;
  const int64_t chunks_per_head = p.head_bytes >> 4;
  const int64_t total = p.num_tokens * chunks_per_row * 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (chunks_per_row * 2);
    const int64_t rem = i - tok * chunks_per_row * 2;
    const bool is_v = rem >= chunks_per_row;
    const int64_t c = is_v ? rem - chunks_per_row : rem;
    const int32_t slot = __ldg(p.slots + tok);
    if (slot < 0) continue;  // padding token: nothing to write
    if (slot >= p.num_slots) {
      if (c == 0 && !is_v) set_device_error(p.err, B2P_DEV_SLOT_RANGE);
      continue;
    }
    const int64_t h = c / chunks_per_head;
    const int64_t within = (c - h * chunks_per_head) << 4;
    const uint8_t* src = is_v ? p.v + tok * p.v_tok + h * p.v_head + within
                              : p.k + tok * p.k_tok + h * p.k_head + within;
    uint8_t* dst = (is_v ? p.v_cache : p.k_cache) + (int64_t)slot * p.row_bytes + (c << 4);
    const int4 val = __ldg(reinterpret_cast<const int4*>(src));
    *reinterpret_cast<int4*>(dst) = val;
  }
}

// Element path for strides or bases that are not 16-byte aligned.
template <typename E>
__global__ void __launch_bounds__(256) kv_write_elem(KvWriteParams p) {
  const int64_t per_row = p.row_bytes / (int64_t)sizeof(E);
  const int64_t per_head = p.head_bytes / (int64_t)sizeof(E);
  const int64_t total = p.num_tokens * per_row * 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (per_row * 2);
    const int64_t rem = i - tok * per_row * 2;
    const bool is_v = rem >= per_row;
    const int64_t e = is_v ? rem - per_row : rem;
    const int32_t slot = __ldg(p.slots + tok);
    if (slot < 0) continue;
    if (slot >= p.num_slots) {
      if (e == 0 && !is_v) set_device_error(p.err, B2P_DEV_SLOT_RANGE);
      continue;
    }
    const int64_t h = e / per_head;
    const int64_t d = e - h * per_head;
    const uint8_t* src = is_v ? p.v + tok * p.v_tok + h * p.v_head
                              : p.k + tok * p.k_tok + h * p.k_head;
    E* dst = reinterpret_cast<E*>((is_v ? p.v_cache : p.k_cache) + (int64_t)slot * p.row_bytes);
    dst[e] = reinterpret_cast<const E*>(src)[d];
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int b2p_kv_write(const void* keys, int64_t k_tok_stride, int64_t k_head_stride,
                            const void* values, int64_t v_tok_stride, int64_t v_head_stride,
                            void* key_cache, void* value_cache, const int32_t* slot_mapping,
                            int64_t num_tokens, int64_t layer_index, int64_t num_layers,
                            int64_t num_slots, int num_kv_heads, int head_dim, int dtype,
                            int32_t* err_flag, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots <= 0 || num_layers <= 0)
    return B2P_EINVAL;
  if (layer_index < 0 || layer_index >= num_layers) return B2P_ERANGE;
  if (num_tokens == 0) return B2P_OK;
  if (!keys || !values || !key_cache || !value_cache || !slot_mapping) return B2P_EINVAL;
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
  KvWriteParams p;
  p.k = static_cast<const uint8_t*>(keys);
  p.v = static_cast<const uint8_t*>(values);
  p.k_tok = k_tok_stride * es;
  p.k_head = k_head_stride * es;
  p.v_tok = v_tok_stride * es;
  p.v_head = v_head_stride * es;
  p.row_bytes = (int64_t)num_kv_heads * head_dim * es;
  p.head_bytes = (int64_t)head_dim * es;
  const int64_t layer_bytes = num_slots * p.row_bytes;
  p.k_cache = static_cast<uint8_t*>(key_cache) + layer_index * layer_bytes;
  p.v_cache = static_cast<uint8_t*>(value_cache) + layer_index * layer_bytes;
  p.slots = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_slots = num_slots;
  p.err = err_flag;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const bool vec = (p.head_bytes % 16 == 0) && (p.k_tok % 16 == 0) && (p.k_head % 16 == 0) &&
                   (p.v_tok % 16 == 0) && (p.v_head % 16 == 0) && aligned16(keys) &&
                   aligned16(values) && aligned16(p.k_cache) && aligned16(p.v_cache);
  const int threads = 256;
  const int64_t items = vec ? num_tokens * (p.row_bytes / 16) * 2 : num_tokens * (p.row_bytes / es) * 2;
  const int64_t max_blocks = (int64_t)b2p_host::sm_count() * 8;
  int64_t blocks = (items + threads - 1) / threads;
  if (blocks > max_blocks) blocks = max_blocks;
  if (vec) {
    kv_write_vec16<<<(unsigned)blocks, threads, 0, s>>>(p);
  } else if (es == 2) {
    kv_write_elem<uint16_t><<<(unsigned)blocks, threads, 0, s>>>(p);
  } else {
    kv_write_elem<uint32_t><<<(unsigned)blocks, threads, 0, s>>>(p);
  }
  return b2p_host::check_launch();
}
