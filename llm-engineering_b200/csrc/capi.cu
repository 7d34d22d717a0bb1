// Host-side plumbing shared by every entry point of the C ABI: status strings, the
// last-CUDA-error record, per-device SM counts and the cached TMA tensor maps over the
// KV pool tensors.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

int b2p_prefill_reset_counters(void* stream);  // prefill_tc.cu

namespace {

thread_local int g_last_cuda_error = 0;

// bf16/f16 launches that ran on the CUDA-core kernels, per kernel (index 2: K2, 3: K3).
std::atomic<int64_t> g_fallbacks[4];

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

struct MapKey {
  const void* base;
  int rank;
  uint64_t dims[5];
  uint64_t strides[4];
  uint32_t box[5];
  int dtype;
  int swizzle;
  bool operator==(const MapKey& o) const {
    if (base != o.base || rank != o.rank || dtype != o.dtype || swizzle != o.swizzle) return false;
    for (int i = 0; i < 5; ++i)
      if (dims[i] != o.dims[i] || box[i] != o.box[i]) return false;
    for (int i = 0; i < 4; ++i)
      if (strides[i] != o.strides[i]) return false;
    return true;
  }
};

struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};

constexpr int kMapCache = 64;
MapEntry g_maps[kMapCache];
int g_next_victim = 0;
std::mutex g_map_mutex;

// Encode (or fetch from the cache) a tiled tensor map with 128-byte swizzle.
int encode_cached(CUtensorMap* out, const MapKey& key) {
  std::lock_guard<std::mutex> lock(g_map_mutex);
  for (auto& e : g_maps) {
    if (e.used && e.key == key) {
      *out = e.map;
      return B2P_OK;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return B2P_EDRIVER;
  cuuint64_t dims[5];
  cuuint64_t strides[4];
  cuuint32_t box[5];
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < 5; ++i) {
    dims[i] = key.dims[i];
    box[i] = key.box[i];
  }
  for (int i = 0; i < 4; ++i) strides[i] = key.strides[i];
  CUtensorMap map;
  CUresult r = fn(&map, static_cast<CUtensorMapDataType>(key.dtype), key.rank,
                  const_cast<void*>(key.base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(key.swizzle),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return B2P_EDRIVER;
  MapEntry& victim = g_maps[g_next_victim];
  g_next_victim = (g_next_victim + 1) % kMapCache;
  victim.key = key;
  victim.map = map;
  victim.used = true;
  *out = map;
  return B2P_OK;
}

}  // namespace

namespace b2p_host {

int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error = static_cast<int>(e);
    return B2P_ELAUNCH;
  }
  return B2P_OK;
}

int record_error(cudaError_t e) {
  cudaGetLastError();
  g_last_cuda_error = static_cast<int>(e);
  return B2P_ELAUNCH;
}

void note_fallback(int kernel) {
  if (kernel >= 0 && kernel < 4) g_fallbacks[kernel].fetch_add(1, std::memory_order_relaxed);
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

// 5-D map over a pool tensor [num_layers, num_slots, num_kv_heads, head_dim] with the box
// {128-byte line, box_chunks lines, 1 head, 16 slots, 1 layer}.
int pool_tensor_map_box(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                        int num_kv_heads, int head_dim, int elem_bytes, int box_chunks) {
  const int inner = 128 / elem_bytes;  // elements per 128-byte swizzle line
  if (head_dim % inner != 0 || box_chunks < 1 || box_chunks > head_dim / inner)
    return B2P_EUNSUPPORTED;
  const uint64_t es = static_cast<uint64_t>(elem_bytes);
  MapKey k{};
  k.base = base;
  k.rank = 5;
  k.dims[0] = inner;
  k.dims[1] = head_dim / inner;
  k.dims[2] = num_kv_heads;
  k.dims[3] = num_slots;
  k.dims[4] = num_layers;
  k.strides[0] = inner * es;
  k.strides[1] = head_dim * es;
  k.strides[2] = static_cast<uint64_t>(num_kv_heads) * head_dim * es;
  k.strides[3] = static_cast<uint64_t>(num_slots) * num_kv_heads * head_dim * es;
  k.box[0] = inner;
  k.box[1] = box_chunks;
  k.box[2] = 1;
  k.box[3] = 16;
  k.box[4] = 1;
  // TMA tile loads copy bytes without conversion, so an unsigned type of the element
  // width serves bf16, f16 and f32 alike.
  k.dtype = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  k.swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
  return encode_cached(out, k);
}

int pool_tensor_map(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                    int num_kv_heads, int head_dim, int elem_bytes) {
  return pool_tensor_map_box(out, base, num_layers, num_slots, num_kv_heads, head_dim, elem_bytes,
                             head_dim / (128 / elem_bytes));
}

// 4-D map over token-major activations [rows, heads, head_dim] (element strides given)
// with the box {128-byte line, 1 line, 1 head, box_rows rows}.
int tensor_map_4d_rows(CUtensorMap* out, const void* base, int64_t rows, int heads, int head_dim,
                       int64_t row_stride_elems, int64_t head_stride_elems, int elem_bytes,
                       int box_rows) {
  const int inner = 128 / elem_bytes;
  if (head_dim % inner != 0 || rows <= 0) return B2P_EUNSUPPORTED;
  const uint64_t es = static_cast<uint64_t>(elem_bytes);
  MapKey k{};
  k.base = base;
  k.rank = 4;
  k.dims[0] = inner;
  k.dims[1] = head_dim / inner;
  k.dims[2] = heads;
  k.dims[3] = rows;
  k.dims[4] = 1;
  k.strides[0] = inner * es;
  k.strides[1] = head_stride_elems * es;
  k.strides[2] = row_stride_elems * es;
  k.box[0] = inner;
  k.box[1] = 1;
  k.box[2] = 1;
  k.box[3] = box_rows;
  k.box[4] = 1;
  k.dtype = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  k.swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
  return encode_cached(out, k);
}

}  // namespace b2p_host

extern "C" {

int b2p_version(void) { return 100; }

int b2p_last_cuda_error(void) { return g_last_cuda_error; }

int b2p_reset_scratch(void* stream) { return b2p_prefill_reset_counters(stream); }

int64_t b2p_cuda_core_fallbacks(int kernel) {
  if (kernel != 2 && kernel != 3) return -1;
  return g_fallbacks[kernel].load(std::memory_order_relaxed);
}

const char* b2p_status_string(int status) {
  switch (status) {
    case B2P_OK:
      return "ok";
    case B2P_EINVAL:
      return "invalid argument";
    case B2P_EUNSUPPORTED:
      return "unsupported shape or dtype";
    case B2P_ERANGE:
      return "index or size outside the KV pool";
    case B2P_EWORKSPACE:
      return "workspace too small";
    case B2P_ELAUNCH:
      return "kernel launch failed";
    case B2P_EDRIVER:
      return "tensor-map encode failed";
    default:
      return "unknown status";
  }
}

}  // extern "C"
