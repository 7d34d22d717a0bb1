// Host-side plumbing shared by every entry point of the C ABI: status strings, the
// last-CUDA-error record, per-device SM counts and the cached TMA tensor maps over the
// KV pool tensors.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace {

thread_local int g_last_cuda_error = 0;

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
  int64_t layers, slots;
  int heads, dim, elem;
  bool operator==(const MapKey& o) const {
    return base == o.base && layers == o.layers && slots == o.slots && heads == o.heads &&
           dim == o.dim && elem == o.elem;
  }
};

struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};

constexpr int kMapCache = 32;
MapEntry g_maps[kMapCache];
int g_next_victim = 0;
std::mutex g_map_mutex;

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

int pool_tensor_map(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                    int num_kv_heads, int head_dim, int elem_bytes) {
  MapKey key{base, num_layers, num_slots, num_kv_heads, head_dim, elem_bytes};
  std::lock_guard<std::mutex> lock(g_map_mutex);
  for (auto& e : g_maps) {
    if (e.used && e.key == key) {
      *out = e.map;
      return B2P_OK;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return B2P_EDRIVER;
  const int inner = 128 / elem_bytes;  // elements per 128-byte swizzle line
  if (head_dim % inner != 0) return B2P_EUNSUPPORTED;
  const uint64_t es = static_cast<uint64_t>(elem_bytes);
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(inner),
                        static_cast<cuuint64_t>(head_dim / inner),
                        static_cast<cuuint64_t>(num_kv_heads),
                        static_cast<cuuint64_t>(num_slots),
                        static_cast<cuuint64_t>(num_layers)};
  // Byte strides of dims 1..4 (dim 0 is the contiguous one).
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(inner * es),
                           static_cast<cuuint64_t>(head_dim * es),
                           static_cast<cuuint64_t>(num_kv_heads) * head_dim * es,
                           static_cast<cuuint64_t>(num_slots) * num_kv_heads * head_dim * es};
  cuuint32_t box[5] = {static_cast<cuuint32_t>(inner), static_cast<cuuint32_t>(head_dim / inner),
                       1u, 16u, 1u};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  // TMA tile loads copy bytes without conversion, so an unsigned type of the element
  // width serves bf16, f16 and f32 alike.
  CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                           : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  CUtensorMap map;
  CUresult r = fn(&map, dt, 5, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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

}  // namespace b2p_host

extern "C" {

int b2p_version(void) { return 100; }

int b2p_last_cuda_error(void) { return g_last_cuda_error; }

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
