// Shared device helpers for the sm_100a paged-attention kernels.
//
// Everything here is inline PTX for the Blackwell data path: mbarriers, TMA tiled
// loads (cp.async.bulk.tensor into this CTA's own shared memory only; no load in this
// library is shared across a cluster), ldmatrix/movmatrix and the m16n8k16 tensor-core MMA used by the
// decode kernel for its tiny per-block contractions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_paged.h"

namespace b2p {

// ---------------------------------------------------------------- error plumbing
__device__ __forceinline__ void set_device_error(int32_t* flag, int bits) {
  if (flag != nullptr) atomicOr(flag, bits);
}

// Bounded spin limits. A wait that runs out sets B2P_DEV_WAIT_TIMEOUT and returns
// false, so no kernel in this library can spin forever on a barrier.
constexpr uint32_t kSpinFast = 1u << 12;
constexpr uint32_t kSpinLimit = 1u << 22;  // with 128 ns naps: ~0.5 s worst case

// ---------------------------------------------------------------- shared-memory ptrs
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false (and sets the
// device error bit) when the wait runs out instead of hanging the SM.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  int32_t* err_flag) {
  uint32_t it = 0;
  while (!mbar_try_wait(bar, parity)) {
    ++it;
    if (it > kSpinFast) __nanosleep(128);
    if (it > kSpinLimit) {
      set_device_error(err_flag, B2P_DEV_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA (tiled, no multicast)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Prefetch of one 5-D tensor-map box into L2 only: no shared-memory destination and no
// completion to wait for. L2 is where every kernel's global writes land, so a prefetch of
// data that another kernel still writes cannot make a later read see stale values.
__device__ __forceinline__ void tma_prefetch_l2_5d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3, int c4) {
  asm volatile("cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];\n" ::
                   "l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
               : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1, int c2, int c3,
                                            int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(c4)
      : "memory");
}

// 128-byte swizzle used by CU_TENSOR_MAP_SWIZZLE_128B on a 1024-byte aligned tile:
// the 16-byte chunk index (bits 4..6) is XORed with the 128-byte line index mod 8
// (bits 7..9).
__device__ __forceinline__ uint32_t swz128(uint32_t byte_off) {
  return byte_off ^ ((byte_off >> 3) & 0x70u);
}

// ---------------------------------------------------------------- warp-level MMA path
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(a));
  return d;
}

template <typename T>
struct MmaOp;

template <>
struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

template <>
struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

// Pack two fp32 values into one 32-bit register of 16-bit elements (lo in bits 0..15).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);

template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Hardware base-2 exponential (MUFU.EX2); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------- element conversion
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace b2p

// ---------------------------------------------------------------- host-side helpers
namespace b2p_host {

// Record a launch result; returns B2P_OK or B2P_ELAUNCH.
int check_launch();

// Record a CUDA error returned by a runtime call (clearing the sticky-free last error)
// and return B2P_ELAUNCH.
int record_error(cudaError_t e);

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

// Count one bf16/f16 launch of kernel 2 (decode) or 3 (prefill) that ran on the CUDA-core
// kernel because the tensor-core kernel's preconditions were not met.
void note_fallback(int kernel);

// Encode a 5-D tiled tensor map over one of the pool tensors
// [num_layers, num_slots, num_kv_heads, head_dim] with the box
// {64 elements, head_dim/64 chunks, 1 head, 16 slots, 1 layer} and 128-byte swizzle.
// Returns B2P_OK or B2P_EDRIVER. Results are cached per (pointer, shape).
int pool_tensor_map(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                    int num_kv_heads, int head_dim, int elem_bytes);

// The same map with a box of box_chunks 128-byte lines per slot (1: one 64-column chunk of
// a bf16/f16 row per slot, so a 16-slot box is 16 consecutive swizzle lines).
int pool_tensor_map_box(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                        int num_kv_heads, int head_dim, int elem_bytes, int box_chunks);

}  // namespace b2p_host
