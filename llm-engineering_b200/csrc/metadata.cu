// K4 — packed batch metadata built on the GPU from a per-step execution descriptor.
//
// Reference computations it reproduces bit for bit:
//   BatchLayout.query_lengths / key_lengths / query_offsets / key_offsets /
//   logit_indices       serving/engine/batch_layout.py:40-81 (offsets = exclusive scan)
//   position_ids        serving/engine/packed_inputs.py:106-131 (prefill 0..L-1, decode L-1)
//   slot ids            serving/engine/engine.py:121-127 + block.py:370-405
//                       (slot = block_id * block_size + pos % block_size)
//   written slots       serving/engine/paged_kv_cache.py:51-58 (prefill: every slot of the
//                       history, decode: the last one)
// Generalised for chunked prefill: an execution with query length q < key length L
// contributes positions L-q .. L-1 (the reference's whole-history prefill is q == L).
//
// Every CTA scans the (small) per-execution arrays in shared memory, so one launch
// produces everything with no inter-CTA dependency; token-level outputs are spread
// over all CTAs.
#include "common.cuh"

namespace {

using namespace b2p;

constexpr int kThreads = 256;
constexpr int kMaxExecs = 8192;

struct MetaParams {
  const int32_t* qlen;
  const int32_t* ctx;
  const int32_t* rows;
  int n;
  const int32_t* mirror;
  int64_t mirror_stride, mirror_rows;
  int block_size;
  int32_t* cu_q;
  int32_t* cu_k;
  int64_t* positions;
  int32_t* slots;
  int64_t* logit_idx;
  int32_t* bt;
  int max_blocks;
  int64_t total_q;
  int32_t* err;
};

// Block-wide exclusive scan of v over kThreads threads; returns the block total.
__device__ int block_exclusive_scan(int v, int& excl, int* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kThreads / 32 ? warp_sums[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < kThreads / 32) warp_sums[lane] = wi - w;  // exclusive warp offsets
    if (lane == kThreads / 32 - 1) warp_sums[kThreads / 32] = wi;
  }
  __syncthreads();
  excl = warp_sums[warp] + incl - v;
  const int total = warp_sums[kThreads / 32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kThreads) build_metadata_kernel(const MetaParams p) {
  extern __shared__ int32_t cuq[];  // [n + 1]
  __shared__ int warp_sums[kThreads / 32 + 1];
  int run_q = 0, run_k = 0;
  for (int base = 0; base < p.n; base += kThreads) {
    const int i = base + threadIdx.x;
    const int q = i < p.n ? __ldg(p.qlen + i) : 0;
    const int k = i < p.n ? __ldg(p.ctx + i) : 0;
    int eq, ek;
    const int tq = block_exclusive_scan(q, eq, warp_sums);
    const int tk = block_exclusive_scan(k, ek, warp_sums);
    if (i < p.n) {
      cuq[i] = run_q + eq;
      if (blockIdx.x == 0) {
        p.cu_q[i] = run_q + eq;
        p.cu_k[i] = run_k + ek;
        p.logit_idx[i] = (int64_t)(run_q + eq + q - 1);
        if (q <= 0 || q > k || p.rows[i] < 0 || p.rows[i] >= p.mirror_rows)
          set_device_error(p.err, B2P_DEV_LENGTH);
      }
    }
    run_q += tq;
    run_k += tk;
  }
  if (threadIdx.x == 0) {
    cuq[p.n] = run_q;
    if (blockIdx.x == 0) {
      p.cu_q[p.n] = run_q;
      p.cu_k[p.n] = run_k;
    }
  }
  __syncthreads();

  const int64_t total = p.total_q < (int64_t)run_q ? p.total_q : (int64_t)run_q;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t r = blockIdx.x * (int64_t)kThreads + threadIdx.x; r < total; r += stride) {
    int lo = 0, hi = p.n - 1;  // last execution with cuq[i] <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cuq[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int i = lo;
    const int q = cuq[i + 1] - cuq[i];
    const int L = __ldg(p.ctx + i);
    const int64_t pos = (int64_t)L - q + (r - cuq[i]);
    p.positions[r] = pos;
    const int32_t row = __ldg(p.rows + i);
    int32_t slot = -1;
    if (pos >= 0 && row >= 0 && row < p.mirror_rows) {
      const int64_t lb = pos / p.block_size;
      if (lb < p.mirror_stride) {
        const int32_t blk = __ldg(p.mirror + (int64_t)row * p.mirror_stride + lb);
        if (blk >= 0) slot = blk * p.block_size + (int32_t)(pos % p.block_size);
      }
    }
    if (slot < 0) set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
    p.slots[r] = slot;
  }

  // Padded per-execution block tables.
  const int64_t cells = (int64_t)p.n * p.max_blocks;
  for (int64_t c = blockIdx.x * (int64_t)kThreads + threadIdx.x; c < cells; c += stride) {
    const int i = (int)(c / p.max_blocks);
    const int k = (int)(c - (int64_t)i * p.max_blocks);
    const int L = __ldg(p.ctx + i);
    const int nblk = L > 0 ? (L + p.block_size - 1) / p.block_size : 0;
    const int32_t row = __ldg(p.rows + i);
    int32_t v = -1;
    if (k < nblk && row >= 0 && row < p.mirror_rows && k < p.mirror_stride)
      v = __ldg(p.mirror + (int64_t)row * p.mirror_stride + k);
    p.bt[c] = v;
  }
}

}  // namespace

extern "C" int b2p_build_metadata(const int32_t* query_lens, const int32_t* context_lens,
                                  const int32_t* table_rows, int num_execs,
                                  const int32_t* block_mirror, int64_t mirror_stride,
                                  int64_t mirror_rows, int block_size, int32_t* cu_seqlens_q,
                                  int32_t* cu_seqlens_k, int64_t* positions,
                                  int32_t* slot_mapping, int64_t* logit_indices,
                                  int32_t* block_tables, int max_blocks_per_seq, int64_t total_q,
                                  int32_t* err_flag, void* stream) {
  if (num_execs <= 0 || num_execs > kMaxExecs || block_size <= 0 || mirror_stride <= 0 ||
      mirror_rows <= 0 || max_blocks_per_seq < 0 || total_q < 0)
    return B2P_EINVAL;
  if (!query_lens || !context_lens || !table_rows || !block_mirror || !cu_seqlens_q ||
      !cu_seqlens_k || !positions || !slot_mapping || !logit_indices ||
      (max_blocks_per_seq > 0 && !block_tables))
    return B2P_EINVAL;
  MetaParams p;
  p.qlen = query_lens;
  p.ctx = context_lens;
  p.rows = table_rows;
  p.n = num_execs;
  p.mirror = block_mirror;
  p.mirror_stride = mirror_stride;
  p.mirror_rows = mirror_rows;
  p.block_size = block_size;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.positions = positions;
  p.slots = slot_mapping;
  p.logit_idx = logit_indices;
  p.bt = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.total_q = total_q;
  p.err = err_flag;
  const int64_t work = total_q > (int64_t)num_execs * max_blocks_per_seq
                           ? total_q
                           : (int64_t)num_execs * max_blocks_per_seq;
  int64_t blocks = (work + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)b2p_host::sm_count() * 2;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const size_t smem = (size_t)(num_execs + 1) * sizeof(int32_t);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(build_metadata_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return b2p_host::check_launch();
  }
  build_metadata_kernel<<<(unsigned)blocks, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return b2p_host::check_launch();
}
