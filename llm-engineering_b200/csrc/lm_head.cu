// K6 — LM head fused with the greedy argmax, on tcgen05.
//
// Reference path replaced (greedy sampling of a step): the LM head over each execution's
// last row (serving/engine/paged_model_runner.py:83-91, `logits[0].index_select(0,
// logit_indices)` after HF's `lm_head`) writes a (B, vocab) logit matrix, and the sampler
// takes `argmax` per row (serving/engine/sampling.py:78-79). Here one kernel computes the
// logits tile by tile in tensor memory and keeps only each row's largest value and its
// index, so the (B, 151936) logits never reach HBM:
//
//   logits tile = H (smem, K-major: rows x hidden) x W^T (smem, K-major: vocab x hidden),
//                 tcgen05.mma kind::f16, M = 128 rows, N <= 256 vocab entries, fp32 in TMEM
//   per row: max and first arg-max over the tile, each logit rounded to the model dtype
//            first (the reference's LM head returns bf16/f16 logits and takes argmax of
//            those, ties to the lowest index)
//
// Work item = (group of up to 256 rows, vocab tile of N entries); the two 128-row halves of
// a group share each W tile (one W read per group), and each hidden chunk serves N vocab
// entries. N (a multiple of 16, at most 256) is chosen per launch so that the items split
// evenly over the SMs: 208 for a 151936-entry vocabulary on 148 SMs (731 items, 4.94 per
// SM) where N = 256 leaves two SMs a fifth 256-entry item. Wide tiles matter: with N = 128
// the MMAs of two row halves measured 1.4x slower. Persistent CTAs walk the items round
// robin; each keeps a running best per row while its items stay in one row group and
// merges it into a per-row 64-bit key with atomicMax (value in the high word, ordered so
// that larger logits give larger keys; ~index in the low word, so equal values keep the
// lowest index). The last CTA to finish turns the keys into token ids and re-zeroes them.
//
// Warp roles (192 threads): warp 0 = TMA producer (hidden and W chunks of 64 elements,
// 128-byte swizzle, 3 stages of 64 KB), warp 1 = tensor-memory owner and MMA issuer, warps
// 2..5 = epilogue (one TMEM lane quarter each). TMEM holds the accumulators of both 128-row
// halves (2 x 256 columns); the next item's first MMA waits for the epilogue's reads.
// Hidden rows are padded by the caller to a multiple of 128, so no box reaches past them
// (boxes that do are filled row by row and measured 1.6x slower for a single row).
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace {

using namespace b2p;

constexpr int kRowsTile = 128;   // rows per MMA (TMEM lanes)
constexpr int kVocabTile = 256;  // largest vocab tile (MMA N)
constexpr int kGroupRows = 2 * kRowsTile;
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr int kEpilogueWarps = 4;
constexpr uint32_t kTmemCols = 512;
constexpr int kChunkBytes = kRowsTile * 128;  // one 128-row x 64-element chunk

struct LmHeadParams {
  int rows;
  int64_t vocab;
  int hidden;            // multiple of 64
  int n_groups;          // ceil(rows / 256)
  int n_tile;            // vocab entries per item (multiple of 16, <= 256)
  int64_t n_vtiles;      // ceil(vocab / n_tile)
  unsigned long long* keys;  // [rows], zero between launches
  int32_t* ctr;          // CTAs done, zero between launches
  int64_t* out_ids;      // [rows]
  float* out_max;        // [rows] or null
  int32_t* err;
};

// Shared-memory plan: per stage the two row halves' hidden chunks and the W chunk (256 rows).
struct Plan {
  static constexpr int kWBytes = kVocabTile * 128;
  static constexpr int kStageBytes = 2 * kChunkBytes + kWBytes;
  static constexpr int kOffBar = kStages * kStageBytes;
  // full[3], empty[3], acc_full[2], acc_empty[2] (one accumulator: index 0 only)
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16;
};

// Orderable 32-bit image of a float: unsigned comparison follows the float order.
__device__ __forceinline__ uint32_t order_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_order_bits(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_tc(const __grid_constant__ CUtensorMap hmap,
                      const __grid_constant__ CUtensorMap wmap, const LmHeadParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Plan::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = bars + 2 * kStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Plan::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  const int kchunks = p.hidden / 64;
  const int64_t n_items = (int64_t)p.n_groups * p.n_vtiles;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpilogueWarps * 32);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&hmap);
      tma_prefetch_desc(&wmap);
      int64_t q = 0;  // chunks issued (stage = q % kStages)
      bool ok = true;
      for (int64_t it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const int grp = (int)(it / p.n_vtiles);
        const int64_t vt = it % p.n_vtiles;
        const int row0 = grp * kGroupRows;
        const int halves = p.rows - row0 > kRowsTile ? 2 : 1;
        for (int kc = 0; kc < kchunks; ++kc, ++q) {
          const int s = (int)(q % kStages);
          if (q >= kStages &&
              !mbar_wait_bounded(&empty[s], (uint32_t)(((q / kStages) - 1) & 1), p.err)) {
            ok = false;
            break;
          }
          if (*abort_flag) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * Plan::kStageBytes;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(halves * kChunkBytes + p.n_tile * 128));
          for (int h = 0; h < halves; ++h)
            tma_load_4d(st + h * kChunkBytes, &hmap, &full[s], 0, kc, 0, row0 + h * kRowsTile);
          tma_load_4d(st + 2 * kChunkBytes, &wmap, &full[s], 0, kc, 0, (int)(vt * p.n_tile));
        }
      }
      if (!ok) *abort_flag = 1;
      // the copies this CTA issued land before it leaves
      for (int64_t r = q > kStages ? q - kStages : 0; r < q; ++r)
        mbar_wait_bounded(&full[r % kStages], (uint32_t)((r / kStages) & 1), nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(ab, kRowsTile, p.n_tile, 0, 0);
      const uint64_t d0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
      int64_t q = 0;
      int li = 0;  // items of this CTA (accumulator phases)
      bool ok = true;
      for (int64_t it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++li) {
        const int grp = (int)(it / p.n_vtiles);
        const int halves = p.rows - grp * kGroupRows > kRowsTile ? 2 : 1;
        // the accumulator is free once the epilogue has read item li - 1
        if (li >= 1 && !mbar_wait_bounded(&acc_empty[0], (uint32_t)((li - 1) & 1), p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < kchunks; ++kc, ++q) {
          const int s = (int)(q % kStages);
          if (!mbar_wait_bounded(&full[s], (uint32_t)((q / kStages) & 1), p.err) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t stage = d0 + (uint64_t)((s * Plan::kStageBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bw = stage + (uint64_t)((2 * kChunkBytes + kk * 32) >> 4);
            for (int h = 0; h < halves; ++h)
              mma_ss(tbase + 256u * h,
                     stage + (uint64_t)((h * kChunkBytes + kk * 32) >> 4), bw, idesc,
                     (kc > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[0]);
      }
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    float best_v[2] = {-INFINITY, -INFINITY};
    int64_t best_i[2] = {-1, -1};
    int cur_grp = -1;
    auto flush = [&]() {
      if (cur_grp < 0) return;
      for (int h = 0; h < 2; ++h) {
        const int r = cur_grp * kGroupRows + h * kRowsTile + row_in_tile;
        if (r < p.rows && best_i[h] >= 0) {
          const unsigned long long key =
              ((unsigned long long)order_bits(best_v[h]) << 32) |
              (unsigned long long)(0xffffffffu - (uint32_t)best_i[h]);
          atomicMax(p.keys + r, key);
        }
        best_v[h] = -INFINITY;
        best_i[h] = -1;
      }
    };
    int li = 0;
    for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x, ++li) {
      const int grp = (int)(it / p.n_vtiles);
      const int64_t vt = it % p.n_vtiles;
      const int halves = p.rows - grp * kGroupRows > kRowsTile ? 2 : 1;
      bool ok = !*abort_flag && mbar_wait_bounded(&acc_full[0], (uint32_t)(li & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      if (grp != cur_grp) {
        flush();
        cur_grp = grp;
      }
      tc_fence_after();
      const int64_t col0 = vt * p.n_tile;
      for (int h = 0; h < halves; ++h) {
#pragma unroll 1
        for (int c0 = 0; c0 < p.n_tile; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(lane_base + 256u * h + c0, v);
          tmem_wait_ld();
          // columns past the tile (a 16-column tail) or past the vocabulary (zero-filled W
          // rows) hold no logits of this item: skip them
          const int64_t left = min((int64_t)(p.n_tile - c0), p.vocab - (col0 + c0));
          const int nvalid = left < 32 ? (int)left : 32;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float x = round_to<T>(__uint_as_float(v[c]));
            // strictly greater: within a row group columns arrive in increasing order, so
            // the first of equal values stays
            if (c < nvalid && x > best_v[h]) {
              best_v[h] = x;
              best_i[h] = col0 + c0 + c;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[0]);
    }
    flush();
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                 "r"(kTmemCols));
  // The last CTA turns the keys into ids and re-zeroes keys and counter.
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(p.ctr, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (last) {
    __threadfence();
    for (int r = threadIdx.x; r < p.rows; r += blockDim.x) {
      const unsigned long long key = __ldcg(p.keys + r);
      // No logit of the row compared above -inf: every one is NaN or -inf (a NaN hidden
      // row makes them all NaN). torch's argmax gives index 0 for such a row; so does this,
      // and the id is always a valid token.
      p.out_ids[r] = key ? (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffu)) : 0;
      if (p.out_max) p.out_max[r] = key ? from_order_bits((uint32_t)(key >> 32))
                                 : __int_as_float(0x7fffffff);
      p.keys[r] = 0;
    }
    if (threadIdx.x == 0) *p.ctr = 0;
  }
}

}  // namespace

namespace b2p_host {
int tensor_map_4d_rows(CUtensorMap* out, const void* base, int64_t rows, int heads, int head_dim,
                       int64_t row_stride_elems, int64_t head_stride_elems, int elem_bytes,
                       int box_rows);
}  // namespace b2p_host

// Workspace: per-row keys then the CTA counter, all zero before the first launch (every
// launch that runs to its end leaves them zero).
size_t b2p_lm_head_argmax_workspace_size(int rows) {
  return (size_t)(rows > 0 ? rows : 0) * 8 + 16;
}

int b2p_lm_head_argmax(const void* hidden, int64_t hidden_row_stride,
                                  const void* weight, int64_t weight_row_stride, int rows,
                                  int64_t vocab, int hidden_size, int dtype, int64_t* out_ids,
                                  float* out_max, void* workspace, size_t workspace_bytes,
                                  int32_t* err_flag, void* stream) {
  if (rows < 0 || vocab <= 0 || hidden_size <= 0 || !out_ids ||
      (rows > 0 && (!hidden || !weight || !workspace)))
    return B2P_EINVAL;
  if (rows == 0) return B2P_OK;
  if ((dtype != B2P_BF16 && dtype != B2P_F16) || hidden_size % 64 != 0 ||
      vocab > 0x7fffffffLL - kVocabTile || rows % kRowsTile != 0)
    return B2P_EUNSUPPORTED;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!al16(hidden) || !al16(weight) || (hidden_row_stride * 2) % 16 ||
      (weight_row_stride * 2) % 16)
    return B2P_EUNSUPPORTED;
  if (workspace_bytes < b2p_lm_head_argmax_workspace_size(rows) ||
      (reinterpret_cast<uintptr_t>(workspace) & 7u))
    return B2P_EWORKSPACE;
  // vocab tile: the multiple of 16 (<= 256) that minimises the most vocab entries one SM
  // processes, ceil(items / SMs) * N; on ties the wider tile
  const int n_groups = (rows + kGroupRows - 1) / kGroupRows;
  const int64_t sms = b2p_host::sm_count();
  int n_tile = kVocabTile;
  int64_t best = INT64_MAX;
  for (int n = kVocabTile; n >= 16; n -= 16) {
    const int64_t items = (int64_t)n_groups * ((vocab + n - 1) / n);
    const int64_t cost = (items + sms - 1) / sms * n;
    if (cost < best) {
      best = cost;
      n_tile = n;
    }
  }
  CUtensorMap hmap, wmap;
  int rc = b2p_host::tensor_map_4d_rows(&hmap, hidden, rows, 1, hidden_size, hidden_row_stride,
                                        hidden_size, 2, kRowsTile);
  if (rc != B2P_OK) return rc;
  rc = b2p_host::tensor_map_4d_rows(&wmap, weight, vocab, 1, hidden_size, weight_row_stride,
                                    hidden_size, 2, n_tile);
  if (rc != B2P_OK) return rc;
  LmHeadParams p;
  p.rows = rows;
  p.vocab = vocab;
  p.hidden = hidden_size;
  p.n_groups = n_groups;
  p.n_tile = n_tile;
  p.n_vtiles = (vocab + n_tile - 1) / n_tile;
  p.keys = static_cast<unsigned long long*>(workspace);
  p.ctr = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + (size_t)rows * 8);
  p.out_ids = out_ids;
  p.out_max = out_max;
  p.err = err_flag;
  const void* fn = dtype == B2P_BF16
                       ? reinterpret_cast<const void*>(&lm_head_argmax_tc<__nv_bfloat16>)
                       : reinterpret_cast<const void*>(&lm_head_argmax_tc<__half>);
  const int smem = Plan::kSmemBytes + 1024;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  const int64_t items = (int64_t)p.n_groups * p.n_vtiles;
  const int grid = (int)std::min<int64_t>(items, b2p_host::sm_count());
  void* args[] = {&hmap, &wmap, &p};
  e = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kThreads), args, (size_t)smem,
                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return b2p_host::record_error(e);
  return b2p_host::check_launch();
}
