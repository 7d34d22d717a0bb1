// K2 — ragged GQA decode attention over the paged KV pool (bf16 / f16).
//
// What it replaces: for DECODE executions the reference gathers every sequence's
// history (PagedKVStorage.gather, serving/engine/paged_kv_storage.py:138-174),
// concatenates them (serving/engine/hf_batched_paged_cache.py:128-148), builds a dense
// block-diagonal mask (serving/engine/attention_mask.py:9-120) and runs SDPA over
// all packed keys for every query (transformers/integrations/sdpa_attention.py:40-104).
// Mathematically each decode query attends to its own history only:
//   out[i, h, :] = softmax_t(q[i, h, :] . K[slot(i, t), h / G, :] * scale) @ V[slot(i, t), h / G, :]
// with G = num_q_heads / num_kv_heads (GQA, repeat_kv in the reference).
//
// Design (HBM-bound: 1 KiB of K+V per token for 2 KV heads x 128 dims in bf16):
//  * Work space = for each KV head, the flattened list of 16-slot sub-blocks of all
//    sequences (a 16-slot sub-block is contiguous in the pool because a block's slots are
//    consecutive). Each KV head's list is cut into gridDim.x equal ranges, one per CTA
//    (stream-K), so every CTA streams the same number of bytes whatever the context-length
//    mix; a sequence cut by a range boundary is finished by the last CTA that works on it
//    (counter in the workspace), which merges the partial softmax states.
//  * One producer thread walks the CTA's range, reads block-table entries and issues TMA
//    tile loads (K and V sub-block of one head: 2 x 16 x head_dim elements) into a ring of
//    NS shared-memory stages guarded by mbarriers (full: TMA bytes landed; empty: the
//    consumer warp is done).
//  * Four consumer warps take sub-blocks round-robin. Per sub-block a warp computes
//    S^T = K Q^T on the tensor cores (m16n8k16: 16 tokens x 8 query heads of the GQA group,
//    K loaded with ldmatrix from the 128-byte-swizzled tile), the online softmax in fp32
//    (warp shuffles over the 8 lanes that share a query head), and O^T += V^T P^T (V^T from
//    ldmatrix.trans, P^T transposed in registers with movmatrix). Each KV tile read from
//    shared memory serves all G query heads of its group.
//  * At a sequence boundary the four warps merge their (max, sum, O) states through shared
//    memory and write the bf16 output, or an fp32 partial for the cross-CTA merge.
#include "common.cuh"

namespace {

using namespace b2p;

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSub = 16;  // slots per sub-block = tokens per MMA tile

struct DecodeParams {
  const uint8_t* q;
  int64_t q_tok, q_head;  // element strides
  uint8_t* out;
  int64_t o_tok, o_head;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* context_lens;
  int num_seqs;
  int group;       // G, query heads per KV head
  int layer;
  int block_size;  // multiple of 16
  int64_t num_blocks;
  float scale_log2;  // softmax scale * log2(e)
  float* partials;   // [num_kv_heads][gridDim.x][2][NT*8*(D+2)]
  int32_t* counters; // [num_kv_heads][num_seqs], zero between launches
  int32_t* err;
};

// Shared-memory plan (dynamic, 1024-byte aligned base).
template <int D, int NT, int NS>
struct Smem {
  // Stage s is only ever consumed by warp s % kConsumerWarps, one use after another, so a
  // consumer can never wait on a stage's phase u while phase u-1 is still pending (the
  // parity of an mbarrier wait cannot tell those two apart).
  static_assert(NS % kConsumerWarps == 0, "stages must be a multiple of the consumer warps");
  static constexpr int kTileBytes = kSub * D * 2;  // one K or V sub-block of one head
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = NS * kStageBytes;
  static constexpr int kCombO = kConsumerWarps * NT * 8 * D * 4;  // fp32 O^T per warp
  static constexpr int kCombML = kConsumerWarps * NT * 8 * 2 * 4;
  static constexpr int kOffComb = kStages;
  static constexpr int kOffML = kOffComb + kCombO;
  static constexpr int kOffBar = kOffML + kCombML;
  static constexpr int kOffMisc = kOffBar + 2 * NS * 8;
  static constexpr int kTotal = kOffMisc + 8 * 8;
};

struct CtaRange {
  int64_t begin, end;  // global sub-block indices of this CTA (per KV head)
  int seq0;            // sequence containing `begin`
  int64_t cb0;         // first global sub-block index of seq0
  int64_t total;       // sub-blocks over all sequences (per KV head)
  int64_t parts;       // ranges actually used: min(gridDim.x, total)
};

__device__ __forceinline__ int64_t range_start(int64_t c, int64_t total, int64_t parts) {
  return (c * total) / parts;
}

__device__ __forceinline__ int64_t owner_cta(int64_t b, int64_t total, int64_t parts) {
  return ((b + 1) * parts - 1) / total;
}

__device__ __forceinline__ int sub_blocks_of(int ctx) { return ctx > 0 ? (ctx + kSub - 1) / kSub : 0; }

// One warp: total sub-blocks over all sequences, then the sequence holding `target`.
// Leaves the answer in lane 0's return value (all lanes return the same).
__device__ void find_range(const DecodeParams& p, int64_t parts, int64_t c, CtaRange& r) {
  const int lane = threadIdx.x & 31;
  int64_t total = 0;
  for (int base = 0; base < p.num_seqs; base += 32) {
    const int i = base + lane;
    int nb = 0;
    if (i < p.num_seqs) nb = sub_blocks_of(__ldg(p.context_lens + i));
    total += __reduce_add_sync(0xffffffffu, (unsigned)nb);
  }
  r.total = total;
  // Never more ranges than sub-blocks, so every range is non-empty and the CTAs that
  // share a sequence are exactly owner(first block) .. owner(last block).
  r.parts = parts < total ? parts : total;
  if (c >= r.parts) {
    r.begin = r.end = 0;
    return;
  }
  r.begin = range_start(c, total, r.parts);
  r.end = range_start(c + 1, total, r.parts);
  r.seq0 = p.num_seqs;
  r.cb0 = total;
  if (r.begin >= r.end) return;
  int64_t run = 0;
  for (int base = 0; base < p.num_seqs; base += 32) {
    const int i = base + lane;
    int nb = 0;
    if (i < p.num_seqs) nb = sub_blocks_of(__ldg(p.context_lens + i));
    // inclusive warp scan
    int incl = nb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t hi = run + incl;  // exclusive end of sequence i
    const unsigned hit = __ballot_sync(0xffffffffu, i < p.num_seqs && hi > r.begin);
    if (hit) {
      const int src = __ffs(hit) - 1;
      r.seq0 = base + src;
      r.cb0 = run + __shfl_sync(0xffffffffu, incl - nb, src);
      return;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
}

template <typename T, int D, int NT, int NS>
__global__ void __launch_bounds__(kThreads) paged_decode_tc(const __grid_constant__ CUtensorMap kmap,
                                                            const __grid_constant__ CUtensorMap vmap,
                                                            const DecodeParams p) {
  using S = Smem<D, NT, NS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* empty = full + NS;
  int64_t* misc = reinterpret_cast<int64_t*>(smem + S::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;  // KV head
  const int64_t cta = blockIdx.x;

  if (warp == kConsumerWarps) {
    CtaRange r;
    find_range(p, (int64_t)gridDim.x, cta, r);
    if (lane == 0) {
      misc[0] = r.begin;
      misc[1] = r.end;
      misc[2] = r.seq0;
      misc[3] = r.cb0;
      misc[6] = r.total;
      misc[7] = r.parts;
      *abort_flag = 0;
      for (int s = 0; s < NS; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], 1);
      }
      fence_mbar_init();
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
  }
  __syncthreads();
  const int64_t begin = misc[0];
  const int64_t end = misc[1];
  if (begin >= end) return;
  const int64_t nloc = end - begin;
  const int64_t parts = misc[7];

  // ------------------------------------------------------------------ producer
  if (warp == kConsumerWarps) {
    if (lane != 0) return;
    int seq = (int)misc[2];
    int64_t cb = misc[3];
    int ctx = __ldg(p.context_lens + seq);
    int nb = sub_blocks_of(ctx);
    const int sub_per_block = p.block_size / kSub;
    const int64_t num_slots = p.num_blocks * p.block_size;
    int64_t issued = 0;
    for (int64_t l = 0; l < nloc; ++l) {
      const int64_t g = begin + l;
      while (g >= cb + nb) {  // advance to the sequence holding g
        cb += nb;
        ++seq;
        ctx = __ldg(p.context_lens + seq);
        nb = sub_blocks_of(ctx);
      }
      const int stage = (int)(l % NS);
      if (l >= NS) {
        if (!mbar_wait_bounded(&empty[stage], (uint32_t)(((l / NS) - 1) & 1), p.err)) {
          *abort_flag = 1;
          break;
        }
      }
      if (*abort_flag) break;
      const int lb = (int)(g - cb);
      const int64_t col = lb / sub_per_block;
      const int32_t blk =
          col < p.bt_stride ? __ldg(p.block_tables + (int64_t)seq * p.bt_stride + col) : -1;
      int64_t slot = (int64_t)blk * p.block_size + (int64_t)(lb % sub_per_block) * kSub;
      if (blk < 0 || (int64_t)blk >= p.num_blocks) {
        set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
        slot = num_slots;  // fully out of bounds: the TMA unit zero-fills the tile
      }
      uint8_t* kdst = smem + stage * S::kStageBytes;
      uint8_t* vdst = kdst + S::kTileBytes;
      mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
      tma_load_5d(kdst, &kmap, &full[stage], 0, 0, head, (int)slot, p.layer);
      tma_load_5d(vdst, &vmap, &full[stage], 0, 0, head, (int)slot, p.layer);
      issued = l + 1;
    }
    // Drain: never leave the CTA while TMA writes into its shared memory are in flight.
    for (int64_t l = (issued > NS ? issued - NS : 0); l < issued; ++l) {
      mbar_wait_bounded(&full[l % NS], (uint32_t)((l / NS) & 1), nullptr);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int g8 = lane >> 2;  // row group (0..7)
  const int t4 = lane & 3;   // thread in group (0..3)
  const int ctid = threadIdx.x;  // 0..127
  float* combO = reinterpret_cast<float*>(smem + S::kOffComb);
  float* combM = reinterpret_cast<float*>(smem + S::kOffML);
  float* combL = combM + kConsumerWarps * NT * 8;
  volatile int* merge_flag = reinterpret_cast<volatile int*>(misc + 5);

  int seq = (int)misc[2];
  int64_t cb = misc[3];
  int64_t g = begin;
  const size_t part_stride = (size_t)NT * 8 * (D + 2);

  while (g < end) {
    const int ctx = __ldg(p.context_lens + seq);
    const int nb = sub_blocks_of(ctx);
    const int lb0 = (int)(g - cb);
    const int64_t seg_end_g = min(end, cb + nb);
    const int lb1 = (int)(seg_end_g - cb);
    if (nb == 0) {
      // A decode sequence always has at least its own token; an empty history has no
      // softmax. Write zeros and flag it.
      if (ctid == 0) set_device_error(p.err, B2P_DEV_LENGTH);
      for (int e = ctid; e < p.group * D; e += kConsumerWarps * 32) {
        const int qh = e / D, d = e - qh * D;
        reinterpret_cast<T*>(p.out)[(int64_t)seq * p.o_tok + (int64_t)(head * p.group + qh) * p.o_head + d] =
            from_f32<T>(0.f);
      }
      ++seq;
      continue;
    }

    // Q fragments (B operand of S^T = K Q^T): Q[qh = g8 + 8n][16kk + 2t4 (+8)].
    uint32_t qf[NT][D / 16][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int qh = n * 8 + g8;
      const bool ok = qh < p.group;
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)seq * p.q_tok +
                      (int64_t)(head * p.group + (ok ? qh : 0)) * p.q_head;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qf[n][kk][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4)) : 0u;
        qf[n][kk][1] =
            ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * t4)) : 0u;
      }
    }

    float m_run[NT][2], l_run[NT][2];
    float acc[D / 16][NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      m_run[n][0] = m_run[n][1] = -INFINITY;
      l_run[n][0] = l_run[n][1] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i)
#pragma unroll
      for (int n = 0; n < NT; ++n) acc[i][n][0] = acc[i][n][1] = acc[i][n][2] = acc[i][n][3] = 0.f;

    // First local index in this segment that belongs to this warp.
    const int64_t l_first = (cb + lb0) - begin;
    int64_t l = l_first + ((warp - (int)(l_first % kConsumerWarps) + kConsumerWarps) % kConsumerWarps);
    const int64_t l_last = (cb + lb1) - begin;  // exclusive
    for (; l < l_last; l += kConsumerWarps) {
      const int stage = (int)(l % NS);
      if (*abort_flag) break;
      if (!mbar_wait_bounded(&full[stage], (uint32_t)((l / NS) & 1), p.err)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* ktile = smem + stage * S::kStageBytes;
      uint8_t* vtile = const_cast<uint8_t*>(ktile) + S::kTileBytes;
      const int lb = (int)(begin + l - cb);
      const int valid = min(kSub, ctx - lb * kSub);
      if (valid < kSub) {
        // Slots past the context may hold anything (the pool is not cleared), and
        // 0 * NaN would poison O: zero the V rows of masked tokens. A token row is
        // D*2 contiguous bytes (whole swizzle lines), so no swizzle math is needed.
        const int zero_bytes = (kSub - valid) * D * 2;
        uint4* z = reinterpret_cast<uint4*>(vtile + valid * D * 2);
        for (int i = lane; i < zero_bytes / 16; i += 32) z[i] = make_uint4(0, 0, 0, 0);
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(ktile);
      const uint32_t vbase = smem_u32(vtile);

      // ---- S^T = K Q^T  (M = 16 tokens, N = 8 query heads per tile, K = D)
      float s[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      {
        const int mat = lane >> 3, r = lane & 7;
        const int tok = r + (mat & 1) * 8;
        const int dsub = (mat >> 1) * 8;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int dcol = kk * 16 + dsub;
          const uint32_t off = (uint32_t)((tok * (D / 64) + dcol / 64) * 128 + (dcol % 64) * 2);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(kbase + swz128(off), a0, a1, a2, a3);
#pragma unroll
          for (int n = 0; n < NT; ++n) MmaOp<T>::run(s[n], a0, a1, a2, a3, qf[n][kk][0], qf[n][kk][1]);
        }
      }

      // ---- online softmax over the tile's tokens (rows g8 and g8+8)
      const bool v0 = g8 < valid, v1 = g8 + 8 < valid;
      uint32_t pb[NT][2];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        float x0 = v0 ? s[n][0] * p.scale_log2 : -INFINITY;
        float x1 = v0 ? s[n][1] * p.scale_log2 : -INFINITY;
        float x2 = v1 ? s[n][2] * p.scale_log2 : -INFINITY;
        float x3 = v1 ? s[n][3] * p.scale_log2 : -INFINITY;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m_run[n][0], mx0), mn1 = fmaxf(m_run[n][1], mx1);
        const float al0 = fast_exp2(m_run[n][0] - mn0), al1 = fast_exp2(m_run[n][1] - mn1);
        m_run[n][0] = mn0;
        m_run[n][1] = mn1;
        const float p0 = fast_exp2(x0 - mn0), p1 = fast_exp2(x1 - mn1);
        const float p2 = fast_exp2(x2 - mn0), p3 = fast_exp2(x3 - mn1);
        l_run[n][0] = l_run[n][0] * al0 + p0 + p2;
        l_run[n][1] = l_run[n][1] * al1 + p1 + p3;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          acc[i][n][0] *= al0;
          acc[i][n][1] *= al1;
          acc[i][n][2] *= al0;
          acc[i][n][3] *= al1;
        }
        pb[n][0] = movmatrix_trans(pack2<T>(p0, p1));
        pb[n][1] = movmatrix_trans(pack2<T>(p2, p3));
      }

      // ---- O^T += V^T P^T  (M = 16 dims per tile, N = 8 query heads, K = 16 tokens)
      {
        const int mat = lane >> 3, r = lane & 7;
        const int tok = r + (mat >> 1) * 8;
        const int dsub = (mat & 1) * 8;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          const int dcol = i * 16 + dsub;
          const uint32_t off = (uint32_t)((tok * (D / 64) + dcol / 64) * 128 + (dcol % 64) * 2);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(vbase + swz128(off), a0, a1, a2, a3);
#pragma unroll
          for (int n = 0; n < NT; ++n) MmaOp<T>::run(acc[i][n], a0, a1, a2, a3, pb[n][0], pb[n][1]);
        }
      }
      if (valid < kSub) fence_proxy_async_smem();  // generic writes before the TMA reuses it
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }

    // ---- merge the four warps' states for this segment
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l_run[n][0] += __shfl_xor_sync(0xffffffffu, l_run[n][0], o);
        l_run[n][1] += __shfl_xor_sync(0xffffffffu, l_run[n][1], o);
      }
      if (g8 == 0) {
        combM[(warp * NT + n) * 8 + 2 * t4] = m_run[n][0];
        combM[(warp * NT + n) * 8 + 2 * t4 + 1] = m_run[n][1];
        combL[(warp * NT + n) * 8 + 2 * t4] = l_run[n][0];
        combL[(warp * NT + n) * 8 + 2 * t4 + 1] = l_run[n][1];
      }
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        float* base = combO + (size_t)(warp * NT + n) * 8 * D;
        base[(2 * t4) * D + i * 16 + g8] = acc[i][n][0];
        base[(2 * t4 + 1) * D + i * 16 + g8] = acc[i][n][1];
        base[(2 * t4) * D + i * 16 + g8 + 8] = acc[i][n][2];
        base[(2 * t4 + 1) * D + i * 16 + g8 + 8] = acc[i][n][3];
      }
    }
    asm volatile("bar.sync 1, %0;\n" ::"r"(kConsumerWarps * 32) : "memory");

    const bool complete = (lb0 == 0) && (lb1 == nb);
    const int nelem = p.group * D;
    float* part = nullptr;
    if (!complete) {
      const int slot_idx = (cb + lb0 == begin) ? 0 : 1;  // first segment of this CTA or not
      part = p.partials + (((size_t)head * parts + cta) * 2 + slot_idx) * part_stride;
    }
    for (int e = ctid; e < nelem; e += kConsumerWarps * 32) {
      const int qh = e / D, d = e - qh * D;
      const int n = qh >> 3, col = qh & 7;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, combM[(w * NT + n) * 8 + col]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float sc = fast_exp2(combM[(w * NT + n) * 8 + col] - M);
        L += combL[(w * NT + n) * 8 + col] * sc;
        O += combO[(size_t)(w * NT + n) * 8 * D + col * D + d] * sc;
      }
      if (complete) {
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)seq * p.o_tok +
                  (int64_t)(head * p.group + qh) * p.o_head;
        orow[d] = from_f32<T>(O / L);
      } else {
        part[qh * D + d] = O;
        if (d == 0) {
          part[NT * 8 * D + qh] = M;
          part[NT * 8 * D + NT * 8 + qh] = L;
        }
      }
    }

    if (!complete) {
      __threadfence();
      asm volatile("bar.sync 1, %0;\n" ::"r"(kConsumerWarps * 32) : "memory");
      if (ctid == 0) {
        const int64_t tot = misc[6];
        const int64_t c_first = owner_cta(cb, tot, parts);
        const int64_t c_last = owner_cta(cb + nb - 1, tot, parts);
        const int expected = (int)(c_last - c_first + 1);
        int32_t* ctr = p.counters + (size_t)head * p.num_seqs + seq;
        const int prev = atomicAdd(ctr, 1);
        const int last = (prev == expected - 1);
        if (last) *ctr = 0;  // leave the workspace zeroed for the next launch
        *merge_flag = last;
      }
      asm volatile("bar.sync 1, %0;\n" ::"r"(kConsumerWarps * 32) : "memory");
      if (*merge_flag) {
        __threadfence();
        const int64_t tot = misc[6];
        const int64_t c_first = owner_cta(cb, tot, parts);
        const int64_t c_last = owner_cta(cb + nb - 1, tot, parts);
        for (int e = ctid; e < nelem; e += kConsumerWarps * 32) {
          const int qh = e / D, d = e - qh * D;
          float M = -INFINITY;
          for (int64_t c = c_first; c <= c_last; ++c) {
            const int si = (c == c_first && range_start(c, tot, parts) != cb) ? 1 : 0;
            const float* pc = p.partials + (((size_t)head * parts + c) * 2 + si) * part_stride;
            M = fmaxf(M, __ldcg(pc + NT * 8 * D + qh));
          }
          float L = 0.f, O = 0.f;
          for (int64_t c = c_first; c <= c_last; ++c) {
            const int si = (c == c_first && range_start(c, tot, parts) != cb) ? 1 : 0;
            const float* pc = p.partials + (((size_t)head * parts + c) * 2 + si) * part_stride;
            const float sc = fast_exp2(__ldcg(pc + NT * 8 * D + qh) - M);
            L += __ldcg(pc + NT * 8 * D + NT * 8 + qh) * sc;
            O += __ldcg(pc + qh * D + d) * sc;
          }
          T* orow = reinterpret_cast<T*>(p.out) + (int64_t)seq * p.o_tok +
                    (int64_t)(head * p.group + qh) * p.o_head;
          orow[d] = from_f32<T>(O / L);
        }
      }
    }
    asm volatile("bar.sync 1, %0;\n" ::"r"(kConsumerWarps * 32) : "memory");
    // After an abort the warps skip all waits and MMA work but still walk every segment,
    // so the named barriers above are always reached by all four consumer warps.
    g = seg_end_g;
    if (lb1 == nb) {
      cb += nb;
      ++seq;
    }
  }
}

}  // namespace

// ====================================================================== host side
namespace {

using KernelFn = void (*)(CUtensorMap, CUtensorMap, DecodeParams);

struct Plan {
  const void* fn = nullptr;
  int smem = 0;
  int ctas_per_sm = 0;
};

template <typename T, int D, int NT, int NS>
Plan make_plan() {
  Plan pl;
  pl.fn = reinterpret_cast<const void*>(&paged_decode_tc<T, D, NT, NS>);
  pl.smem = Smem<D, NT, NS>::kTotal + 1024;  // + alignment slack for the 1024-byte base
  return pl;
}

// Pick the kernel instantiation for (dtype, head_dim, group). Stage counts keep roughly
// 48-64 KiB of K/V tiles in flight per CTA.
bool select_plan(int dtype, int head_dim, int group, Plan& pl) {
  const int nt = group <= 8 ? 1 : (group <= 16 ? 2 : 0);
  if (nt == 0) return false;
#define B2P_CASE(TT, DD, NN, SS)                                                  \
  if (head_dim == DD && nt == NN) {                                               \
    pl = make_plan<TT, DD, NN, SS>();                                             \
    return true;                                                                  \
  }
  if (dtype == B2P_BF16) {
    B2P_CASE(__nv_bfloat16, 64, 1, 12)
    B2P_CASE(__nv_bfloat16, 64, 2, 12)
    B2P_CASE(__nv_bfloat16, 128, 1, 8)
    B2P_CASE(__nv_bfloat16, 128, 2, 8)
    B2P_CASE(__nv_bfloat16, 256, 1, 4)
  } else if (dtype == B2P_F16) {
    B2P_CASE(__half, 64, 1, 12)
    B2P_CASE(__half, 64, 2, 12)
    B2P_CASE(__half, 128, 1, 8)
    B2P_CASE(__half, 128, 2, 8)
    B2P_CASE(__half, 256, 1, 4)
  }
#undef B2P_CASE
  return false;
}

int prepare(Plan& pl) {
  static thread_local const void* last_fn[16] = {nullptr};
  static thread_local int last_occ[16] = {0};
  static thread_local int last_dev[16] = {-1};
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < 16; ++i) {
    if (last_fn[i] == pl.fn && last_dev[i] == dev) {
      pl.ctas_per_sm = last_occ[i];
      return B2P_OK;
    }
  }
  if (cudaFuncSetAttribute(pl.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) !=
      cudaSuccess)
    return b2p_host::check_launch();
  int occ = 0;
  cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pl.fn, kThreads, pl.smem);
  if (oe != cudaSuccess) return b2p_host::record_error(oe);
  if (occ <= 0) return B2P_EUNSUPPORTED;
  for (int i = 0; i < 16; ++i) {
    if (last_fn[i] == nullptr) {
      last_fn[i] = pl.fn;
      last_occ[i] = occ;
      last_dev[i] = dev;
      break;
    }
  }
  pl.ctas_per_sm = occ;
  return B2P_OK;
}

int64_t parts_per_head(int ctas_per_sm, int num_kv_heads) {
  if (ctas_per_sm > 8) ctas_per_sm = 8;  // the workspace is sized for at most 8 per SM
  const int64_t slots = (int64_t)b2p_host::sm_count() * ctas_per_sm;
  int64_t parts = slots / num_kv_heads;
  return parts < 1 ? 1 : parts;
}

size_t workspace_bytes(int num_seqs, int num_kv_heads, int head_dim, int nt, int64_t parts) {
  const size_t counters = ((size_t)num_kv_heads * num_seqs * 4 + 255) & ~size_t(255);
  const size_t part = (size_t)num_kv_heads * parts * 2 * nt * 8 * (head_dim + 2) * 4;
  return counters + part;
}

}  // namespace

extern "C" size_t b2p_paged_decode_workspace_size(int num_seqs, int num_q_heads,
                                                  int num_kv_heads, int head_dim) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  const int nt = group <= 8 ? 1 : 2;
  // Upper bound over the instantiations: at most 8 CTAs of this kernel fit on an SM.
  return workspace_bytes(num_seqs, num_kv_heads, head_dim, nt, parts_per_head(8, num_kv_heads));
}

int b2p_decode_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                    const void* key_cache, const void* value_cache, int64_t layer_index,
                    int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                    int64_t block_table_stride, const int32_t* context_lens, int num_seqs,
                    int num_q_heads, int num_kv_heads, int head_dim, int block_size, float scale,
                    void* out, int64_t out_tok_stride, int64_t out_head_stride, int dtype,
                    int32_t* err_flag, void* stream);

extern "C" int b2p_paged_decode(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                                const void* key_cache, const void* value_cache,
                                int64_t layer_index, int64_t num_layers, int64_t num_slots,
                                const int32_t* block_tables, int64_t block_table_stride,
                                const int32_t* context_lens, int num_seqs, int num_q_heads,
                                int num_kv_heads, int head_dim, int block_size, float scale,
                                void* out, int64_t out_tok_stride, int64_t out_head_stride,
                                void* workspace, size_t workspace_size, int dtype,
                                int32_t* err_flag, void* stream) {
  if (num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_slots <= 0 || num_layers <= 0)
    return B2P_EINVAL;
  if (num_q_heads % num_kv_heads != 0) return B2P_EINVAL;
  if (layer_index < 0 || layer_index >= num_layers) return B2P_ERANGE;
  if (num_slots % block_size != 0) return B2P_EINVAL;
  if (num_seqs == 0) return B2P_OK;
  if (!q || !key_cache || !value_cache || !block_tables || !context_lens || !out)
    return B2P_EINVAL;
  const int group = num_q_heads / num_kv_heads;

  Plan pl;
  const bool tc = (dtype == B2P_BF16 || dtype == B2P_F16) && block_size % 16 == 0 &&
                  (q_tok_stride % 2 == 0) && (q_head_stride % 2 == 0) &&
                  ((reinterpret_cast<uintptr_t>(q) & 3u) == 0) &&
                  ((reinterpret_cast<uintptr_t>(key_cache) & 15u) == 0) &&
                  ((reinterpret_cast<uintptr_t>(value_cache) & 15u) == 0) &&
                  select_plan(dtype, head_dim, group, pl);
  if (!tc) {
    return b2p_decode_simt(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                           num_layers, num_slots, block_tables, block_table_stride, context_lens,
                           num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                           out_tok_stride, out_head_stride, dtype, err_flag, stream);
  }
  if (!workspace) return B2P_EWORKSPACE;
  int rc = prepare(pl);
  if (rc != B2P_OK) return rc;
  const int nt = group <= 8 ? 1 : 2;
  const int64_t parts = parts_per_head(pl.ctas_per_sm, num_kv_heads);
  const size_t need = workspace_bytes(num_seqs, num_kv_heads, head_dim, nt, parts);
  if (workspace_size < need) return B2P_EWORKSPACE;

  CUtensorMap kmap, vmap;
  rc = b2p_host::pool_tensor_map(&kmap, key_cache, num_layers, num_slots, num_kv_heads,
                                 head_dim, 2);
  if (rc != B2P_OK) return rc;
  rc = b2p_host::pool_tensor_map(&vmap, value_cache, num_layers, num_slots, num_kv_heads,
                                 head_dim, 2);
  if (rc != B2P_OK) return rc;

  DecodeParams p;
  p.q = static_cast<const uint8_t*>(q);
  p.q_tok = q_tok_stride;
  p.q_head = q_head_stride;
  p.out = static_cast<uint8_t*>(out);
  p.o_tok = out_tok_stride;
  p.o_head = out_head_stride;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.context_lens = context_lens;
  p.num_seqs = num_seqs;
  p.group = group;
  p.layer = (int)layer_index;
  p.block_size = block_size;
  p.num_blocks = num_slots / block_size;
  p.scale_log2 = scale * kLog2e;
  const size_t counters_bytes = ((size_t)num_kv_heads * num_seqs * 4 + 255) & ~size_t(255);
  p.counters = static_cast<int32_t*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + counters_bytes);
  p.err = err_flag;

  dim3 grid((unsigned)parts, (unsigned)num_kv_heads);
  void* args[] = {&kmap, &vmap, &p};
  cudaError_t e = cudaLaunchKernel(pl.fn, grid, dim3(kThreads), args, (size_t)pl.smem,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return b2p_host::record_error(e);
  return b2p_host::check_launch();
}
