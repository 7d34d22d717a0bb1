// K3 — packed variable-length causal prefill / chunked-prefill attention on tcgen05.
//
// Reference path replaced (PREFILL executions): HFBatchedPagedCache.update gathers every
// history (serving/engine/hf_batched_paged_cache.py:52-148), build_attention_mask adds a
// dense tril block per prefill (serving/engine/attention_mask.py:37-45) and HF SDPA runs
// over all packed keys (transformers/integrations/sdpa_attention.py:40-104). Here each CTA
// computes one tile of 128 query rows of one (sequence, query head) against the sequence's
// keys read in place from the paged pool:
//
//   S = Q K^T   tcgen05.mma kind::f16, A = Q (smem, K-major), B = K tile (smem, K-major),
//               D = S in tensor memory (fp32, 128 lanes x 64 columns, two buffers)
//   P = softmax rows of S, one thread per query row (tcgen05.ld -> fp32 -> exp2), written
//       back as bf16/f16 over its own S buffer (tcgen05.st)
//   O += P V    tcgen05.mma with A = P from tensor memory, B = V tile (smem, MN-major),
//               D = O in tensor memory (fp32, 128 x head_dim)
//
// K/V tiles of 64 tokens are assembled from four 16-slot pool sub-blocks (TMA tile loads,
// 128-byte swizzle, no multicast) into a two-stage ring. A query row j of sequence i sits
// at position ctx_i - q_len_i + j and sees keys 0..position (whole-history prefill when
// q_len == ctx, chunked prefill otherwise). The running max is only moved (and O rescaled)
// when a row's max grows by more than 2^8, so exp2 values stay below 256 and the O
// correction is rare.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = tensor-memory owner and MMA
// issuer (one thread), warps 2..5 = softmax + epilogue (thread = TMEM lane = query row).
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace {

using namespace b2p;

constexpr int kM = 128;     // query rows per tile
constexpr int kN = 64;      // keys per KV tile
constexpr int kD = 128;     // head_dim handled by this kernel
constexpr int kThreads = 192;
constexpr int kSub = 16;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillParams {
  int hq;                  // query heads
  int32_t* ctr;            // {next work item, CTAs done}: zero at launch, re-zeroed at the end
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* cu_q;
  const int32_t* ctx;
  int num_seqs;
  int group;
  int layer;
  int block_size;
  int64_t num_blocks;
  float scale_log2;
  uint8_t* out;
  int64_t o_tok, o_head;
  int32_t* err;
};

// Shared-memory plan (bytes from the 1024-aligned base).
constexpr int kQBytes = 2 * kM * 128;        // 2 chunks x 128 rows x 128 B
constexpr int kKVBytes = 2 * kN * 128;       // 2 chunks x 64 rows x 128 B
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;       // 2 stages
constexpr int kOffV = kOffK + 2 * kKVBytes;  // 2 stages
constexpr int kOffBar = kOffV + 2 * kKVBytes;
constexpr int kNumBars = 1 + 2 * 7 + 1 + 1 + 4;  // q_full, k_full[2], v_full[2], k_empty[2],
                                                // s_full[2], p_full[2], o_done[2], v_empty[2],
                                                // mma_done, q_empty, item_full[2], item_empty[2]
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kOffItems = kOffMisc + 64;
constexpr int kSmemBytes = kOffItems + 2 * 48;

// TMEM columns: S buffers at 0 and 64, O at 128 (256 allocated).
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS0 = 0, kColS1 = 64, kColO = 128;

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B of `ab` format (0 = f16,
// 1 = bf16), A/B major (0 = K-major, 1 = MN-major), M x N.
__device__ __forceinline__ uint32_t idesc_f16(uint32_t ab, int m, int n, uint32_t a_mn,
                                              uint32_t b_mn) {
  return (1u << 4) | (ab << 7) | (ab << 10) | (a_mn << 15) | (b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

#define B2P_R32(v)                                                                        \
  "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),    \
      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),          \
      "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),       \
      "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),       \
      "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
#define B2P_W32(v)                                                                        \
  "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), \
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),   \
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), \
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), \
      "r"(v[29]), "r"(v[30]), "r"(v[31])

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : B2P_R32(v)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      B2P_W32(v));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Row max of a 64-key S tile (columns 0..31 in r0, 32..63 in r1), four independent
// chains. kMasked: keys at or past `nvis` are ignored.
template <bool kMasked>
__device__ __forceinline__ float row_max64(const uint32_t (&r0)[32], const uint32_t (&r1)[32],
                                           int nvis) {
  float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const float x0 = __uint_as_float(r0[c]), x1 = __uint_as_float(r0[c + 1]);
    const float x2 = __uint_as_float(r1[c]), x3 = __uint_as_float(r1[c + 1]);
    a0 = fmaxf(a0, (!kMasked || c < nvis) ? x0 : -INFINITY);
    a1 = fmaxf(a1, (!kMasked || c + 1 < nvis) ? x1 : -INFINITY);
    a2 = fmaxf(a2, (!kMasked || 32 + c < nvis) ? x2 : -INFINITY);
    a3 = fmaxf(a3, (!kMasked || 33 + c < nvis) ? x3 : -INFINITY);
  }
  return fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
}

// P = exp2(S * scale_log2 - m) of a 64-key row, packed in pairs for tcgen05.st; returns
// the row sum. kMasked: keys at or past `nvis` get 0.
template <typename T, bool kMasked>
__device__ __forceinline__ float row_exp64(const uint32_t (&r0)[32], const uint32_t (&r1)[32],
                                           int nvis, float scale_log2, float m,
                                           uint32_t (&pk)[32]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int c = 0; c < 16; ++c) {  // tokens 0..31 from r0, 32..63 from r1
    const float e0 = (!kMasked || 2 * c < nvis) ? fast_exp2(__uint_as_float(r0[2 * c]) * scale_log2 - m) : 0.f;
    const float e1 = (!kMasked || 2 * c + 1 < nvis) ? fast_exp2(__uint_as_float(r0[2 * c + 1]) * scale_log2 - m) : 0.f;
    const float e2 = (!kMasked || 32 + 2 * c < nvis) ? fast_exp2(__uint_as_float(r1[2 * c]) * scale_log2 - m) : 0.f;
    const float e3 = (!kMasked || 33 + 2 * c < nvis) ? fast_exp2(__uint_as_float(r1[2 * c + 1]) * scale_log2 - m) : 0.f;
    s0 += e0 + e1;
    s1 += e2 + e3;
    pk[c] = pack2<T>(e0, e1);
    pk[16 + c] = pack2<T>(e2, e3);
  }
  return s0 + s1;
}

// Work items. Sequence s has ntiles(s) = ceil(q_len_s / 128) query tiles; tile-items are
// ordered round by round from the end: round r holds tile ntiles(s) - 1 - r of every
// sequence with more than r tiles, sequences in index order. A sequence's later tiles see
// more keys, so the order runs close to longest first (LPT) whatever the prompt mix. Work
// item k is tile-item k / HQ for query head k % HQ: the query heads of one tile are
// neighbours, so the heads of a GQA group, which read the same K/V tiles, run together and
// share them through L2.
struct ItemInfo {
  int seq;  // -1: no more work for this CTA
  int qt, qh, q0, qlen, ctx, rows_valid, pos0, n_kv, pad[3];
};

__device__ __forceinline__ int ntiles_of(const PrefillParams& p, int s) {
  const int q = __ldg(p.cu_q + s + 1) - __ldg(p.cu_q + s);
  return q > 0 ? ceil_div(q, kM) : 0;
}

__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Tile-items in rounds before r: sum over sequences of min(ntiles, r). One warp.
__device__ int64_t items_before_round(const PrefillParams& p, int r, int lane) {
  int64_t acc = 0;
  for (int s = lane; s < p.num_seqs; s += 32) acc += min(ntiles_of(p, s), r);
  return warp_sum64(acc);
}

// Tile-item t -> (sequence, query tile). One warp; all lanes get the result.
__device__ bool decode_tile_item(const PrefillParams& p, int64_t t, int maxnt, int lane,
                                 int& seq, int& tile) {
  int lo = 0, hi = maxnt - 1;  // largest r with items_before_round(r) <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (items_before_round(p, mid, lane) <= t) lo = mid; else hi = mid - 1;
  }
  int64_t i = t - items_before_round(p, lo, lane);
  for (int base = 0; base < p.num_seqs; base += 32) {
    const int s = base + lane;
    const int nt = s < p.num_seqs ? ntiles_of(p, s) : 0;
    const unsigned m = __ballot_sync(0xffffffffu, nt > lo);
    const int c = __popc(m);
    if (i < c) {
      const int pos = __fns(m, 0, (int)i + 1);
      seq = base + pos;
      tile = __shfl_sync(0xffffffffu, nt, pos) - 1 - lo;
      return true;
    }
    i -= c;
  }
  return false;
}

// Persistent CTAs (two per SM) claim work items in the order above from an atomic counter
// (dynamic, so faster SMs take more items and the short items come last). Tensor memory, barriers and descriptors are set up once; the stage, S-buffer and
// item counters run on across items, so the next item's Q and first K/V tiles load while
// the current item finishes, and its first QK^T MMAs run during the current epilogue.
template <typename T>
__global__ void __launch_bounds__(kThreads, 2) paged_prefill_tc(const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap,
                                                                const PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 3;
  uint64_t* k_empty = bars + 5;
  uint64_t* s_full = bars + 7;
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 11;
  uint64_t* v_empty = bars + 13;
  uint64_t* mma_done = bars + 15;
  uint64_t* q_empty = bars + 16;
  uint64_t* item_full = bars + 17;
  uint64_t* item_empty = bars + 19;
  int32_t* misc = reinterpret_cast<int32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 5);
  ItemInfo* items = reinterpret_cast<ItemInfo*>(smem + kOffItems);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0;
    misc[0] = misc[1] = misc[2] = misc[3] = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kM);
      mbar_init(&o_done[s], 1);
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], 5);  // the MMA issuer and the four softmax warps
    }
    mbar_init(mma_done, 1);
    mbar_init(q_empty, 1);
    fence_mbar_init();
  }
  if (warp == 1) {  // tensor memory for S0, S1, O
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  // An item as seen by the consumer warps: wait for its slot, copy it, hand the slot back.
  auto take_item = [&](int i, ItemInfo& it) -> bool {
    const int b = i & 1;
    bool ok = true;
    if (lane == 0) ok = mbar_wait_bounded(&item_full[b], (uint32_t)((i >> 1) & 1), p.err);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) {
      *abort_flag = 1;
      return false;
    }
    __syncwarp();
    it = items[b];
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[b]);
    return it.seq >= 0;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- scheduler + producer
    int64_t total = 0;
    int maxnt = 0;
    for (int s = lane; s < p.num_seqs; s += 32) {
      const int nt = ntiles_of(p, s);
      total += nt;
      maxnt = max(maxnt, nt);
    }
    total = warp_sum64(total);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maxnt = max(maxnt, __shfl_xor_sync(0xffffffffu, maxnt, o));
    const int64_t n_items = total * p.hq;
    const int spb = p.block_size / kSub;
    const int64_t num_slots = p.num_blocks * p.block_size;
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int64_t g = 0;  // K/V tiles issued by this CTA (stage = g & 1)
    int nq = 0;     // Q tiles issued
    bool aborted = false;
    int64_t v_slots[4] = {0, 0, 0, 0};  // slots of the V tile not yet issued (lane 0)
    // V(gv) into stage gv & 1 once PV(gv - 2) has read that stage (lane 0 only).
    auto issue_v = [&](int64_t gv, const int64_t (&sl)[4], int kvh_) -> bool {
      const int sv = (int)(gv & 1);
      if (gv >= 2 && !mbar_wait_bounded(&v_empty[sv], (uint32_t)(((gv >> 1) - 1) & 1), p.err))
        return false;
      if (*abort_flag) return false;
      uint8_t* vdst = smem + kOffV + sv * kKVBytes;
      mbar_arrive_expect_tx(&v_full[sv], kKVBytes);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_load_5d(vdst + c * (kN * 128) + u * (kSub * 128), &vmap, &v_full[sv], 0, c, kvh_,
                      (int)sl[u], p.layer);
      misc[3] = (int)(gv + 1);  // V tiles issued
      return true;
    };
    // Claims run one item ahead: the next item's claim is in flight while this one's tiles
    // are issued.
    int32_t claim = 0;
    if (lane == 0) claim = atomicAdd(p.ctr, 1);
    for (int i = 0;; ++i) {
      const int64_t k = __shfl_sync(0xffffffffu, claim, 0);
      ItemInfo it;
      it.seq = -1;
      if (k < n_items && !aborted) {
        int seq = 0, tile = 0;
        if (decode_tile_item(p, k / p.hq, maxnt, lane, seq, tile)) {
          it.seq = seq;
          it.qt = tile;
          it.qh = (int)(k % p.hq);
          it.q0 = __ldg(p.cu_q + seq);
          it.qlen = __ldg(p.cu_q + seq + 1) - it.q0;
          it.ctx = __ldg(p.ctx + seq);
          it.rows_valid = min(kM, it.qlen - tile * kM);
          it.pos0 = it.ctx - it.qlen + tile * kM;  // position of the tile's first row
          const int last_pos = it.pos0 + it.rows_valid - 1;
          it.n_kv = last_pos >= 0 ? ceil_div(last_pos + 1, kN) : 0;
          if (lane == 0 && (it.ctx < it.qlen || it.n_kv == 0)) set_device_error(p.err, B2P_DEV_LENGTH);
        }
      }
      const int b = i & 1;
      bool ok = true;
      if (lane == 0) {
        if (i >= 2) ok = mbar_wait_bounded(&item_empty[b], (uint32_t)(((i >> 1) - 1) & 1), p.err);
        if (ok) {
          items[b] = it;
          mbar_arrive(&item_full[b]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) {
        *abort_flag = 1;
        aborted = true;
      }
      if (it.seq < 0 || aborted) break;
      if (lane == 0) claim = atomicAdd(p.ctr, 1);
      if (it.n_kv == 0) continue;
      const int kvh = it.qh / p.group;
      if (lane == 0) {
        // The previous item's QK^T MMAs are done with the Q buffer before it is refilled.
        if (nq >= 1 && !mbar_wait_bounded(q_empty, (uint32_t)((nq - 1) & 1), p.err)) {
          *abort_flag = 1;
          aborted = true;
        } else {
          mbar_arrive_expect_tx(q_full, kQBytes);
          for (int c = 0; c < 2; ++c)
            tma_load_4d(smem + kOffQ + c * (kM * 128), &qmap, q_full, 0, c, it.qh,
                        it.q0 + it.qt * kM);
          misc[1] = nq + 1;  // Q tiles issued
        }
      }
      aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
      if (aborted) break;
      ++nq;
      const int32_t* bt = p.block_tables + (int64_t)it.seq * p.bt_stride;
      // lane l holds the slot of sub-block (win + l); 8 KV tiles per window
      int win = -32;
      int64_t my_slot = 0;
      for (int j = 0; j < it.n_kv && !aborted; ++j, ++g) {
        const int s = (int)(g & 1);
        if (j * 4 >= win + 32) {
          win = j * 4;
          const int sb = win + lane;  // sub-block index within the sequence
          const int64_t col = sb / spb;
          int32_t blk = -1;
          if ((int64_t)sb * kSub < it.ctx && col < p.bt_stride) blk = __ldg(bt + col);
          if ((int64_t)sb * kSub < it.ctx && (blk < 0 || (int64_t)blk >= p.num_blocks)) {
            set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
            blk = -1;
          }
          my_slot = blk < 0 ? num_slots : (int64_t)blk * p.block_size + (int64_t)(sb % spb) * kSub;
        }
        int64_t slots[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) slots[u] = __shfl_sync(0xffffffffu, my_slot, j * 4 - win + u);
        if (lane == 0) {
          // K(g) first, then V(g - 1): K stages free up as soon as their QK^T MMAs finish, so
          // the next K load is in flight while the softmax of the current tile runs.
          if (g >= 2 && !mbar_wait_bounded(&k_empty[s], (uint32_t)(((g >> 1) - 1) & 1), p.err)) {
            aborted = true;
          } else if (*abort_flag) {
            aborted = true;
          } else {
            uint8_t* kdst = smem + kOffK + s * kKVBytes;
            mbar_arrive_expect_tx(&k_full[s], kKVBytes);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int c = 0; c < 2; ++c)
                tma_load_5d(kdst + c * (kN * 128) + u * (kSub * 128), &kmap, &k_full[s], 0, c,
                            kvh, (int)slots[u], p.layer);
            misc[2] = (int)(g + 1);  // K tiles issued
            if (j > 0 && !issue_v(g - 1, v_slots, kvh)) aborted = true;
          }
          if (aborted) *abort_flag = 1;
#pragma unroll
          for (int u = 0; u < 4; ++u) v_slots[u] = slots[u];
        }
        aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
      }
      // the item's last V tile
      if (lane == 0 && !aborted && !issue_v(g - 1, v_slots, kvh)) {
        *abort_flag = 1;
        aborted = true;
      }
      aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
      if (aborted) break;
    }
    if (aborted && lane == 0) {  // the consumers learn it from the flag or their waits
      *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t id_qk = idesc_f16(ab, kM, kN, 0, 0);
    const uint32_t id_pv = idesc_f16(ab, kM, kD, 0, 1);
    const uint32_t q_addr = smem_u32(smem + kOffQ);
    int64_t g = 0;
    int nq = 0;
    bool ok = true;
    for (int i = 0; ok; ++i) {
      ItemInfo it;
      if (!take_item(i, it)) break;
      if (it.n_kv == 0) continue;
      if (lane == 0) {
        auto issue_qk = [&](int64_t gg) {
          const int s = (int)(gg & 1);
          const uint32_t k_addr = smem_u32(smem + kOffK + s * kKVBytes);
          const uint32_t d = tbase + (s ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t da = smem_desc_sw128(q_addr + (kk >> 2) * (kM * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(k_addr + (kk >> 2) * (kN * 128) + (kk & 3) * 32, 16, 1024);
            mma_ss(d, da, db, id_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[s]);
          mma_commit(&k_empty[s]);  // K stage s is free once these MMAs have read it
        };
        // S buffer g & 1 held P of tile g - 2: PV(g - 2) must be done reading it.
        auto s_free = [&](int64_t gg) -> bool {
          return gg < 2 || mbar_wait_bounded(&o_done[(gg - 2) & 1], (uint32_t)(((gg - 2) >> 1) & 1), p.err);
        };
        ok = mbar_wait_bounded(q_full, (uint32_t)(nq & 1), p.err);
        if (ok) ok = s_free(g) && mbar_wait_bounded(&k_full[g & 1], (uint32_t)((g >> 1) & 1), p.err);
        if (ok) {
          tc_fence_after();
          issue_qk(g);
          if (it.n_kv == 1) mma_commit(q_empty);  // the item's last read of Q
        }
        for (int j = 0; j < it.n_kv && ok && !*abort_flag; ++j, ++g) {
          const int s = (int)(g & 1);
          if (j + 1 < it.n_kv) {
            ok = s_free(g + 1) &&
                 mbar_wait_bounded(&k_full[(g + 1) & 1], (uint32_t)(((g + 1) >> 1) & 1), p.err);
            if (!ok) break;
            tc_fence_after();
            issue_qk(g + 1);
            if (j + 2 == it.n_kv) mma_commit(q_empty);
          }
          ok = mbar_wait_bounded(&p_full[s], (uint32_t)((g >> 1) & 1), p.err);
          if (ok) ok = mbar_wait_bounded(&v_full[s], (uint32_t)((g >> 1) & 1), p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + kOffV + s * kKVBytes);
          const uint32_t p_tmem = tbase + (s ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            const uint64_t db = smem_desc_sw128(v_addr + kk * (16 * 128), kN * 128, 1024);
            mma_ts(tbase + kColO, p_tmem + kk * 8, db, id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&v_empty[s]);
          mma_commit(&o_done[s]);
        }
        if (!ok) *abort_flag = 1;
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      g = __shfl_sync(0xffffffffu, g, 0);
      ++nq;
    }
    if (lane == 0) {
      // every MMA issued above has completed once this commit arrives
      mma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quarter = warp & 3;        // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    int64_t g = 0;
    bool ok = true;
    for (int i = 0; ok; ++i) {
      ItemInfo it;
      if (!take_item(i, it)) break;
      if (it.n_kv == 0) continue;
      const bool valid_row = row < it.rows_valid;
      const int pos = it.pos0 + row;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++g) {
        const int s = (int)(g & 1);
        if (ok && !mbar_wait_bounded(&s_full[s], (uint32_t)((g >> 1) & 1), p.err)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_col = lane_base + (s ? kColS1 : kColS0);
        uint32_t r0[32], r1[32];
        tmem_ld32(s_col, r0);
        tmem_ld32(s_col + 32, r1);
        tmem_wait_ld();
        const int key0 = j * kN;
        // key c of this tile is visible iff key0 + c <= pos (then also < ctx). Tiles that
        // every row of the warp sees whole (all but the diagonal ones) skip the masks.
        const int nvis = valid_row ? min(kN, pos - key0 + 1) : 0;
        const bool whole = __all_sync(0xffffffffu, nvis == kN);
        float mx = whole ? row_max64<false>(r0, r1, nvis) : row_max64<true>(r0, r1, nvis);
        mx = mx * p.scale_log2;  // scale_log2 > 0 keeps the arg-max
        bool rescale = false;
        float alpha = 1.f;
        if (mx > -INFINITY) {
          if (m == -INFINITY) {
            m = mx;
          } else if (mx > m + kRescaleThreshold) {
            alpha = fast_exp2(m - mx);
            m = mx;
            rescale = true;
          }
        }
        // Rows that move their reference max fix O once PV of the previous tile has landed.
        if (__any_sync(0xffffffffu, rescale)) {
          if (!mbar_wait_bounded(&o_done[(g - 1) & 1], (uint32_t)(((g - 1) >> 1) & 1), p.err)) ok = false;
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
          for (int c0 = 0; c0 < kD; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + kColO + c0, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(lane_base + kColO + c0, o);
          }
          tmem_wait_st();
          l *= alpha;
        }
        uint32_t pk[32];
        const float rs = whole ? row_exp64<T, false>(r0, r1, nvis, p.scale_log2, m, pk)
                               : row_exp64<T, true>(r0, r1, nvis, p.scale_log2, m, pk);
        l += rs;
        tmem_st32(s_col, pk);
        tmem_wait_st();
        // Keys past the context (the last KV tile's tail) may hold NaN/Inf in the pool;
        // P is 0 there but 0 * NaN is not: zero those V rows before the PV MMA reads them.
        const int tail0 = it.ctx - key0;  // first row of this tile past the context
        if (j == it.n_kv - 1 && tail0 < kN) {
          if (!mbar_wait_bounded(&v_full[s], (uint32_t)((g >> 1) & 1), p.err)) ok = false;
          uint8_t* vt = smem + kOffV + s * kKVBytes;
          const int zrows = kN - max(tail0, 0);
          for (int e = threadIdx.x - 64; e < 2 * zrows * 8; e += 128) {
            const int c = e / (zrows * 8);         // d chunk
            const int rem = e - c * zrows * 8;
            const int r = max(tail0, 0) + rem / 8;  // token row
            const int q16 = rem % 8;                // 16-byte piece of the 128-byte line
            reinterpret_cast<uint4*>(vt + c * (kN * 128) + r * 128)[q16] = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(&p_full[s]);
      }
      // ---- epilogue: O / l -> out (the next item's first PV waits for this warp's arrival
      // on its first P, which comes after these reads)
      if (ok) {
        const int64_t gl = g - 1;
        if (!mbar_wait_bounded(&o_done[gl & 1], (uint32_t)((gl >> 1) & 1), p.err)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(it.q0 + it.qt * kM + row) * p.o_tok +
                  (int64_t)it.qh * p.o_head;
        for (int c0 = 0; c0 < kD; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(lane_base + kColO + c0, o);
          tmem_wait_ld();
          if (valid_row) {
            uint32_t pk[16];
#pragma unroll
            for (int c = 0; c < 16; ++c)
              pk[c] = pack2<T>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              reinterpret_cast<uint4*>(orow + c0)[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          }
        }
        tc_fence_before();
      }
      if (!ok) *abort_flag = 1;
    }
  }

  // ---- teardown: every TMA and MMA of this CTA has finished before TMEM is freed
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Loads this CTA issued land before it leaves: the last Q tile, and the last two K/V
    // tiles (at most two are ever in flight).
    const int nq_issued = misc[1];
    if (nq_issued > 0) mbar_wait_bounded(q_full, (uint32_t)((nq_issued - 1) & 1), nullptr);
    const int k_issued = misc[2];
    for (int gg = max(0, k_issued - 2); gg < k_issued; ++gg)
      mbar_wait_bounded(&k_full[gg & 1], (uint32_t)((gg >> 1) & 1), nullptr);
    const int v_issued = misc[3];
    for (int gg = max(0, v_issued - 2); gg < v_issued; ++gg)
      mbar_wait_bounded(&v_full[gg & 1], (uint32_t)((gg >> 1) & 1), nullptr);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                 "r"(kTmemCols));
  // The last CTA to finish re-zeroes the counters (every claim has been made by then).
  if (threadIdx.x == 0 && atomicAdd(p.ctr + 1, 1) == (int)gridDim.x - 1) {
    p.ctr[0] = 0;
    p.ctr[1] = 0;
    __threadfence();
  }
}

// Claim counters of prefill launches. A launch takes the next of these slots (round robin)
// and leaves it zeroed, so up to 64 launches can be in flight on a device at once.
constexpr int kCounterSlots = 64;
__device__ int32_t g_prefill_counters[kCounterSlots][2];

}  // namespace

// ====================================================================== host side
namespace b2p_host {
int tensor_map_4d_rows(CUtensorMap* out, const void* base, int64_t rows, int heads, int head_dim,
                       int64_t row_stride_elems, int64_t head_stride_elems, int elem_bytes,
                       int box_rows);
int pool_tensor_map_box(CUtensorMap* out, const void* base, int64_t num_layers, int64_t num_slots,
                        int num_kv_heads, int head_dim, int elem_bytes, int box_chunks);
}  // namespace b2p_host

// Launches the tcgen05 prefill when the shape allows it; returns B2P_EUNSUPPORTED otherwise
// (the caller then runs the CUDA-core kernel).
int b2p_prefill_tc(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                   const void* key_cache, const void* value_cache, int64_t layer_index,
                   int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                   int64_t block_table_stride, const int32_t* cu_seqlens_q,
                   const int32_t* context_lens, int num_seqs, int64_t total_q, int num_q_heads,
                   int num_kv_heads, int head_dim, int block_size, float scale, void* out,
                   int64_t out_tok_stride, int64_t out_head_stride, int dtype, int32_t* err_flag,
                   void* stream) {
  if (head_dim != kD || (dtype != B2P_BF16 && dtype != B2P_F16) || block_size % kSub != 0)
    return B2P_EUNSUPPORTED;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!al16(q) || !al16(out) || !al16(key_cache) || !al16(value_cache) ||
      (q_tok_stride * 2) % 16 || (q_head_stride * 2) % 16 || (out_tok_stride * 2) % 16 ||
      (out_head_stride * 2) % 16 || num_slots > 0x7fffffffLL || total_q > 0x7fffffffLL)
    return B2P_EUNSUPPORTED;
  CUtensorMap qmap, kmap, vmap;
  int rc = b2p_host::tensor_map_4d_rows(&qmap, q, total_q, num_q_heads, head_dim, q_tok_stride,
                                        q_head_stride, 2, kM);
  if (rc != B2P_OK) return rc;
  rc = b2p_host::pool_tensor_map_box(&kmap, key_cache, num_layers, num_slots, num_kv_heads,
                                     head_dim, 2, 1);
  if (rc != B2P_OK) return rc;
  rc = b2p_host::pool_tensor_map_box(&vmap, value_cache, num_layers, num_slots, num_kv_heads,
                                     head_dim, 2, 1);
  if (rc != B2P_OK) return rc;
  PrefillParams p;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.cu_q = cu_seqlens_q;
  p.ctx = context_lens;
  p.num_seqs = num_seqs;
  p.group = num_q_heads / num_kv_heads;
  p.layer = (int)layer_index;
  p.block_size = block_size;
  p.num_blocks = num_slots / block_size;
  p.scale_log2 = scale * kLog2e;
  p.out = static_cast<uint8_t*>(out);
  p.o_tok = out_tok_stride;
  p.o_head = out_head_stride;
  p.err = err_flag;
  p.hq = num_q_heads;
  {
    static void* base[64] = {nullptr};
    static std::mutex mu;
    static std::atomic<uint32_t> next_slot{0};
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return b2p_host::record_error(ce);
    if (dev < 0 || dev >= 64) return B2P_EUNSUPPORTED;
    void* addr = nullptr;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (base[dev] == nullptr) {
        ce = cudaGetSymbolAddress(&base[dev], g_prefill_counters);
        if (ce != cudaSuccess) return b2p_host::record_error(ce);
      }
      addr = base[dev];
    }
    const uint32_t slot = next_slot.fetch_add(1) % kCounterSlots;
    p.ctr = static_cast<int32_t*>(addr) + 2 * slot;
  }
  const void* fn = dtype == B2P_BF16
                       ? reinterpret_cast<const void*>(&paged_prefill_tc<__nv_bfloat16>)
                       : reinterpret_cast<const void*>(&paged_prefill_tc<__half>);
  const int smem = kSmemBytes + 1024;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  // Persistent: every resident CTA walks the work items (tile-items x query heads). The
  // residency comes from the SM's own limits (shared memory with the per-CTA reservation,
  // the register file, tensor memory: two CTAs' 256 columns fill it), computed once per
  // device. cudaOccupancyMaxActiveBlocksPerMultiprocessor answers 1 for this kernel on
  // B200 although two CTAs run side by side (measured: 296 CTAs started within 1 us on
  // 148 SMs, at TMEM columns 0 and 256), and a grid of one CTA per SM ran 1.6x slower.
  static int resident[64] = {0};
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  if (dev < 0 || dev >= 64) return B2P_EUNSUPPORTED;
  if (resident[dev] == 0) {
    cudaFuncAttributes fa;
    int smem_sm = 0, reserved = 0, regs_sm = 0;
    if ((e = cudaFuncGetAttributes(&fa, fn)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor,
                                    dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) !=
            cudaSuccess)
      return b2p_host::record_error(e);
    // registers are handed out per warp in 256-register units
    const int warp_regs = (fa.numRegs * 32 + 255) / 256 * 256;
    const int by_regs = regs_sm / (warp_regs * (kThreads / 32));
    const int by_smem = smem_sm / (smem + (int)fa.sharedSizeBytes + reserved);
    int n = by_regs < by_smem ? by_regs : by_smem;
    if (n > 2) n = 2;
    resident[dev] = n;
  }
  const int per_sm = resident[dev];
  if (per_sm <= 0) return B2P_EUNSUPPORTED;
  dim3 grid((unsigned)(b2p_host::sm_count() * per_sm));
  void* args[] = {&qmap, &kmap, &vmap, &p};
  e = cudaLaunchKernel(fn, grid, dim3(kThreads), args, (size_t)smem,
                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return b2p_host::record_error(e);
  return b2p_host::check_launch();
}
