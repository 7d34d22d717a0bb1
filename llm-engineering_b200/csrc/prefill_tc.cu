// K3 — packed variable-length causal prefill / chunked-prefill attention on tcgen05.
//
// Reference path replaced (PREFILL executions): HFBatchedPagedCache.update gathers every
// history (serving/engine/hf_batched_paged_cache.py:52-148), build_attention_mask adds a
// dense tril block per prefill (serving/engine/attention_mask.py:37-45) and HF SDPA runs
// over all packed keys (transformers/integrations/sdpa_attention.py:40-104). Here a work
// item is one tile of 128 query rows of one sequence for two query heads of the same GQA
// group (A and B), attended against the sequence's keys read in place from the paged pool:
//
//   S = Q K^T   tcgen05.mma kind::f16, A = Q (smem, K-major), B = K tile (smem, K-major),
//               D = S in tensor memory (fp32, 128 lanes x 128 columns, one per head)
//   P = softmax rows of S, two threads per query row (two warps share a TMEM lane
//       quarter, one per 64-key half of the tile: tcgen05.ld -> fp32 -> exp2), written back
//       as bf16/f16 (tcgen05.st) over the first 32 of each half's own 64 S columns (head_dim
//       128) or into columns of its own (head_dim 64)
//   O += P V    tcgen05.mma with A = P from tensor memory, B = V tile (smem, MN-major),
//               D = O in tensor memory (fp32, 128 x head_dim, one per head)
//
// Tensor memory holds S_A, S_B, O_A, O_B (512 columns, one CTA per SM). The MMA warp
// issues PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1), ..., so the softmax of one head runs
// while the tensor cores work on the other head, and both heads read each K/V tile once.
// QK_h(j+1) follows PV_h(j) with no wait for it to complete: the tensor pipe runs the MMAs
// of the issuing thread in order, so PV_h(j) has read P_h(j) before QK_h(j+1) overwrites
// those columns of S_h.
// With head_dim 64 the order is QK_A(j+1), QK_B(j+1), PV_A(j), PV_B(j): P has columns of
// its own there, so the next QK^T only waits for the softmax to have read S.
// K/V tiles of 128 tokens are assembled from eight 16-slot pool sub-blocks (TMA tile
// loads, 128-byte swizzle, no multicast) into two-stage K and V rings. A query row j of
// sequence i sits at position ctx_i - q_len_i + j and sees keys 0..position (whole-history
// prefill when q_len == ctx, chunked prefill otherwise). The first KV tile of an item sets
// each row's reference max; later tiles take exp2 against that reference in one pass (the
// row sum flags the rare rows whose scores outgrow it by more than 2^8, which then move
// the reference and rescale O and l before any P of the tile is stored). The two warps of a
// row agree on its reference max, on a move of it and on aborts through shared memory, at
// one 64-thread named barrier per tile. One softmax warp per row ran alone on its SM
// sub-partition while the other head waited, latency-bound; two warps per row there were
// measured 5.4 % faster (673.7 against 712.2 us per launch on the 32-prompt workload). The
// softmax is bound by neither exp2 throughput nor its tensor-memory loads, and the
// exponent arithmetic runs as packed f32x2 FMA/ADD.
//
// Warp roles (576 threads): warp 0 = TMA producer and work-item scheduler, warp 1 =
// tensor-memory owner and MMA issuer (one thread), warps 2..9 = softmax + epilogue of head
// A, warps 10..17 = the same for head B. Softmax warp w serves TMEM lanes 32 * (w % 4)
// .. +31 (thread = lane = query row), keys 0..63 of each tile for w - 2 in {0..3, 8..11},
// keys 64..127 otherwise.
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace {

using namespace b2p;

constexpr int kM = 128;     // query rows per tile
constexpr int kN = 128;     // keys per KV tile
constexpr int kSeqCache = 512;    // scheduler tables: sequences cached in shared memory
constexpr int kSizeCache = 1024;  // ... and tile sizes (KV tiles per query tile)
constexpr int kThreads = 576;
constexpr int kSub = 16;
constexpr int kSubPerTile = kN / kSub;
constexpr int kConsumerWarps = 17;  // the MMA issuer and sixteen softmax warps
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

// Shared-memory plan (bytes from the 1024-aligned base) for head_dim D (64 or 128): Q, K
// and V tiles are D / 64 chunks of 128-byte lines (64 elements), 128 rows each.
template <int D>
struct Plan {
  static constexpr int kChunks = D / 64;
  static constexpr int kQBytes = kChunks * kM * 128;   // one head
  static constexpr int kKVBytes = kChunks * kN * 128;  // one K or V tile
  static constexpr int kOffQ = 0;                      // heads A and B
  static constexpr int kOffK = kOffQ + 2 * kQBytes;    // 2 stages
  static constexpr int kOffV = kOffK + 2 * kKVBytes;   // 2 stages
  static constexpr int kOffBar = kOffV + 2 * kKVBytes;
  static constexpr int kNumBars = 23;  // q_full, q_empty, k_full[2], k_empty[2], v_full[2],
                                       // v_empty[2], s_full[2], p_full[2], o_done[2] (by
                                       // head), item_full[2], item_empty[2], mma_done,
                                       // s_read[2] (by head; head_dim 64)
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kOffItems = kOffMisc + 64;
  // epilogue staging: 16 warps x 32 rows x 32 B
  static constexpr int kOffStage = (kOffItems + 2 * 48 + 127) / 128 * 128;
  // row exchange between the two warps of a lane quarter: 8 pairs x [2 parity][2 half]
  // x (32 floats), then 8 pairs x [2 parity][2 half] flags
  static constexpr int kOffXch = kOffStage + 16 * 32 * 32;
  static constexpr int kOffXok = kOffXch + 8 * 4 * 32 * 4;
  static constexpr int kOffSched = kOffXok + 8 * 4 * 4;  // scheduler tables
  static constexpr int kSmemBytes = kOffSched + (3 * kSeqCache + kSizeCache + 1) * 4;
};

// TMEM columns (512 allocated): S of head A at 0, of head B at 128. head_dim 128: O_A at
// 256, O_B at 384, and P overwrites part of its S: each key half's softmax warp writes its
// 64 keys' P (two keys per column) over the first 32 of that half's own 64 S columns (S + 0
// .. 31 for keys 0..63, S + 64 .. 95 for keys 64..127; see col_p_keys). head_dim 64: O_A at
// 256, O_B at 320, and P has columns of its own (P_A at 384, P_B at 448), so S is free for
// the next QK^T as soon as the softmax has read it.
constexpr uint32_t kTmemCols = 512;
__device__ __forceinline__ uint32_t col_s(int h) { return h ? 128u : 0u; }
template <int D>
__device__ __forceinline__ uint32_t col_o(int h) {
  return D == 64 ? 256u + 64u * h : (h ? 384u : 256u);
}
template <int D>
__device__ __forceinline__ uint32_t col_p(int h) {
  return D == 64 ? 384u + 64u * h : col_s(h) + 64u;
}
// TMEM column of P for keys 16*kk .. 16*kk+15 (two keys per column). head_dim 64: P has 64
// columns of its own. head_dim 128: the softmax warp of key half `half` stores its 64 keys'
// P over the first 32 columns of its own 64 S columns (keys 0..63 at S + 0, keys 64..127 at
// S + 64), which it alone has read.
template <int D>
__device__ __forceinline__ uint32_t col_p_keys(int h, int kk) {
  return D == 64 ? col_p<D>(h) + 8u * kk : col_s(h) + (kk < 4 ? 8u * kk : 64u + 8u * (kk - 4));
}
template <int D>
__device__ __forceinline__ uint32_t col_p_half(int h, int half) {
  return D == 64 ? col_p<D>(h) + 32u * half : col_s(h) + 64u * half;
}

__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Two fp32 values in one 64-bit register for the packed f32x2 FMA-pipe instructions.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Row max of 32 S columns (keys base .. base+31 of the row's visible range), two chains.
template <bool kMasked>
__device__ __forceinline__ float row_max32(const uint32_t (&r)[32], int base, int nvis) {
  float a0 = -INFINITY, a1 = -INFINITY;
#pragma unroll
  for (int c = 0; c < 32; c += 4) {
    auto v = [&](int cc) {
      const float x = __uint_as_float(r[cc]);
      return (!kMasked || base + cc < nvis) ? x : -INFINITY;
    };
    a0 = fmax3(a0, v(c), v(c + 1));
    a1 = fmax3(a1, v(c + 2), v(c + 3));
  }
  return fmaxf(a0, a1);
}

// P of 32 S columns (keys base .. base+31) into pk[16] (two keys per word); returns their sum.
// (Computing 1 to 3 of every 8 pairs' exp2 on the FMA pipe instead, by range reduction and a
// cubic, was measured slower: 791 to 964 us per launch against 714 with one softmax warp
// per row: the softmax is not bound by MUFU throughput.)
template <typename T, bool kMasked>
__device__ __forceinline__ float row_exp32(const uint32_t (&r)[32], int base, int nvis,
                                           float scale_log2, float m, uint32_t* pk) {
  const uint64_t sc = f2pack(scale_log2, scale_log2);
  const uint64_t nm = f2pack(-m, -m);
  uint64_t acc0 = f2pack(0.f, 0.f), acc1 = f2pack(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const uint64_t x =
        ffma2(f2pack(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1])), sc, nm);
    float x0, x1, e0, e1;
    f2unpack(x, x0, x1);
    e0 = fast_exp2(x0);
    e1 = fast_exp2(x1);
    if (kMasked) {
      e0 = base + 2 * q < nvis ? e0 : 0.f;
      e1 = base + 2 * q + 1 < nvis ? e1 : 0.f;
    }
    if (q & 1) acc1 = fadd2(acc1, f2pack(e0, e1)); else acc0 = fadd2(acc0, f2pack(e0, e1));
    pk[q] = pack2<T>(e0, e1);
  }
  float s0, s1, s2, s3;
  f2unpack(acc0, s0, s1);
  f2unpack(acc1, s2, s3);
  return (s0 + s1) + (s2 + s3);
}

// Work items. Sequence s has ntiles(s) = ceil(q_len_s / 128) query tiles; its tile t
// needs size(s, t) KV tiles: t + 1 + ceil((ctx_s - q_len_s) / 128) for every full tile and
// ceil(ctx_s / 128) for the last one. Tile-items are claimed longest first: by size
// descending, then by sequence, a sequence's full tile before its last tile. Work item k is
// tile-item k / (HKV * pairs) for head pair k % (HKV * pairs): the query heads of a GQA
// group go two by two (the last one alone when the group is odd), and the pairs of one
// tile are neighbours, so the whole group reads the same K/V tiles close together.
struct ItemInfo {
  int seq;  // -1: no more work for this CTA
  int qt, kvh, qh_a, qh_b;  // qh_b = -1: head A only
  int q0, qlen, ctx, rows_valid, pos0, n_kv, pad;
};

__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// What the scheduler needs of one sequence: query tiles, the size of its first full tile
// minus one (c = ceil((ctx - q_len) / 128)), and the size of its last tile.
struct SeqTiles {
  int nt, c, last;
};

__device__ __forceinline__ SeqTiles seq_tiles_global(const PrefillParams& p, int s) {
  const int q0 = __ldg(p.cu_q + s);
  const int q = __ldg(p.cu_q + s + 1) - q0;
  const int ctx = __ldg(p.ctx + s);
  SeqTiles t;
  t.nt = q > 0 ? ceil_div(q, kM) : 0;
  t.c = ctx > q ? ceil_div(ctx - q, kN) : 0;
  t.last = max(1, ceil_div(max(ctx, 1), kN));
  return t;
}

// Tiles of a sequence whose size is larger than v.
__device__ __forceinline__ int tiles_above(const SeqTiles& t, int v) {
  if (t.nt == 0) return 0;
  const int full = max(0, (t.nt - 1 + t.c) - max(v, t.c));  // full sizes 1+c .. nt-1+c
  return full + (t.last > v ? 1 : 0);
}

// Scheduler tables in shared memory, built once per CTA by the producer warp: the
// SeqTiles of the first kSeqCache sequences, and the tile-items larger than each size v
// when no tile needs more than kSizeCache KV tiles. Past either limit the scheduler reads
// cu_seqlens and the context lengths directly (same order, more global round trips).
struct SchedTables {
  int32_t* seq;     // [kSeqCache][3]: nt, c, last
  int32_t* above;   // [kSizeCache + 1]: tile-items of size > v
  bool sizes;       // `above` holds sizes 0..maxv
};

__device__ __forceinline__ SeqTiles seq_tiles(const PrefillParams& p, const SchedTables& st, int s) {
  if (s < kSeqCache) return SeqTiles{st.seq[3 * s], st.seq[3 * s + 1], st.seq[3 * s + 2]};
  return seq_tiles_global(p, s);
}

// Tile-items larger than v. One warp; all lanes get the result.
__device__ __forceinline__ int64_t items_above(const PrefillParams& p, const SchedTables& st,
                                               int v, int lane) {
  if (st.sizes) return st.above[v];
  int64_t acc = 0;
  for (int s = lane; s < p.num_seqs; s += 32) acc += tiles_above(seq_tiles(p, st, s), v);
  return warp_sum64(acc);
}

// Fills the tables and returns the total tile-items (all lanes); maxv gets the largest
// tile size. One warp.
__device__ __forceinline__ int64_t build_sched_tables(const PrefillParams& p, SchedTables& st,
                                                      int lane, int& maxv) {
  int64_t total = 0;
  maxv = 0;
  for (int s = lane; s < p.num_seqs; s += 32) {
    const SeqTiles t = seq_tiles_global(p, s);
    if (s < kSeqCache) {
      st.seq[3 * s] = t.nt;
      st.seq[3 * s + 1] = t.c;
      st.seq[3 * s + 2] = t.last;
    }
    total += t.nt;
    if (t.nt > 0) maxv = max(maxv, max(t.nt - 1 + t.c, t.last));
  }
  total = warp_sum64(total);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxv = max(maxv, __shfl_xor_sync(0xffffffffu, maxv, o));
  st.sizes = maxv <= kSizeCache;
  if (st.sizes) {
    int32_t* h = st.above;
    for (int v = lane; v <= maxv + 1 && v <= kSizeCache; v += 32) h[v] = 0;
    __syncwarp();
    // full tiles: a range of sizes per sequence (difference array), prefix-summed below
    for (int s = lane; s < p.num_seqs; s += 32) {
      const SeqTiles t = seq_tiles(p, st, s);
      if (t.nt >= 2) {
        atomicAdd(&h[1 + t.c], 1);
        if (t.nt + t.c <= maxv) atomicAdd(&h[t.nt + t.c], -1);
      }
    }
    __syncwarp();
    if (lane == 0) {
      int run = 0;
      for (int v = 1; v <= maxv; ++v) {
        run += h[v];
        h[v] = run;
      }
    }
    __syncwarp();
    for (int s = lane; s < p.num_seqs; s += 32) {  // last tiles: one size each
      const SeqTiles t = seq_tiles(p, st, s);
      if (t.nt >= 1) atomicAdd(&h[t.last], 1);
    }
    __syncwarp();
    if (lane == 0) {  // histogram of sizes -> tile-items larger than v
      int acc = 0;
      for (int v = maxv; v >= 1; --v) {
        const int c = h[v];
        h[v] = acc;
        acc += c;
      }
      h[0] = acc;
    }
    __syncwarp();
  }
  return total;
}

// Tile-item t -> (sequence, query tile). One warp; all lanes get the result.
__device__ __forceinline__ bool decode_tile_item(const PrefillParams& p, const SchedTables& st,
                                                 int64_t t, int maxv, int lane, int& seq,
                                                 int& tile) {
  int lo = 1, hi = maxv;  // smallest v with items_above(v) <= t
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (items_above(p, st, mid, lane) <= t) hi = mid; else lo = mid + 1;
  }
  const int v = lo;
  int64_t i = t - items_above(p, st, v, lane);
  for (int base = 0; base < p.num_seqs; base += 32) {
    const int s = base + lane;
    int full = 0, last = 0;
    SeqTiles ts{0, 0, 0};
    if (s < p.num_seqs) {
      ts = seq_tiles(p, st, s);
      full = (ts.nt >= 2 && v >= 1 + ts.c && v <= ts.nt - 1 + ts.c) ? 1 : 0;
      last = (ts.nt >= 1 && ts.last == v) ? 1 : 0;
    }
    int incl = full + last;  // inclusive scan over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (i < total) {
      const unsigned m = __ballot_sync(0xffffffffu, incl > i);
      const int pos = __ffs(m) - 1;
      const int before = __shfl_sync(0xffffffffu, incl - full - last, pos);
      const int f = __shfl_sync(0xffffffffu, full, pos);
      const int nt = __shfl_sync(0xffffffffu, ts.nt, pos);
      const int c = __shfl_sync(0xffffffffu, ts.c, pos);
      seq = base + pos;
      tile = (f && i - before == 0) ? v - 1 - c : nt - 1;
      return true;
    }
    i -= total;
  }
  return false;
}

// Persistent CTAs (one per SM) claim work items in the order above from an atomic counter
// (dynamic, so faster SMs take more items and the short items come last). Tensor memory,
// barriers and descriptors are set up once; the stage and per-head counters run on across
// items, so the next item's Q and first K/V tiles load while the current item finishes.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) paged_prefill_tc(const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap,
                                                                const PrefillParams p) {
  using L = Plan<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;       // by stage
  uint64_t* k_empty = bars + 4;
  uint64_t* v_full = bars + 6;
  uint64_t* v_empty = bars + 8;
  uint64_t* s_full = bars + 10;      // by head (A, B)
  uint64_t* p_full = bars + 12;
  uint64_t* o_done = bars + 14;
  uint64_t* item_full = bars + 16;   // by ring slot
  uint64_t* item_empty = bars + 18;
  uint64_t* mma_done = bars + 20;
  uint64_t* s_read = bars + 21;      // by head: the softmax has read S (head_dim 64)
  int32_t* misc = reinterpret_cast<int32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 5);
  ItemInfo* items = reinterpret_cast<ItemInfo*>(smem + L::kOffItems);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0;
    misc[0] = misc[1] = misc[2] = misc[3] = 0;
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 2 * kM);
      mbar_init(&s_read[s], 2 * kM);
      mbar_init(&o_done[s], 1);
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], kConsumerWarps);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {  // tensor memory for S_A, S_B, O_A, O_B
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
    SchedTables st;
    st.seq = reinterpret_cast<int32_t*>(smem + L::kOffSched);
    st.above = st.seq + 3 * kSeqCache;
    int maxv = 0;
    const int64_t total = build_sched_tables(p, st, lane, maxv);
    const int pairs = (p.group + 1) >> 1;
    const int64_t per_tile = (int64_t)(p.hq / p.group) * pairs;
    const int64_t n_items = total * per_tile;
    const int spb = p.block_size / kSub;
    const int64_t num_slots = p.num_blocks * p.block_size;
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int64_t g = 0;  // K/V tiles issued by this CTA (stage = g & 1)
    int nq = 0;     // Q loads issued
    bool aborted = false;
    // V(gv) into stage gv & 1 once PV of tile gv - 2 has read that stage (lane 0 only).
    auto issue_v = [&](int64_t gv, const int32_t (&sl)[kSubPerTile], int kvh_) -> bool {
      const int sv = (int)(gv & 1);
      if (gv >= 2 && !mbar_wait_bounded(&v_empty[sv], (uint32_t)(((gv >> 1) - 1) & 1), p.err))
        return false;
      if (*abort_flag) return false;
      uint8_t* vdst = smem + L::kOffV + sv * L::kKVBytes;
      mbar_arrive_expect_tx(&v_full[sv], L::kKVBytes);
#pragma unroll
      for (int u = 0; u < kSubPerTile; ++u)
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_5d(vdst + c * (kN * 128) + u * (kSub * 128), &vmap, &v_full[sv], 0, c, kvh_,
                      sl[u], p.layer);
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
        if (decode_tile_item(p, st, k / per_tile, maxv, lane, seq, tile)) {
          const int r = (int)(k % per_tile);
          const int pr = r % pairs;
          it.seq = seq;
          it.qt = tile;
          it.kvh = r / pairs;
          it.qh_a = it.kvh * p.group + 2 * pr;
          it.qh_b = 2 * pr + 1 < p.group ? it.qh_a + 1 : -1;
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
      const int kvh = it.kvh;
      if (lane == 0) {
        // The previous item's QK^T MMAs are done with the Q buffers before they are refilled.
        if (nq >= 1 && !mbar_wait_bounded(q_empty, (uint32_t)((nq - 1) & 1), p.err)) {
          *abort_flag = 1;
          aborted = true;
        } else {
          const int nh = it.qh_b >= 0 ? 2 : 1;
          mbar_arrive_expect_tx(q_full, nh * L::kQBytes);
          for (int h = 0; h < nh; ++h)
            for (int c = 0; c < L::kChunks; ++c)
              tma_load_4d(smem + L::kOffQ + h * L::kQBytes + c * (kM * 128), &qmap, q_full, 0, c,
                          h ? it.qh_b : it.qh_a, it.q0 + it.qt * kM);
          misc[1] = nq + 1;  // Q loads issued
        }
      }
      aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
      if (aborted) break;
      ++nq;
      const int32_t* bt = p.block_tables + (int64_t)it.seq * p.bt_stride;
      // lane l holds the slot of sub-block (win + l); 4 KV tiles per window
      int win = -32;
      int32_t my_slot = 0;  // slot indices fit in int32 (checked on the host)
      for (int j = 0; j < it.n_kv && !aborted; ++j, ++g) {
        const int s = (int)(g & 1);
        if (j * kSubPerTile >= win + 32) {
          win = j * kSubPerTile;
          const int sb = win + lane;  // sub-block index within the sequence
          const int64_t col = sb / spb;
          int32_t blk = -1;
          if ((int64_t)sb * kSub < it.ctx && col < p.bt_stride) blk = __ldg(bt + col);
          if ((int64_t)sb * kSub < it.ctx && (blk < 0 || (int64_t)blk >= p.num_blocks)) {
            set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
            blk = -1;
          }
          my_slot = (int32_t)(blk < 0 ? num_slots : (int64_t)blk * p.block_size + (int64_t)(sb % spb) * kSub);
        }
        int32_t slots[kSubPerTile];
#pragma unroll
        for (int u = 0; u < kSubPerTile; ++u)
          slots[u] = __shfl_sync(0xffffffffu, my_slot, j * kSubPerTile - win + u);
        if (lane == 0) {
          // K(g), then V(g). V(g) waits for PV_B(g - 2), which the MMA warp issues before
          // QK_B(g - 1), the MMA that K(g + 1) waits for: issuing V right behind K never
          // holds up the next K.
          if (g >= 2 && !mbar_wait_bounded(&k_empty[s], (uint32_t)(((g >> 1) - 1) & 1), p.err)) {
            aborted = true;
          } else if (*abort_flag) {
            aborted = true;
          } else {
            uint8_t* kdst = smem + L::kOffK + s * L::kKVBytes;
            mbar_arrive_expect_tx(&k_full[s], L::kKVBytes);
#pragma unroll
            for (int u = 0; u < kSubPerTile; ++u)
#pragma unroll
              for (int c = 0; c < L::kChunks; ++c)
                tma_load_5d(kdst + c * (kN * 128) + u * (kSub * 128), &kmap, &k_full[s], 0, c,
                            kvh, slots[u], p.layer);
            misc[2] = (int)(g + 1);  // K tiles issued
            if (!issue_v(g, slots, kvh)) aborted = true;
          }
          if (aborted) *abort_flag = 1;
        }
        aborted = __shfl_sync(0xffffffffu, aborted ? 1 : 0, 0) != 0;
      }
      if (aborted) break;
    }
    if (aborted && lane == 0) {  // the consumers learn it from the flag or their waits
      *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t id_qk = idesc_f16(ab, kM, kN, 0, 0);
    const uint32_t id_pv = idesc_f16(ab, kM, D, 0, 1);
    int64_t g = 0;
    int nq = 0;
    int n0 = 0, n1 = 0;  // PV MMAs issued for head A / head B (S, P and O barrier phases)
    bool ok = true;
    for (int i = 0; ok; ++i) {
      ItemInfo it;
      if (!take_item(i, it)) break;
      if (it.n_kv == 0) continue;
      const int nh = it.qh_b >= 0 ? 2 : 1;
      if (lane == 0) {
        auto issue_qk = [&](int h, int64_t gg) {
          const uint32_t q_addr = smem_u32(smem + L::kOffQ + h * L::kQBytes);
          const uint32_t k_addr = smem_u32(smem + L::kOffK + (int)(gg & 1) * L::kKVBytes);
          const uint32_t d = tbase + col_s(h);
          // base descriptors once; each K step adds its byte offset / 16 to the address
          // field (shared-memory addresses stay below 2^18 bytes, so the field never
          // carries into the next one)
          const uint64_t qa = smem_desc_sw128(q_addr, 16, 1024);
          const uint64_t kb = smem_desc_sw128(k_addr, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t da = qa + (uint64_t)(((kk >> 2) * (kM * 128) + (kk & 3) * 32) >> 4);
            const uint64_t db = kb + (uint64_t)(((kk >> 2) * (kN * 128) + (kk & 3) * 32) >> 4);
            mma_ss(d, da, db, id_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[h]);
        };
        auto issue_pv = [&](int h, int64_t gg, bool first) {
          const uint32_t v_addr = smem_u32(smem + L::kOffV + (int)(gg & 1) * L::kKVBytes);
          const uint64_t vb = smem_desc_sw128(v_addr, kN * 128, 1024);
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            const uint64_t db = vb + (uint64_t)((kk * (16 * 128)) >> 4);
            mma_ts(tbase + col_o<D>(h), tbase + col_p_keys<D>(h, kk), db, id_pv,
                   (!first || kk > 0) ? 1u : 0u);
          }
          mma_commit(&o_done[h]);
        };
        // S of head h may be overwritten once the softmax has read the previous S (head_dim
        // 64, where P has columns of its own). With head_dim 128, P overwrites S and the
        // next QK^T only has to come after the PV that reads P, which the tensor pipe
        // guarantees for MMAs issued in that order by this thread.
        auto s_free = [&](int h) -> bool {
          const int n = h ? n1 : n0;
          if constexpr (D != 64) return true;
          return n == 0 || mbar_wait_bounded(&s_read[h], (uint32_t)((n - 1) & 1), p.err);
        };
        ok = mbar_wait_bounded(q_full, (uint32_t)(nq & 1), p.err);
        if (ok) ok = mbar_wait_bounded(&k_full[g & 1], (uint32_t)((g >> 1) & 1), p.err);
        for (int h = 0; h < nh && ok; ++h) {
          ok = s_free(h);
          if (ok) {
            tc_fence_after();
            issue_qk(h, g);
          }
        }
        if (ok) {
          mma_commit(&k_empty[g & 1]);
          if (it.n_kv == 1) mma_commit(q_empty);  // the item's last read of Q
        }
        if constexpr (D == 64) {
          // QK_A(j+1), QK_B(j+1) as soon as each head's softmax has read S(j), then PV_A(j),
          // PV_B(j): the next S is ready when the softmax of this tile ends.
          for (int j = 0; j < it.n_kv && ok && !*abort_flag; ++j, ++g) {
            const int s = (int)(g & 1);
            if (j + 1 < it.n_kv) {
              ok = mbar_wait_bounded(&k_full[(g + 1) & 1], (uint32_t)(((g + 1) >> 1) & 1), p.err);
              for (int h = 0; h < nh && ok; ++h) {
                const int n = h ? n1 : n0;
                ok = mbar_wait_bounded(&s_read[h], (uint32_t)(n & 1), p.err);
                if (!ok) break;
                tc_fence_after();
                issue_qk(h, g + 1);
              }
              if (!ok) break;
              mma_commit(&k_empty[(g + 1) & 1]);
              if (j + 2 == it.n_kv) mma_commit(q_empty);
            }
            ok = mbar_wait_bounded(&v_full[s], (uint32_t)((g >> 1) & 1), p.err);
            for (int h = 0; h < nh && ok; ++h) {
              const int n = h ? n1 : n0;
              ok = mbar_wait_bounded(&p_full[h], (uint32_t)(n & 1), p.err);
              if (!ok) break;
              tc_fence_after();
              issue_pv(h, g, j == 0);
              if (h) ++n1; else ++n0;
            }
            if (!ok) break;
            mma_commit(&v_empty[s]);
          }
        } else {
          for (int j = 0; j < it.n_kv && ok && !*abort_flag; ++j, ++g) {
            const int s = (int)(g & 1);
            const bool more = j + 1 < it.n_kv;
            ok = mbar_wait_bounded(&v_full[s], (uint32_t)((g >> 1) & 1), p.err);
            // PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1): each head's next S is computed while
            // the other head's softmax runs.
            for (int h = 0; h < nh && ok; ++h) {
              const int n = h ? n1 : n0;
              ok = mbar_wait_bounded(&p_full[h], (uint32_t)(n & 1), p.err);
              if (!ok) break;
              tc_fence_after();
              issue_pv(h, g, j == 0);
              if (h) ++n1; else ++n0;
              if (more) {
                // QK_h(j+1) overwrites the S columns that hold P_h(j), which PV_h(j) just
                // issued reads: both MMAs come from this thread and the tensor pipe runs
                // them in issue order, so no wait for PV_h(j) to complete is needed here.
                if (h == 0)
                  ok = mbar_wait_bounded(&k_full[(g + 1) & 1], (uint32_t)(((g + 1) >> 1) & 1), p.err);
                if (!ok) break;
                tc_fence_after();
                issue_qk(h, g + 1);
              }
            }
            if (!ok) break;
            if (more) {
              mma_commit(&k_empty[(g + 1) & 1]);
              if (j + 2 == it.n_kv) mma_commit(q_empty);
            }
            mma_commit(&v_empty[s]);
          }
        }
        if (!ok) *abort_flag = 1;
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      g = __shfl_sync(0xffffffffu, g, 0);
      n0 = __shfl_sync(0xffffffffu, n0, 0);
      n1 = __shfl_sync(0xffffffffu, n1, 0);
      ++nq;
    }
    if (lane == 0) {
      // every MMA issued above has completed once this commit arrives
      mma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    // Two warps per TMEM lane quarter and head: warp half 0 takes keys 0..63 of every KV
    // tile, half 1 keys 64..127, so each SM sub-partition runs two softmax warps of a head
    // at once. The pair agrees on each row's reference max (and on aborts) through shared
    // memory at one 64-thread named barrier per tile, before either stores P.
    const int local = warp - 2;
    const int h = local >> 3;             // 0: head A, 1: head B
    const int half = (local >> 2) & 1;    // key half of every tile
    const int quarter = warp & 3;         // TMEM lanes 32*quarter .. +31
    const int row = quarter * 32 + lane;  // query row within the tile
    const int pair = h * 4 + quarter;     // named barrier 1 + pair (ids 1..8)
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = lane_base + col_s(h) + 64u * half;        // my 64 S columns
    const uint32_t p_col = lane_base + col_p_half<D>(h, half);       // my 32 P columns
    const uint32_t o_col = lane_base + col_o<D>(h) + (uint32_t)(D / 2) * half;  // D/2 O cols
    float* xv = reinterpret_cast<float*>(smem + L::kOffXch) + pair * (4 * 32);
    int* xo = reinterpret_cast<int*>(smem + L::kOffXok) + pair * 4;
    int ex_n = 0;  // exchanges so far (the pair runs them in lock step)
    // Publish v and this warp's status, wait for the partner, return its v; both_ok tells
    // whether both warps are still fine (then both go on, else both leave: the pair always
    // meets at the same barriers).
    auto exchange = [&](float v, bool mine_ok, bool& both_ok) -> float {
      const int par = ex_n & 1;
      ++ex_n;
      xv[(par * 2 + half) * 32 + lane] = v;
      if (lane == 0) xo[par * 2 + half] = mine_ok ? 1 : 0;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
      const float pv = xv[(par * 2 + (half ^ 1)) * 32 + lane];
      both_ok = mine_ok && xo[par * 2 + (half ^ 1)] != 0;
      return pv;
    };
    int64_t g = 0;  // K/V tiles of the items seen so far (V stage of the tail fix-up)
    int n = 0;      // tiles of this head so far (S, P and O barrier phases)
    bool ok = true;
    for (int i = 0;; ++i) {
      ItemInfo it;
      it.seq = -1;
      const bool got = ok && take_item(i, it);
      bool both = false;
      (void)exchange(0.f, got, both);
      if (!both) {
        if (got || it.seq >= 0) *abort_flag = 1;  // left on the partner's failure
        break;
      }
      if (it.n_kv == 0) continue;
      if (h == 1 && it.qh_b < 0) {  // an odd group's last head: head A alone
        g += it.n_kv;
        continue;
      }
      const int qh = h ? it.qh_b : it.qh_a;
      const bool valid_row = row < it.rows_valid;
      const int pos = it.pos0 + row;
      float m = -INFINITY, l = 0.f;  // l: this warp's half of the row sum
      bool left = false;             // the pair left the item together
      for (int j = 0; j < it.n_kv; ++j, ++g, ++n) {
        bool okw = ok;
        if (okw && !mbar_wait_bounded(&s_full[h], (uint32_t)(n & 1), p.err)) okw = false;
        okw = __all_sync(0xffffffffu, okw) && !*abort_flag;
        const int key0 = j * kN + 64 * half;
        // key c of my half is visible iff key0 + c <= pos (then also < ctx); chunks that
        // every row of the warp sees whole (all but the diagonal tiles) skip the masks
        const int nv = valid_row ? pos - key0 + 1 : 0;
        const bool whole0 = __all_sync(0xffffffffu, nv >= 32);
        const bool whole1 = __all_sync(0xffffffffu, nv >= 64);
        uint32_t r[32], pk[32];
        auto load = [&](int c) {
          tmem_ld32(s_col + 32u * c, r);
          tmem_wait_ld();
        };
        auto max_chunk = [&](int c) -> float {
          const bool w = c ? whole1 : whole0;
          return w ? row_max32<false>(r, 32 * c, nv) : row_max32<true>(r, 32 * c, nv);
        };
        auto exp_chunk = [&](int c) -> float {
          const bool w = c ? whole1 : whole0;
          return w ? row_exp32<T, false>(r, 32 * c, nv, p.scale_log2, m, pk + 16 * c)
                   : row_exp32<T, true>(r, 32 * c, nv, p.scale_log2, m, pk + 16 * c);
        };
        // the largest S * scale_log2 over my 64 keys (two loads of S, still in TMEM)
        auto max_half = [&]() -> float {
          load(0);
          const float a = max_chunk(0);
          load(1);
          return fmaxf(a, max_chunk(1)) * p.scale_log2;
        };
        auto exps = [&]() -> float {
          load(0);
          const float a = exp_chunk(0);
          load(1);
          return a + exp_chunk(1);
        };
        float v = -INFINITY, rs = 0.f;
        if (okw) {
          tc_fence_after();
          if (j == 0) {
            v = max_half();  // the first tile of an item sets each row's reference max
          } else {
            // one pass with the running reference m. exp2(x - m) is exact for any
            // reference as long as x = S * scale - m stays small; the sum of my 64 keys is
            // at most 64 * 2^8 when every x <= 8 and above 2^8 when any x > 8 (or on
            // overflow), so rows whose sum passes 2^8 look at their true max
            rs = exps();
            // tcgen05.ld is .sync.aligned: the whole warp loads S again when any row needs
            // its max (never inside a per-row branch)
            const bool look = !(rs <= 256.f);
            if (__any_sync(0xffffffffu, look)) {
              const float xm = max_half() - m;
              if (look) v = xm;
            }
          }
        }
        const float pv = exchange(v, okw, both);
        if (!both) {
          ok = false;
          left = true;
          break;
        }
        bool step_ok = true;
        if (j == 0) {
          m = fmaxf(v, pv);  // scale_log2 > 0 keeps the arg-max; -inf for empty rows
          rs = exps();
        } else {
          const float xm = fmaxf(v, pv);
          const bool mv = xm > kRescaleThreshold;
          if (__any_sync(0xffffffffu, mv)) {
            // move m; O (my D/2 columns) and l follow once the previous PV has landed
            const float alpha = mv ? fast_exp2(-xm) : 1.f;
            if (mv) m += xm;
            if (!mbar_wait_bounded(&o_done[h], (uint32_t)((n - 1) & 1), p.err)) step_ok = false;
            step_ok = __all_sync(0xffffffffu, step_ok);
            if (step_ok) {
              tc_fence_after();
              for (int c0 = 0; c0 < D / 2; c0 += 16) {
                uint32_t o[16];
                tmem_ld16(o_col + c0, o);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; ++c)
                  o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                tmem_st16(o_col + c0, o);
              }
              tmem_wait_st();
              l *= alpha;
              rs = exps();
            }
          }
        }
        if constexpr (D == 64) {
          // P has columns of its own: S may be overwritten by the next QK^T now, and P may
          // be stored once the previous tile's PV has read the P before it
          tc_fence_before();
          mbar_arrive(&s_read[h]);
          if (step_ok && n > 0 &&
              !mbar_wait_bounded(&o_done[h], (uint32_t)((n - 1) & 1), p.err))
            step_ok = false;
          step_ok = __all_sync(0xffffffffu, step_ok);
          if (step_ok) tc_fence_after();
        }
        if (!step_ok) {  // skip the rest of the tile; the next exchange tells the partner
          ok = false;
          continue;
        }
        tmem_st32(p_col, pk);
        l += rs;
        tmem_wait_st();
        // Keys past the context (the last KV tile's tail) may hold NaN/Inf in the pool;
        // P is 0 there but 0 * NaN is not: zero those V rows before the PV MMAs read them.
        // Head A's warps do it; head B's PV is issued after head A's.
        const int tail0 = it.ctx - j * kN;  // first row of this tile past the context
        if (h == 0 && j == it.n_kv - 1 && tail0 < kN) {
          const int64_t gv = g;
          if (!mbar_wait_bounded(&v_full[gv & 1], (uint32_t)((gv >> 1) & 1), p.err)) ok = false;
          uint8_t* vt = smem + L::kOffV + (int)(gv & 1) * L::kKVBytes;
          const int zrows = kN - max(tail0, 0);
          for (int e = threadIdx.x - 64; e < L::kChunks * zrows * 8; e += 256) {
            const int c = e / (zrows * 8);         // d chunk
            const int rem = e - c * zrows * 8;
            const int rr = max(tail0, 0) + rem / 8;  // token row
            const int q16 = rem % 8;                 // 16-byte piece of the 128-byte line
            reinterpret_cast<uint4*>(vt + c * (kN * 128) + rr * 128)[q16] =
                make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(&p_full[h]);
      }
      if (left) {
        *abort_flag = 1;
        break;
      }
      // ---- epilogue: O / l -> out, each warp its D/2 columns (the next item's first PV of
      // this head waits for this warp's arrival on its first P, which comes after these
      // reads)
      bool okw = ok;
      if (okw && !mbar_wait_bounded(&o_done[h], (uint32_t)((n - 1) & 1), p.err)) okw = false;
      okw = __all_sync(0xffffffffu, okw);
      const float lp = exchange(l, okw, both);
      if (!both) {
        ok = false;
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const float lt = l + lp;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      // 16 columns at a time: each thread puts its row's 32 bytes in the warp's staging
      // buffer (16-byte pieces swapped on every fourth row), then the warp writes 16 rows x
      // 32 B per store instruction
      uint8_t* stage = smem + L::kOffStage + local * (32 * 32);
      const int64_t row0 = (int64_t)it.q0 + it.qt * kM + quarter * 32;  // this warp's rows
      const int nrows = min(32, it.rows_valid - quarter * 32);
      T* obase = reinterpret_cast<T*>(p.out) + (int64_t)qh * p.o_head + (D / 2) * half;
      const int sw = (lane >> 2) & 1;
      for (int c0 = 0; c0 < D / 2; c0 += 16) {
        uint32_t o[16];
        tmem_ld16(o_col + c0, o);
        tmem_wait_ld();
        uint32_t pk8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          pk8[c] = pack2<T>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
        *reinterpret_cast<uint4*>(stage + lane * 32 + sw * 16) =
            make_uint4(pk8[0], pk8[1], pk8[2], pk8[3]);
        *reinterpret_cast<uint4*>(stage + lane * 32 + (sw ^ 1) * 16) =
            make_uint4(pk8[4], pk8[5], pk8[6], pk8[7]);
        __syncwarp();
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const int rr = pass * 16 + (lane >> 1);
          const int c = lane & 1;
          if (rr < nrows)
            *reinterpret_cast<uint4*>(obase + (row0 + rr) * p.o_tok + c0 + c * 8) =
                *reinterpret_cast<const uint4*>(stage + rr * 32 + ((c ^ ((rr >> 2) & 1)) * 16));
        }
        __syncwarp();
      }
      tc_fence_before();
    }
    if (!ok) *abort_flag = 1;
  }

  // ---- teardown: every TMA and MMA of this CTA has finished before TMEM is freed
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Loads this CTA issued land before it leaves: the last Q tiles, and the last two K and
    // V tiles (at most two of each are ever in flight).
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

// Device address of g_prefill_counters on the current device (looked up once per device).
int prefill_counter_base(int32_t** out) {
  static void* base[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return b2p_host::record_error(ce);
  if (dev < 0 || dev >= 64) return B2P_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (base[dev] == nullptr) {
    ce = cudaGetSymbolAddress(&base[dev], g_prefill_counters);
    if (ce != cudaSuccess) return b2p_host::record_error(ce);
  }
  *out = static_cast<int32_t*>(base[dev]);
  return B2P_OK;
}

}  // namespace

// Zero every prefill claim slot of the current device on `stream` (after a launch that
// did not run to its end, e.g. one whose bounded waits gave up).
int b2p_prefill_reset_counters(void* stream) {
  int32_t* base = nullptr;
  const int rc = prefill_counter_base(&base);
  if (rc != B2P_OK) return rc;
  const cudaError_t e = cudaMemsetAsync(base, 0, sizeof(int32_t) * 2 * kCounterSlots,
                                        static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B2P_OK : b2p_host::record_error(e);
}

// ====================================================================== host side
namespace b2p_host {
int tensor_map_4d_rows(CUtensorMap* out, const void* base, int64_t rows, int heads, int head_dim,
                       int64_t row_stride_elems, int64_t head_stride_elems, int elem_bytes,
                       int box_rows);
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
  if ((head_dim != 64 && head_dim != 128) || (dtype != B2P_BF16 && dtype != B2P_F16) ||
      block_size % kSub != 0)
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
    static std::atomic<uint32_t> next_slot{0};
    int32_t* addr = nullptr;
    const int crc = prefill_counter_base(&addr);
    if (crc != B2P_OK) return crc;
    const uint32_t slot = next_slot.fetch_add(1) % kCounterSlots;
    p.ctr = addr + 2 * slot;
  }
  const bool bf16 = dtype == B2P_BF16;
  const int variant = (bf16 ? 0 : 1) + (head_dim == 64 ? 2 : 0);
  const void* fn =
      head_dim == 64
          ? (bf16 ? reinterpret_cast<const void*>(&paged_prefill_tc<__nv_bfloat16, 64>)
                  : reinterpret_cast<const void*>(&paged_prefill_tc<__half, 64>))
          : (bf16 ? reinterpret_cast<const void*>(&paged_prefill_tc<__nv_bfloat16, 128>)
                  : reinterpret_cast<const void*>(&paged_prefill_tc<__half, 128>));
  const int smem = (head_dim == 64 ? Plan<64>::kSmemBytes : Plan<128>::kSmemBytes) + 1024;
  // Persistent: one CTA per SM walks the work items (its 512 TMEM columns and, for head_dim
  // 128, ~222 KB of shared memory fill the SM). Once per device and kernel variant: the
  // kernel's shared-memory attributes, and whether one CTA fits the SM's limits.
  static int resident[64][4] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  if (dev < 0 || dev >= 64) return B2P_EUNSUPPORTED;
  int& fit = resident[dev][variant];
  if (fit == 0) {
    cudaFuncAttributes fa;
    int smem_sm = 0, reserved = 0, regs_sm = 0;
    if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  cudaSharedmemCarveoutMaxShared)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&fa, fn)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor,
                                    dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) !=
            cudaSuccess)
      return b2p_host::record_error(e);
    // registers are handed out per warp in 256-register units
    const int warp_regs = (fa.numRegs * 32 + 255) / 256 * 256;
    const bool fits = regs_sm >= warp_regs * (kThreads / 32) &&
                      smem_sm >= smem + (int)fa.sharedSizeBytes + reserved;
    fit = fits ? 1 : -1;
  }
  if (fit < 0) return B2P_EUNSUPPORTED;
  dim3 grid((unsigned)b2p_host::sm_count());
  void* args[] = {&qmap, &kmap, &vmap, &p};
  e = cudaLaunchKernel(fn, grid, dim3(kThreads), args, (size_t)smem,
                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return b2p_host::record_error(e);
  return b2p_host::check_launch();
}
