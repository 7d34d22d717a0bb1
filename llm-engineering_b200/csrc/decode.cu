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
//    consecutive). Each KV head's list is cut into equal ranges, one per WARP (stream-K at
//    warp granularity), so every warp streams the same number of bytes whatever the
//    context-length mix. Warps of a CTA never wait for one another.
//  * Each warp owns a private ring of S shared-memory stages. Lane 0 issues TMA tile loads
//    (K and V sub-block of one head: 2 x 16 x head_dim elements, 128-byte swizzle, no
//    multicast) and refills a stage as soon as the warp has consumed it; the physical
//    block of every upcoming sub-block is resolved 32 at a time with parallel loads, one
//    chunk ahead, so no TMA waits on a dependent global load.
//  * Per sub-block the warp computes S^T = K Q^T on the tensor cores (m16n8k16: 16 tokens
//    x 8 query heads of the GQA group, K via ldmatrix), the online softmax in fp32 (warp
//    shuffles over the 8 lanes that share a query head), and O^T += V^T P^T (V^T via
//    ldmatrix.trans, P^T transposed in registers with movmatrix). Each KV tile read from
//    shared memory serves all G query heads of its group.
//  * A sequence that lies inside one warp's range is finished from registers. A sequence
//    cut by range boundaries leaves a partial per warp in the workspace (O / l scaled into
//    [-1, 1] in fp16, with the running max, running sum and scale in fp32); once a warp's
//    stream is done it counts its partials in (atomic counter per sequence) and the last
//    warp to report a sequence merges its partials.
#include <mutex>

#include "common.cuh"

namespace {

using namespace b2p;

constexpr int kSub = 16;  // slots per sub-block = tokens per MMA tile
// Sub-blocks per warp prefetched into L2 before the dependent-launch wait (at most 32).
// Measured on the 256-sequence workload: 104.8 us per launch with 4, 105.2 with 8, 106.6
// with 16, 105.6 without.
constexpr int kL2Prefetch = 4;

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
  int heads_per_unit;  // KV heads whose warps stream the same sub-block range in one CTA
  int block_size;      // multiple of 16
  int64_t num_blocks;
  float scale_log2;  // softmax scale * log2(e)
  float* partials;   // [num_kv_heads][units][2][record]
  int32_t* counters; // [num_kv_heads][num_seqs], zero between launches
  int32_t* err;
  // Append mode (new_k != nullptr): each sequence's newest K/V row (the key at position
  // ctx - 1) comes in here; the warp that streams the sequence's last sub-block puts it
  // into its shared-memory tile and stores it into the pool at the slot the block table
  // gives for that position (what a KV write with the step's slot mapping would do).
  const uint8_t* new_k;
  int64_t nk_tok, nk_head;  // element strides
  const uint8_t* new_v;
  int64_t nv_tok, nv_head;
  uint8_t* kpool;
  uint8_t* vpool;
  int num_kv_heads;
};

template <int D, int NT>
struct Record {
  // Partial of one (unit, sequence): O^T / (l * s) in fp16, in MMA fragment order
  // ([D/16][NT][32 lanes][4 halves] = one 8-byte access per lane), then per query head in
  // fp32 the running max, the running sum and the scale s = max_d |O / l|. Normalised
  // values are bounded by max|v|, which a bf16 pool can push far past fp16's 65504; divided
  // by s they lie in [-1, 1], so fp16 keeps its 11-bit precision relative to the head's
  // largest value at any magnitude. The merge re-weights them with the fp32 sums and scales.
  static constexpr int kOBytes = (D / 16) * NT * 32 * 8;
  static constexpr int kFloats = kOBytes / 4 + 3 * NT * 8;
  static constexpr int kM = kOBytes / 4;           // float index of the maxima
  static constexpr int kL = kOBytes / 4 + NT * 8;  // float index of the sums
  static constexpr int kS = kOBytes / 4 + 2 * NT * 8;  // float index of the scales
};

struct Range {
  int64_t begin, end;  // global sub-block indices of this unit (per KV head)
  int seq0;            // sequence containing `begin`
  int64_t cb0;         // first global sub-block index of seq0
  int64_t total;       // sub-blocks over all sequences (per KV head)
  int64_t parts;       // ranges actually used: min(requested, total)
};

__device__ __forceinline__ int64_t range_start(int64_t c, int64_t total, int64_t parts) {
  return (c * total) / parts;
}

__device__ __forceinline__ int64_t owner_unit(int64_t b, int64_t total, int64_t parts) {
  return ((b + 1) * parts - 1) / total;
}

__device__ __forceinline__ int sub_blocks_of(int ctx) { return ctx > 0 ? (ctx + kSub - 1) / kSub : 0; }

// One warp: total sub-blocks over all sequences, then the sequence holding unit c's first
// sub-block. Each lane owns kPer consecutive sequences of a 32*kPer chunk and issues all
// its loads before any arithmetic, so a batch of up to 256 sequences costs one memory
// round trip; the second pass reuses the registers in that case.
__device__ void find_range(const DecodeParams& p, int64_t parts, int64_t c, Range& r) {
  constexpr int kPer = 8;
  constexpr int kChunk = 32 * kPer;
  const int lane = threadIdx.x & 31;
  int nbv[kPer];
  int64_t total = 0;
  for (int base = 0; base < p.num_seqs; base += kChunk) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = base + lane * kPer + j;
      nbv[j] = i < p.num_seqs ? __ldg(p.context_lens + i) : 0;
    }
    int sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      nbv[j] = sub_blocks_of(nbv[j]);
      sum += nbv[j];
    }
    total += __reduce_add_sync(0xffffffffu, (unsigned)sum);
  }
  r.total = total;
  // Never more ranges than sub-blocks, so every range is non-empty and the units that
  // share a sequence are exactly owner(first block) .. owner(last block).
  r.parts = parts < total ? parts : total;
  r.seq0 = p.num_seqs;
  r.cb0 = total;
  if (c >= r.parts) {
    r.begin = r.end = 0;
    return;
  }
  r.begin = range_start(c, total, r.parts);
  r.end = range_start(c + 1, total, r.parts);
  int64_t run = 0;
  for (int base = 0; base < p.num_seqs; base += kChunk) {
    if (p.num_seqs > kChunk) {  // registers hold the last chunk only: reload this one
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int i = base + lane * kPer + j;
        nbv[j] = sub_blocks_of(i < p.num_seqs ? __ldg(p.context_lens + i) : 0);
      }
    }
    int sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) sum += nbv[j];
    int incl = sum;  // inclusive scan of per-lane sums
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t lane_lo = run + incl - sum;
    const unsigned hit = __ballot_sync(0xffffffffu, run + incl > r.begin);
    if (hit) {
      const int src = __ffs(hit) - 1;
      if (lane == src) {
        int64_t cb = lane_lo;
        int k = 0;
        while (k < kPer - 1 && cb + nbv[k] <= r.begin) cb += nbv[k++];
        r.seq0 = base + lane * kPer + k;
        r.cb0 = cb;
      }
      r.seq0 = __shfl_sync(0xffffffffu, r.seq0, src);
      r.cb0 = __shfl_sync(0xffffffffu, r.cb0, src);
      return;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
}

// Maps a warp's consecutive sub-blocks to pool slot coordinates, 32 at a time: lane j
// resolves sub-block (chunk0 + j) of the range. Sequences are found by a scan over windows
// of 32 context lengths plus a per-lane binary search, then every lane reads its block
// id; all loads of one call are independent of each other.
struct SlotResolver {
  int win_seq;     // first sequence that can hold the next chunk
  int64_t win_cb;  // its first sub-block
  int64_t begin, n;

  __device__ int64_t operator()(const DecodeParams& p, int64_t chunk0, int lane,
                                int64_t num_slots) {
    const unsigned full_mask = 0xffffffffu;
    const int spb = p.block_size / kSub;
    const int64_t g = begin + chunk0 + lane;
    const bool valid = chunk0 + lane < n;
    int my_seq = -1;
    int64_t my_cb = 0;
    for (int guard = 0; guard < 1024; ++guard) {  // windows of 32 sequences
      const int si = win_seq + lane;
      const int nbj = si < p.num_seqs ? sub_blocks_of(__ldg(p.context_lens + si)) : 0;
      int incl = nbj;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(full_mask, incl, o);
        if (lane >= o) incl += v;
      }
      const int64_t endj = win_cb + incl;  // exclusive end of sequence win_seq + lane
      int lo = 0, hi = 32;  // smallest j with end_j > g
#pragma unroll
      for (int step = 0; step < 6; ++step) {
        const int mid = (lo + hi) >> 1;
        const int64_t e = __shfl_sync(full_mask, endj, mid < 32 ? mid : 31);
        if (lo < hi) {
          if (e > g) hi = mid; else lo = mid + 1;
        }
      }
      const int64_t start_lo = __shfl_sync(full_mask, endj - nbj, lo < 32 ? lo : 31);
      if (valid && my_seq < 0 && lo < 32) {
        my_seq = win_seq + lo;
        my_cb = start_lo;
      }
      if (!__any_sync(full_mask, valid && my_seq < 0)) break;
      win_cb = __shfl_sync(full_mask, endj, 31);
      win_seq += 32;
      if (win_seq >= p.num_seqs) break;
    }
    // The next chunk starts in the sequence of this chunk's last sub-block.
    const unsigned vmask = __ballot_sync(full_mask, valid && my_seq >= 0);
    if (vmask) {
      const int last = 31 - __clz(vmask);
      win_seq = __shfl_sync(full_mask, my_seq, last);
      win_cb = __shfl_sync(full_mask, my_cb, last);
    }
    if (!valid) return -1;
    if (my_seq < 0) {
      set_device_error(p.err, B2P_DEV_LENGTH);
      return num_slots;
    }
    const int lb = (int)(g - my_cb);
    const int64_t col = lb / spb;
    const int32_t blk =
        col < p.bt_stride ? __ldg(p.block_tables + (int64_t)my_seq * p.bt_stride + col) : -1;
    if (blk < 0 || (int64_t)blk >= p.num_blocks) {
      set_device_error(p.err, B2P_DEV_BLOCK_RANGE);
      return num_slots;  // fully out of bounds: the TMA unit zero-fills the tile
    }
    return (int64_t)blk * p.block_size + (int64_t)(lb % spb) * kSub;
  }
};

template <typename T, int D, int NT, int S, int W>
__global__ void __launch_bounds__(W * 32) paged_decode_tc(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap,
                                                          const DecodeParams p) {
  constexpr int kTileBytes = kSub * D * 2;  // one K or V sub-block of one head
  constexpr int kStageBytes = 2 * kTileBytes;
  // A tile is stored as D/64 chunks of [16 tokens][64 elements] (one TMA box each), so the
  // 8 token rows that one ldmatrix phase reads are 8 consecutive 128-byte lines: their
  // 128-byte swizzle phases all differ and the reads are free of bank conflicts (with
  // 256-byte token rows, rows t and t + 4 would share a phase).
  constexpr int kChunks = D / 64;
  constexpr int kChunkBytes = kSub * 128;
  using Rec = Record<D, NT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // Programmatic dependent launch: this grid may be scheduled while the previous kernel on
  // the stream is finishing, and lets the next launch be scheduled the same way (the
  // trigger). Before the wait it reads only the context lengths and block tables (to find
  // its range and resolve its first blocks), which no kernel that triggers early writes:
  // this one never writes them, and a kernel that does not trigger (block-table builds,
  // host copies, PyTorch ops) has completed before this grid starts. Errors found there go
  // to the error word with atomic ORs, which commute. The pool, the outputs and the
  // workspace are touched only after the wait, once the previous kernel has completed and
  // its writes are visible.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  auto pdl_wait = []() { asm volatile("griddepcontrol.wait;" ::: "memory"); };
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Warps w and w+1 (2 KV heads) or w..w+3 (4 heads) stream the same sub-blocks for
  // different heads, so both halves of every 512-byte slot row are fetched by one SM at
  // nearly the same time (one DRAM page opening instead of two).
  const int hpu = p.heads_per_unit;
  const int head = blockIdx.y * hpu + warp % hpu;  // KV head
  uint8_t* ring = smem + (size_t)warp * S * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)W * S * kStageBytes) + warp * S;
  // slot of each stage's first row (append mode stores the new row relative to it)
  int32_t* stage_slot =
      reinterpret_cast<int32_t*>(smem + (size_t)W * S * kStageBytes + W * S * 8) + warp * S;

  // A decode sequence always has at least its own token; an empty history has no softmax.
  // One warp per KV head writes the zero rows and the flag of every empty history (a range
  // never starts on one, so no stream unit sees those that sit on range boundaries).
  auto write_empties = [&]() {
    for (int base = 0; base < p.num_seqs; base += 32) {
      const int sq = base + lane;
      unsigned m = __ballot_sync(0xffffffffu, sq < p.num_seqs && __ldg(p.context_lens + sq) <= 0);
      while (m) {
        const int s2 = base + __ffs(m) - 1;
        m &= m - 1;
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)s2 * p.o_tok;
        for (int e = lane; e < p.group * D; e += 32) {
          const int qh = e / D, d = e - qh * D;
          orow[(int64_t)(head * p.group + qh) * p.o_head + d] = from_f32<T>(0.f);
        }
        if (lane == 0) set_device_error(p.err, B2P_DEV_LENGTH);
      }
    }
  };
  const bool empties_warp = blockIdx.x == 0 && warp == W - 1;

  Range r;
  const int64_t units_per_cta = W / hpu;
  const int64_t unit = (int64_t)blockIdx.x * units_per_cta + warp / hpu;
  find_range(p, (int64_t)gridDim.x * units_per_cta, unit, r);
  if (r.begin >= r.end) {
    pdl_wait();
    if (empties_warp) write_empties();
    return;
  }
  const int64_t n = r.end - r.begin;
  const int64_t parts = r.parts;
  const int64_t num_slots = p.num_blocks * p.block_size;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  __syncwarp();

  SlotResolver res{r.seq0, r.cb0, r.begin, n};
  int64_t buf_base = 0;  // items [buf_base, buf_base + 32) are in slot_lo
  int64_t slot_lo = res(p, 0, lane, num_slots);
  int64_t slot_hi = -1;  // resolved right after the first copies are out
  int64_t issued = 0;
  bool aborted = false;

  // Issue item k into stage k % S (all lanes call it; lane 0 issues the copies).
  auto issue = [&](int64_t k) {
    if (k >= buf_base + 32) {  // every item below k is issued: rotate the slot buffers
      buf_base += 32;
      slot_lo = slot_hi;
      slot_hi = buf_base + 32 < n ? res(p, buf_base + 32, lane, num_slots) : -1;
    }
    const int64_t slot = __shfl_sync(0xffffffffu, slot_lo, (int)(k - buf_base));
    if (lane == 0) {
      const int stage = (int)(k % S);
      uint8_t* kdst = ring + stage * kStageBytes;
      const int c3 = (int)(slot < 0 ? num_slots : slot);
      stage_slot[stage] = c3;
      mbar_arrive_expect_tx(&full[stage], kStageBytes);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        tma_load_5d(kdst + c * kChunkBytes, &kmap, &full[stage], 0, c, head, c3, p.layer);
        tma_load_5d(kdst + kTileBytes + c * kChunkBytes, &vmap, &full[stage], 0, c, head, c3,
                    p.layer);
      }
    }
    issued = k + 1;
  };
  // While the previous kernel finishes (this CTA may start early under programmatic
  // dependent launch, when HBM is mostly idle), pull the warp's first sub-blocks into L2:
  // lane j prefetches item j's K and V boxes. The prefetches write no shared memory, so
  // they need no wait of their own; the loads after the wait then hit L2.
  if (lane < kL2Prefetch && lane < n && slot_lo >= 0 && slot_lo < num_slots) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      tma_prefetch_l2_5d(&kmap, 0, c, head, (int)slot_lo, p.layer);
      tma_prefetch_l2_5d(&vmap, 0, c, head, (int)slot_lo, p.layer);
    }
  }
  pdl_wait();  // the first access to memory the previous kernel may write
  for (int64_t k = 0; k < S && k < n; ++k) issue(k);
  if (empties_warp) write_empties();  // while the first tiles are in flight
  if (n > 32) slot_hi = res(p, 32, lane, num_slots);

  const int g8 = lane >> 2;  // row group (0..7)
  const int t4 = lane & 3;   // thread in group (0..3)
  int seq = r.seq0;
  int64_t cb = r.cb0;
  int64_t gidx = r.begin;
  int64_t k = 0;  // local item index

  // Normalised output rows of one sequence from O^T fragments and per-head sums.
  auto write_out = [&](int sq, float (&o)[D / 16][NT][4], float (&lsum)[NT][2]) {
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int qh = nn * 8 + 2 * t4 + cc;
        if (qh >= p.group) continue;
        const float inv = lsum[nn][cc] > 0.f ? 1.f / lsum[nn][cc] : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)sq * p.o_tok +
                  (int64_t)(head * p.group + qh) * p.o_head;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          orow[i * 16 + g8] = from_f32<T>(o[i][nn][cc] * inv);
          orow[i * 16 + g8 + 8] = from_f32<T>(o[i][nn][2 + cc] * inv);
        }
      }
    }
  };
  int npend = 0;  // sequences this warp left a partial for (at most its first and last)
  int pend_seq[2] = {0, 0};
  int64_t pend_cb[2] = {0, 0};
  int pend_nb[2] = {0, 0};

  while (gidx < r.end) {
    const int ctx = __ldg(p.context_lens + seq);
    const int nb = sub_blocks_of(ctx);
    if (nb == 0) {  // written by the empties warp
      ++seq;
      continue;
    }
    const int lb0 = (int)(gidx - cb);
    const int64_t seg_end = min(r.end, cb + nb);
    const int lb1 = (int)(seg_end - cb);

    // Append mode: warm L1 with this sequence's new K/V rows if its last sub-block is in
    // the segment (they are put into that tile when it arrives).
    const bool appends = p.new_k != nullptr && lb1 == nb;
    if (appends && lane < 2 * (D * (int)sizeof(T) / 128)) {
      const int lines = D * (int)sizeof(T) / 128;
      const bool isv = lane >= lines;
      const uint8_t* row = isv ? p.new_v + ((int64_t)seq * p.nv_tok + (int64_t)head * p.nv_head) * sizeof(T)
                               : p.new_k + ((int64_t)seq * p.nk_tok + (int64_t)head * p.nk_head) * sizeof(T);
      asm volatile("prefetch.global.L1 [%0];" ::"l"(row + (isv ? lane - lines : lane) * 128));
    }

    // Warm L1 with the next sequence's query rows (read when its segment starts).
    if (seg_end < r.end && lb1 == nb && seq + 1 < p.num_seqs) {
      const T* nq = reinterpret_cast<const T*>(p.q) + (int64_t)(seq + 1) * p.q_tok +
                    (int64_t)head * p.group * p.q_head;
      const int lines = (p.group * D * (int)sizeof(T) + 127) / 128;
      if (lane < lines && p.q_head == D)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const uint8_t*>(nq) + lane * 128));
    }

    // Q fragments (B operand of S^T = K Q^T): Q[qh = g8 + 8n][16kk + 2t4 (+8)].
    uint32_t qf[NT][D / 16][2];
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
      const int qh = nn * 8 + g8;
      const bool ok = qh < p.group;
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)seq * p.q_tok +
                      (int64_t)(head * p.group + (ok ? qh : 0)) * p.q_head;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qf[nn][kk][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4)) : 0u;
        qf[nn][kk][1] =
            ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * t4)) : 0u;
      }
    }

    float m_run[NT][2], l_run[NT][2];
    float acc[D / 16][NT][4];
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
      m_run[nn][0] = m_run[nn][1] = -INFINITY;
      l_run[nn][0] = l_run[nn][1] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i)
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) acc[i][nn][0] = acc[i][nn][1] = acc[i][nn][2] = acc[i][nn][3] = 0.f;

    for (int lb = lb0; lb < lb1; ++lb, ++k) {
      const int stage = (int)(k % S);
      if (!aborted && !mbar_wait_bounded(&full[stage], (uint32_t)((k / S) & 1), p.err))
        aborted = true;
      aborted = __any_sync(0xffffffffu, aborted);
      if (aborted) continue;  // keep walking so every sequence still gets written
      uint8_t* ktile = ring + stage * kStageBytes;
      uint8_t* vtile = ktile + kTileBytes;
      const int valid = min(kSub, ctx - lb * kSub);
      if (valid < kSub) {
        // Slots past the context may hold anything (the pool is not cleared), and
        // 0 * NaN would poison O: zero the V rows of masked tokens. In each 64-column chunk
        // a token is one whole 128-byte swizzle line, so no swizzle math is needed.
        const int per_chunk = (kSub - valid) * 8;  // 16-byte pieces per chunk
        for (int i = lane; i < kChunks * per_chunk; i += 32) {
          const int c = i / per_chunk;
          const int j = i - c * per_chunk;
          reinterpret_cast<uint4*>(vtile + c * kChunkBytes + valid * 128)[j] =
              make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      const bool patched = appends && lb == nb - 1;
      if (patched) {
        // The newest token (row valid - 1 of this tile): its K and V rows replace what the
        // pool held at its slot, in the tile (16-byte chunks at their swizzled places) and
        // in the pool. No other stream unit reads that slot in this launch.
        const int rrow = valid - 1;
        const int32_t slot = stage_slot[stage] + rrow;
        const bool in_pool = stage_slot[stage] < (int32_t)num_slots;
        constexpr int kChunks = D * 2 / 16;  // 16-byte chunks per row
        for (int c = lane; c < 2 * kChunks; c += 32) {
          const bool isv = c >= kChunks;
          const int cc = isv ? c - kChunks : c;
          const uint4 val = __ldg(reinterpret_cast<const uint4*>(
                                isv ? p.new_v + ((int64_t)seq * p.nv_tok + (int64_t)head * p.nv_head) * 2
                                    : p.new_k + ((int64_t)seq * p.nk_tok + (int64_t)head * p.nk_head) * 2) + cc);
          const int d = cc * 8;
          const uint32_t off = (uint32_t)(((d / 64) * kSub + rrow) * 128 + (d % 64) * 2);
          *reinterpret_cast<uint4*>((isv ? vtile : ktile) + swz128(off)) = val;
          if (in_pool) {
            uint8_t* pool = isv ? p.vpool : p.kpool;
            const int64_t e = (((int64_t)p.layer * num_slots + slot) * p.num_kv_heads + head) * D + d;
            *reinterpret_cast<uint4*>(pool + e * 2) = val;
          }
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(ktile);
      const uint32_t vbase = smem_u32(vtile);

      // ---- S^T = K Q^T  (M = 16 tokens, N = 8 query heads per tile, K = D); two
      // accumulator sets (even / odd k-steps) halve the dependent MMA chain.
      float s[NT][4], s2[NT][4];
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        s[nn][0] = s[nn][1] = s[nn][2] = s[nn][3] = 0.f;
        s2[nn][0] = s2[nn][1] = s2[nn][2] = s2[nn][3] = 0.f;
      }
      {
        const int mat = lane >> 3, rr = lane & 7;
        const int tok = rr + (mat & 1) * 8;
        const int dsub = (mat >> 1) * 8;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int dcol = kk * 16 + dsub;
          const uint32_t off = (uint32_t)(((dcol / 64) * kSub + tok) * 128 + (dcol % 64) * 2);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(kbase + swz128(off), a0, a1, a2, a3);
#pragma unroll
          for (int nn = 0; nn < NT; ++nn)
            MmaOp<T>::run((kk & 1) ? s2[nn] : s[nn], a0, a1, a2, a3, qf[nn][kk][0], qf[nn][kk][1]);
        }
#pragma unroll
        for (int nn = 0; nn < NT; ++nn)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[nn][e] += s2[nn][e];
      }

      // ---- online softmax over the tile's tokens (rows g8 and g8+8)
      const bool v0 = g8 < valid, v1 = g8 + 8 < valid;
      uint32_t pb[NT][2];
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        const float x0 = v0 ? s[nn][0] * p.scale_log2 : -INFINITY;
        const float x1 = v0 ? s[nn][1] * p.scale_log2 : -INFINITY;
        const float x2 = v1 ? s[nn][2] * p.scale_log2 : -INFINITY;
        const float x3 = v1 ? s[nn][3] * p.scale_log2 : -INFINITY;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m_run[nn][0], mx0), mn1 = fmaxf(m_run[nn][1], mx1);
        const float al0 = fast_exp2(m_run[nn][0] - mn0), al1 = fast_exp2(m_run[nn][1] - mn1);
        m_run[nn][0] = mn0;
        m_run[nn][1] = mn1;
        const float p0 = fast_exp2(x0 - mn0), p1 = fast_exp2(x1 - mn1);
        const float p2 = fast_exp2(x2 - mn0), p3 = fast_exp2(x3 - mn1);
        l_run[nn][0] = l_run[nn][0] * al0 + p0 + p2;
        l_run[nn][1] = l_run[nn][1] * al1 + p1 + p3;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          acc[i][nn][0] *= al0;
          acc[i][nn][1] *= al1;
          acc[i][nn][2] *= al0;
          acc[i][nn][3] *= al1;
        }
        pb[nn][0] = movmatrix_trans(pack2<T>(p0, p1));
        pb[nn][1] = movmatrix_trans(pack2<T>(p2, p3));
      }

      // ---- O^T += V^T P^T  (M = 16 dims per tile, N = 8 query heads, K = 16 tokens)
      {
        const int mat = lane >> 3, rr = lane & 7;
        const int tok = rr + (mat >> 1) * 8;
        const int dsub = (mat & 1) * 8;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          const int dcol = i * 16 + dsub;
          const uint32_t off = (uint32_t)(((dcol / 64) * kSub + tok) * 128 + (dcol % 64) * 2);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(vbase + swz128(off), a0, a1, a2, a3);
#pragma unroll
          for (int nn = 0; nn < NT; ++nn)
            MmaOp<T>::run(acc[i][nn], a0, a1, a2, a3, pb[nn][0], pb[nn][1]);
        }
      }
      // Refill this stage with the item S ahead. All reads of the stage are complete (their
      // results fed the MMAs above); generic writes (the zeroed rows) need a proxy fence
      // before the TMA unit writes the same bytes.
      if (valid < kSub || patched) fence_proxy_async_smem();
      __syncwarp();
      if (k + S < n) issue(k + S);
    }

    // ---- finish the segment: full sums per query head
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l_run[nn][0] += __shfl_xor_sync(0xffffffffu, l_run[nn][0], o);
        l_run[nn][1] += __shfl_xor_sync(0xffffffffu, l_run[nn][1], o);
      }
    }
    const bool complete = (lb0 == 0) && (lb1 == nb);
    if (complete) {
      write_out(seq, acc, l_run);
    } else {
      const int slot_idx = (cb + lb0 == r.begin) ? 0 : 1;  // first segment of this unit or not
      float* rec = p.partials + (((size_t)head * parts + unit) * 2 + slot_idx) * Rec::kFloats;
      float sc[NT][2];  // per query head: max_d |O / l|
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          a0 = fmaxf(a0, fmaxf(fabsf(acc[i][nn][0]), fabsf(acc[i][nn][2])));
          a1 = fmaxf(a1, fmaxf(fabsf(acc[i][nn][1]), fabsf(acc[i][nn][3])));
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {  // the 8 lanes holding one query head's rows
          a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, o));
          a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, o));
        }
        const float i0 = l_run[nn][0] > 0.f ? 1.f / l_run[nn][0] : 0.f;
        const float i1 = l_run[nn][1] > 0.f ? 1.f / l_run[nn][1] : 0.f;
        sc[nn][0] = a0 * i0;
        sc[nn][1] = a1 * i1;
        // O / l / s = O / max_d |O|: every stored value lies in [-1, 1].
        const float f0 = a0 > 0.f ? 1.f / a0 : 0.f;
        const float f1 = a1 > 0.f ? 1.f / a1 : 0.f;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          __half2 lo = __floats2half2_rn(acc[i][nn][0] * f0, acc[i][nn][1] * f1);
          __half2 hi = __floats2half2_rn(acc[i][nn][2] * f0, acc[i][nn][3] * f1);
          uint2 v;
          v.x = *reinterpret_cast<uint32_t*>(&lo);
          v.y = *reinterpret_cast<uint32_t*>(&hi);
          reinterpret_cast<uint2*>(rec)[(i * NT + nn) * 32 + lane] = v;
        }
      }
      if (g8 == 0) {
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
          rec[Rec::kM + nn * 8 + 2 * t4] = m_run[nn][0];
          rec[Rec::kM + nn * 8 + 2 * t4 + 1] = m_run[nn][1];
          rec[Rec::kL + nn * 8 + 2 * t4] = l_run[nn][0];
          rec[Rec::kL + nn * 8 + 2 * t4 + 1] = l_run[nn][1];
          rec[Rec::kS + nn * 8 + 2 * t4] = sc[nn][0];
          rec[Rec::kS + nn * 8 + 2 * t4 + 1] = sc[nn][1];
        }
      }
      // The counter update (which needs a fence) and the possible merge wait until this
      // warp's stream is finished: a fence issued mid-stream stalls behind the warp's
      // outstanding loads and leaves its stages unrefilled.
      if (npend < 2) {
        pend_seq[npend] = seq;
        pend_cb[npend] = cb;
        pend_nb[npend] = nb;
        ++npend;
      }
    }
    gidx = seg_end;
    if (lb1 == nb) {
      cb += nb;
      ++seq;
    }
  }
  // Never leave while TMA writes into this warp's stages are in flight (only possible
  // after an abort; otherwise every issued item has been waited for).
  if (lane == 0) {
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(&full[kk % S], (uint32_t)((kk / S) & 1), nullptr);
  }

  // Count this warp's partials in; the last unit to report a sequence merges all of its
  // partials (its own included), reading through L2 since other SMs wrote them.
  if (npend == 0) return;
  __syncwarp();
  int last_mask = 0;
  if (lane == 0) {
    // Release: the partial records written above (by every lane, ordered before this by
    // __syncwarp) are visible before the counts say so. fence.acq_rel with relaxed atomics
    // is the release/acquire pattern of the PTX memory model, lighter than a full fence.
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    int prev[2] = {0, 0};
    for (int j = 0; j < npend; ++j)  // both atomics in flight together
      prev[j] = atomicAdd(p.counters + (size_t)head * p.num_seqs + pend_seq[j], 1);
    for (int j = 0; j < npend; ++j) {
      const int64_t uf = owner_unit(pend_cb[j], r.total, parts);
      const int64_t ul = owner_unit(pend_cb[j] + pend_nb[j] - 1, r.total, parts);
      if (prev[j] == (int)(ul - uf)) {
        p.counters[(size_t)head * p.num_seqs + pend_seq[j]] = 0;  // zeroed for the next launch
        last_mask |= 1 << j;
      }
    }
    // acquire: a last contributor reads the others' records after their counts
    if (last_mask) asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  last_mask = __shfl_sync(0xffffffffu, last_mask, 0);
  for (int j = 0; j < npend; ++j) {
    if (!((last_mask >> j) & 1)) continue;
    const int sq = pend_seq[j];
    const int64_t scb = pend_cb[j];
    const int64_t u_first = owner_unit(scb, r.total, parts);
    const int64_t u_last = owner_unit(scb + pend_nb[j] - 1, r.total, parts);
    float M[NT][2], L[NT][2];
    float O[D / 16][NT][4];
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
      M[nn][0] = M[nn][1] = -INFINITY;
      L[nn][0] = L[nn][1] = 0.f;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) O[i][nn][0] = O[i][nn][1] = O[i][nn][2] = O[i][nn][3] = 0.f;
    }
    // One online pass; four contributors' loads are issued before any of them is used.
    constexpr int kBatch = 4;
    for (int64_t u0 = u_first; u0 <= u_last; u0 += kBatch) {
      float mv[kBatch][NT][2], lv[kBatch][NT][2], sv[kBatch][NT][2];
      uint2 ov[kBatch][D / 16][NT];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int64_t u = u0 + b;
        const bool have = u <= u_last;
        const int si = (u == u_first && range_start(u, r.total, parts) != scb) ? 1 : 0;
        const float* pr =
            p.partials + (((size_t)head * parts + (have ? u : u_first)) * 2 + si) * Rec::kFloats;
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
          mv[b][nn][0] = have ? __ldcg(pr + Rec::kM + nn * 8 + 2 * t4) : -INFINITY;
          mv[b][nn][1] = have ? __ldcg(pr + Rec::kM + nn * 8 + 2 * t4 + 1) : -INFINITY;
          lv[b][nn][0] = have ? __ldcg(pr + Rec::kL + nn * 8 + 2 * t4) : 0.f;
          lv[b][nn][1] = have ? __ldcg(pr + Rec::kL + nn * 8 + 2 * t4 + 1) : 0.f;
          sv[b][nn][0] = have ? __ldcg(pr + Rec::kS + nn * 8 + 2 * t4) : 0.f;
          sv[b][nn][1] = have ? __ldcg(pr + Rec::kS + nn * 8 + 2 * t4 + 1) : 0.f;
#pragma unroll
          for (int i = 0; i < D / 16; ++i)
            ov[b][i][nn] = have ? __ldcg(reinterpret_cast<const uint2*>(pr) + (i * NT + nn) * 32 + lane)
                                : make_uint2(0u, 0u);
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
          float w[2], a[2];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const float mn = fmaxf(M[nn][cc], mv[b][nn][cc]);
            a[cc] = mn == -INFINITY ? 0.f : fast_exp2(M[nn][cc] - mn);  // rescale old
            w[cc] = mn == -INFINITY ? 0.f : fast_exp2(mv[b][nn][cc] - mn) * lv[b][nn][cc];
            L[nn][cc] = L[nn][cc] * a[cc] + w[cc];
            M[nn][cc] = mn;
            w[cc] *= sv[b][nn][cc];  // stored values are O / (l * s)
          }
#pragma unroll
          for (int i = 0; i < D / 16; ++i) {
            const uint2 v = ov[b][i][nn];
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
            O[i][nn][0] = O[i][nn][0] * a[0] + lo.x * w[0];
            O[i][nn][1] = O[i][nn][1] * a[1] + lo.y * w[1];
            O[i][nn][2] = O[i][nn][2] * a[0] + hi.x * w[0];
            O[i][nn][3] = O[i][nn][3] * a[1] + hi.y * w[1];
          }
        }
      }
    }
    write_out(sq, O, L);
  }
}

}  // namespace

// ====================================================================== host side
namespace {

struct Plan {
  const void* fn = nullptr;
  int smem = 0;
  int warps = 0;        // W: stream units per CTA
  int record = 0;       // floats per partial record
  int max_ctas = 8;     // CTAs per SM at most (the workspace is sized for 8)
  int ctas_per_sm = 0;
};

template <typename T, int D, int NT, int S, int W>
Plan make_plan(int max_ctas) {
  Plan pl;
  pl.fn = reinterpret_cast<const void*>(&paged_decode_tc<T, D, NT, S, W>);
  // W rings of S stages (K and V tile each), W*S mbarriers, W*S stage slots, + slack for
  // the 1024 alignment.
  pl.smem = W * S * (2 * kSub * D * 2) + W * S * 8 + W * S * 4 + 1024;
  pl.warps = W;
  pl.record = Record<D, NT>::kFloats;
  pl.max_ctas = max_ctas;
  return pl;
}

// Kernel instantiation for (dtype, head_dim, group): S stages of K+V tiles per warp, W warps
// (stream units) per CTA, at most C CTAs per SM. For head_dim 128 and groups up to 8 (the
// Qwen2.5-1.5B and -7B shapes) one CTA of 7 warps per SM with 2-stage rings (112 KiB of
// reads in flight per SM) was measured fastest on the 256-sequence benchmark workload:
// 107.7 us per launch against 111.9 us for three CTAs of 4 warps (the previous layout),
// 108.4 for 8 warps, 109.2 for 6, 112.0 for 10, 110.7 for 12, 109.6 for two CTAs of 4,
// 111.9 for 3-stage rings of 6 warps. Fewer stream units cut fewer sequences, and the
// partial records and merges they save outweigh the reads in flight they give up.
bool select_plan(int dtype, int head_dim, int group, Plan& pl) {
  const int nt = group <= 8 ? 1 : (group <= 16 ? 2 : 0);
  if (nt == 0) return false;
#define B2P_CASE(TT, DD, NN, SS, WW, CC)         \
  if (head_dim == DD && nt == NN) {              \
    pl = make_plan<TT, DD, NN, SS, WW>(CC);      \
    return true;                                 \
  }
  if (dtype == B2P_BF16) {
    B2P_CASE(__nv_bfloat16, 64, 1, 4, 4, 8)
    B2P_CASE(__nv_bfloat16, 64, 2, 4, 4, 8)
    B2P_CASE(__nv_bfloat16, 128, 1, 2, 7, 1)
    B2P_CASE(__nv_bfloat16, 128, 2, 2, 4, 8)
    B2P_CASE(__nv_bfloat16, 256, 1, 2, 4, 8)
  } else if (dtype == B2P_F16) {
    B2P_CASE(__half, 64, 1, 4, 4, 8)
    B2P_CASE(__half, 64, 2, 4, 4, 8)
    B2P_CASE(__half, 128, 1, 2, 7, 1)
    B2P_CASE(__half, 128, 2, 2, 4, 8)
    B2P_CASE(__half, 256, 1, 2, 4, 8)
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
  cudaError_t e = cudaFuncSetAttribute(pl.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pl.fn, pl.warps * 32, pl.smem);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  if (occ <= 0) return B2P_EUNSUPPORTED;
  if (occ > pl.max_ctas) occ = pl.max_ctas;  // never above 8: the workspace bound
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

// KV heads that share one sub-block range inside a CTA (a divisor of the head count that
// fits the CTA's warps).
int heads_per_unit(int num_kv_heads, int warps) {
  // Measured on B200: pairing the warps of both KV heads on one range (both halves of each
  // slot row fetched by one SM) was slower than one head per CTA (121 vs 113 us on the
  // 256-sequence, 12/2-head benchmark), so every warp streams its own range.
  (void)num_kv_heads;
  (void)warps;
  return 1;
}

// CTAs along x (one wave over all SMs for the grid.y head groups).
int64_t ctas_x(int ctas_per_sm, int num_kv_heads, int hpu) {
  const int64_t slots = (int64_t)b2p_host::sm_count() * ctas_per_sm;
  const int64_t c = slots / (num_kv_heads / hpu);
  return c < 1 ? 1 : c;
}

// Workspace layout: the partial records first (their size depends only on the launch
// shape: heads, head_dim, group, dtype and SM occupancy), then one count-in counter per
// (kv head, sequence). The counters therefore sit at the same offset for every launch of a
// shape, in bytes that only counters ever use; every launch that completes leaves them zero
// (each last contributor re-zeroes its own). Counters placed first, sized by this launch's
// sequence count, would grow into bytes that an earlier launch with fewer sequences filled
// with partial records, and a stale non-zero count there never reaches the merge.
size_t counters_bytes(int num_seqs, int num_kv_heads) {
  return ((size_t)num_kv_heads * num_seqs * 4 + 255) & ~size_t(255);
}

size_t partials_bytes(int num_kv_heads, int64_t units, int record) {
  return ((size_t)num_kv_heads * units * 2 * record * sizeof(float) + 255) & ~size_t(255);
}

size_t workspace_bytes(int num_seqs, int num_kv_heads, int64_t units, int record) {
  return partials_bytes(num_kv_heads, units, record) + counters_bytes(num_seqs, num_kv_heads);
}

}  // namespace

extern "C" size_t b2p_paged_decode_workspace_size(int num_seqs, int num_q_heads,
                                                  int num_kv_heads, int head_dim) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  Plan pl;
  if (!select_plan(B2P_BF16, head_dim, group, pl)) return 16;  // CUDA-core path: none needed
  // Upper bound over occupancies (at most pl.max_ctas CTAs per SM are used).
  const int hpu = heads_per_unit(num_kv_heads, pl.warps);
  const int64_t units = ctas_x(pl.max_ctas, num_kv_heads, hpu) * (pl.warps / hpu);
  return workspace_bytes(num_seqs, num_kv_heads, units, pl.record);
}

int b2p_decode_simt(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                    const void* key_cache, const void* value_cache, int64_t layer_index,
                    int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                    int64_t block_table_stride, const int32_t* context_lens, int num_seqs,
                    int num_q_heads, int num_kv_heads, int head_dim, int block_size, float scale,
                    void* out, int64_t out_tok_stride, int64_t out_head_stride, int dtype,
                    int32_t* err_flag, void* stream);

namespace {

// The newest row of each sequence in append mode (null `k`: plain decode).
struct AppendRows {
  const void* k = nullptr;
  int64_t k_tok = 0, k_head = 0;
  const void* v = nullptr;
  int64_t v_tok = 0, v_head = 0;
};

// CUDA-core path of append mode: puts each sequence's new row at the slot the block table
// gives for position ctx - 1 (the plain decode kernel then reads it like any other key).
template <int ES>
__global__ void append_rows_by_table(AppendRows rows, uint8_t* kpool, uint8_t* vpool,
                                     const int32_t* bt, int64_t bt_stride, const int32_t* ctx,
                                     int num_seqs, int64_t layer, int64_t num_slots,
                                     int block_size, int num_kv_heads, int head_dim,
                                     int32_t* err) {
  const int sq = blockIdx.x;
  if (sq >= num_seqs) return;
  const int c = ctx[sq];
  if (c <= 0) return;  // empty history: nothing to append to (decode flags it)
  const int64_t col = (c - 1) / block_size;
  const int32_t blk = col < bt_stride ? bt[(int64_t)sq * bt_stride + col] : -1;
  const int64_t slot = (int64_t)blk * block_size + (c - 1) % block_size;
  if (blk < 0 || slot >= num_slots) {
    if (threadIdx.x == 0) set_device_error(err, B2P_DEV_BLOCK_RANGE);
    return;
  }
  const int words = head_dim * ES / 4;  // 4-byte words per head row
  for (int e = threadIdx.x; e < 2 * num_kv_heads * words; e += blockDim.x) {
    const bool isv = e >= num_kv_heads * words;
    const int r = isv ? e - num_kv_heads * words : e;
    const int h = r / words, w = r - h * words;
    const uint8_t* src = static_cast<const uint8_t*>(isv ? rows.v : rows.k) +
                         ((int64_t)sq * (isv ? rows.v_tok : rows.k_tok) +
                          (int64_t)h * (isv ? rows.v_head : rows.k_head)) * ES;
    uint8_t* dst = (isv ? vpool : kpool) +
                   (((layer * num_slots + slot) * num_kv_heads + h) * head_dim) * ES;
    reinterpret_cast<uint32_t*>(dst)[w] = reinterpret_cast<const uint32_t*>(src)[w];
  }
}

// How a decode call runs: validated arguments, the kernel chosen, and for the tensor-core
// kernel the plan and the workspace bytes it needs. Shared by every decode entry point so
// that argument and size checks all happen before anything is queued on the stream.
struct DecodeRoute {
  bool empty = false;  // num_seqs == 0: nothing to launch
  bool tc = false;     // tensor-core kernel (else the CUDA-core kernel)
  Plan pl;
  int hpu = 1;
  int64_t ctas = 0;
  size_t need = 0;         // workspace bytes of the tensor-core kernel
  size_t counters_at = 0;  // byte offset of the counters (after the partial records)
};

int decode_route(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                 const void* key_cache, const void* value_cache, int64_t layer_index,
                 int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                 const int32_t* context_lens, int num_seqs, int num_q_heads, int num_kv_heads,
                 int head_dim, int block_size, const void* out, int dtype, DecodeRoute& rt,
                 size_t workspace_limit = SIZE_MAX) {
  if (num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_slots <= 0 || num_layers <= 0)
    return B2P_EINVAL;
  if (num_q_heads % num_kv_heads != 0) return B2P_EINVAL;
  if (layer_index < 0 || layer_index >= num_layers) return B2P_ERANGE;
  if (num_slots % block_size != 0) return B2P_EINVAL;
  if (dtype < B2P_BF16 || dtype > B2P_F32) return B2P_EINVAL;
  if (num_seqs == 0) {
    rt.empty = true;
    return B2P_OK;
  }
  if (!q || !key_cache || !value_cache || !block_tables || !context_lens || !out)
    return B2P_EINVAL;
  const int group = num_q_heads / num_kv_heads;
  rt.tc = (dtype == B2P_BF16 || dtype == B2P_F16) && block_size % 16 == 0 &&
          (q_tok_stride % 2 == 0) && (q_head_stride % 2 == 0) &&
          ((reinterpret_cast<uintptr_t>(q) & 3u) == 0) &&
          ((reinterpret_cast<uintptr_t>(key_cache) & 15u) == 0) &&
          ((reinterpret_cast<uintptr_t>(value_cache) & 15u) == 0) &&
          num_slots <= 0x7fffffffLL && select_plan(dtype, head_dim, group, rt.pl);
  if (!rt.tc) return B2P_OK;
  // The per-sequence counters alone bound the workspace from below (checked before any
  // device query, so an oversized problem is refused without touching the GPU).
  if (counters_bytes(num_seqs, num_kv_heads) > workspace_limit) return B2P_EWORKSPACE;
  const int rc = prepare(rt.pl);
  if (rc != B2P_OK) return rc;
  rt.hpu = heads_per_unit(num_kv_heads, rt.pl.warps);
  rt.ctas = ctas_x(rt.pl.ctas_per_sm, num_kv_heads, rt.hpu);
  const int64_t units = rt.ctas * (rt.pl.warps / rt.hpu);
  rt.need = workspace_bytes(num_seqs, num_kv_heads, units, rt.pl.record);
  rt.counters_at = partials_bytes(num_kv_heads, units, rt.pl.record);
  return B2P_OK;
}

int decode_impl(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                const void* key_cache, const void* value_cache, int64_t layer_index,
                int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
                int64_t block_table_stride, const int32_t* context_lens, int num_seqs,
                int num_q_heads, int num_kv_heads, int head_dim, int block_size, float scale,
                void* out, int64_t out_tok_stride, int64_t out_head_stride, void* workspace,
                size_t workspace_size, int dtype, int32_t* err_flag, void* stream,
                const AppendRows& app) {
  DecodeRoute rt;
  int rc = decode_route(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                        num_layers, num_slots, block_tables, context_lens, num_seqs,
                        num_q_heads, num_kv_heads, head_dim, block_size, out, dtype, rt);
  if (rc != B2P_OK || rt.empty) return rc;
  const int group = num_q_heads / num_kv_heads;
  const bool tc = rt.tc;
  // A bf16/f16 call that misses the tensor-core kernel's preconditions (block size, GQA
  // group, head_dim, alignment) runs on CUDA cores at a fraction of the speed: count it.
  if (!tc && dtype != B2P_F32) b2p_host::note_fallback(2);
  if (!tc) {
    if (app.k != nullptr) {
      const int es = dtype == B2P_F32 ? 4 : 2;
      if ((head_dim * es) % 4 != 0) return B2P_EINVAL;
      const cudaStream_t st = static_cast<cudaStream_t>(stream);
      uint8_t* kp = static_cast<uint8_t*>(const_cast<void*>(key_cache));
      uint8_t* vp = static_cast<uint8_t*>(const_cast<void*>(value_cache));
      if (es == 4)
        append_rows_by_table<4><<<num_seqs, 128, 0, st>>>(app, kp, vp, block_tables,
                                                          block_table_stride, context_lens,
                                                          num_seqs, layer_index, num_slots,
                                                          block_size, num_kv_heads, head_dim,
                                                          err_flag);
      else
        append_rows_by_table<2><<<num_seqs, 128, 0, st>>>(app, kp, vp, block_tables,
                                                          block_table_stride, context_lens,
                                                          num_seqs, layer_index, num_slots,
                                                          block_size, num_kv_heads, head_dim,
                                                          err_flag);
      const int rc = b2p_host::check_launch();
      if (rc != B2P_OK) return rc;
    }
    return b2p_decode_simt(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                           num_layers, num_slots, block_tables, block_table_stride, context_lens,
                           num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                           out_tok_stride, out_head_stride, dtype, err_flag, stream);
  }
  if (!workspace || workspace_size < rt.need) return B2P_EWORKSPACE;
  const Plan& pl = rt.pl;
  const int hpu = rt.hpu;
  const int64_t ctas = rt.ctas;

  CUtensorMap kmap, vmap;
  rc = b2p_host::pool_tensor_map_box(&kmap, key_cache, num_layers, num_slots, num_kv_heads,
                                     head_dim, 2, 1);
  if (rc != B2P_OK) return rc;
  rc = b2p_host::pool_tensor_map_box(&vmap, value_cache, num_layers, num_slots, num_kv_heads,
                                     head_dim, 2, 1);
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
  p.heads_per_unit = hpu;
  p.block_size = block_size;
  p.num_blocks = num_slots / block_size;
  p.scale_log2 = scale * kLog2e;
  p.partials = static_cast<float*>(workspace);
  p.counters = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + rt.counters_at);
  p.err = err_flag;
  p.new_k = static_cast<const uint8_t*>(app.k);
  p.nk_tok = app.k_tok;
  p.nk_head = app.k_head;
  p.new_v = static_cast<const uint8_t*>(app.v);
  p.nv_tok = app.v_tok;
  p.nv_head = app.v_head;
  p.kpool = static_cast<uint8_t*>(const_cast<void*>(key_cache));
  p.vpool = static_cast<uint8_t*>(const_cast<void*>(value_cache));
  p.num_kv_heads = num_kv_heads;

  void* args[] = {&kmap, &vmap, &p};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, (unsigned)(num_kv_heads / hpu));
  cfg.blockDim = dim3(pl.warps * 32);
  cfg.dynamicSmemBytes = (size_t)pl.smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelExC(&cfg, pl.fn, args);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  return b2p_host::check_launch();
}

}  // namespace

extern "C" int b2p_paged_decode(const void* q, int64_t q_tok_stride, int64_t q_head_stride,
                                const void* key_cache, const void* value_cache,
                                int64_t layer_index, int64_t num_layers, int64_t num_slots,
                                const int32_t* block_tables, int64_t block_table_stride,
                                const int32_t* context_lens, int num_seqs, int num_q_heads,
                                int num_kv_heads, int head_dim, int block_size, float scale,
                                void* out, int64_t out_tok_stride, int64_t out_head_stride,
                                void* workspace, size_t workspace_size, int dtype,
                                int32_t* err_flag, void* stream) {
  return decode_impl(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                     num_layers, num_slots, block_tables, block_table_stride, context_lens,
                     num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                     out_tok_stride, out_head_stride, workspace, workspace_size, dtype, err_flag,
                     stream, AppendRows{});
}

extern "C" int b2p_paged_decode_append(
    const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* new_keys,
    int64_t k_tok_stride, int64_t k_head_stride, const void* new_values, int64_t v_tok_stride,
    int64_t v_head_stride, void* key_cache, void* value_cache, int64_t layer_index,
    int64_t num_layers, int64_t num_slots, const int32_t* block_tables,
    int64_t block_table_stride, const int32_t* context_lens, int num_seqs, int num_q_heads,
    int num_kv_heads, int head_dim, int block_size, float scale, void* out,
    int64_t out_tok_stride, int64_t out_head_stride, void* workspace, size_t workspace_size,
    int dtype, int32_t* err_flag, void* stream) {
  if (num_seqs > 0 && (!new_keys || !new_values)) return B2P_EINVAL;
  // 16-byte rows: the tensor-core path moves each new row as 16-byte pieces.
  const int es = dtype == B2P_F32 ? 4 : 2;
  if (((reinterpret_cast<uintptr_t>(new_keys) | reinterpret_cast<uintptr_t>(new_values)) & 15u) ||
      (k_tok_stride * es) % 16 || (k_head_stride * es) % 16 || (v_tok_stride * es) % 16 ||
      (v_head_stride * es) % 16)
    return B2P_EINVAL;
  AppendRows app;
  app.k = new_keys;
  app.k_tok = k_tok_stride;
  app.k_head = k_head_stride;
  app.v = new_values;
  app.v_tok = v_tok_stride;
  app.v_head = v_head_stride;
  return decode_impl(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                     num_layers, num_slots, block_tables, block_table_stride, context_lens,
                     num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                     out_tok_stride, out_head_stride, workspace, workspace_size, dtype, err_flag,
                     stream, app);
}

// ====================================================================== scratch-free decode
// Some callers cannot hand this library device scratch. Examples: a runtime that
// reserves all device memory in its own arena at start-up and cannot carve out more,
// and a language binding (Go, Java, Node) that drives these kernels without any device
// allocator of its own. For them, the decode entry point below keeps the split-K
// counters and partial records in a fixed array compiled into the library.
namespace {

// 16 MiB holds the counters and partial records of, for example, 256 sequences of a
// 12/2-head, head_dim-128 layer (about 7.5 MiB on a 148-SM B200). Every GPU that loads
// the library keeps this array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

// Device address of g_decode_scratch on the current device (its host-side name is only
// a stand-in, not a device pointer). Looked up once per device.
int noalloc_scratch(void** ptr) {
  static void* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b2p_host::record_error(e);
  if (dev < 0 || dev >= 64) return B2P_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return b2p_host::record_error(e);
    addr[dev] = p;
  }
  *ptr = addr[dev];
  return B2P_OK;
}

}  // namespace

extern "C" int b2p_paged_decode_noalloc(const void* q, int64_t q_tok_stride,
                                        int64_t q_head_stride, const void* key_cache,
                                        const void* value_cache, int64_t layer_index,
                                        int64_t num_layers, int64_t num_slots,
                                        const int32_t* block_tables, int64_t block_table_stride,
                                        const int32_t* context_lens, int num_seqs,
                                        int num_q_heads, int num_kv_heads, int head_dim,
                                        int block_size, float scale, void* out,
                                        int64_t out_tok_stride, int64_t out_head_stride,
                                        int dtype, int32_t* err_flag, void* stream) {
  // Every argument and the workspace the chosen kernel needs are checked first, so a
  // rejected call queues nothing on the stream.
  DecodeRoute rt;
  int rc = decode_route(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                        num_layers, num_slots, block_tables, context_lens, num_seqs,
                        num_q_heads, num_kv_heads, head_dim, block_size, out, dtype, rt,
                        kNoAllocScratchBytes);
  if (rc != B2P_OK || rt.empty) return rc;
  void* scratch = nullptr;
  if (rt.tc) {  // the CUDA-core kernel uses no scratch
    if (rt.need > kNoAllocScratchBytes) return B2P_EWORKSPACE;
    rc = noalloc_scratch(&scratch);
    if (rc != B2P_OK) return rc;
    // The array keeps whatever the previous call left; the counters must start at zero.
    const cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + rt.counters_at, 0,
                                          counters_bytes(num_seqs, num_kv_heads),
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return b2p_host::record_error(e);
  }
  return b2p_paged_decode(q, q_tok_stride, q_head_stride, key_cache, value_cache, layer_index,
                          num_layers, num_slots, block_tables, block_table_stride, context_lens,
                          num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, scale, out,
                          out_tok_stride, out_head_stride, scratch,
                          rt.tc ? kNoAllocScratchBytes : 0, dtype, err_flag, stream);
}
