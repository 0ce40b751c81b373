// Paged single-token decode attention for B200 (sm_100a).
//
// One kernel covers the reference's three attention kernels
// (flashdec/kernels/paged_decode.py: per-head MHA :28-121, grouped GQA
// :124-327, split-KV :330-543) and the fused current-token append of its
// vLLM launcher (:728-919).  A standalone reducer covers :546-642.
//
// Work decomposition.  The unit of work is a 32-token tile of one
// (sequence, head block) pair; a head block is up to 16 query heads that share
// one KV head, so every K/V byte is read once per head block (once per KV head
// whenever the GQA group is <= 16).  Schedules:
//   * num_splits == 0 (auto), large batches: the tiles of the whole batch are
//     laid out in (sequence, head block, tile) order and cut into near-equal
//     ranges, one per persistent CTA; cuts that fall inside a short pair move
//     to its boundary when that costs little balance.  A CTA's range may
//     cover the tail of one pair, whole pairs and the head of another; every
//     piece is a "segment".  Ragged batches balance to within a tile per SM.
//   * num_splits == 0 (auto), small batches: every pair is split into S equal
//     ranges (3-D grid split x head block x sequence).  When all pairs fit as
//     co-resident thread-block clusters, the S CTAs of a pair form one
//     cluster and merge through distributed shared memory.
//   * num_splits == S: the reference's fixed split of every sequence into S
//     chunks of cdiv(tiles, S) tiles (paged_decode.py:395-411), one CTA each.
// A segment that covers a whole pair writes the output directly.  In a
// cluster, each CTA pushes its rows' (max, sum, acc) into the row owner's
// shared memory and the owner merges them.  Otherwise a segment writes an
// un-normalised partial to global memory and takes a ticket; the CTA that
// takes the last ticket of the pair merges all partials (no second launch, no
// CTA ever waits for another) and re-arms the ticket for the next call.
//
// Inside a CTA: warp 4 is the producer.  It resolves block-table entries
// (32 at a time, one per lane) and issues TMA boxes into a ring of
// shared-memory stages (128B swizzle; one "full" and one "empty" mbarrier per
// stage): one box per (page, 64-dim half), or for head_dim 128 with 16- or
// 8-token pages one box per page plane through a 5-D map.  Caches whose
// strides a tensor map cannot describe are copied by the producer warp with
// ordinary loads instead.  Warps 0-3 are consumers: each owns the stages
// s with s % 4 == warp and runs S = Q K^T and O += P V on the tensor cores
// (mma.sync m16n8k16, fp32 accumulate) with an online softmax in fp32
// (base-2 exponent, scale folded in).  At the end of a segment the four
// warps' (m, l, O) are merged through shared memory.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <mutex>
#include <utility>
#include <vector>

#include "fd_host.h"
#include "fd_ptx.cuh"
#include "fd_tile.cuh"
#include "fd_wave_decode.h"

namespace fd {

constexpr int kConsumerWarps = 4;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kMaxRows = 16;  // query heads per head block (mma M)
constexpr int kMaxStages = 16;
// fused-append RoPE: cos and sin of the current sequence's angles
// (rope_dim / 2 <= 64 each)
constexpr int kRopeFloats = 2 * 64;
// fused-append row of the current segment: slot (int64) + K and V [2][128]
// 16-bit values (the rotated K when RoPE is on)
constexpr int kAppendInts = 2 + 128;
constexpr int kMiscInts = 16;  // [0] abort, [1] ticket winner, [2] stream-K cut test,
                               // [8..9] cluster mbarrier
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kBarConsumers = 1;  // named barrier id for the consumer warps
constexpr int kMergeBatch = 10;   // partials merged per register batch
constexpr int kMaxClusterSize = 8;  // portable thread-block cluster size
constexpr int kSnapSlackTiles = 16; // stream-K: extra tiles tolerated for pair-aligned cuts

struct AttnParams {
  int num_seqs, num_q_heads, num_kv_heads, block_size, num_blocks, max_blocks;
  int group, hb_per_kv, rows, nhb;
  float scale_log2;  // sm_scale * log2(e)
  const void* q;
  int64_t qs0, qs1, qs2;
  void* out;
  int64_t os0, os1, os2;
  void* k;
  int64_t ks0, ks1, ks2, ks3;
  void* v;
  int64_t vs0, vs1, vs2, vs3;
  int kperm[4], vperm[4];  // tensor-map axis order (0 token, 1 head, 2 block, 3 half)
  const void* bt;
  int bt64;
  int64_t bts0, bts1;
  const void* sl;
  int sl64;
  int64_t sls;
  const void* ak;
  int64_t aks0, aks1, aks2;
  const void* av;
  int64_t avs0, avs1, avs2;
  const void* slot;
  int slot64;
  int64_t slots;
  int fused_append;
  // fused append with RoPE (rope_dim > 0): q rows and the appended K row are
  // rotated by rope_pos[b] with the fp32 table rope_inv_freq[rope_dim / 2]
  int rope_dim;
  const float* rope_inv_freq;
  const void* rope_pos;
  int rope_pos64;
  int64_t rope_pos_stride;
  // cascade tail pass: sequence b attends only to its tokens after its first
  // pre_pages[b] pages (a shared prefix handled by the prefix pass), and the
  // final merge of a member (pre_pages[b] > 0) also takes the prefix pass's
  // pre_slots partials in split slots [num_splits, num_splits + pre_slots)
  const int* pre_pages;
  int pre_slots;
  int num_splits;  // 0 = length-balanced (stream-K) schedule
  int epilogue;    // FD_EPILOGUE_*
  int balanced;    // split mode: equal tile ranges instead of cdiv chunks
  int cluster;     // split mode: the S CTAs of a pair form one thread-block
                   // cluster and merge through distributed shared memory
  int cap_tiles;   // tiles of a full block-table row (speculative prefetch)
  int min_tiles_per_cta;
  // split-mode partials [seq, q_head, split, dim] / [seq, q_head, split]
  float* pacc;
  int64_t pas0, pas1, pas2, pas3;
  float* pmax;
  float* psum;
  int64_t pss0, pss1, pss2;
  // stream-K partial slots: acc[(slot*rows + r)*D + d], m/l[slot*rows + r]
  float* slot_acc;
  float* slot_m;
  float* slot_l;
  int* tickets;
  int* status;
  int num_stages;
};

template <int D>
struct Smem {
  static constexpr int kHalves = D / 64;
  static constexpr int kHalfBytes = kTile * 128;  // [32 rows][64 dims] x 2 B
  static constexpr int kStageBytes = 2 * kHalves * kHalfBytes;
  static constexpr int kMergeFloats = kConsumerWarps * kMaxRows * D;
  static constexpr int kMergeBytes = kMergeFloats * 4 + kConsumerWarps * kMaxRows * 8;
};


struct SeqInfo {
  int n;      // tokens attended (0 => nothing to attend: zero output)
  int tiles;  // cdiv(n, 32)
  int off;    // pages skipped at the start of the block-table row (cascade tail)
};

// Reference semantics (paged_decode.py:263-264, :398-403): the sequence is
// active when seq_len > 0 and, with a fused append, slot >= 0.  seq_len is
// clamped to the block-table capacity so no read leaves the table row.
template <bool kAppend>
__device__ __forceinline__ SeqInfo seq_info(const AttnParams& p, int b) {
  int64_t n = load_index(p.sl, p.sl64, static_cast<int64_t>(b) * p.sls);
  const int64_t cap = static_cast<int64_t>(p.max_blocks) * p.block_size;
  n = n < 0 ? 0 : (n > cap ? cap : n);
  bool live = true;
  if constexpr (kAppend) {
    // the slot is read alongside the length (one memory round trip)
    const int64_t slot = load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots);
    if (slot < 0) {
      n = 0;
      live = false;  // reference MASK_INVALID_SLOT: a zero row, no prefix either
    }
  }
  SeqInfo r;
  r.off = 0;
  if (p.pre_pages && live) {
    // cascade tail: the first pre_pages[b] pages are attended by the prefix pass
    const int off = min(max(p.pre_pages[b], 0), p.max_blocks);
    const int64_t skip = static_cast<int64_t>(off) * p.block_size;
    n = n > skip ? n - skip : 0;
    r.off = off;
  }
  r.n = static_cast<int>(n);
  r.tiles = static_cast<int>((n + kTile - 1) / kTile);
  return r;
}

// A piece of work: tiles [t0, t1) of pair (b, hb).
struct Segment {
  int b, hb, t0, t1, n, tiles;
  int off;        // block-table pages before tile 0 (cascade tail pass)
  int extra;      // cascade member: prefix-pass partials merged after the nseg splits
  int whole;      // covers the whole pair: write the output directly
  int part_slot;  // stream-K slot id or split index
  int nseg;       // contributors to the pair's ticket
  int c_first;    // stream-K: first contributing CTA
};

// Largest b with nhb * prefix[b] <= x; empty sequences before a non-empty
// one share its start, and the search lands on the last of them, i.e. the
// non-empty one that actually contains x.
__device__ __forceinline__ int find_seq(const int* prefix, int num_seqs, int nhb, int64_t x) {
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (static_cast<int64_t>(nhb) * prefix[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct Sched {
  const int* prefix;  // smem, tiles prefix over sequences [num_seqs + 1]
  const int* seqn;    // smem, attended tokens per sequence [num_seqs]
  int num_seqs, nhb;
  int64_t U;          // total tiles of the batch
  int g;              // CTAs that own work (<= gridDim.x)
  int64_t x, hi;      // this CTA's cursor / end (stream-K)
  int done;           // split mode: the single segment was produced
  const int* cut;     // smem, start of every CTA's range [g + 1] (stream-K; U < 2^31)
  // Start of CTA c's tile range.  The ideal cut c * U / g is moved to the
  // nearer end of the (sequence, head block) pair it falls in whenever that
  // pair is no longer than a CTA's average share U / g: splitting a short
  // pair costs a partial write, a ticket and a merge, while snapping shifts
  // at most half a short pair between two neighbours.  Long pairs are cut
  // where the ideal boundary falls.  The cuts stay non-decreasing (two ideal
  // cuts are U / g apart, so they never share a short pair).
  __device__ __forceinline__ int64_t snapped_cut(int c) const {
    if (c <= 0) return 0;
    if (c >= g) return U;
    const int64_t xc = (static_cast<int64_t>(c) * U) / g;
    const int b = find_seq(prefix, num_seqs, nhb, xc);
    const int tiles = prefix[b + 1] - prefix[b];
    if (tiles <= 0 || static_cast<int64_t>(tiles) * g > U) return xc;
    const int64_t base = static_cast<int64_t>(nhb) * prefix[b];
    const int64_t ps = base + ((xc - base) / tiles) * tiles;
    const int64_t pe = ps + tiles;
    return (xc - ps <= pe - xc) ? ps : pe;
  }
  // CTA owning linear tile x: the largest c < g with cut[c] <= x.
  __device__ __forceinline__ int owner(int64_t x_) const {
    int lo_c = 0, hi_c = g - 1;
    while (lo_c < hi_c) {
      const int mid = (lo_c + hi_c + 1) >> 1;
      if (cut[mid] <= x_) lo_c = mid; else hi_c = mid - 1;
    }
    return lo_c;
  }
};

// Tiles of split `split` out of `tiles`: equal ranges when p.balanced
// (within one tile), else the reference's cdiv chunks (paged_decode.py:405-411).
__device__ __forceinline__ void split_range(const AttnParams& p, int split, int tiles, int& t0,
                                            int& t1) {
  const int S = p.num_splits;
  if (p.balanced) {
    // (split + 1) * tiles < 2^32 for any block table a device can hold
    t0 = static_cast<int>(static_cast<uint32_t>(split) * static_cast<uint32_t>(tiles) /
                          static_cast<uint32_t>(S));
    t1 = static_cast<int>(static_cast<uint32_t>(split + 1) * static_cast<uint32_t>(tiles) /
                          static_cast<uint32_t>(S));
  } else {
    const int bps = (tiles + S - 1) / S;
    t0 = min(split * bps, tiles);
    t1 = min(t0 + bps, tiles);
  }
}

template <bool kAppend>
__device__ __forceinline__ bool next_segment(const AttnParams& p, Sched& sc, Segment& s) {
  if (p.num_splits == 0) {
    if (sc.x >= sc.hi) return false;
    const int b = find_seq(sc.prefix, p.num_seqs, p.nhb, sc.x);
    const int tiles = sc.prefix[b + 1] - sc.prefix[b];
    const int64_t seq_base = static_cast<int64_t>(p.nhb) * sc.prefix[b];
    const int hb = static_cast<int>((sc.x - seq_base) / tiles);
    const int64_t pair_start = seq_base + static_cast<int64_t>(hb) * tiles;
    const int64_t pair_end = pair_start + tiles;
    const int64_t seg_end = pair_end < sc.hi ? pair_end : sc.hi;
    s.b = b;
    s.hb = hb;
    s.tiles = tiles;
    s.t0 = static_cast<int>(sc.x - pair_start);
    s.t1 = static_cast<int>(seg_end - pair_start);
    s.whole = (s.t0 == 0 && s.t1 == tiles);
    s.c_first = sc.owner(pair_start);
    s.nseg = sc.owner(pair_end - 1) - s.c_first + 1;
    s.part_slot = static_cast<int>(blockIdx.x) + b * p.nhb + hb;
    s.n = sc.seqn[b];
    s.off = 0;  // (the cascade tail pass runs the split schedule)
    s.extra = 0;
    sc.x = seg_end;
    return true;
  }
  if (sc.done) return false;
  sc.done = 1;
  // split schedule: grid = (splits, head blocks, sequences)
  const int S = p.num_splits;
  const int split = static_cast<int>(blockIdx.x);
  s.hb = static_cast<int>(blockIdx.y);
  s.b = static_cast<int>(blockIdx.z);
  const SeqInfo si = seq_info<kAppend>(p, s.b);
  s.n = si.n;
  s.off = si.off;
  s.extra = si.off > 0 ? p.pre_slots : 0;
  s.tiles = si.tiles;
  split_range(p, split, si.tiles, s.t0, s.t1);
  s.whole = (S == 1) && p.epilogue == FD_EPILOGUE_FUSED && s.extra == 0;
  s.part_slot = split;
  s.nseg = S;
  s.c_first = 0;
  return true;
}

// ---------------------------------------------------------------------------
// partial storage
// ---------------------------------------------------------------------------
template <int D>
struct PartRef {
  float* acc;  // points at element d = 0 of (slot, row)
  int64_t acc_step_d;
  float* m;
  float* l;
};

template <int D>
__device__ __forceinline__ PartRef<D> part_ref(const AttnParams& p, const Segment& s, int slot,
                                               int row, int qhead) {
  PartRef<D> r;
  if (p.num_splits == 0) {
    const int64_t i = static_cast<int64_t>(slot) * p.rows + row;
    r.acc = p.slot_acc + i * D;
    r.acc_step_d = 1;
    r.m = p.slot_m + i;
    r.l = p.slot_l + i;
  } else {
    r.acc = p.pacc + s.b * p.pas0 + qhead * p.pas1 + slot * p.pas2;
    r.acc_step_d = p.pas3;
    const int64_t o = s.b * p.pss0 + qhead * p.pss1 + slot * p.pss2;
    r.m = p.pmax + o;
    r.l = p.psum + o;
  }
  return r;
}

template <typename T>
__device__ __forceinline__ void store_out4(const AttnParams& p, int b, int h, int d, float a0,
                                           float a1, float a2, float a3) {
  T* o = static_cast<T*>(p.out) + b * p.os0 + h * p.os1 + d * p.os2;
  if (p.os2 == 1 && (reinterpret_cast<uintptr_t>(o) & 7u) == 0) {
    uint2 v;
    v.x = pack2<T>(a0, a1);
    v.y = pack2<T>(a2, a3);
    *reinterpret_cast<uint2*>(o) = v;
    return;
  }
  o[0] = from_f32<T>(a0);
  o[p.os2] = from_f32<T>(a1);
  o[2 * p.os2] = from_f32<T>(a2);
  o[3 * p.os2] = from_f32<T>(a3);
}


// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename T, int D, bool kTma, int kPageRows, bool kAppend>
__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_kernel(const __grid_constant__ AttnParams p,
                        const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v) {
  using SM = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int NST = p.num_stages;
  uint8_t* stages = smem;
  float* obuf = reinterpret_cast<float*>(stages + NST * SM::kStageBytes);
  float2* mlbuf = reinterpret_cast<float2*>(obuf + SM::kMergeFloats);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(mlbuf + kConsumerWarps * kMaxRows);
  uint64_t* empty_bar = full_bar + NST;
  uint32_t* stage_mask = reinterpret_cast<uint32_t*>(empty_bar + NST);
  // misc starts 16-byte aligned whatever the stage count: it holds the
  // cluster mbarrier and the fused-append slot (8-byte objects)
  int* misc = reinterpret_cast<int*>(
      (reinterpret_cast<uintptr_t>(stage_mask + NST) + 15) & ~static_cast<uintptr_t>(15));
  float* rope_tab = reinterpret_cast<float*>(misc + kMiscInts);  // [2][64]: cos, sin
  int64_t* app_slot = reinterpret_cast<int64_t*>(misc + kMiscInts + kRopeFloats);
  T* app_row = reinterpret_cast<T*>(app_slot + 1);  // [2][D]: K, V
  // the RoPE table and the append row exist only for a fused append (the
  // other calls keep that shared memory for the stage ring)
  int* prefix = misc + kMiscInts + (kAppend ? kRopeFloats + kAppendInts : 0);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  volatile int* abort_flag = misc;

  // cluster mode: arrivals of the S CTAs that push partials into this one
  uint64_t* merge_bar = reinterpret_cast<uint64_t*>(misc + 8);
  if (tid < NST) {  // one stage's barriers per thread
    mbar_init(smem_u32(&full_bar[tid]), 1);
    mbar_init(smem_u32(&empty_bar[tid]), 1);
    fence_mbar_init();
  }
  if (tid == 0) {
    misc[0] = 0;
    misc[1] = 0;
    if (p.cluster) {
      mbar_init(smem_u32(merge_bar), static_cast<uint32_t>(p.num_splits));
      fence_mbar_init();
    }
  }
  if (kTma && warp == kConsumerWarps && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  // Everything above touches no global memory and may overlap the previous
  // kernel of the stream; from here on its writes (KV cache, q, metadata,
  // the shared tickets) must be visible.
  pdl_wait();
  pdl_launch_dependents();

  // ---- schedule ----------------------------------------------------------
  Sched sc;
  sc.prefix = prefix;
  sc.num_seqs = p.num_seqs;
  sc.nhb = p.nhb;
  int* seqn = prefix + p.num_seqs + 1;
  sc.seqn = seqn;
  sc.U = 0;
  sc.g = 1;
  sc.x = sc.hi = 0;
  sc.done = 0;
  sc.cut = nullptr;
  const bool streamk = (p.num_splits == 0);
  if (streamk) {
    for (int b = tid; b < p.num_seqs; b += kThreads) {
      const SeqInfo si = seq_info<kAppend>(p, b);
      prefix[b + 1] = si.tiles;
      seqn[b] = si.n;
    }
    if (tid == 0) prefix[0] = 0;
  }
  __syncthreads();
  if (streamk) {
    if (warp == 0) {  // chunked inclusive scan of prefix[1..num_seqs]
      const int n = p.num_seqs;
      const int per = (n + 31) / 32;
      const int beg = 1 + lane * per;
      const int end = min(beg + per, n + 1);
      int run = 0;
      for (int i = beg; i < end; ++i) {
        run += prefix[i];
        prefix[i] = run;
      }
      int incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - run;
      for (int i = beg; i < end; ++i) prefix[i] += excl;
    }
    __syncthreads();
    sc.U = static_cast<int64_t>(p.nhb) * prefix[p.num_seqs];
    int64_t g = (sc.U + p.min_tiles_per_cta - 1) / p.min_tiles_per_cta;
    if (g > static_cast<int64_t>(gridDim.x)) g = gridDim.x;
    sc.g = static_cast<int>(g < 1 ? 1 : g);
    // Every CTA's range start, computed once, in parallel, into shared
    // memory.  Pair-aligned cuts are kept only if the busiest CTA gets at
    // most kSnapSlackTiles more than with the ideal cuts: a split pair costs
    // a partial write, a ticket and a merge (about a dozen tiles of ingest),
    // so a little imbalance is cheaper, a lot is not (ragged batches).
    int* cut = seqn + p.num_seqs;
    for (int c = tid; c <= sc.g; c += kThreads) cut[c] = static_cast<int>(sc.snapped_cut(c));
    if (tid == 0) misc[2] = 0;
    __syncthreads();
    int worst = 0;
    for (int c = tid; c < sc.g; c += kThreads) worst = max(worst, cut[c + 1] - cut[c]);
    if (worst > 0) atomicMax(&misc[2], worst);
    __syncthreads();
    const int64_t ideal_worst = (sc.U + sc.g - 1) / sc.g;
    if (static_cast<int64_t>(misc[2]) > ideal_worst + kSnapSlackTiles) {
      __syncthreads();  // every thread has read misc[2] before the table changes
      for (int c = tid; c <= sc.g; c += kThreads) {
        cut[c] = static_cast<int>((static_cast<int64_t>(c) * sc.U) / sc.g);
      }
    }
    sc.cut = cut;
    __syncthreads();
    if (sc.U > 0 && static_cast<int>(blockIdx.x) < sc.g) {
      sc.x = cut[blockIdx.x];
      sc.hi = cut[blockIdx.x + 1];
    }
  }

  const int bs = p.block_size;
  const int PPT = kTile / bs;  // pages per tile: 1, 2 or 4
  // Per-tile index math uses shifts and incrementally tracked (stage, phase)
  // pairs: runtime division is a long dependent instruction sequence.
  const int ppt_shift = bs == 32 ? 0 : (bs == 16 ? 1 : 2);
  const int bs_shift = 5 - ppt_shift;  // log2(block_size)

  // =========================================================================
  // producer warp.  Tiles are produced in groups of TG tiles (TG * PPT <= 32
  // pages, TG <= NST / 2 so a group only waits on stages freed by earlier
  // groups).  Lane j resolves the block id of page j of the group; lane i
  // (< group tiles) waits on its tile's "empty" barrier and posts the byte
  // count on the tile's "full" barrier; then all lanes issue the group's TMA
  // boxes together.  One warp instruction thus covers many tiles instead of
  // one lane walking tile by tile.
  // =========================================================================
  if (warp == kConsumerWarps) {
    // The producer touches no other CTA's memory; it arrives at the cluster
    // barrier (paired with the consumers' wait before their first remote
    // store) and may exit once its tiles are issued.
    if (p.cluster) cluster_arrive();
    const uint64_t policy = l2_policy_evict_first();
    const int TG = max(1, min(32 >> ppt_shift, NST / 2));
    constexpr int kOps = 2 * SM::kHalves;  // boxes per page: K and V halves
    // (stage, phase parity) of the next tile to produce; a group of
    // ntile <= NST / 2 tiles wraps the ring at most once.
    int pst = 0;
    uint32_t pph = 0;
    auto stage_of = [&](int i, uint32_t& ph) {
      int st = pst + i;
      ph = pph;
      if (st >= NST) {
        st -= NST;
        ph ^= 1u;
      }
      return st;
    };
    bool bad = false;
    // Block-table window: lane l holds the entry of page wb + l (win) and of
    // page wb + 32 + l (win_next, prefetched); win_b is the sequence.
    int64_t wb = -1;
    int win_b = -1, win = -1, win_next = -1;
    int seg_off = 0;  // the current segment's leading pages (cascade tail)
    auto bt_entry = [&](int b, int64_t lb) -> int {
      lb += seg_off;
      return lb < p.max_blocks
                 ? static_cast<int>(load_index(p.bt, p.bt64,
                                               static_cast<int64_t>(b) * p.bts0 + lb * p.bts1))
                 : -1;
    };
    if (!streamk && !p.pre_pages) {
      // Split schedule: this CTA's pair and (for a full-length sequence) its
      // pages are known from blockIdx alone, so the first window is fetched
      // speculatively, in parallel with the sequence-length load.
      int st0, st1;
      split_range(p, static_cast<int>(blockIdx.x), p.cap_tiles, st0, st1);
      win_b = static_cast<int>(blockIdx.z);
      wb = static_cast<int64_t>(st0) << ppt_shift;
      win = bt_entry(win_b, wb + lane);
      win_next = bt_entry(win_b, wb + 32 + lane);
    }
    Segment s;
    while (next_segment<kAppend>(p, sc, s)) {
      if (s.t1 <= s.t0) continue;
      seg_off = s.off;  // fixed per sequence, so a window of this sequence stays valid
      const int kv_head = s.hb / p.hb_per_kv;
      const int limit_cache = kAppend ? s.n - 1 : s.n;  // tokens read from the cache
      const int64_t nlb = (limit_cache + bs - 1) >> bs_shift;  // pages holding them
      for (int tg = s.t0; tg < s.t1;) {
        const int64_t pg0 = static_cast<int64_t>(tg) << ppt_shift;
        if (win_b != s.b || pg0 < wb || pg0 >= wb + 64) {
          wb = pg0;  // (re)load the window at this group
          win_b = s.b;
          win = bt_entry(s.b, wb + lane);
          win_next = bt_entry(s.b, wb + 32 + lane);
        } else if (pg0 >= wb + 32) {
          wb += 32;  // slide by one window; prefetch the following one
          win = win_next;
          win_next = bt_entry(s.b, wb + 32 + lane);
        }
        // a group never crosses the window end
        const int room = static_cast<int>((wb + 32 - pg0) >> ppt_shift);
        const int ntile = min(min(TG, s.t1 - tg), room);
        const int npage = ntile << ppt_shift;
        const int64_t lb = pg0 + lane;
        const bool has_tokens = lane < npage && lb < nlb;
        int blk = __shfl_sync(0xffffffffu, win, static_cast<int>(pg0 - wb + lane) & 31);
        if (!has_tokens) blk = -1;
        const bool pvalid = has_tokens && blk >= 0 && blk < p.num_blocks;
        bad = bad || (has_tokens && !pvalid);
        const uint32_t pages = __ballot_sync(0xffffffffu, pvalid);
        bool ok = true;
        if (lane < ntile) {
          uint32_t ph;
          const int stage = stage_of(lane, ph);
          ok = mbar_wait(smem_u32(&empty_bar[stage]), ph ^ 1u, p.status, abort_flag);
          const uint32_t tmask = (pages >> (lane << ppt_shift)) & ((1u << PPT) - 1u);
          stage_mask[stage] = tmask;
          if (kTma && ok) {
            mbar_arrive_expect_tx(smem_u32(&full_bar[stage]),
                                  static_cast<uint32_t>(__popc(tmask)) * (bs * D * 2 * 2));
          }
        }
        if (__all_sync(0xffffffffu, ok)) {
          if constexpr (kTma && kPageRows > 0) {
            // one box per (page, plane): kPageRows tokens x both 64-dim halves
            const int nops = npage * 2;
            for (int base = 0; base < nops; base += 32) {
              const int op = base + lane;
              const int page = op >> 1;
              const int pblk = __shfl_sync(0xffffffffu, blk, page & 31);
              if (op < nops && ((pages >> page) & 1u)) {
                const int plane = op & 1;  // 0: K, 1: V
                uint32_t ph;
                const int stage = stage_of(page >> ppt_shift, ph);
                const uint32_t dst = smem_u32(stages + stage * SM::kStageBytes) +
                                     plane * (SM::kHalves * SM::kHalfBytes) +
                                     (page & (PPT - 1)) * (kPageRows * 256);
                const int* perm = plane ? p.vperm : p.kperm;
                tma_load_5d(dst, plane ? &tmap_v : &tmap_k, smem_u32(&full_bar[stage]), 0,
                            tmap_coord(perm[0], kv_head, pblk), tmap_coord(perm[1], kv_head, pblk),
                            tmap_coord(perm[2], kv_head, pblk), tmap_coord(perm[3], kv_head, pblk),
                            policy);
              }
            }
          } else if constexpr (kTma) {
            const int nops = npage * kOps;
            for (int base = 0; base < nops; base += 32) {
              const int op = base + lane;
              const int page = op / kOps;  // kOps is a compile-time power of two
              const int pblk = __shfl_sync(0xffffffffu, blk, page & 31);
              if (op < nops && ((pages >> page) & 1u)) {
                const int rem = op - page * kOps;
                const int plane = rem / SM::kHalves;  // 0: K, 1: V
                const int h = rem - plane * SM::kHalves;
                const int ti = page >> ppt_shift;
                const int j = page & (PPT - 1);
                uint32_t ph;
                const int stage = stage_of(ti, ph);
                const uint32_t dst = smem_u32(stages + stage * SM::kStageBytes) +
                                     plane * (SM::kHalves * SM::kHalfBytes) + h * SM::kHalfBytes +
                                     ((j * bs) << 7);
                const int* perm = plane ? p.vperm : p.kperm;
                tma_load_4d(dst, plane ? &tmap_v : &tmap_k, smem_u32(&full_bar[stage]), h * 64,
                            tmap_coord(perm[0], kv_head, pblk), tmap_coord(perm[1], kv_head, pblk),
                            tmap_coord(perm[2], kv_head, pblk), policy);
              }
            }
          } else {
            // generic strides: the producer warp copies the valid pages itself
            for (int page = 0; page < npage; ++page) {
              const int pblk = __shfl_sync(0xffffffffu, blk, page);
              if (!((pages >> page) & 1u)) continue;
              const int ti = page >> ppt_shift;
              const int j = page & (PPT - 1);
              uint32_t ph;
              uint8_t* sb = stages + stage_of(ti, ph) * SM::kStageBytes;
              const uint16_t* kp =
                  static_cast<const uint16_t*>(p.k) + pblk * p.ks0 + kv_head * p.ks1;
              const uint16_t* vp =
                  static_cast<const uint16_t*>(p.v) + pblk * p.vs0 + kv_head * p.vs1;
              for (int e = lane; e < bs * D; e += 32) {
                const int r = e / D;
                const int d = e - r * D;
                const uint32_t off = stage_tile_offset<kPageRows>(j * bs + r, d);
                *reinterpret_cast<uint16_t*>(sb + off) = kp[r * p.ks2 + d * p.ks3];
                *reinterpret_cast<uint16_t*>(sb + SM::kHalves * SM::kHalfBytes + off) =
                    vp[r * p.vs2 + d * p.vs3];
              }
            }
            __syncwarp();
            if (lane < ntile) {
              uint32_t ph;
              mbar_arrive(smem_u32(&full_bar[stage_of(lane, ph)]));
            }
          }
        }
        // (aborted groups are skipped; the consumers' waits then time out too)
        pst += ntile;
        if (pst >= NST) {
          pst -= NST;
          pph ^= 1u;
        }
        tg += ntile;
      }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
    return;
  }

  // =========================================================================
  // consumer warps
  // =========================================================================
  const int g8 = lane >> 2;  // mma group (row) index
  const int t4 = lane & 3;   // thread in group
  const int mi = lane >> 3;  // ldmatrix matrix index
  const int r8 = lane & 7;   // ldmatrix row
  // Per-lane ldmatrix offsets, the same for every tile (StageStrides): K
  // rows (mi >> 1) * 8 + r8 with chunk 2 j + (mi & 1) of a half, V rows
  // (mi & 1) * 8 + r8 with chunk 2 j + (mi >> 1).
  using SS = StageStrides<kPageRows>;
  const uint32_t k_lane = stage_row_base<kPageRows>((mi >> 1) * 8 + r8, 0);
  const uint32_t v_lane = stage_row_base<kPageRows>((mi & 1) * 8 + r8, 0);
  uint32_t k_sw[4], v_sw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    k_sw[j] = k_lane + ((((2 * j) + (mi & 1)) ^ r8) << 4);
    v_sw[j] = v_lane + ((((2 * j) + (mi >> 1)) ^ r8) << 4);
  }
  int cst = 0;        // (stage, phase parity) of the next tile
  uint32_t cph = 0;
  // ---- Q fragments (A operand, rows = query heads of the head block) ----
  uint32_t qf[D / 16][4];
  int q_b = -1, q_hb = -1;
  // Q of the head block is staged into shared memory (the merge buffer, idle
  // at a segment start) with 16-byte loads, in the swizzled tile layout, and
  // read back as mma A fragments with ldmatrix.  Called by all consumer
  // warps together.
  auto load_q = [&](int b, int hb) {
    const int kvh = hb / p.hb_per_kv;
    const int jb = hb % p.hb_per_kv;
    const int h0 = kvh * p.group + jb * p.rows;
    const int nr = min(p.rows, p.group - jb * p.rows);
    const T* qb = static_cast<const T*>(p.q) + b * p.qs0;
    uint8_t* qs = reinterpret_cast<uint8_t*>(obuf);
    // RoPE position of this sequence (its load is in flight with q's)
    const bool rope_pair = kAppend && tid < (p.rope_dim >> 1);
    const float posf =
        rope_pair ? static_cast<float>(load_index(p.rope_pos, p.rope_pos64,
                                                  static_cast<int64_t>(b) * p.rope_pos_stride))
                  : 0.f;
    const float invf = rope_pair ? p.rope_inv_freq[tid] : 0.f;
    // Fused append: this sequence's new K/V row and its slot are staged with
    // q (same memory round trip), so the tile that receives the row reads
    // shared memory only.  2 * D / 128 values per thread (1 or 2).
    constexpr int kAppPer = (2 * D) / kConsumerThreads;
    T app_v[kAppPer];
    if (kAppend) {
#pragma unroll
      for (int j = 0; j < kAppPer; ++j) {
        const int e = tid + j * kConsumerThreads;
        const int plane = e / D;
        const int d = e - plane * D;
        app_v[j] = plane ? static_cast<const T*>(p.av)[b * p.avs0 + kvh * p.avs1 + d * p.avs2]
                         : static_cast<const T*>(p.ak)[b * p.aks0 + kvh * p.aks1 + d * p.aks2];
      }
      if (tid == 0) *app_slot = load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots);
    }
    for (int c = tid; c < kMaxRows * (D / 8); c += kConsumerThreads) {
      const int row = c / (D / 8);
      const int ch = c - row * (D / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < nr) {
        const T* src = qb + (h0 + row) * p.qs1 + ch * 8 * p.qs2;
        if (p.qs2 == 1 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
          v = *reinterpret_cast<const uint4*>(src);
        } else {
          __align__(16) T e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) e[i] = src[i * p.qs2];
          v = *reinterpret_cast<const uint4*>(e);
        }
      }
      *reinterpret_cast<uint4*>(qs + chunk_offset(row, ch)) = v;
    }
    if (kAppend) {
#pragma unroll
      for (int j = 0; j < kAppPer; ++j) app_row[tid + j * kConsumerThreads] = app_v[j];
    }
    if (rope_pair) {
      // cos / sin of this sequence's angles, once per pair index (the same
      // for every q row and the K row)
      float sn, cs;
      sincosf(__fmul_rn(posf, invf), &sn, &cs);
      rope_tab[tid] = cs;
      rope_tab[64 + tid] = sn;
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    if (kAppend && p.rope_dim > 0) {
      // RoPE in place of the staged q rows and (row nr) the appended K row:
      // pair (i, i + rope_dim / 2)
      const int half = p.rope_dim >> 1;
      for (int e = tid; e < (nr + 1) * half; e += kConsumerThreads) {
        const int row = e / half;
        const int i = e - row * half;
        T* x1p = row < nr ? reinterpret_cast<T*>(qs + tile_offset(row, i)) : app_row + i;
        T* x2p = row < nr ? reinterpret_cast<T*>(qs + tile_offset(row, i + half))
                          : app_row + i + half;
        float y1, y2;
        rope_rotate_pair_cs(to_f32<T>(*x1p), to_f32<T>(*x2p), rope_tab[i], rope_tab[64 + i], y1,
                            y2);
        *x1p = from_f32<T>(y1);
        *x2p = from_f32<T>(y2);
      }
      named_barrier(kBarConsumers, kConsumerThreads);
    }
    const uint32_t qbase = smem_u32(qs);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      ldsm_x4(qbase + chunk_offset(r8 + (mi & 1) * 8, ks * 2 + (mi >> 1)), qf[ks][0], qf[ks][1],
              qf[ks][2], qf[ks][3]);
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    q_b = b;
    q_hb = hb;
  };
  if (!streamk) {
    // split schedule: the pair is known from blockIdx; load Q before the
    // sequence length arrives
    load_q(static_cast<int>(blockIdx.z), static_cast<int>(blockIdx.y));
    // Cluster mode: obuf (which just held Q) becomes the receive buffer for
    // the peers' partials.  This arrival, made after Q left obuf and after
    // merge_bar was initialised, is what a peer waits for before its first
    // store into this CTA.  The wait follows at once: the peers reach this
    // point at about the same time, and the consumers would otherwise only
    // wait for their first tile here.
    if (p.cluster) {
      cluster_arrive();
      cluster_wait();
    }
  }

  Segment s;
  while (next_segment<kAppend>(p, sc, s)) {
    const int kv_head = s.hb / p.hb_per_kv;
    const int jblk = s.hb % p.hb_per_kv;
    const int head0 = kv_head * p.group + jblk * p.rows;
    const int nrows = min(p.rows, p.group - jblk * p.rows);
    if (s.b != q_b || s.hb != q_hb) load_q(s.b, s.hb);

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    const int limit_cache = kAppend ? s.n - 1 : s.n;
    for (int t = s.t0; t < s.t1; ++t) {
      const int stage = cst;
      const uint32_t phase = cph;
      // each stage is always consumed by the same warp (stage % 4), so a warp
      // waits on its stages' phases in order whatever the stage count
      const bool mine = (stage & (kConsumerWarps - 1)) == warp;
      if (++cst == NST) {
        cst = 0;
        cph ^= 1u;
      }
      if (!mine) continue;
      if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, abort_flag)) continue;
      uint8_t* sb = stages + stage * SM::kStageBytes;
      const uint32_t kbase = smem_u32(sb);
      const uint32_t vbase = kbase + SM::kHalves * SM::kHalfBytes;
      const uint32_t pmask = stage_mask[stage];
      const int base = t * kTile;

      // valid rows of this tile
      const int pos = base + lane;
      const bool from_cache = pos < limit_cache && ((pmask >> (lane >> bs_shift)) & 1u);
      const bool appended = kAppend && pos == s.n - 1;
      const uint32_t vmask = __ballot_sync(0xffffffffu, from_cache || appended);
      bool touched = false;
      if (vmask != 0xffffffffu) {
        // rows without data: zero V so that P (= 0 there) times V stays 0
        // even if the stale bytes are NaN/Inf.
        const uint32_t inv = ~vmask;
        for (int e = lane; e < kTile * (D / 8); e += 32) {
          const int r = e / (D / 8);
          const int c = e - r * (D / 8);
          if ((inv >> r) & 1u) {
            *reinterpret_cast<uint4*>(sb + SM::kHalves * SM::kHalfBytes +
                                      stage_chunk_offset<kPageRows>(r, c)) =
                make_uint4(0u, 0u, 0u, 0u);
          }
        }
        touched = true;
      }
      if (kAppend && (s.n - 1) >= base && (s.n - 1) < base + kTile) {
        // current token: K/V come from the call (staged with q, K rotated
        // when RoPE is on); patch the tile and store the token into its cache
        // slot (reference paged_decode.py:193-221).
        const int ra = s.n - 1 - base;
        const int64_t slot = *app_slot;
        const int64_t sblk = slot >> bs_shift;
        const int64_t soff = slot - sblk * bs;
        const bool store = (jblk == 0) && sblk < p.num_blocks;
        T* kc = static_cast<T*>(p.k) + sblk * p.ks0 + kv_head * p.ks1 + soff * p.ks2;
        T* vc = static_cast<T*>(p.v) + sblk * p.vs0 + kv_head * p.vs1 + soff * p.vs2;
        for (int d = lane; d < D; d += 32) {
          const T kv = app_row[d];
          const T vv = app_row[D + d];
          *reinterpret_cast<T*>(sb + stage_tile_offset<kPageRows>(ra, d)) = kv;
          *reinterpret_cast<T*>(sb + SM::kHalves * SM::kHalfBytes +
                                stage_tile_offset<kPageRows>(ra, d)) = vv;
          if (store) {
            kc[d * p.ks3] = kv;
            vc[d * p.vs3] = vv;
          }
        }
        if (!store && jblk == 0 && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
        touched = true;
      }
      if (touched) __syncwarp();

      // ---- S = Q K^T  (16 heads x 32 tokens) ----
      float sacc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b0a, b1a, b0b, b1b;
          ldsm_x4(kbase + k_sw[ks & 3] + np * SS::kRows16Bytes + (ks >> 2) * SS::kHalfStride, b0a,
                  b1a, b0b, b1b);
          mma_16816<T>(sacc[2 * np], qf[ks], b0a, b1a);
          mma_16816<T>(sacc[2 * np + 1], qf[ks], b0b, b1b);
        }
      }

      // ---- online softmax (base 2, scale folded in) ----
      float mx0 = -INFINITY, mx1 = -INFINITY;
      if (vmask == 0xffffffffu) {  // a full tile: no masking
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int e = 0; e < 4; ++e) sacc[j][e] *= p.scale_log2;
          mx0 = fmaxf(mx0, fmaxf(sacc[j][0], sacc[j][1]));
          mx1 = fmaxf(mx1, fmaxf(sacc[j][2], sacc[j][3]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tok = 8 * j + 2 * t4 + e;
            const bool valid = (vmask >> tok) & 1u;
            const float x0 = valid ? sacc[j][e] * p.scale_log2 : -INFINITY;
            const float x1 = valid ? sacc[j][2 + e] * p.scale_log2 : -INFINITY;
            sacc[j][e] = x0;
            sacc[j][2 + e] = x1;
            mx0 = fmaxf(mx0, x0);
            mx1 = fmaxf(mx1, x1);
          }
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0);
      const float mn1 = fmaxf(m1, mx1);
      const float ref0 = (mn0 == -INFINITY) ? 0.f : mn0;
      const float ref1 = (mn1 == -INFINITY) ? 0.f : mn1;
      const float alpha0 = exp2f(m0 - ref0);
      const float alpha1 = exp2f(m1 - ref1);
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sacc[j][0] = exp2f(sacc[j][0] - ref0);
        sacc[j][1] = exp2f(sacc[j][1] - ref0);
        sacc[j][2] = exp2f(sacc[j][2] - ref1);
        sacc[j][3] = exp2f(sacc[j][3] - ref1);
        ps0 += sacc[j][0] + sacc[j][1];
        ps1 += sacc[j][2] + sacc[j][3];
      }
      l0 = l0 * alpha0 + ps0;
      l1 = l1 * alpha1 + ps1;
      m0 = mn0;
      m1 = mn1;
      // Once the running maxima settle (alpha == 1: exactly the old max) the
      // rescale multiplies by 1.0; skipping it changes no bit.
      if (!__all_sync(0xffffffffu, alpha0 == 1.f && alpha1 == 1.f)) {
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
          o[j][0] *= alpha0;
          o[j][1] *= alpha0;
          o[j][2] *= alpha1;
          o[j][3] *= alpha1;
        }
      }

      // ---- O += P V ----
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t a[4];
        a[0] = pack2<T>(sacc[2 * kk][0], sacc[2 * kk][1]);
        a[1] = pack2<T>(sacc[2 * kk][2], sacc[2 * kk][3]);
        a[2] = pack2<T>(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
        a[3] = pack2<T>(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t b0a, b1a, b0b, b1b;
          ldsm_x4_t(vbase + v_sw[dp & 3] + kk * SS::kRows16Bytes + (dp >> 2) * SS::kHalfStride,
                    b0a, b1a, b0b, b1b);
          mma_16816<T>(o[2 * dp], a, b0a, b1a);
          mma_16816<T>(o[2 * dp + 1], a, b0b, b1b);
        }
      }
      __syncwarp();
      if (touched) fence_proxy_async_smem();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[stage]));
    }

    // ---- merge the four warps' states of this segment ----
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    // Cluster mode keeps obuf free for the peers' partials and merges in the
    // stage ring instead, which is idle once every warp has consumed its
    // last tile (one segment per CTA; the producer has nothing left to load).
    float* wbuf = obuf;
    if (p.cluster) {
      named_barrier(kBarConsumers, kConsumerThreads);
      wbuf = reinterpret_cast<float*>(stages);
    }
    if (t4 == 0) {
      mlbuf[warp * kMaxRows + g8] = make_float2(m0, l0);
      mlbuf[warp * kMaxRows + g8 + 8] = make_float2(m1, l1);
    }
    // Rows of the merge buffer are 128-float aligned, so the eight rows one
    // store instruction touches would share banks; the column is XORed with
    // 8 * (row % 4) (merge_col), which keeps float2/float4 groups contiguous
    // and spreads a store over all 32 banks.
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int d = 8 * j + 2 * t4;
      const int r0 = warp * kMaxRows + g8;
      *reinterpret_cast<float2*>(&wbuf[r0 * D + merge_col(r0, d)]) =
          make_float2(o[j][0], o[j][1]);
      *reinterpret_cast<float2*>(&wbuf[(r0 + 8) * D + merge_col(r0 + 8, d)]) =
          make_float2(o[j][2], o[j][3]);
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    const int pid = s.b * p.nhb + s.hb;
    // Cluster mode: row r of the pair is finished by CTA (r % S) of the
    // cluster, which receives every CTA's (max, sum, acc) of that row in its
    // obuf: acc at [(src * RI + r / S) * D + d], (max, sum) at
    // mlr[src * RI + r / S].  Wait until every CTA of the cluster has made
    // its obuf available (the arrival after Q staging).
    const int csz = p.num_splits;
    const int crank = p.cluster ? static_cast<int>(cluster_ctarank()) : 0;
    const int cri = (nrows + csz - 1) / csz;  // rows finished per CTA (at most)
    float2* mlr = reinterpret_cast<float2*>(obuf + csz * cri * D);
    for (int e = tid; e < nrows * (D / 4); e += kConsumerThreads) {
      const int r = e / (D / 4);
      const int d = (e - r * (D / 4)) * 4;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mlbuf[w * kMaxRows + r].x);
      float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float2 ml = mlbuf[w * kMaxRows + r];
          const float wgt = exp2f(ml.x - M);
          const int wr = w * kMaxRows + r;
          const float4 ov = *reinterpret_cast<const float4*>(&wbuf[wr * D + merge_col(wr, d)]);
          L += wgt * ml.y;
          a0 += wgt * ov.x;
          a1 += wgt * ov.y;
          a2 += wgt * ov.z;
          a3 += wgt * ov.w;
        }
      }
      if (p.cluster) {
        // push this CTA's partial of row r to the row's owner (base-2 max)
        const int owner = r % csz;
        const int slot = crank * cri + r / csz;
        st_cluster_v4(map_to_rank(smem_u32(&obuf[slot * D + d]), owner), a0, a1, a2, a3);
        if (d == 0) st_cluster_v2(map_to_rank(smem_u32(&mlr[slot]), owner), M, L);
      } else if (s.whole) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        store_out4<T>(p, s.b, head0 + r, d, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
      } else {
        PartRef<D> pr = part_ref<D>(p, s, s.part_slot, r, head0 + r);
        float* ap = pr.acc + d * pr.acc_step_d;
        if (pr.acc_step_d == 1 && (reinterpret_cast<uintptr_t>(ap) & 15u) == 0) {
          *reinterpret_cast<float4*>(ap) = make_float4(a0, a1, a2, a3);
        } else {
          ap[0] = a0;
          ap[pr.acc_step_d] = a1;
          ap[2 * pr.acc_step_d] = a2;
          ap[3 * pr.acc_step_d] = a3;
        }
        if (d == 0) {
          *pr.m = (M == -INFINITY) ? -INFINITY : M * kLn2;  // natural-log units
          *pr.l = L;
        }
      }
    }
    if (p.cluster) {
      // The named barrier orders every consumer thread's pushes before the
      // release arrivals on the owners' merge barriers (one lane per owner);
      // each owner waits for all S arrivals, which also tells it that no CTA
      // will touch its shared memory again.
      named_barrier(kBarConsumers, kConsumerThreads);
      if (tid < csz) mbar_arrive_remote(map_to_rank(smem_u32(merge_bar), tid));
      if (mbar_wait_cluster(smem_u32(merge_bar), 0u, p.status, abort_flag)) {
        for (int e = tid; e < cri * (D / 4); e += kConsumerThreads) {
          const int ri = e / (D / 4);
          const int r = crank + ri * csz;
          if (r >= nrows) continue;
          const int d = (e - ri * (D / 4)) * 4;
          // all loads first (independent), then the merge
          float2 ml[kMaxClusterSize];
          float4 ov[kMaxClusterSize];
#pragma unroll
          for (int src = 0; src < kMaxClusterSize; ++src) {
            ml[src] = make_float2(-INFINITY, 0.f);
            ov[src] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (src < csz) {
              ml[src] = mlr[src * cri + ri];
              ov[src] = *reinterpret_cast<const float4*>(&obuf[(src * cri + ri) * D + d]);
            }
          }
          float M = -INFINITY;
#pragma unroll
          for (int src = 0; src < kMaxClusterSize; ++src) M = fmaxf(M, ml[src].x);
          float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
          if (M != -INFINITY) {
#pragma unroll
            for (int src = 0; src < kMaxClusterSize; ++src) {
              const float wgt = exp2f(ml[src].x - M);  // 0 for an empty or absent split
              L += wgt * ml[src].y;
              a0 += wgt * ov[src].x;
              a1 += wgt * ov[src].y;
              a2 += wgt * ov[src].z;
              a3 += wgt * ov[src].w;
            }
          }
          const float inv = L > 0.f ? 1.f / L : 0.f;
          store_out4<T>(p, s.b, head0 + r, d, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
        }
      }
    } else if (!s.whole && p.epilogue == FD_EPILOGUE_FUSED) {
      // The barrier orders every consumer thread's partial stores before
      // thread 0's acq_rel ticket, which publishes them at GPU scope
      // (release) and, for the last arriver, makes the other CTAs' partials
      // visible (acquire); the second barrier extends that to all threads.
      named_barrier(kBarConsumers, kConsumerThreads);
      if (tid == 0) {
        const int prev = atom_add_acq_rel_gpu(&p.tickets[pid], 1);
        const int last = (prev == s.nseg - 1);
        // Re-arm for the next call: every contributor has arrived, nothing
        // else touches this ticket before the kernel ends.
        if (last) p.tickets[pid] = 0;
        misc[1] = last;
      }
      named_barrier(kBarConsumers, kConsumerThreads);
      if (misc[1]) {
        // Final merge of the pair's nseg partials (reference reducer
        // semantics, paged_decode.py:593-635).  One warp per output row, one
        // lane per 4 dims (D/4 lanes); the (max, sum, acc) of up to
        // kMergeBatch partials are loaded into registers by a fully unrolled,
        // predicated loop -- all independent, so one memory round trip --
        // and merged afterwards.
        constexpr int kLanesPerRow = D / 4;
        constexpr int kRowsPerWarp = 32 / kLanesPerRow;  // 1 (D=128) or 2 (D=64)
        constexpr int kSlots = kConsumerWarps * kRowsPerWarp;
        constexpr int kRowPass = 2;  // rows a lane merges together (loads overlap)
        const int sub = lane / kLanesPerRow;
        const int d = (lane - sub * kLanesPerRow) * 4;
        for (int r0 = warp * kRowsPerWarp + sub; r0 < nrows; r0 += kSlots * kRowPass) {
          float M[kRowPass], L[kRowPass], A[kRowPass][4];
#pragma unroll
          for (int q = 0; q < kRowPass; ++q) {
            M[q] = -INFINITY;
            L[q] = 0.f;
            A[q][0] = A[q][1] = A[q][2] = A[q][3] = 0.f;
          }
          const int nmerge = s.nseg + s.extra;  // + the prefix pass's chunks
          for (int i0 = 0; i0 < nmerge; i0 += kMergeBatch) {
            float mv[kRowPass][kMergeBatch], lv[kRowPass][kMergeBatch];
            float4 av[kRowPass][kMergeBatch];
#pragma unroll
            for (int q = 0; q < kRowPass; ++q) {
              const int r = r0 + q * kSlots;
#pragma unroll
              for (int j = 0; j < kMergeBatch; ++j) {
                mv[q][j] = -INFINITY;
                lv[q][j] = 0.f;
                av[q][j] = make_float4(0.f, 0.f, 0.f, 0.f);
                const int i = i0 + j;
                if (r < nrows && i < nmerge) {
                  const int sl = (p.num_splits == 0) ? (s.c_first + i + pid) : i;
                  const PartRef<D> pr = part_ref<D>(p, s, sl, r, head0 + r);
                  mv[q][j] = __ldcg(pr.m);
                  lv[q][j] = __ldcg(pr.l);
                  const float* ap = pr.acc + d * pr.acc_step_d;
                  if (pr.acc_step_d == 1 && (reinterpret_cast<uintptr_t>(ap) & 15u) == 0) {
                    av[q][j] = __ldcg(reinterpret_cast<const float4*>(ap));
                  } else {
                    av[q][j] = make_float4(__ldcg(ap), __ldcg(ap + pr.acc_step_d),
                                           __ldcg(ap + 2 * pr.acc_step_d),
                                           __ldcg(ap + 3 * pr.acc_step_d));
                  }
                }
              }
            }
#pragma unroll
            for (int q = 0; q < kRowPass; ++q) {
              float Mn = M[q];
#pragma unroll
              for (int j = 0; j < kMergeBatch; ++j) Mn = fmaxf(Mn, mv[q][j]);
              if (Mn == -INFINITY) continue;  // only empty splits so far
              const float sa = exp2f((M[q] - Mn) * kLog2e);  // 0 while M is -inf
              L[q] *= sa;
              A[q][0] *= sa;
              A[q][1] *= sa;
              A[q][2] *= sa;
              A[q][3] *= sa;
#pragma unroll
              for (int j = 0; j < kMergeBatch; ++j) {
                const float w = exp2f((mv[q][j] - Mn) * kLog2e);  // 0 for empty splits
                L[q] += w * lv[q][j];
                A[q][0] += w * av[q][j].x;
                A[q][1] += w * av[q][j].y;
                A[q][2] += w * av[q][j].z;
                A[q][3] += w * av[q][j].w;
              }
              M[q] = Mn;
            }
          }
#pragma unroll
          for (int q = 0; q < kRowPass; ++q) {
            const int r = r0 + q * kSlots;
            if (r < nrows) {
              const float inv = L[q] > 0.f ? 1.f / L[q] : 0.f;
              store_out4<T>(p, s.b, head0 + r, d, A[q][0] * inv, A[q][1] * inv, A[q][2] * inv,
                            A[q][3] * inv);
            }
          }
        }
      }
    }
    named_barrier(kBarConsumers, kConsumerThreads);
  }

  // ---- zero outputs of pairs with nothing to attend (stream-K) ----
  if (streamk) {
    for (int b = 0; b < p.num_seqs; ++b) {
      if (prefix[b + 1] != prefix[b]) continue;
      for (int hb = 0; hb < p.nhb; ++hb) {
        if ((b * p.nhb + hb) % static_cast<int>(gridDim.x) != static_cast<int>(blockIdx.x)) continue;
        const int kvh = hb / p.hb_per_kv;
        const int jb = hb % p.hb_per_kv;
        const int h0 = kvh * p.group + jb * p.rows;
        const int nr = min(p.rows, p.group - jb * p.rows);
        for (int e = tid; e < nr * (D / 4); e += kConsumerThreads) {
          const int r = e / (D / 4);
          store_out4<T>(p, b, h0 + r, (e - r * (D / 4)) * 4, 0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// standalone split-KV reducer (reference _paged_decode_gqa_reduce_kernel)
// ---------------------------------------------------------------------------
struct ReduceParams {
  int num_seqs, num_q_heads, head_dim, num_splits;
  const float* acc;
  int64_t as0, as1, as2, as3;
  const float* mx;
  const float* sm;
  int64_t ss0, ss1, ss2;
  const void* sl;
  int sl64;
  int64_t sls;
  const void* slot;
  int slot64;
  int64_t slots;
  void* out;
  int64_t os0, os1, os2;
  // cascade: a sequence with pre_pages[b] > 0 also merges the prefix pass's
  // pre_slots partials in slots [num_splits, num_splits + pre_slots)
  const int* pre_pages;
  int pre_slots;
};

constexpr int kReduceMaxSlots = 512;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  // blockDim.x <= 128 (at most 4 warps)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float y = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, y) : v + y;
  }
  const int warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  __syncthreads();  // red is free (an earlier reduction has been read)
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// One CTA per (sequence, q head); thread = dimension.  The slot maxima and
// weights are formed once per row in shared memory, then every thread sums
// its dimension over the slots with eight independent loads in flight, so a
// row with many partials costs a few memory round trips instead of one per
// partial.
template <typename T>
__global__ void split_reduce_kernel(const __grid_constant__ ReduceParams p) {
  __shared__ float w_sh[kReduceMaxSlots];
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int h = blockIdx.y;
  const int tid = threadIdx.x;
  const int nt = blockDim.x;
  const int64_t n = load_index(p.sl, p.sl64, static_cast<int64_t>(b) * p.sls);
  bool has = n > 0;
  if (p.slot) has = has && load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots) >= 0;
  const int S = min(p.num_splits + ((p.pre_pages && p.pre_pages[b] > 0) ? p.pre_slots : 0),
                    kReduceMaxSlots);
  const int64_t so = b * p.ss0 + h * p.ss1;
  float mloc = -INFINITY;
  if (has) {
    for (int s = tid; s < S; s += nt) mloc = fmaxf(mloc, p.mx[so + s * p.ss2]);
  }
  const float M = block_reduce(mloc, red, true);
  float lloc = 0.f;
  for (int s = tid; s < S; s += nt) {
    float w = 0.f;
    if (has && M != -INFINITY) {
      const float m = p.mx[so + s * p.ss2];
      if (m != -INFINITY) {
        w = exp2f((m - M) * kLog2e);
        lloc += w * p.sm[so + s * p.ss2];
      }
    }
    w_sh[s] = w;
  }
  const float L = block_reduce(lloc, red, false);  // its barriers publish w_sh
  const float* ab = p.acc + b * p.as0 + h * p.as1;
  for (int d = tid; d < p.head_dim; d += nt) {
    const float* ad = ab + d * p.as3;
    float a = 0.f;
    int s = 0;
    for (; s + 8 <= S; s += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = w_sh[s + j] != 0.f ? ad[(s + j) * p.as2] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) a += w_sh[s + j] * v[j];
    }
    for (; s < S; ++s) {
      if (w_sh[s] != 0.f) a += w_sh[s] * ad[s * p.as2];
    }
    T* o = static_cast<T*>(p.out) + b * p.os0 + h * p.os1 + d * p.os2;
    *o = from_f32<T>(L > 0.f ? a / L : 0.f);
  }
}

// ---------------------------------------------------------------------------
// shared-prefix (cascade) pass
// ---------------------------------------------------------------------------
// A group is a set of sequences whose block-table rows start with the same
// grp_pages[g] physical pages (a shared prompt prefix registered once and
// attached to every member).  The plain decode reads those pages once per
// member; this pass reads them once per KV head for all of the group's query
// rows, rows = members x (q heads of the KV head).  CTA (chunk c, row block
// rb, group g x KV head h) serves 128 rows -- one m16 tile per consumer warp,
// every warp consuming every stage of the TMA ring -- over prefix tiles
// [c T / C, (c + 1) T / C) of T = pages * block_size / 32, and writes its
// rows' (max, sum, acc) into slot slot0 + c of the split workspace.  The
// split reducer then merges these slots with the tail pass's partials
// (same LSE merge as reference paged_decode.py:593-635).
constexpr int kCascadeMaxGroups = 32;
constexpr int kCascadeMaxMembers = 512;

struct PrefixParams {
  int num_seqs, num_kv_heads, group, block_size, num_blocks, max_blocks;
  float scale_log2;
  const void* q;
  int64_t qs0, qs1, qs2;
  int rope_dim;  // > 0: q rows are rotated by their sequence's position
  const float* rope_inv_freq;
  const void* rope_pos;
  int rope_pos64;
  int64_t rope_pos_stride;
  const void* bt;
  int bt64;
  int64_t bts0, bts1;
  // the groups travel in the launch parameters (no dependent loads before
  // the first page): CSR offsets, member sequence indices (the first
  // member's table row is read), shared pages (pages * block_size % 32 == 0)
  int grp_start[kCascadeMaxGroups + 1];
  int grp_pages[kCascadeMaxGroups];
  int grp_members[kCascadeMaxMembers];
  int chunks;
  float* pacc;
  int64_t pas0, pas1, pas2, pas3;
  float* pmax;
  float* psum;
  int64_t pss0, pss1, pss2;
  int slot0;
  int kperm[4], vperm[4];
  int* status;
  int num_stages;
};

// Eight consumer warps (two per SM sub-partition, so one warp's mma and
// exp2 latencies hide behind the other's) plus the producer warp.
constexpr int kPrefixWarps = 8;
constexpr int kPrefixThreads = 32 * kPrefixWarps + 32;
constexpr int kPrefixRows = kPrefixWarps * 16;  // query rows per prefix CTA

template <int D>
constexpr int prefix_q_bytes() {
  return (D / 64) * (kTile * 128);  // one warp's Q block: [D/64][32 rows][64], rows 0-15 used
}

template <int D>
size_t prefix_smem_bytes(int stages) {
  return 1024 + static_cast<size_t>(stages) * Smem<D>::kStageBytes +
         kPrefixWarps * prefix_q_bytes<D>() + 2 * kPrefixRows * sizeof(int) +
         static_cast<size_t>(stages) * 16 + 64;
}

template <typename T, int D, int kPageRows>
__global__ void __launch_bounds__(kPrefixThreads, 1)
    prefix_kernel(const __grid_constant__ PrefixParams p,
                  const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v) {
  using SM = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int NST = p.num_stages;
  uint8_t* stages = smem;
  uint8_t* qsm = stages + NST * SM::kStageBytes;
  int* row_seq = reinterpret_cast<int*>(qsm + kPrefixWarps * prefix_q_bytes<D>());
  float* row_pos = reinterpret_cast<float*>(row_seq + kPrefixRows);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(row_pos + kPrefixRows);
  uint64_t* empty_bar = full_bar + NST;
  int* misc = reinterpret_cast<int*>(empty_bar + NST);  // [0] abort
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  volatile int* abort_flag = misc;

  if (tid < NST) {
    mbar_init(smem_u32(&full_bar[tid]), 1);
    mbar_init(smem_u32(&empty_bar[tid]), kPrefixWarps);  // every warp reads every stage
    fence_mbar_init();
  }
  if (tid == 0) misc[0] = 0;
  if (warp == kPrefixWarps && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  pdl_wait();
  pdl_launch_dependents();

  const int c = static_cast<int>(blockIdx.x);
  const int row0 = static_cast<int>(blockIdx.y) * kPrefixRows;
  const int g = static_cast<int>(blockIdx.z) / p.num_kv_heads;
  const int h = static_cast<int>(blockIdx.z) - g * p.num_kv_heads;
  const int m0 = p.grp_start[g];
  const int rows = (p.grp_start[g + 1] - m0) * p.group;
  const int64_t ptok = static_cast<int64_t>(p.grp_pages[g]) * p.block_size;
  const int tiles = static_cast<int>(ptok / kTile);
  const int t0 = static_cast<int>(static_cast<int64_t>(c) * tiles / p.chunks);
  const int t1 = static_cast<int>(static_cast<int64_t>(c + 1) * tiles / p.chunks);
  __syncthreads();  // barrier initialisation is visible to every warp
  if (row0 >= rows) return;  // this group has fewer row blocks (whole CTA)

  const int bs = p.block_size;
  const int ppt_shift = bs == 32 ? 0 : (bs == 16 ? 1 : 2);

  // =========================================================================
  // producer warp: the group's first member's pages, tile by tile
  // =========================================================================
  if (warp == kPrefixWarps) {
    const int rep = p.grp_members[m0];
    const uint64_t policy = l2_policy_evict_first();
    const int PPT = 1 << ppt_shift;  // pages per tile
    const int TG = max(1, min(32 >> ppt_shift, NST / 2));
    constexpr int kOps = 2 * SM::kHalves;
    int pst = 0;
    uint32_t pph = 0;
    bool bad = false;
    for (int tg = t0; tg < t1;) {
      const int ntile = min(TG, t1 - tg);
      const int npage = ntile << ppt_shift;
      const int64_t lb = (static_cast<int64_t>(tg) << ppt_shift) + lane;
      int blk = -1;
      if (lane < npage && lb < p.max_blocks) {
        blk = static_cast<int>(
            load_index(p.bt, p.bt64, static_cast<int64_t>(rep) * p.bts0 + lb * p.bts1));
      }
      const bool pvalid = lane < npage && blk >= 0 && blk < p.num_blocks;
      bad = bad || (lane < npage && !pvalid);
      const uint32_t pages = __ballot_sync(0xffffffffu, pvalid);
      bool ok = true;
      if (lane < ntile) {
        int st = pst + lane;
        uint32_t ph = pph;
        if (st >= NST) {
          st -= NST;
          ph ^= 1u;
        }
        ok = mbar_wait(smem_u32(&empty_bar[st]), ph ^ 1u, p.status, abort_flag);
        const uint32_t tmask = (pages >> (lane << ppt_shift)) & ((1u << PPT) - 1u);
        if (ok) {
          mbar_arrive_expect_tx(smem_u32(&full_bar[st]),
                                static_cast<uint32_t>(__popc(tmask)) * (bs * D * 2 * 2));
        }
      }
      if (__all_sync(0xffffffffu, ok)) {
        if constexpr (kPageRows > 0) {
          const int nops = npage * 2;  // one box per (page, plane)
          for (int base = 0; base < nops; base += 32) {
            const int op = base + lane;
            const int page = op >> 1;
            const int pblk = __shfl_sync(0xffffffffu, blk, page & 31);
            if (op < nops && ((pages >> page) & 1u)) {
              const int plane = op & 1;
              int st = pst + (page >> ppt_shift);
              if (st >= NST) st -= NST;
              const uint32_t dst = smem_u32(stages + st * SM::kStageBytes) +
                                   plane * (SM::kHalves * SM::kHalfBytes) +
                                   (page & (PPT - 1)) * (kPageRows * 256);
              const int* perm = plane ? p.vperm : p.kperm;
              tma_load_5d(dst, plane ? &tmap_v : &tmap_k, smem_u32(&full_bar[st]), 0,
                          tmap_coord(perm[0], h, pblk), tmap_coord(perm[1], h, pblk),
                          tmap_coord(perm[2], h, pblk), tmap_coord(perm[3], h, pblk), policy);
            }
          }
        } else {
          const int nops = npage * kOps;
          for (int base = 0; base < nops; base += 32) {
            const int op = base + lane;
            const int page = op / kOps;
            const int pblk = __shfl_sync(0xffffffffu, blk, page & 31);
            if (op < nops && ((pages >> page) & 1u)) {
              const int rem = op - page * kOps;
              const int plane = rem / SM::kHalves;
              const int hh = rem - plane * SM::kHalves;
              int st = pst + (page >> ppt_shift);
              if (st >= NST) st -= NST;
              const uint32_t dst = smem_u32(stages + st * SM::kStageBytes) +
                                   plane * (SM::kHalves * SM::kHalfBytes) + hh * SM::kHalfBytes +
                                   (((page & (PPT - 1)) * bs) << 7);
              const int* perm = plane ? p.vperm : p.kperm;
              tma_load_4d(dst, plane ? &tmap_v : &tmap_k, smem_u32(&full_bar[st]), hh * 64,
                          tmap_coord(perm[0], h, pblk), tmap_coord(perm[1], h, pblk),
                          tmap_coord(perm[2], h, pblk), policy);
            }
          }
        }
      }
      pst += ntile;
      if (pst >= NST) {
        pst -= NST;
        pph ^= 1u;
      }
      tg += ntile;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
    return;
  }

  // =========================================================================
  // consumer warps: warp w owns rows row0 + 16 w .. + 15
  // =========================================================================
  const int g8 = lane >> 2;
  const int t4 = lane & 3;
  const int mi = lane >> 3;
  const int r8 = lane & 7;
  uint8_t* qw = qsm + warp * prefix_q_bytes<D>();
  const int wrow0 = row0 + 16 * warp;
  if (lane < 16) {
    const int gr = wrow0 + lane;
    int seq = -1;
    float posf = 0.f;
    if (gr < rows) {
      seq = p.grp_members[m0 + gr / p.group];  // checked on the host
      if (p.rope_dim > 0) {
        posf = static_cast<float>(
            load_index(p.rope_pos, p.rope_pos64, static_cast<int64_t>(seq) * p.rope_pos_stride));
      }
    }
    row_seq[16 * warp + lane] = seq;
    row_pos[16 * warp + lane] = posf;
  }
  __syncwarp();
  for (int e = lane; e < 16 * (D / 8); e += 32) {
    const int r = e / (D / 8);
    const int ch = e - r * (D / 8);
    const int gr = wrow0 + r;
    const int seq = row_seq[16 * warp + r];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (seq >= 0) {
      const int qh = h * p.group + (gr - (gr / p.group) * p.group);
      const T* src = static_cast<const T*>(p.q) + seq * p.qs0 + qh * p.qs1 + ch * 8 * p.qs2;
      if (p.qs2 == 1 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        __align__(16) T el[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) el[i] = src[i * p.qs2];
        v = *reinterpret_cast<const uint4*>(el);
      }
    }
    *reinterpret_cast<uint4*>(qw + chunk_offset(r, ch)) = v;
  }
  __syncwarp();
  if (p.rope_dim > 0) {
    // RoPE of the rows in place; rows of one member share their angles
    const int half = p.rope_dim >> 1;
    for (int i = lane; i < half; i += 32) {
      const float invf = p.rope_inv_freq[i];
      int last = -1;
      float cs = 1.f, sn = 0.f;
      for (int r = 0; r < 16; ++r) {
        const int seq = row_seq[16 * warp + r];
        if (seq < 0) continue;  // rows past the group's end (or invalid members)
        if (seq != last) {
          sincosf(__fmul_rn(row_pos[16 * warp + r], invf), &sn, &cs);
          last = seq;
        }
        T* x1p = reinterpret_cast<T*>(qw + tile_offset(r, i));
        T* x2p = reinterpret_cast<T*>(qw + tile_offset(r, i + half));
        float y1, y2;
        rope_rotate_pair_cs(to_f32<T>(*x1p), to_f32<T>(*x2p), cs, sn, y1, y2);
        *x1p = from_f32<T>(y1);
        *x2p = from_f32<T>(y2);
      }
    }
    __syncwarp();
  }
  uint32_t qf[D / 16][4];
  const uint32_t qbase = smem_u32(qw);
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    ldsm_x4(qbase + chunk_offset(r8 + (mi & 1) * 8, ks * 2 + (mi >> 1)), qf[ks][0], qf[ks][1],
            qf[ks][2], qf[ks][3]);
  }

  float m0r = -INFINITY, m1r = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  int cst = 0;
  uint32_t cph = 0;
  for (int t = t0; t < t1; ++t) {
    const int stage = cst;
    const uint32_t phase = cph;
    if (++cst == NST) {
      cst = 0;
      cph ^= 1u;
    }
    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, abort_flag)) continue;
    const uint32_t kbase = smem_u32(stages + stage * SM::kStageBytes);
    const uint32_t vbase = kbase + SM::kHalves * SM::kHalfBytes;
    // ---- S = Q K^T (16 rows x 32 tokens; every prefix token is valid) ----
    float sacc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int tok = np * 16 + (mi >> 1) * 8 + r8;
        const int chunk = ks * 2 + (mi & 1);
        uint32_t b0a, b1a, b0b, b1b;
        ldsm_x4(kbase + stage_chunk_offset<kPageRows>(tok, chunk), b0a, b1a, b0b, b1b);
        mma_16816<T>(sacc[2 * np], qf[ks], b0a, b1a);
        mma_16816<T>(sacc[2 * np + 1], qf[ks], b0b, b1b);
      }
    }
    // ---- online softmax (base 2, scale folded in) ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sacc[j][e] *= p.scale_log2;
        sacc[j][2 + e] *= p.scale_log2;
        mx0 = fmaxf(mx0, sacc[j][e]);
        mx1 = fmaxf(mx1, sacc[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0r, mx0);
    const float mn1 = fmaxf(m1r, mx1);
    const float alpha0 = exp2f(m0r - mn0);  // 0 on the first tile (m = -inf)
    const float alpha1 = exp2f(m1r - mn1);
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sacc[j][0] = exp2f(sacc[j][0] - mn0);
      sacc[j][1] = exp2f(sacc[j][1] - mn0);
      sacc[j][2] = exp2f(sacc[j][2] - mn1);
      sacc[j][3] = exp2f(sacc[j][3] - mn1);
      ps0 += sacc[j][0] + sacc[j][1];
      ps1 += sacc[j][2] + sacc[j][3];
    }
    l0 = l0 * alpha0 + ps0;
    l1 = l1 * alpha1 + ps1;
    m0r = mn0;
    m1r = mn1;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha0;
      o[j][1] *= alpha0;
      o[j][2] *= alpha1;
      o[j][3] *= alpha1;
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t a[4];
      a[0] = pack2<T>(sacc[2 * kk][0], sacc[2 * kk][1]);
      a[1] = pack2<T>(sacc[2 * kk][2], sacc[2 * kk][3]);
      a[2] = pack2<T>(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      a[3] = pack2<T>(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int tok = kk * 16 + (mi & 1) * 8 + r8;
        const int chunk = dp * 2 + (mi >> 1);
        uint32_t b0a, b1a, b0b, b1b;
        ldsm_x4_t(vbase + stage_chunk_offset<kPageRows>(tok, chunk), b0a, b1a, b0b, b1b);
        mma_16816<T>(o[2 * dp], a, b0a, b1a);
        mma_16816<T>(o[2 * dp + 1], a, b0b, b1b);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[stage]));
  }

  // ---- this chunk's partial of the warp's rows ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int slot = p.slot0 + c;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = g8 + 8 * hr;
    const int gr = wrow0 + r;
    const int seq = row_seq[16 * warp + r];
    if (seq < 0) continue;
    const int qh = h * p.group + (gr - (gr / p.group) * p.group);
    float* acc = p.pacc + seq * p.pas0 + qh * p.pas1 + slot * p.pas2;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int d = 8 * j + 2 * t4;
      if (p.pas3 == 1 && (reinterpret_cast<uintptr_t>(acc + d) & 7u) == 0) {
        *reinterpret_cast<float2*>(acc + d) = make_float2(o[j][2 * hr], o[j][2 * hr + 1]);
      } else {
        acc[d * p.pas3] = o[j][2 * hr];
        acc[(d + 1) * p.pas3] = o[j][2 * hr + 1];
      }
    }
    if (t4 == 0) {
      const float M = hr ? m1r : m0r;
      const int64_t so = seq * p.pss0 + qh * p.pss1 + slot * p.pss2;
      p.pmax[so] = (M == -INFINITY) ? -INFINITY : M * kLn2;  // natural-log units
      p.psum[so] = hr ? l1 : l0;
    }
  }
}

// ---------------------------------------------------------------------------
// shared-prefix pass on the 5th-generation tensor cores (tcgen05 / UMMA)
// ---------------------------------------------------------------------------
// Same work unit and output as prefix_kernel, for head_dim 128 and 32-token
// pages: CTA (chunk, 128-row block, group x KV head) holds the chunk's n <= 8
// tiles in shared memory -- K and V each as one [half][256 tokens][64 dims]
// operand (TMA, 128B swizzle; tile i at token 32 i) -- and its 128 query rows
// (K-major, 128B swizzle), one TMEM lane per row.
//   1. one thread issues S = Q K^T for the whole chunk (M 128, N 32 n, K 128:
//      8 UMMAs) into TMEM columns [0, 32 n);
//   2. each consumer thread (one row) takes its row max over the chunk's
//      scores, then P = exp2(S - max) (no online rescale needed), and writes P
//      as bf16 over K (no longer needed; core-matrix layout, K-major);
//   3. the thread issues O = P V (M 128, N 128, K 32 n: 2 n UMMAs, V as the
//      MN-major operand) into TMEM columns [256, 384);
//   4. O goes through shared memory to coalesced row writes of the
//      (max, sum, acc) partial.
constexpr int kUmmaMaxTiles = 8;
constexpr int kUmmaMaxMembers = 33;  // RoPE table rows (members of one 128-row block, group >= 4)
constexpr int kUmmaQBytes = 2 * 128 * 128;  // [half][128 rows][128 B]
constexpr int kUmmaTmemCols = 512;
constexpr int kUmmaOCol = 256;
constexpr int kUmmaKBytes = 2 * kUmmaMaxTiles * kTile * 128;  // [half][256 tokens][128 B]

constexpr size_t prefix_umma_smem_bytes() {
  return 1024 + kUmmaQBytes + static_cast<size_t>(kUmmaMaxTiles) * Smem<128>::kStageBytes +
         kUmmaMaxMembers * 128 * sizeof(float) + 2 * 128 * sizeof(int64_t) +
         4 * 128 * sizeof(int) + 16 * sizeof(uint64_t) + 64;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefix_umma_kernel(const __grid_constant__ PrefixParams p,
                       const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v) {
  constexpr int D = 128;
  using SM = Smem<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qsm = smem;
  uint8_t* tiles = qsm + kUmmaQBytes;  // K operand, then V operand (kUmmaKBytes each)
  uint8_t* kreg = tiles;
  uint8_t* vreg = tiles + kUmmaKBytes;
  float* rtab = reinterpret_cast<float*>(tiles + kUmmaMaxTiles * SM::kStageBytes);
  int64_t* row_qoff = reinterpret_cast<int64_t*>(rtab + kUmmaMaxMembers * 128);  // q element
  int64_t* row_ooff = row_qoff + 128;  // partial acc element offset of the row
  int* row_seq = reinterpret_cast<int*>(row_ooff + 128);  // -1: padding row
  float* row_pos = reinterpret_cast<float*>(row_seq + 128);  // RoPE position
  int* row_mm = reinterpret_cast<int*>(row_pos + 128);  // RoPE table row (member - first)
  uint64_t* bars = reinterpret_cast<uint64_t*>(row_mm + 128);  // 8-byte aligned: 2 KB + 2 KB above
  uint64_t* full_bar = bars;                     // every tile of the chunk landed (TMA bytes)
  uint64_t* q_ready = bars + kUmmaMaxTiles;      // Q staged (consumer arrivals)
  uint64_t* s_done = q_ready + 1;                // S UMMAs complete (commit)
  uint64_t* p_ready = s_done + 1;                // P written (consumer arrivals)
  uint64_t* o_done = p_ready + 1;                // PV UMMAs complete (commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  int* misc = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  volatile int* abort_flag = misc;

  if (tid == 0) {
    mbar_init(smem_u32(full_bar), 1);
    mbar_init(smem_u32(q_ready), kConsumerThreads);
    mbar_init(smem_u32(s_done), 1);
    mbar_init(smem_u32(p_ready), kConsumerThreads);
    mbar_init(smem_u32(o_done), 1);
    fence_mbar_init();
    misc[0] = 0;
  }
  if (warp == 0) tmem_alloc(smem_u32(tmem_slot), kUmmaTmemCols);
  if (warp == kConsumerWarps && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  pdl_wait();
  pdl_launch_dependents();

  const int c = static_cast<int>(blockIdx.x);
  const int row0 = static_cast<int>(blockIdx.y) * 128;
  const int g = static_cast<int>(blockIdx.z) / p.num_kv_heads;
  const int h = static_cast<int>(blockIdx.z) - g * p.num_kv_heads;
  const int m0 = p.grp_start[g];
  const int rows = (p.grp_start[g + 1] - m0) * p.group;
  const int tiles_all = p.grp_pages[g] * p.block_size / kTile;
  const int t0 = static_cast<int>(static_cast<int64_t>(c) * tiles_all / p.chunks);
  const int t1 = static_cast<int>(static_cast<int64_t>(c + 1) * tiles_all / p.chunks);
  const int nt = min(t1 - t0, kUmmaMaxTiles);  // the host keeps chunks <= 8 tiles
  const bool active = row0 < rows;

  if (active && warp == kConsumerWarps) {
    // ======== producer (TMA, lane i: tile t0 + i) and UMMA issue (lane 0) ========
    const int rep = p.grp_members[m0];
    const uint64_t policy = l2_policy_evict_first();
    bool bad = false;
    int blk = -1;
    if (lane < nt) {
      const int64_t lb = t0 + lane;  // 32-token pages: page = tile
      blk = lb < p.max_blocks ? static_cast<int>(load_index(
                                    p.bt, p.bt64, static_cast<int64_t>(rep) * p.bts0 + lb * p.bts1))
                              : -1;
    }
    const bool valid = lane < nt && blk >= 0 && blk < p.num_blocks;
    bad = lane < nt && !valid;
    const uint32_t nvalid = __popc(__ballot_sync(0xffffffffu, valid));
    // one barrier for the chunk; the byte count is posted before any copy
    if (lane == 0) mbar_arrive_expect_tx(smem_u32(full_bar), nvalid * SM::kStageBytes);
    __syncwarp();
    if (valid) {
#pragma unroll
      for (int op = 0; op < 4; ++op) {
        const int plane = op >> 1;
        const int hh = op & 1;
        const int* perm = plane ? p.vperm : p.kperm;
        tma_load_4d(smem_u32((plane ? vreg : kreg) + hh * (kUmmaKBytes / 2) + lane * SM::kHalfBytes),
                    plane ? &tmap_v : &tmap_k, smem_u32(full_bar), hh * 64,
                    tmap_coord(perm[0], h, blk), tmap_coord(perm[1], h, blk),
                    tmap_coord(perm[2], h, blk), policy);
      }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
    if (lane == 0) {
      const uint32_t id_s = umma_idesc_f16(kBf16, false, 128, 32 * max(nt, 1));
      constexpr uint32_t kIdO = umma_idesc_f16(kBf16, true, 128, 128);
      bool ok = mbar_wait(smem_u32(q_ready), 0u, p.status, abort_flag);
      ok = ok && mbar_wait(smem_u32(full_bar), 0u, p.status, abort_flag);
      tc_fence_after();
      const uint32_t qbase = smem_u32(qsm);
      const uint32_t kbase = smem_u32(kreg);
      if (ok && nt > 0) {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {  // S = Q K^T over the chunk (N = 32 nt)
          const uint32_t koff = (k & 3) * 32u;
          const uint64_t a = umma_smem_desc(qbase + (k >> 2) * (kUmmaQBytes / 2) + koff, 16, 1024, 2);
          const uint64_t b = umma_smem_desc(kbase + (k >> 2) * (kUmmaKBytes / 2) + koff, 16, 1024, 2);
          umma_f16(taddr, a, b, id_s, k > 0);
        }
      }
      umma_commit(smem_u32(s_done));  // also when nothing was issued: the waiters go on
      ok = ok && mbar_wait(smem_u32(p_ready), 0u, p.status, abort_flag);
      tc_fence_after();
      const uint32_t vbase = smem_u32(vreg);
      for (int kk = 0; ok && kk < 2 * nt; ++kk) {  // O = P V, 16 tokens per UMMA
        const uint64_t a = umma_smem_desc(kbase + kk * 256, 128, 4096, 0);   // P over K
        const uint64_t b = umma_smem_desc(vbase + kk * 2048, kUmmaKBytes / 2, 1024, 2);
        umma_f16(taddr + kUmmaOCol, a, b, kIdO, kk > 0 ? 1u : 0u);
      }
      umma_commit(smem_u32(o_done));
    }
    __syncwarp();
  } else if (active) {
    // ======== consumers: thread = query row = TMEM lane ========
    const int r = tid;  // warps 0-3 -> rows 0-127 -> TMEM lanes 0-127
    const int slot = p.slot0 + c;
    const int half = p.rope_dim >> 1;
    const int mem_first = row0 / p.group;
    int seq_r = -1;     // this thread's row: sequence (-1: padding row)
    int64_t so_r = 0;   // and (max, sum) element offset
    {
      const int gr = row0 + r;
      int seq = -1, mem = mem_first;
      int64_t qo = 0, oo = 0;
      float posf = 0.f;
      if (gr < rows) {
        mem = gr / p.group;
        seq = p.grp_members[m0 + mem];
        const int qh = h * p.group + (gr - mem * p.group);
        qo = seq * p.qs0 + qh * p.qs1;
        oo = seq * p.pas0 + qh * p.pas1 + slot * p.pas2;
        so_r = seq * p.pss0 + qh * p.pss1 + slot * p.pss2;
        if (p.rope_dim > 0)
          posf = static_cast<float>(
              load_index(p.rope_pos, p.rope_pos64, static_cast<int64_t>(seq) * p.rope_pos_stride));
      }
      row_seq[r] = seq;
      row_qoff[r] = qo;
      row_ooff[r] = oo;
      row_pos[r] = posf;
      row_mm[r] = mem - mem_first;
      seq_r = seq;
    }
    // RoPE table: cos / sin per (member of this block, pair index)
    const int nmem = min((row0 + 127) / p.group, p.grp_start[g + 1] - m0 - 1) - mem_first + 1;
    const bool table = p.rope_dim > 0 && nmem <= kUmmaMaxMembers;
    if (table) {
      for (int e = tid; e < nmem * half; e += kConsumerThreads) {
        const int mm = e / half;
        const int i = e - mm * half;
        const int sq = p.grp_members[m0 + mem_first + mm];
        const float posf = static_cast<float>(
            load_index(p.rope_pos, p.rope_pos64, static_cast<int64_t>(sq) * p.rope_pos_stride));
        float sn, cs;
        sincosf(__fmul_rn(posf, p.rope_inv_freq[i]), &sn, &cs);
        rtab[mm * 128 + i] = cs;
        rtab[mm * 128 + 64 + i] = sn;
      }
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    // ---- Q rows into the K-major 128B-swizzled operand: 16-byte chunks, 16
    // lanes per row (coalesced), RoPE applied in registers on the way.  With
    // rope_dim / 2 a multiple of 8, chunk cc < hp (hp = rope_dim / 16) pairs
    // with chunk cc + hp of the same row, one warp shuffle away. ----
    auto q_chunk = [&](int row, int cc) -> uint8_t* {
      return qsm + (cc >> 3) * (kUmmaQBytes / 2) + row * 128 + (((cc & 7) ^ (row & 7)) << 4);
    };
    const int hp = (p.rope_dim > 0 && (half & 7) == 0) ? (half >> 3) : 0;
    {
      // 16 chunks per thread (2048 / 128): every load is issued before the
      // first store, so the staging costs one memory round trip
      constexpr int kPer = 128 * (D / 8) / kConsumerThreads;
      uint4 v[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int rr = (tid + k * kConsumerThreads) >> 4;
        const int cc = lane & 15;
        v[k] = make_uint4(0u, 0u, 0u, 0u);
        if (row_seq[rr] >= 0) {
          const T* src = static_cast<const T*>(p.q) + row_qoff[rr] + cc * 8 * p.qs2;
          if (p.qs2 == 1 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
            v[k] = __ldg(reinterpret_cast<const uint4*>(src));
          } else {
            __align__(16) T el[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) el[i] = src[i * p.qs2];
            v[k] = *reinterpret_cast<const uint4*>(el);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int rr = (tid + k * kConsumerThreads) >> 4;
        const int cc = lane & 15;
        if (hp > 0) {  // warp-uniform
          const bool lo = cc < hp;
          const bool hi = !lo && cc < 2 * hp;
          const int src = lo ? lane + hp : (hi ? lane - hp : lane);
          uint4 w;
          w.x = __shfl_sync(0xffffffffu, v[k].x, src);
          w.y = __shfl_sync(0xffffffffu, v[k].y, src);
          w.z = __shfl_sync(0xffffffffu, v[k].z, src);
          w.w = __shfl_sync(0xffffffffu, v[k].w, src);
          if ((lo || hi) && row_seq[rr] >= 0) {
            // y1 = x1 cos - x2 sin (own = x1), y2 = x2 cos + x1 sin (own = x2):
            // the operations and order of rope_rotate_pair_cs
            const int i0 = 8 * (lo ? cc : cc - hp);
            float cs[8], sn[8];
            if (table) {
              const float* tr = rtab + row_mm[rr] * 128;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                cs[j] = tr[i0 + j];
                sn[j] = tr[64 + i0 + j];
              }
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                sincosf(__fmul_rn(row_pos[rr], p.rope_inv_freq[i0 + j]), &sn[j], &cs[j]);
            }
            const uint32_t own[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
            const uint32_t oth[4] = {w.x, w.y, w.z, w.w};
            uint32_t res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 a = unpack2<T>(own[e]);
              const float2 b = unpack2<T>(oth[e]);
              float y0, y1;
              if (lo) {
                y0 = __fsub_rn(__fmul_rn(a.x, cs[2 * e]), __fmul_rn(b.x, sn[2 * e]));
                y1 = __fsub_rn(__fmul_rn(a.y, cs[2 * e + 1]), __fmul_rn(b.y, sn[2 * e + 1]));
              } else {
                y0 = __fadd_rn(__fmul_rn(a.x, cs[2 * e]), __fmul_rn(b.x, sn[2 * e]));
                y1 = __fadd_rn(__fmul_rn(a.y, cs[2 * e + 1]), __fmul_rn(b.y, sn[2 * e + 1]));
              }
              res[e] = pack2<T>(y0, y1);
            }
            v[k] = make_uint4(res[0], res[1], res[2], res[3]);
          }
        }
        *reinterpret_cast<uint4*>(q_chunk(rr, cc)) = v[k];
      }
    }
    if (p.rope_dim > 0 && hp == 0) {
      // rope_dim / 2 not a multiple of 8: element pairs in shared memory
      named_barrier(kBarConsumers, kConsumerThreads);
      for (int e = tid; e < 128 * half; e += kConsumerThreads) {
        const int rr = e / half;
        const int i = e - rr * half;
        if (row_seq[rr] < 0) continue;
        float cs, sn;
        if (table) {
          cs = rtab[row_mm[rr] * 128 + i];
          sn = rtab[row_mm[rr] * 128 + 64 + i];
        } else {
          sincosf(__fmul_rn(row_pos[rr], p.rope_inv_freq[i]), &sn, &cs);
        }
        T* x1p = reinterpret_cast<T*>(q_chunk(rr, i >> 3) + (i & 7) * 2);
        T* x2p = reinterpret_cast<T*>(q_chunk(rr, (i + half) >> 3) + ((i + half) & 7) * 2);
        float y1, y2;
        rope_rotate_pair_cs(to_f32<T>(*x1p), to_f32<T>(*x2p), cs, sn, y1, y2);
        *x1p = from_f32<T>(y1);
        *x2p = from_f32<T>(y2);
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(q_ready));

    // ---- scores -> row max -> P (bf16) over the K area of each tile ----
    // tcgen05.ld is warp-collective (.sync.aligned): every TMEM load below
    // runs on all 32 lanes under warp-uniform conditions; only the global
    // writes depend on the row.
    const uint32_t lane_addr = taddr + (static_cast<uint32_t>(warp * 32) << 16);
    bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(s_done), 0u, p.status, abort_flag));
    tc_fence_after();
    float mrow = -INFINITY, lrow = 0.f;
    if (ok && nt > 0) {
      for (int i = 0; i < nt; ++i) {
        float v[32];
        tmem_ld32(lane_addr + 32 * i, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) mrow = fmaxf(mrow, v[j] * p.scale_log2);
      }
      // P in the no-swizzle K-major core-matrix layout over the K operand:
      // row r, tokens 8 k .. 8 k + 7 at (r / 8) * 4096 + k * 128 + (r % 8) * 16
      for (int i = 0; i < nt; ++i) {
        float v[32];
        tmem_ld32(lane_addr + 32 * i, v);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {  // tokens 32 i + 8 cc .. + 7
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a0 = exp2f(v[8 * cc + 2 * e] * p.scale_log2 - mrow);
            const float a1 = exp2f(v[8 * cc + 2 * e + 1] * p.scale_log2 - mrow);
            lrow += a0 + a1;
            w[e] = pack2<T>(a0, a1);
          }
          *reinterpret_cast<uint4*>(kreg + (r >> 3) * 4096 + (4 * i + cc) * 128 + (r & 7) * 16) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(p_ready));

    // ---- this row's (max, sum, acc) partial ----
    ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(o_done), 0u, p.status, abort_flag)) && ok;
    tc_fence_after();
    {
      // O rows go through shared memory (the tile area: the PV UMMAs that read
      // it have completed) so that each warp writes whole 512-byte rows.
      // Row r's 16-byte chunk k sits at r * 512 + ((k ^ (r % 32)) * 16): the
      // XOR spreads a warp's same-chunk writes over all banks.
      float* ob = reinterpret_cast<float*>(tiles);
      for (int j = 0; j < 4; ++j) {
        float v[32];
        if (ok && nt > 0) {
          tmem_ld32(lane_addr + kUmmaOCol + 32 * j, v);  // all lanes
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const int k = (32 * j + e) >> 2;
          *reinterpret_cast<float4*>(ob + r * 128 + ((k ^ (r & 31)) << 2)) =
              make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
      }
      if (seq_r >= 0) {
        const bool empty = !(ok && nt > 0);
        p.pmax[so_r] = (empty || mrow == -INFINITY) ? -INFINITY : mrow * kLn2;  // natural-log units
        p.psum[so_r] = empty ? 0.f : lrow;
      }
      named_barrier(kBarConsumers, kConsumerThreads);
      // warp w writes rows w, w + 4, ...: lane l moves 16-byte chunk l
#pragma unroll 4
      for (int rr = warp; rr < 128; rr += kConsumerWarps) {
        if (row_seq[rr] < 0) continue;  // warp-uniform (one row per iteration)
        float* acc = p.pacc + row_ooff[rr];
        const float4 val = *reinterpret_cast<const float4*>(ob + rr * 128 + ((lane ^ (rr & 31)) << 2));
        if (p.pas3 == 1 && (reinterpret_cast<uintptr_t>(acc) & 15u) == 0) {
          reinterpret_cast<float4*>(acc)[lane] = val;
        } else {
          acc[(4 * lane) * p.pas3] = val.x;
          acc[(4 * lane + 1) * p.pas3] = val.y;
          acc[(4 * lane + 2) * p.pas3] = val.z;
          acc[(4 * lane + 3) * p.pas3] = val.w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(taddr, kUmmaTmemCols);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

template <int D>
size_t smem_bytes(int stages, int sched_ints, bool fused_append) {
  using SM = Smem<D>;
  return 1024 + static_cast<size_t>(stages) * SM::kStageBytes + SM::kMergeBytes +
         static_cast<size_t>(stages) * 20 + 16 +
         (kMiscInts + (fused_append ? kRopeFloats + kAppendInts : 0) + sched_ints) * sizeof(int);
}

struct Derived {
  int group, hb_per_kv, rows, nhb;
};

Derived derive(const fd_paged_decode_args& a) {
  Derived d;
  d.group = a.num_q_heads / a.num_kv_heads;
  d.hb_per_kv = (d.group + kMaxRows - 1) / kMaxRows;
  d.rows = (d.group + d.hb_per_kv - 1) / d.hb_per_kv;
  d.nhb = a.num_kv_heads * d.hb_per_kv;
  return d;
}

int validate(const fd_paged_decode_args* a) {
  if (!a || a->struct_size != static_cast<int32_t>(sizeof(fd_paged_decode_args)))
    return FD_ERR_INVALID_ARGUMENT;
  if (a->dtype != FD_DTYPE_F16 && a->dtype != FD_DTYPE_BF16) return FD_ERR_UNSUPPORTED;
  if (a->head_dim != 64 && a->head_dim != 128) return FD_ERR_UNSUPPORTED;
  if (a->block_size != 8 && a->block_size != 16 && a->block_size != 32) return FD_ERR_UNSUPPORTED;
  if (a->num_seqs < 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->num_blocks <= 0 ||
      a->max_blocks_per_seq <= 0)
    return FD_ERR_INVALID_ARGUMENT;
  if (a->num_q_heads % a->num_kv_heads != 0) return FD_ERR_INVALID_ARGUMENT;
  if (!a->q || !a->out || !a->k_cache || !a->v_cache || !a->block_tables || !a->seq_lens)
    return FD_ERR_INVALID_ARGUMENT;
  if (a->append_k && (!a->append_v || !a->slot_mapping)) return FD_ERR_INVALID_ARGUMENT;
  if (a->rope_dim != 0) {
    // RoPE applies to the fused-append row: q and the appended K
    if (!a->append_k || a->rope_dim < 0 || (a->rope_dim & 1) || a->rope_dim > a->head_dim ||
        !a->rope_inv_freq || !a->rope_positions)
      return FD_ERR_INVALID_ARGUMENT;
  }
  if (a->num_splits < 0 || a->num_splits > 4096) return FD_ERR_INVALID_ARGUMENT;
  if (a->epilogue != FD_EPILOGUE_FUSED && a->epilogue != FD_EPILOGUE_PARTIALS)
    return FD_ERR_INVALID_ARGUMENT;
  if (a->epilogue == FD_EPILOGUE_PARTIALS && a->num_splits == 0) return FD_ERR_INVALID_ARGUMENT;
  if (a->num_splits > 0 && a->num_seqs > 65535) return FD_ERR_UNSUPPORTED;  // grid.z limit
  return FD_OK;
}

// Launch plan.  An explicit num_splits keeps the reference's fixed split.
// Automatic (num_splits == 0):
//   * few (sequence, head block) pairs and short block tables -- the
//     latency regime of small decode batches -- every pair gets
//     S = SMs / pairs CTAs with equal tile ranges, so each CTA owns one
//     segment and knows its pages from blockIdx alone;
//   * otherwise (or when max_ctas is given) the persistent length-balanced
//     schedule over the whole batch.
constexpr int kSplitMaxTilesPerCta = 32;
constexpr int kSplitMinTilesPerCta = 2;
constexpr int kWaveSplitCap = 14;
constexpr int kWaveBalancedMaxTiles = 64;
constexpr int kWaveFillCap = 12;

// FLASHDEC_B200_BALANCED_MAX_TILES=n: a batch takes the balanced split plan
// while pairs x tiles <= SMs x n (tuning sweeps; default kSplitMaxTilesPerCta)
int balanced_max_tiles_per_cta() {
  static const int n = [] {
    const char* v = std::getenv("FLASHDEC_B200_BALANCED_MAX_TILES");
    const int x = v ? std::atoi(v) : 0;
    return x > 0 ? x : kSplitMaxTilesPerCta;
  }();
  return n;
}
constexpr int kWaveLongTiles = 12;

struct Plan {
  int splits;    // 0: length-balanced persistent schedule
  int balanced;
  int grid;
  int cap_tiles;
};

Plan make_plan(const fd_paged_decode_args& a, const Derived& dv, const DeviceInfo& dev) {
  Plan pl;
  const int64_t pairs = static_cast<int64_t>(a.num_seqs) * dv.nhb;
  const int64_t cap_tokens = static_cast<int64_t>(a.max_blocks_per_seq) * a.block_size;
  pl.cap_tiles = static_cast<int>((cap_tokens + kTile - 1) / kTile);
  pl.balanced = 0;
  if (a.num_splits > 0) {
    pl.splits = a.num_splits;
    pl.grid = static_cast<int>(pairs * a.num_splits);
    return pl;
  }
  const int64_t nsm = dev.num_sms;
  const bool wave = wave_enabled() && a.epilogue == FD_EPILOGUE_FUSED;
  const int64_t work = pairs * pl.cap_tiles;
  if (a.max_ctas <= 0 && pairs <= nsm &&
      work <= nsm * (wave ? kWaveBalancedMaxTiles : balanced_max_tiles_per_cta())) {
    int64_t s = nsm / pairs;
    s = std::min<int64_t>(s, std::max(1, pl.cap_tiles / kSplitMinTilesPerCta));
    if (wave) {
      // One-wave kernel (two CTAs fit an SM): clusters above 14 CTAs cost
      // more in residency than they add; once a split would hold 12 tiles or
      // more, about 1.3 CTAs per SM beat one (measured over B1-B16,
      // contexts 1k-8k).
      s = std::min<int64_t>(s, kWaveSplitCap);
      if (pl.cap_tiles >= kWaveLongTiles * s) {
        s = std::max<int64_t>(s, std::min<int64_t>(kWaveSplitCap, nsm * 13 / 10 / pairs));
        // Splits that still hold 16 tiles or more go up to one full wave at
        // two CTAs per SM (clusters of at most 12, whose co-residency holds
        // at 16 pairs): B16 x 5120 tokens 21.9 -> 18.8 us, the c5 layer 15.1
        // -> 13.3 us; fewer tiles per split (B16 x 2048) keep the rule above.
        const int64_t fill = std::min<int64_t>(
            {kWaveFillCap, 2 * nsm / pairs, static_cast<int64_t>(pl.cap_tiles) / 16});
        s = std::max<int64_t>(s, fill);
      }
      if (wave_splits_override() > 0) s = wave_splits_override();
    }
    s = std::max<int64_t>(1, s);
    // Past the plain limit the even split pays only while its CTAs cover
    // every SM (B16 x 5k tokens: 21.3 us against 26.8 us for stream-K; B4 x
    // 32k, 112 CTAs: 44.9 against 35.2).  The split is even over the block
    // table width, not the true lengths: a ragged batch in this range can
    // run up to about twice the stream-K time, which bounds the range.
    const bool fits = work <= nsm * balanced_max_tiles_per_cta() || pairs * s >= nsm;
    if (fits) {
      pl.splits = static_cast<int>(s);
      pl.balanced = 1;
      pl.grid = static_cast<int>(pairs * pl.splits);
      return pl;
    }
  }
  pl.splits = 0;
  // Two resident CTAs per SM when a ring of at least 4 stages fits in half
  // an SM's shared memory next to the schedule tables.
  const int g = a.max_ctas > 0 ? a.max_ctas : dev.num_sms;
  pl.grid = g < 1 ? 1 : g;
  return pl;
}

struct WorkspaceNeed {
  size_t scratch_bytes = 0;
  int64_t tickets = 0;
};

WorkspaceNeed workspace_need(const fd_paged_decode_args& a, const Derived& dv, const Plan& pl) {
  WorkspaceNeed w;
  const int64_t pairs = static_cast<int64_t>(a.num_seqs) * dv.nhb;
  if (pl.splits == 0) {
    const int64_t slots = static_cast<int64_t>(pl.grid) + pairs;
    w.scratch_bytes = static_cast<size_t>(slots) * dv.rows * (a.head_dim + 2) * sizeof(float);
    w.tickets = pairs;
  } else {
    const bool partials = pl.splits > 1 || a.epilogue == FD_EPILOGUE_PARTIALS;
    if (partials && !a.part_acc) {
      w.scratch_bytes = static_cast<size_t>(a.num_seqs) * a.num_q_heads * pl.splits *
                        (a.head_dim + 2) * sizeof(float);
    }
    if (pl.splits > 1 && a.epilogue == FD_EPILOGUE_FUSED) w.tickets = pairs;
  }
  return w;
}

// Clusters of the split schedule.  The S CTAs of a (sequence, head block)
// pair can merge through distributed shared memory only if all clusters of
// the launch are resident at once; cudaOccupancyMaxActiveClusters answers
// that for this kernel, smem size and S (cached: the answer depends on the
// device only).

struct ClusterKey {
  int device;
  const void* kern;
  size_t smem;
  int size;
};

std::mutex g_cluster_mu;
std::vector<std::pair<ClusterKey, int>> g_cluster_cache;

template <typename K>
int max_active_clusters(K kern, size_t smem, int size, const DeviceInfo& dev) {
  {
    std::lock_guard<std::mutex> lock(g_cluster_mu);
    for (const auto& e : g_cluster_cache) {
      if (e.first.device == dev.device && e.first.kern == reinterpret_cast<const void*>(kern) &&
          e.first.smem == smem && e.first.size == size)
        return e.second;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(size));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(size);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();  // not fatal: the launch falls back to the ticket merge
    n = 0;
  }
  std::lock_guard<std::mutex> lock(g_cluster_mu);
  g_cluster_cache.push_back({ClusterKey{dev.device, reinterpret_cast<const void*>(kern), smem, size}, n});
  return n;
}

template <typename T, int D, bool kTma, int kPageRows, bool kAppend>
int launch(AttnParams prm, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
           size_t smem, const DeviceInfo& dev, cudaStream_t stream) {
  auto kern = paged_decode_kernel<T, D, kTma, kPageRows, kAppend>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  const int slot = dev.device & 63;
  std::call_once(once[slot], [&] {
    attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          dev.max_smem_optin);
  });
  if (attr_err[slot] != cudaSuccess) return cuda_status(attr_err[slot]);
  // Balanced split of a small batch: use the largest cluster size S <= the
  // planned split count whose clusters all fit on the device at once.
  int csize = 0;
  if (prm.balanced && prm.num_splits >= 2 && prm.epilogue == FD_EPILOGUE_FUSED &&
      cluster_enabled()) {
    const int64_t clusters = static_cast<int64_t>(grid.y) * grid.z;
    for (int sz = std::min(prm.num_splits, kMaxClusterSize); sz >= 2; --sz) {
      if (max_active_clusters(kern, smem, sz, dev) >= clusters) {
        csize = sz;
        break;
      }
    }
  }
  if (csize >= 2) {
    prm.num_splits = csize;
    prm.cluster = 1;
    grid.x = static_cast<unsigned>(csize);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int nattr = 1;
  if (csize >= 2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(csize);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    nattr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, prm, mk, mv));
}

template <typename T, int D, bool kAppend>
int dispatch_tma(bool tma, const AttnParams& prm, const CUtensorMap& mk, const CUtensorMap& mv,
                 dim3 grid, size_t smem, const DeviceInfo& dev, cudaStream_t st) {
  if (!tma) return launch<T, D, false, 0, kAppend>(prm, mk, mv, grid, smem, dev, st);
  if constexpr (D == 128) {
    // whole-plane boxes (5-D maps) for 16- and 8-token pages
    if (prm.kperm[3] >= 0) {
      return prm.block_size == 16
                 ? launch<T, D, true, 16, kAppend>(prm, mk, mv, grid, smem, dev, st)
                 : launch<T, D, true, 8, kAppend>(prm, mk, mv, grid, smem, dev, st);
    }
  }
  return launch<T, D, true, 0, kAppend>(prm, mk, mv, grid, smem, dev, st);
}

// The fused-append variant (current token from the call, optional RoPE) is a
// separate instantiation, so the plain decode carries none of its code.
template <typename T, int D>
int dispatch(bool tma, const AttnParams& prm, const CUtensorMap& mk, const CUtensorMap& mv,
             dim3 grid, size_t smem, const DeviceInfo& dev, cudaStream_t st) {
  return prm.fused_append ? dispatch_tma<T, D, true>(tma, prm, mk, mv, grid, smem, dev, st)
                          : dispatch_tma<T, D, false>(tma, prm, mk, mv, grid, smem, dev, st);
}

}  // namespace
}  // namespace fd

using namespace fd;

extern "C" int fd_paged_decode_workspace(const fd_paged_decode_args* a, size_t* scratch_bytes,
                                         int64_t* tickets_needed) {
  int rc = validate(a);
  if (rc) return rc;
  const DeviceInfo* dev = current_device_info();
  if (!dev) return FD_ERR_CUDA;
  const Derived dv = derive(*a);
  const WorkspaceNeed w = workspace_need(*a, dv, make_plan(*a, dv, *dev));
  if (scratch_bytes) *scratch_bytes = w.scratch_bytes;
  if (tickets_needed) *tickets_needed = w.tickets;
  return FD_OK;
}

namespace fd {
namespace {
int paged_decode_impl(const fd_paged_decode_args* a, const int* pre_pages, int pre_slots,
                      void* cuda_stream);
}
}  // namespace fd

extern "C" int fd_paged_decode(const fd_paged_decode_args* a, void* cuda_stream) {
  return fd::paged_decode_impl(a, nullptr, 0, cuda_stream);
}

namespace fd {
namespace {
// fd_paged_decode; pre_pages (cascade tail pass, split schedule only) skips
// each sequence's leading shared pages, and a member's final merge also takes
// the pre_slots prefix partials after the split partials.
int paged_decode_impl(const fd_paged_decode_args* a, const int* pre_pages, int pre_slots,
                      void* cuda_stream) {
  int rc = validate(a);
  if (rc) return rc;
  if (a->num_seqs == 0) return FD_OK;
  const DeviceInfo* dev = current_device_info();
  if (!dev) return FD_ERR_CUDA;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  const Derived dv = derive(*a);
  const Plan plan = make_plan(*a, dv, *dev);
  if (pre_pages && plan.splits == 0) return FD_ERR_INVALID_ARGUMENT;  // split schedule only
  const int grid = plan.grid;
  // split schedule: (split, head block, sequence) -- no division in-kernel
  const dim3 gdim = plan.splits == 0 ? dim3(static_cast<unsigned>(grid))
                                     : dim3(static_cast<unsigned>(plan.splits),
                                            static_cast<unsigned>(dv.nhb),
                                            static_cast<unsigned>(a->num_seqs));
  const WorkspaceNeed need = workspace_need(*a, dv, plan);
  if (need.scratch_bytes > 0 && (!a->scratch || a->scratch_bytes < need.scratch_bytes))
    return FD_ERR_WORKSPACE;
  if (need.tickets > 0 && (!a->tickets || a->tickets_capacity < need.tickets))
    return FD_ERR_WORKSPACE;

  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.num_seqs = a->num_seqs;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.block_size = a->block_size;
  p.num_blocks = a->num_blocks;
  p.max_blocks = a->max_blocks_per_seq;
  p.group = dv.group;
  p.hb_per_kv = dv.hb_per_kv;
  p.rows = dv.rows;
  p.nhb = dv.nhb;
  p.scale_log2 = a->sm_scale * kLog2e;
  p.q = a->q;
  p.qs0 = a->q_stride[0];
  p.qs1 = a->q_stride[1];
  p.qs2 = a->q_stride[2];
  p.out = a->out;
  p.os0 = a->out_stride[0];
  p.os1 = a->out_stride[1];
  p.os2 = a->out_stride[2];
  p.k = a->k_cache;
  p.ks0 = a->k_stride[0];
  p.ks1 = a->k_stride[1];
  p.ks2 = a->k_stride[2];
  p.ks3 = a->k_stride[3];
  p.v = a->v_cache;
  p.vs0 = a->v_stride[0];
  p.vs1 = a->v_stride[1];
  p.vs2 = a->v_stride[2];
  p.vs3 = a->v_stride[3];
  p.bt = a->block_tables;
  p.bt64 = a->block_tables_index == FD_INDEX_I64;
  p.bts0 = a->block_tables_stride[0];
  p.bts1 = a->block_tables_stride[1];
  p.sl = a->seq_lens;
  p.sl64 = a->seq_lens_index == FD_INDEX_I64;
  p.sls = a->seq_lens_stride;
  p.pre_pages = pre_pages;
  p.pre_slots = pre_pages ? pre_slots : 0;
  p.fused_append = a->append_k != nullptr;
  if (p.fused_append) {
    p.ak = a->append_k;
    p.aks0 = a->append_k_stride[0];
    p.aks1 = a->append_k_stride[1];
    p.aks2 = a->append_k_stride[2];
    p.av = a->append_v;
    p.avs0 = a->append_v_stride[0];
    p.avs1 = a->append_v_stride[1];
    p.avs2 = a->append_v_stride[2];
    p.slot = a->slot_mapping;
    p.slot64 = a->slot_mapping_index == FD_INDEX_I64;
    p.slots = a->slot_mapping_stride;
    p.rope_dim = a->rope_dim;
    if (a->rope_dim > 0) {
      p.rope_inv_freq = a->rope_inv_freq;
      p.rope_pos = a->rope_positions;
      p.rope_pos64 = a->rope_positions_index == FD_INDEX_I64;
      p.rope_pos_stride = a->rope_positions_stride;
    }
  }
  p.num_splits = plan.splits;
  p.balanced = plan.balanced;
  p.cap_tiles = plan.cap_tiles;
  p.epilogue = a->epilogue;
  p.min_tiles_per_cta = a->min_tiles_per_cta > 0 ? a->min_tiles_per_cta : 4;
  p.tickets = a->tickets;
  p.status = device_status_ptr();
  if (!p.status) return FD_ERR_CUDA;

  const int D = a->head_dim;
  if (plan.splits == 0) {
    const int64_t slots = static_cast<int64_t>(grid) + static_cast<int64_t>(a->num_seqs) * dv.nhb;
    p.slot_acc = a->scratch;
    p.slot_m = a->scratch + slots * dv.rows * D;
    p.slot_l = p.slot_m + slots * dv.rows;
  } else if (plan.splits > 1 || a->epilogue == FD_EPILOGUE_PARTIALS) {
    if (a->part_acc) {
      p.pacc = a->part_acc;
      p.pas0 = a->part_acc_stride[0];
      p.pas1 = a->part_acc_stride[1];
      p.pas2 = a->part_acc_stride[2];
      p.pas3 = a->part_acc_stride[3];
      p.pmax = a->part_max;
      p.psum = a->part_sum;
      p.pss0 = a->part_stat_stride[0];
      p.pss1 = a->part_stat_stride[1];
      p.pss2 = a->part_stat_stride[2];
    } else {
      const int64_t S = plan.splits;
      p.pacc = a->scratch;
      p.pas3 = 1;
      p.pas2 = D;
      p.pas1 = S * D;
      p.pas0 = static_cast<int64_t>(a->num_q_heads) * S * D;
      p.pmax = a->scratch + static_cast<int64_t>(a->num_seqs) * a->num_q_heads * S * D;
      p.psum = p.pmax + static_cast<int64_t>(a->num_seqs) * a->num_q_heads * S;
      p.pss2 = 1;
      p.pss1 = S;
      p.pss0 = static_cast<int64_t>(a->num_q_heads) * S;
    }
  }

  // loader: TMA when both planes are expressible as tensor maps
  CUtensorMap mk, mv;
  std::memset(&mk, 0, sizeof(mk));
  std::memset(&mv, 0, sizeof(mv));
  bool tma = true;
  for (int plane = 0; plane < 2 && tma; ++plane) {
    CacheDesc cd;
    cd.base = plane ? a->v_cache : a->k_cache;
    cd.elem_bytes = 2;
    cd.is_bf16 = a->dtype == FD_DTYPE_BF16;
    cd.head_dim = D;
    cd.block_size = a->block_size;
    cd.num_heads = a->num_kv_heads;
    cd.num_blocks = a->num_blocks;
    const int64_t* st = plane ? a->v_stride : a->k_stride;
    for (int i = 0; i < 4; ++i) cd.stride[i] = st[i];
    if (cd.num_heads == 1) cd.stride[1] = cd.stride[0];  // size-1 axis: any legal stride
    tma = get_cache_tensor_map(cd, plane ? &mv : &mk, plane ? p.vperm : p.kperm);
  }

  // stream-K: tiles prefix and lengths per sequence, and the start of every
  // CTA's range (grid + 1 entries; the batch has fewer than 2^31 tiles)
  const int sched_ints = (plan.splits == 0) ? (2 * a->num_seqs + 1 + (grid + 1)) : 0;
  if (plan.splits == 0 &&
      static_cast<int64_t>(a->num_seqs) * dv.nhb * plan.cap_tiles >= (int64_t(1) << 31))
    return FD_ERR_UNSUPPORTED;
  // The stage count is sized as if the fused-append area were present, for
  // both variants: tile t is consumed by warp (t mod stages) mod 4, so equal
  // stage counts give the plain and the fused-append launch the same
  // per-warp summation order (bit-identical results for the same tiles).
  const bool fa = p.fused_append != 0;
  const size_t fixed =
      (D == 128 ? smem_bytes<128>(0, sched_ints, true) : smem_bytes<64>(0, sched_ints, true));
  const size_t stage_bytes = (D == 128 ? Smem<128>::kStageBytes : Smem<64>::kStageBytes) + 20;
  const size_t cap = static_cast<size_t>(dev->max_smem_optin);
  if (fixed + 2 * stage_bytes > cap) return FD_ERR_UNSUPPORTED;  // batch too large for the schedule
  int stages = static_cast<int>((cap - fixed) / stage_bytes);
  stages = std::min(stages, kMaxStages);
  // Tile i uses stage i % stages and is consumed by warp (stage % 4): every
  // stage always belongs to the same warp, so each warp waits on a stage's
  // phases in order and a parity wait can never alias a phase one ring
  // ahead, for any stage count of at least four.
  if (stages < kConsumerWarps) return FD_ERR_UNSUPPORTED;
  p.num_stages = stages;
  const size_t smem = D == 128 ? smem_bytes<128>(stages, sched_ints, fa)
                                : smem_bytes<64>(stages, sched_ints, fa);

  const bool bf16 = a->dtype == FD_DTYPE_BF16;
  // Small batches (the balanced split plan) run as one wave of CTAs that fit
  // two per SM, so the next call's CTAs overlap this one (fd_wave_decode.cu).
  if (tma && plan.balanced && !pre_pages && a->epilogue == FD_EPILOGUE_FUSED && wave_enabled()) {
    WaveParams w;
    std::memset(&w, 0, sizeof(w));
    w.num_seqs = p.num_seqs;
    w.num_blocks = p.num_blocks;
    w.max_blocks = p.max_blocks;
    w.block_size = p.block_size;
    w.group = p.group;
    w.hb_per_kv = p.hb_per_kv;
    w.rows = p.rows;
    w.cap_tiles = p.cap_tiles;
    w.scale_log2 = p.scale_log2;
    w.q = p.q;
    w.qs0 = p.qs0;
    w.qs1 = p.qs1;
    w.qs2 = p.qs2;
    w.out = p.out;
    w.os0 = p.os0;
    w.os1 = p.os1;
    w.os2 = p.os2;
    std::copy(p.kperm, p.kperm + 4, w.kperm);
    std::copy(p.vperm, p.vperm + 4, w.vperm);
    w.k = p.k;
    w.ks0 = p.ks0;
    w.ks1 = p.ks1;
    w.ks2 = p.ks2;
    w.v = p.v;
    w.vs0 = p.vs0;
    w.vs1 = p.vs1;
    w.vs2 = p.vs2;
    w.bt = p.bt;
    w.bt64 = p.bt64;
    w.bts0 = p.bts0;
    w.bts1 = p.bts1;
    w.sl = p.sl;
    w.sl64 = p.sl64;
    w.sls = p.sls;
    w.pacc = p.pacc;
    w.pas0 = p.pas0;
    w.pas1 = p.pas1;
    w.pas2 = p.pas2;
    w.pas3 = p.pas3;
    w.pmax = p.pmax;
    w.psum = p.psum;
    w.pss0 = p.pss0;
    w.pss1 = p.pss1;
    w.pss2 = p.pss2;
    w.tickets = p.tickets;
    w.status = p.status;
    w.fused_append = p.fused_append;
    w.ks3 = p.ks3;
    w.vs3 = p.vs3;
    w.ak = p.ak;
    w.aks0 = p.aks0;
    w.aks1 = p.aks1;
    w.aks2 = p.aks2;
    w.av = p.av;
    w.avs0 = p.avs0;
    w.avs1 = p.avs1;
    w.avs2 = p.avs2;
    w.slot = p.slot;
    w.slot64 = p.slot64;
    w.slots = p.slots;
    w.rope_dim = p.rope_dim;
    w.rope_inv_freq = p.rope_inv_freq;
    w.rope_pos = p.rope_pos;
    w.rope_pos64 = p.rope_pos64;
    w.rope_pos_stride = p.rope_pos_stride;
    // head_dim 128: maps whose box is a whole page plane (the 32-token
    // maps above move one 64-dim half per box)
    CUtensorMap wk = mk, wv = mv;
    bool wtma = true;
    w.num_kv_heads = a->num_kv_heads;
    w.spec_skew = wave_spec_skew();
    if (D == 128 && (a->block_size == 32 || a->block_size == 16)) {
      // K and V of a page in one box: a token-major pair of caches with
      // evenly spaced planes, or vLLM's per-block interleaved planes
      CacheDesc cd;
      cd.base = a->k_cache;
      cd.elem_bytes = 2;
      cd.is_bf16 = a->dtype == FD_DTYPE_BF16;
      cd.head_dim = D;
      cd.block_size = a->block_size;
      cd.num_heads = a->num_kv_heads;
      cd.num_blocks = a->num_blocks;
      for (int i = 0; i < 4; ++i) cd.stride[i] = a->k_stride[i];
      w.kv_box = kv_pair_enabled() &&
                 get_kv_pair_tensor_map(cd, a->v_cache, a->v_stride, &wk, &w.v_first, w.pair_m);
    }
    if (D == 128 && a->block_size == 32 && !w.kv_box) {
      for (int plane = 0; plane < 2 && wtma; ++plane) {
        CacheDesc cd;
        cd.base = plane ? a->v_cache : a->k_cache;
        cd.elem_bytes = 2;
        cd.is_bf16 = a->dtype == FD_DTYPE_BF16;
        cd.head_dim = D;
        cd.block_size = a->block_size;
        cd.num_heads = a->num_kv_heads;
        cd.num_blocks = a->num_blocks;
        const int64_t* st = plane ? a->v_stride : a->k_stride;
        for (int i = 0; i < 4; ++i) cd.stride[i] = st[i];
        if (cd.num_heads == 1) cd.stride[1] = cd.stride[0];
        cd.plane_box = 1;
        wtma = get_cache_tensor_map(cd, plane ? &wv : &wk, plane ? w.vperm : w.kperm);
      }
    }
    if (wtma) {
      const int page_rows = (D == 128 && a->block_size < 32) ? a->block_size : 0;
      const int wrc = wave_decode(w, wk, wv, bf16, D, page_rows, gdim, *dev, stream);
      if (wrc != FD_ERR_UNSUPPORTED) return wrc;
    }
  }
  if (D == 128) {
    return bf16 ? dispatch<__nv_bfloat16, 128>(tma, p, mk, mv, gdim, smem, *dev, stream)
                : dispatch<__half, 128>(tma, p, mk, mv, gdim, smem, *dev, stream);
  }
  return bf16 ? dispatch<__nv_bfloat16, 64>(tma, p, mk, mv, gdim, smem, *dev, stream)
              : dispatch<__half, 64>(tma, p, mk, mv, gdim, smem, *dev, stream);
}

}  // namespace
}  // namespace fd

extern "C" int fd_split_kv_reduce(const fd_split_kv_reduce_args* a, void* cuda_stream) {
  if (!a || a->struct_size != static_cast<int32_t>(sizeof(fd_split_kv_reduce_args)))
    return FD_ERR_INVALID_ARGUMENT;
  if (a->dtype != FD_DTYPE_F16 && a->dtype != FD_DTYPE_BF16 && a->dtype != FD_DTYPE_F32)
    return FD_ERR_UNSUPPORTED;
  if (a->num_seqs < 0 || a->num_q_heads <= 0 || a->head_dim <= 0 || a->num_splits <= 0)
    return FD_ERR_INVALID_ARGUMENT;
  if (a->num_splits > kReduceMaxSlots) return FD_ERR_UNSUPPORTED;
  if (!a->part_acc || !a->part_max || !a->part_sum || !a->seq_lens || !a->out)
    return FD_ERR_INVALID_ARGUMENT;
  if (a->num_seqs == 0) return FD_OK;
  ReduceParams p;
  std::memset(&p, 0, sizeof(p));
  p.num_seqs = a->num_seqs;
  p.num_q_heads = a->num_q_heads;
  p.head_dim = a->head_dim;
  p.num_splits = a->num_splits;
  p.acc = a->part_acc;
  p.as0 = a->part_acc_stride[0];
  p.as1 = a->part_acc_stride[1];
  p.as2 = a->part_acc_stride[2];
  p.as3 = a->part_acc_stride[3];
  p.mx = a->part_max;
  p.sm = a->part_sum;
  p.ss0 = a->part_stat_stride[0];
  p.ss1 = a->part_stat_stride[1];
  p.ss2 = a->part_stat_stride[2];
  p.sl = a->seq_lens;
  p.sl64 = a->seq_lens_index == FD_INDEX_I64;
  p.sls = a->seq_lens_stride;
  p.slot = a->slot_mapping;
  p.slot64 = a->slot_mapping_index == FD_INDEX_I64;
  p.slots = a->slot_mapping_stride;
  p.out = a->out;
  p.os0 = a->out_stride[0];
  p.os1 = a->out_stride[1];
  p.os2 = a->out_stride[2];
  dim3 grid(a->num_seqs, a->num_q_heads);
  const int threads = a->head_dim >= 128 ? 128 : 64;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  switch (a->dtype) {
    case FD_DTYPE_BF16:
      return cuda_status(launch_pdl(split_reduce_kernel<__nv_bfloat16>, grid, dim3(threads), 0,
                                    stream, p));
    case FD_DTYPE_F16:
      return cuda_status(launch_pdl(split_reduce_kernel<__half>, grid, dim3(threads), 0, stream, p));
    default:
      return cuda_status(launch_pdl(split_reduce_kernel<float>, grid, dim3(threads), 0, stream, p));
  }
}

// ---------------------------------------------------------------------------
// cascade (shared-prefix) decode
// ---------------------------------------------------------------------------
namespace fd {
namespace {

struct CascadePlan {
  int chunks, splits, row_blocks;
  bool umma;  // prefix pass on tcgen05 (head_dim 128, 32-token pages)
};

// Host checks of the group description (it is copied into the prefix
// kernel's launch parameters).
int cascade_check(const fd_paged_decode_args* a, const fd_cascade_args* c) {
  int rc = validate(a);
  if (rc) return rc;
  if (!c || c->struct_size != static_cast<int32_t>(sizeof(fd_cascade_args)))
    return FD_ERR_INVALID_ARGUMENT;
  if (c->num_groups <= 0 || !c->group_start || !c->group_members || !c->group_pages ||
      !c->seq_prefix_pages || c->chunks < 0 || c->tail_splits < 0 || c->chunks > 256 ||
      c->tail_splits > 256)
    return FD_ERR_INVALID_ARGUMENT;
  if (c->num_groups > kCascadeMaxGroups) return FD_ERR_UNSUPPORTED;
  if (c->group_start[0] != 0) return FD_ERR_INVALID_ARGUMENT;
  const int total = c->group_start[c->num_groups];
  if (total > kCascadeMaxMembers) return FD_ERR_UNSUPPORTED;
  for (int g = 0; g < c->num_groups; ++g) {
    if (c->group_start[g + 1] <= c->group_start[g]) return FD_ERR_INVALID_ARGUMENT;
    const int64_t tok = static_cast<int64_t>(c->group_pages[g]) * a->block_size;
    if (c->group_pages[g] <= 0 || c->group_pages[g] > a->max_blocks_per_seq || tok % kTile)
      return FD_ERR_INVALID_ARGUMENT;
  }
  for (int i = 0; i < total; ++i) {
    if (c->group_members[i] < 0 || c->group_members[i] >= a->num_seqs)
      return FD_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(c->num_groups) * a->num_kv_heads > 65535) return FD_ERR_UNSUPPORTED;
  return FD_OK;
}

CascadePlan cascade_plan(const fd_paged_decode_args& a, const fd_cascade_args& c,
                         const Derived& dv, const DeviceInfo& dev) {
  CascadePlan pl;
  int max_members = 0, max_tiles = 0;
  for (int g = 0; g < c.num_groups; ++g) {
    max_members = std::max(max_members, c.group_start[g + 1] - c.group_start[g]);
    max_tiles = std::max(max_tiles, c.group_pages[g] * a.block_size / kTile);
  }
  const int64_t rows = static_cast<int64_t>(max_members) * dv.group;
  pl.row_blocks = static_cast<int>((rows + kPrefixRows - 1) / kPrefixRows);
  // The concurrent cascade shares the SMs between the two passes, and its
  // prefix pass is fastest as many short mma.sync chunks (c5 layer: 24.5 us
  // against 26.1 us for the best tcgen05 split); the serial cascade uses
  // the tcgen05 pass.
  const bool conc = cascade_concurrent_enabled();
  pl.umma = a.head_dim == 128 && a.block_size == 32 && prefix_umma_enabled() && !conc;
  const int64_t units = static_cast<int64_t>(c.num_groups) * a.num_kv_heads * pl.row_blocks;
  if (c.chunks > 0) {
    pl.chunks = c.chunks;
  } else {
    // about one prefix CTA per SM, at least two tiles per chunk
    int64_t ch = (dev.num_sms + units - 1) / units;
    ch = std::min<int64_t>(ch, std::max(1, max_tiles / 2));
    pl.chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ch, 32)));
  }
  if (pl.umma) {
    // a UMMA prefix CTA holds its whole chunk in shared memory
    pl.chunks = std::max(pl.chunks, (max_tiles + kUmmaMaxTiles - 1) / kUmmaMaxTiles);
  }
  if (c.tail_splits > 0) {
    pl.splits = c.tail_splits;
  } else {
    const int64_t pairs = std::max<int64_t>(1, static_cast<int64_t>(a.num_seqs) * dv.nhb);
    // serial: the tail has every SM; concurrent: the SMs the prefix CTAs leave
    const int64_t sms = conc ? std::max<int64_t>(pairs, dev.num_sms - pl.chunks * units)
                             : dev.num_sms;
    const int64_t s = conc ? sms / pairs : (sms + pairs - 1) / pairs;
    pl.splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(s, 8)));
  }
  return pl;
}

size_t cascade_scratch_bytes(const fd_paged_decode_args& a, const CascadePlan& pl) {
  return static_cast<size_t>(a.num_seqs) * a.num_q_heads * (pl.splits + pl.chunks) *
         (a.head_dim + 2) * sizeof(float);
}

template <typename T, int D, int kPageRows>
int launch_prefix(const PrefixParams& prm, const CUtensorMap& mk, const CUtensorMap& mv,
                  dim3 grid, size_t smem, const DeviceInfo& dev, cudaStream_t stream, bool pdl) {
  auto kern = prefix_kernel<T, D, kPageRows>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  const int slot = dev.device & 63;
  std::call_once(once[slot], [&] {
    attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          dev.max_smem_optin);
  });
  if (attr_err[slot] != cudaSuccess) return cuda_status(attr_err[slot]);
  return cuda_status(pdl ? launch_pdl(kern, grid, dim3(kPrefixThreads), smem, stream, prm, mk, mv)
                         : launch_plain(kern, grid, dim3(kPrefixThreads), smem, stream, prm, mk, mv));
}

template <typename T>
int launch_prefix_umma(const PrefixParams& prm, const CUtensorMap& mk, const CUtensorMap& mv,
                       dim3 grid, const DeviceInfo& dev, cudaStream_t stream, bool pdl) {
  auto kern = prefix_umma_kernel<T>;
  const size_t smem = prefix_umma_smem_bytes();
  if (smem > static_cast<size_t>(dev.max_smem_optin)) return FD_ERR_UNSUPPORTED;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  const int slot = dev.device & 63;
  std::call_once(once[slot], [&] {
    attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
  });
  if (attr_err[slot] != cudaSuccess) return cuda_status(attr_err[slot]);
  return cuda_status(pdl ? launch_pdl(kern, grid, dim3(kThreads), smem, stream, prm, mk, mv)
                         : launch_plain(kern, grid, dim3(kThreads), smem, stream, prm, mk, mv));
}

template <typename T, int D>
int dispatch_prefix(const PrefixParams& prm, const CUtensorMap& mk, const CUtensorMap& mv,
                    dim3 grid, size_t smem, const DeviceInfo& dev, cudaStream_t st, bool pdl) {
  if constexpr (D == 128) {
    if (prm.kperm[3] >= 0) {
      return prm.block_size == 16
                 ? launch_prefix<T, D, 16>(prm, mk, mv, grid, smem, dev, st, pdl)
                 : launch_prefix<T, D, 8>(prm, mk, mv, grid, smem, dev, st, pdl);
    }
  }
  return launch_prefix<T, D, 0>(prm, mk, mv, grid, smem, dev, st, pdl);
}

// Per-device second stream and fork / join events of the concurrent cascade
// (created on the first such call on the device, with that device current;
// a mutex keeps calls from different host threads from interleaving their
// fork and join).
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex mu;
  cudaError_t err = cudaSuccess;
};
SideStream g_side[64];
std::once_flag g_side_once[64];

SideStream* side_stream(int device) {
  SideStream& ss = g_side[device & 63];
  std::call_once(g_side_once[device & 63], [&] {
    ss.err = cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking);
    if (ss.err == cudaSuccess) ss.err = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming);
    if (ss.err == cudaSuccess) ss.err = cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming);
  });
  return ss.err == cudaSuccess ? &ss : nullptr;
}

template <typename T>
int launch_reduce(const ReduceParams& p, int head_dim, cudaStream_t stream) {
  const dim3 grid(p.num_seqs, p.num_q_heads);
  const int threads = head_dim >= 128 ? 128 : 64;
  return cuda_status(launch_plain(split_reduce_kernel<T>, grid, dim3(threads), 0, stream, p));
}

}  // namespace
}  // namespace fd

extern "C" int fd_cascade_workspace(const fd_paged_decode_args* a, const fd_cascade_args* c,
                                    size_t* scratch_bytes, int64_t* tickets_needed) {
  int rc = cascade_check(a, c);
  if (rc) return rc;
  const DeviceInfo* dev = current_device_info();
  if (!dev) return FD_ERR_CUDA;
  const Derived dv = derive(*a);
  const CascadePlan pl = cascade_plan(*a, *c, dv, *dev);
  if (scratch_bytes) *scratch_bytes = cascade_scratch_bytes(*a, pl);
  if (tickets_needed) *tickets_needed = static_cast<int64_t>(a->num_seqs) * dv.nhb;
  return FD_OK;
}

extern "C" int fd_cascade_decode(const fd_paged_decode_args* a, const fd_cascade_args* c,
                                 void* cuda_stream) {
  int rc = cascade_check(a, c);
  if (rc) return rc;
  if (a->num_seqs == 0) return FD_OK;
  const DeviceInfo* dev = current_device_info();
  if (!dev) return FD_ERR_CUDA;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  const Derived dv = derive(*a);
  const CascadePlan pl = cascade_plan(*a, *c, dv, *dev);
  if (!a->scratch || a->scratch_bytes < cascade_scratch_bytes(*a, pl)) return FD_ERR_WORKSPACE;
  if (!a->tickets || a->tickets_capacity < static_cast<int64_t>(a->num_seqs) * dv.nhb)
    return FD_ERR_WORKSPACE;
  const int D = a->head_dim;
  const int64_t slots = pl.splits + pl.chunks;
  float* acc = a->scratch;
  float* mx = acc + static_cast<int64_t>(a->num_seqs) * a->num_q_heads * slots * D;
  float* sm = mx + static_cast<int64_t>(a->num_seqs) * a->num_q_heads * slots;

  // ---- prefix pass ----
  PrefixParams pp;
  std::memset(&pp, 0, sizeof(pp));
  pp.num_seqs = a->num_seqs;
  pp.num_kv_heads = a->num_kv_heads;
  pp.group = dv.group;
  pp.block_size = a->block_size;
  pp.num_blocks = a->num_blocks;
  pp.max_blocks = a->max_blocks_per_seq;
  pp.scale_log2 = a->sm_scale * kLog2e;
  pp.q = a->q;
  pp.qs0 = a->q_stride[0];
  pp.qs1 = a->q_stride[1];
  pp.qs2 = a->q_stride[2];
  if (a->rope_dim > 0) {
    pp.rope_dim = a->rope_dim;
    pp.rope_inv_freq = a->rope_inv_freq;
    pp.rope_pos = a->rope_positions;
    pp.rope_pos64 = a->rope_positions_index == FD_INDEX_I64;
    pp.rope_pos_stride = a->rope_positions_stride;
  }
  pp.bt = a->block_tables;
  pp.bt64 = a->block_tables_index == FD_INDEX_I64;
  pp.bts0 = a->block_tables_stride[0];
  pp.bts1 = a->block_tables_stride[1];
  for (int g = 0; g <= c->num_groups; ++g) pp.grp_start[g] = c->group_start[g];
  for (int g = 0; g < c->num_groups; ++g) pp.grp_pages[g] = c->group_pages[g];
  for (int i = 0; i < c->group_start[c->num_groups]; ++i) pp.grp_members[i] = c->group_members[i];
  pp.chunks = pl.chunks;
  pp.pacc = acc;
  pp.pas3 = 1;
  pp.pas2 = D;
  pp.pas1 = slots * D;
  pp.pas0 = static_cast<int64_t>(a->num_q_heads) * slots * D;
  pp.pmax = mx;
  pp.psum = sm;
  pp.pss2 = 1;
  pp.pss1 = slots;
  pp.pss0 = static_cast<int64_t>(a->num_q_heads) * slots;
  pp.slot0 = pl.splits;
  pp.status = device_status_ptr();
  if (!pp.status) return FD_ERR_CUDA;
  CUtensorMap mk, mv;
  std::memset(&mk, 0, sizeof(mk));
  std::memset(&mv, 0, sizeof(mv));
  for (int plane = 0; plane < 2; ++plane) {
    CacheDesc cd;
    cd.base = plane ? a->v_cache : a->k_cache;
    cd.elem_bytes = 2;
    cd.is_bf16 = a->dtype == FD_DTYPE_BF16;
    cd.head_dim = D;
    cd.block_size = a->block_size;
    cd.num_heads = a->num_kv_heads;
    cd.num_blocks = a->num_blocks;
    const int64_t* st = plane ? a->v_stride : a->k_stride;
    for (int i = 0; i < 4; ++i) cd.stride[i] = st[i];
    if (cd.num_heads == 1) cd.stride[1] = cd.stride[0];
    if (!get_cache_tensor_map(cd, plane ? &mv : &mk, plane ? pp.vperm : pp.kperm))
      return FD_ERR_UNSUPPORTED;
  }
  const size_t fixed = D == 128 ? prefix_smem_bytes<128>(0) : prefix_smem_bytes<64>(0);
  const size_t stage_bytes = (D == 128 ? Smem<128>::kStageBytes : Smem<64>::kStageBytes) + 16;
  const size_t cap = static_cast<size_t>(dev->max_smem_optin);
  if (fixed + 2 * stage_bytes > cap) return FD_ERR_UNSUPPORTED;
  const int stages = std::min(static_cast<int>((cap - fixed) / stage_bytes), kMaxStages);
  pp.num_stages = stages;
  const size_t psmem = D == 128 ? prefix_smem_bytes<128>(stages) : prefix_smem_bytes<64>(stages);
  const dim3 pgrid(static_cast<unsigned>(pl.chunks), static_cast<unsigned>(pl.row_blocks),
                   static_cast<unsigned>(c->num_groups * a->num_kv_heads));
  const bool bf16 = a->dtype == FD_DTYPE_BF16;
  auto launch_prefix_pass = [&](cudaStream_t st, bool pdl) {
    if (pl.umma && pp.kperm[3] < 0) {
      return bf16 ? launch_prefix_umma<__nv_bfloat16>(pp, mk, mv, pgrid, *dev, st, pdl)
                  : launch_prefix_umma<__half>(pp, mk, mv, pgrid, *dev, st, pdl);
    }
    if (D == 128) {
      return bf16 ? dispatch_prefix<__nv_bfloat16, 128>(pp, mk, mv, pgrid, psmem, *dev, st, pdl)
                  : dispatch_prefix<__half, 128>(pp, mk, mv, pgrid, psmem, *dev, st, pdl);
    }
    return bf16 ? dispatch_prefix<__nv_bfloat16, 64>(pp, mk, mv, pgrid, psmem, *dev, st, pdl)
                : dispatch_prefix<__half, 64>(pp, mk, mv, pgrid, psmem, *dev, st, pdl);
  };

  // tail pass: split decode after the shared pages, partials in slots [0, S)
  fd_paged_decode_args t = *a;
  t.num_splits = pl.splits;
  t.part_acc = acc;
  t.part_acc_stride[0] = pp.pas0;
  t.part_acc_stride[1] = pp.pas1;
  t.part_acc_stride[2] = pp.pas2;
  t.part_acc_stride[3] = 1;
  t.part_max = mx;
  t.part_sum = sm;
  t.part_stat_stride[0] = pp.pss0;
  t.part_stat_stride[1] = pp.pss1;
  t.part_stat_stride[2] = 1;

  if (!cascade_concurrent_enabled()) {
    // prefix pass, then the tail, whose pair-last CTA merges the S tail
    // splits and (members) the C prefix chunks through the tickets
    rc = launch_prefix_pass(stream, true);
    if (rc) return rc;
    t.epilogue = FD_EPILOGUE_FUSED;
    return paged_decode_impl(&t, c->seq_prefix_pages, pl.chunks, cuda_stream);
  }

  // Concurrent: the prefix pass runs on a second stream beside the tail pass
  // (neither reads what the other writes; together they fit the SMs of a
  // small batch), then one reduction merges S tail + C prefix partials per
  // member row and the S tail partials of the other rows.
  SideStream* ss = side_stream(dev->device);
  if (!ss) return FD_ERR_CUDA;
  std::lock_guard<std::mutex> lock(ss->mu);
  cudaError_t e = cudaEventRecord(ss->fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ss->stream, ss->fork, 0);
  if (e != cudaSuccess) return cuda_status(e);
  int prc = launch_prefix_pass(ss->stream, false);
  // the join is recorded and waited on whatever happened, so the caller's
  // stream (or its capture) never leaves the second stream behind
  e = cudaEventRecord(ss->join, ss->stream);
  t.epilogue = FD_EPILOGUE_PARTIALS;
  int trc = paged_decode_impl(&t, c->seq_prefix_pages, 0, cuda_stream);
  const cudaError_t e2 = cudaStreamWaitEvent(stream, ss->join, 0);
  if (prc) return prc;
  if (trc) return trc;
  if (e != cudaSuccess) return cuda_status(e);
  if (e2 != cudaSuccess) return cuda_status(e2);

  ReduceParams rp;
  std::memset(&rp, 0, sizeof(rp));
  rp.num_seqs = a->num_seqs;
  rp.num_q_heads = a->num_q_heads;
  rp.head_dim = D;
  rp.num_splits = pl.splits;
  rp.pre_pages = c->seq_prefix_pages;
  rp.pre_slots = pl.chunks;
  rp.acc = acc;
  rp.as0 = pp.pas0;
  rp.as1 = pp.pas1;
  rp.as2 = pp.pas2;
  rp.as3 = 1;
  rp.mx = mx;
  rp.sm = sm;
  rp.ss0 = pp.pss0;
  rp.ss1 = pp.pss1;
  rp.ss2 = 1;
  rp.sl = a->seq_lens;
  rp.sl64 = a->seq_lens_index == FD_INDEX_I64;
  rp.sls = a->seq_lens_stride;
  rp.slot = a->slot_mapping;
  rp.slot64 = a->slot_mapping_index == FD_INDEX_I64;
  rp.slots = a->slot_mapping_stride;
  rp.out = a->out;
  rp.os0 = a->out_stride[0];
  rp.os1 = a->out_stride[1];
  rp.os2 = a->out_stride[2];
  return bf16 ? launch_reduce<__nv_bfloat16>(rp, D, stream) : launch_reduce<__half>(rp, D, stream);
}
