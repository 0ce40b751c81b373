// Paged single-token decode for small batches on B200 (sm_100a): one wave.
//
// Covers the reference's split-KV decode (flashdec/kernels/paged_decode.py:
// grouped GQA :124-327, split :330-543, reducer :546-642) for batches whose
// (sequence, head block) pairs are few enough to split: every pair gets S
// CTAs (grid = S x head blocks x sequences, S * pairs <= SMs) and each CTA
// streams an equal range of the pair's 32-token tiles.
//
// A decode batch of this size moves a few MB, so the design is about
// latency:
//  * 192 threads and at most 112 KB of shared memory, so two CTAs fit on one
//    SM.  With programmatic dependent launch the CTAs of the next call on the
//    stream become resident while this call still runs; before
//    griddepcontrol.wait their prefetch warp (warp 5) prefetches the pages
//    they will read into L2.  The sequence length and block-table entries it
//    reads for that (through L2, no L1 allocation) may be stale, because the
//    previous kernel may still be writing them: they only choose what to
//    prefetch, and a prefetch cannot make any later read stale (L2 is where
//    every SM's writes become visible).  Every load that feeds the result is
//    made after the wait.
//  * warp 4 resolves the block table and issues the TMA boxes into a ring of
//    stages (one "full" mbarrier per tile, one "empty" mbarrier per stage).
//  * warps 0-3 take the tiles in turn (tile i: warp i % 4).  S^T = K Q^T runs
//    with tokens as the mma M dimension (a GQA group of up to 8 query heads
//    is one n8 tile, so no half-empty M tile is multiplied), the softmax is
//    per query head in fp32 (base 2, scale folded in), and O^T += V^T P^T
//    (P^T moves from the accumulator layout into the B operand by
//    movmatrix).  The four warps' (max, sum, acc) are merged in the idle
//    stage ring at the end.
//  * the S partials of a pair are merged either inside a thread-block
//    cluster (each CTA pushes its rows into the row owner's shared memory
//    and arrives on the owner's mbarrier; the owner merges and stores) or,
//    when the clusters do not all fit, by the CTA that takes the pair's last
//    ticket (atom.add.acq_rel.gpu), which re-arms the ticket for the next
//    call.  No CTA waits for another CTA that is not resident.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "fd_host.h"
#include "fd_ptx.cuh"
#include "fd_tile.cuh"
#include "fd_wave_decode.h"

namespace fd {

namespace {

constexpr int kWaveConsumerWarps = 4;
constexpr int kWaveProducerWarp = 4;
constexpr int kWavePrefetchWarp = 5;
constexpr int kWaveThreads = 32 * 6;
constexpr int kWaveConsumerThreads = 32 * kWaveConsumerWarps;
constexpr int kWaveTileBars = 32;    // tile i completes on full barrier i % 32
constexpr int kWaveMaxStages = 16;
constexpr int kWaveMiscInts = 16;    // [0] abort, [1] last ticket, [2] prefetch hint,
                                     // [3] cluster merge arrived, [4..5] appended slot,
                                     // [6] speculative first page, [7] speculative length + 1,
                                     // [8] speculative window ready
constexpr int kWaveBarConsumers = 1;  // named barrier of the consumer warps
constexpr int kWavePrefetchPages = 64;
// barriers (full, empty, cluster merge), tile masks, misc
constexpr int kWaveCtlBytes = (2 * kWaveTileBars + kWaveMaxStages + 2) * 8 + kWaveTileBars * 4 +
                              kWaveMiscInts * 4 + 2 * 64 * 4 + 2 * 128 * 2 + 32 * 4;
// Shared-memory budget that keeps two CTAs resident per SM (228 KB per SM,
// 1 KB reserved per CTA).
constexpr size_t kWaveSmemBudget = 112 * 1024;

template <int D>
struct WaveSmem {
  static constexpr int kHalves = D / 64;
  static constexpr int kHalfBytes = kTile * 128;  // [32 rows][64 dims] x 2 B
  static constexpr int kStageBytes = 2 * kHalves * kHalfBytes;
  // q rows in the tile layout (16 of its 32 rows)
  static constexpr int kQBytes = kHalves * kHalfBytes;
  // the four warps' fp32 [16 rows][D] accumulators and (max, sum), staged in
  // the stage ring for the merge inside the CTA
  static constexpr int kWarpMergeBytes = kWaveConsumerWarps * 16 * (D * 4 + 8);
};

// Column of (row, dim) in fp32 rows of D floats: dims XORed with
// 8 * ((row / 2) % 4), so that the four heads one store instruction covers
// land on different banks (float4 groups stay contiguous).
__device__ __forceinline__ int wave_col(int row, int d) { return d ^ (((row >> 1) & 3) << 3); }

template <typename T>
__device__ __forceinline__ void wave_store_out4(const WaveParams& p, int b, int h, int d, float a0,
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

// Tokens attended by a sequence of length n, clamped to the block-table capacity.
__device__ __forceinline__ int64_t wave_clamp_len(const WaveParams& p, int64_t n) {
  const int64_t cap = static_cast<int64_t>(p.max_blocks) * p.block_size;
  return n < 0 ? 0 : (n > cap ? cap : n);
}

// Equal tile ranges (within one tile) of `tiles` over `splits` CTAs.
__device__ __forceinline__ void wave_range(int split, int splits, int tiles, int& t0, int& t1) {
  t0 = static_cast<int>(static_cast<uint32_t>(split) * static_cast<uint32_t>(tiles) /
                        static_cast<uint32_t>(splits));
  t1 = static_cast<int>(static_cast<uint32_t>(split + 1) * static_cast<uint32_t>(tiles) /
                        static_cast<uint32_t>(splits));
}

// Tokens of one tile whose page is valid, as a 32-bit row mask (bit r = token
// r of the tile), from the per-page validity bits of the tile.
__device__ __forceinline__ uint32_t wave_page_rows(uint32_t pmask, int bs_shift) {
  if (bs_shift == 5) return (pmask & 1u) ? 0xffffffffu : 0u;
  uint32_t m = 0;
  const int ppt = 32 >> bs_shift;
  const uint32_t page_bits = (1u << (1 << bs_shift)) - 1u;
  for (int j = 0; j < ppt; ++j) {
    if ((pmask >> j) & 1u) m |= page_bits << (j << bs_shift);
  }
  return m;
}

template <typename T, int D, int kPageRows, int kNT, bool kCluster, bool kAppend>
__global__ void __launch_bounds__(kWaveThreads, 2)
    wave_decode_kernel(const __grid_constant__ WaveParams p,
                       const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v) {
  using SM = WaveSmem<D>;
  using SS = StageStrides<kPageRows>;
  constexpr int kMTD = D / 16;                // m16 tiles of head_dim in O^T
  constexpr int kKS = D / 16;                 // k16 steps of Q K^T
  constexpr int kQA = kNT == 1 ? 2 : 1;       // independent Q K^T accumulator sets
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int NST = p.num_stages;
  uint8_t* stages = smem;
  uint8_t* qbuf = stages + NST * SM::kStageBytes;  // q rows
  uint8_t* rbuf = qbuf + SM::kQBytes;               // cluster receive area (recv_bytes)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(rbuf + p.recv_bytes);
  uint64_t* empty_bar = full_bar + kWaveTileBars;
  uint64_t* merge_bar = empty_bar + kWaveMaxStages;
  // "verified": tile i's pages are the ones the real block table names (the
  // first group may be issued from the prefetch warp's speculative read)
  uint64_t* ver_bar = merge_bar + 2;
  uint32_t* tile_mask = reinterpret_cast<uint32_t*>(ver_bar + kWaveTileBars);
  int* misc = reinterpret_cast<int*>(tile_mask + kWaveTileBars);
  // fused append: the appended token's slot (misc[4..5]), the cos / sin of
  // its position per pair index, and its K (rotated) and V rows
  int64_t* app_slot = reinterpret_cast<int64_t*>(misc + 4);
  float* rope_tab = reinterpret_cast<float*>(misc + kWaveMiscInts);  // [2][64]
  T* app_row = reinterpret_cast<T*>(rope_tab + 2 * 64);              // [2][D]
  int* spec_win = reinterpret_cast<int*>(app_row + 2 * 128);           // [32] speculative block ids

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = static_cast<int>(blockIdx.x);
  const int S = static_cast<int>(gridDim.x);
  const int hb = static_cast<int>(blockIdx.y);
  const int b = static_cast<int>(blockIdx.z);
  const int kv_head = hb / p.hb_per_kv;
  const int jb = hb - kv_head * p.hb_per_kv;
  const int head0 = kv_head * p.group + jb * p.rows;
  const int nrows = min(p.rows, p.group - jb * p.rows);
  const int bs = p.block_size;
  const int ppt_shift = bs == 32 ? 0 : (bs == 16 ? 1 : 2);  // log2(pages per tile)
  const int bs_shift = 5 - ppt_shift;                        // log2(block_size)
  volatile int* abort_flag = misc;

  // The next kernel of the stream may become resident now; it waits for
  // this one to finish before it reads anything this one writes.
  pdl_launch_dependents();
  if (tid < kWaveTileBars) {
    mbar_init(smem_u32(&full_bar[tid]), 1);
    mbar_init(smem_u32(&ver_bar[tid]), 1);
  }
  if (tid >= 32 && tid < 32 + NST) mbar_init(smem_u32(&empty_bar[tid - 32]), 1);
  if (kCluster && tid == 64) {
    // The peers' pushes land on this CTA's merge barrier as bytes (st.async);
    // the barrier is armed now with all it will receive: every split's
    // (max, sum, acc) of each row this CTA finishes (rows r with r % S ==
    // its cluster rank).
    const int rank = static_cast<int>(cluster_ctarank());
    const int owned = rank < nrows ? (nrows - rank + S - 1) / S : 0;
    mbar_init(smem_u32(merge_bar), 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(smem_u32(merge_bar), static_cast<uint32_t>(owned * S * (D * 4 + 8)));
  }
  if (tid < kWaveMiscInts) misc[tid] = 0;
  if (tid < 32 + NST || tid == 64) fence_mbar_init();
  if (warp == kWaveProducerWarp && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  __syncthreads();
  // Cluster barrier: every thread arrives now (the merge barrier's init is
  // ordered before it by fence.mbarrier_init); the consumers wait on it
  // before their first store into another CTA.
  if constexpr (kCluster) cluster_arrive_relaxed();

  // =========================================================================
  // prefetch warp: L2 prefetch of this CTA's pages and q rows, then exit
  // =========================================================================
  if (warp == kWavePrefetchWarp) {
    int64_t n = 0;
    if (lane == 0) n = wave_clamp_len(p, load_index_cg(p.sl, p.sl64, static_cast<int64_t>(b) * p.sls));
    n = __shfl_sync(0xffffffffu, n, 0);
    if (lane == 0) abort_flag[2] = static_cast<int>(n) + 1;  // hint for the producer (volatile)
    const int tiles = static_cast<int>((n + kTile - 1) / kTile);
    int t0, t1;
    wave_range(split, S, tiles, t0, t1);
    const int64_t nlb = ((kAppend && n > 0 ? n - 1 : n) + bs - 1) >> bs_shift;
    const int64_t pg0 = static_cast<int64_t>(t0) << ppt_shift;
    int64_t pg1 = min(static_cast<int64_t>(t1) << ppt_shift, nlb);
    pg1 = min(pg1, pg0 + kWavePrefetchPages);
    // block ids first (one per lane), then each page: one TMA prefetch of
    // its K and V planes through the pair map when there is one, else every
    // 128-byte line of its K and V rows with all 32 lanes (one warp
    // instruction covers 32 lines) through the load unit
    constexpr int kLinesPerRow = D * 2 / 128;
    const int lines = bs * kLinesPerRow;  // lines of one page plane
    for (int64_t lb0 = pg0; lb0 < pg1; lb0 += 32) {
      const int64_t lb = lb0 + lane;
      int64_t blk = -1;
      if (lb < pg1) blk = load_index_cg(p.bt, p.bt64, static_cast<int64_t>(b) * p.bts0 + lb * p.bts1);
      const int npg = static_cast<int>(min(static_cast<int64_t>(32), pg1 - lb0));
      if (lb0 == pg0) {
        // the first window, for the producer to issue from before its own
        // (real) read of the block table returns
        spec_win[lane] = (p.spec_skew && blk >= 0)
                             ? static_cast<int>((blk + p.spec_skew) % p.num_blocks)
                             : static_cast<int>(blk);
        __syncwarp();
        if (lane == 0) {
          abort_flag[6] = static_cast<int>(pg0);
          abort_flag[7] = static_cast<int>(n) + 1;
          __threadfence_block();
          abort_flag[8] = 1;
        }
      }
      for (int j = 0; j < npg; ++j) {
        const int64_t bj = __shfl_sync(0xffffffffu, blk, j);
        if (bj < 0 || bj >= p.num_blocks) continue;  // warp-uniform
        if (p.kv_box) {
          // one TMA prefetch per page through the K + V pair map (cheaper to
          // issue than 256 line prefetches)
          if (lane == 0) {
            tma_prefetch_5d(&tmap_k, 0, 0, 0,
                            static_cast<int>(bj) * p.pair_m[0] + kv_head * p.pair_m[1],
                            static_cast<int>(bj) * p.pair_m[2]);
          }
          continue;
        }
        const char* kp = static_cast<const char*>(p.k) + (bj * p.ks0 + kv_head * p.ks1) * 2;
        const char* vp = static_cast<const char*>(p.v) + (bj * p.vs0 + kv_head * p.vs1) * 2;
        for (int e = lane; e < lines; e += 32) {
          const int r = e / kLinesPerRow;
          const int c = e - r * kLinesPerRow;
          prefetch_l2(kp + r * p.ks2 * 2 + c * 128);
          prefetch_l2(vp + r * p.vs2 * 2 + c * 128);
        }
      }
    }
    // q rows of the head block (D * 2 bytes each: one or two 128-byte lines)
    if (p.qs2 == 1) {
      constexpr int kLines = D * 2 / 128;
      const int line = lane;
      if (line < nrows * kLines) {
        const int r = line / kLines;
        const T* src = static_cast<const T*>(p.q) + b * p.qs0 + (head0 + r) * p.qs1 +
                       (line - r * kLines) * 64;
        prefetch_l2(src);
      }
    }
    return;
  }

  // From here on this CTA reads what the previous kernel may have written.
  pdl_wait();

  // =========================================================================
  // producer warp: block table -> TMA boxes
  // =========================================================================
  if (warp == kWaveProducerWarp) {
    const uint64_t policy = l2_policy_evict_first();
    int64_t n = 0;
    int64_t slotv = 0;
    if (lane == 0) {
      n = load_index(p.sl, p.sl64, static_cast<int64_t>(b) * p.sls);
      if constexpr (kAppend) slotv = load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots);
    }
    // Block-table window (lane j: page wb + j; next window prefetched), first
    // placed where the prefetch warp's length says this CTA starts (or, when
    // its hint is not there yet, at the start for a full row); the real
    // length is read in parallel.
    const int hint = abort_flag[2];  // volatile: written by the prefetch warp, maybe not yet
    const int64_t ng = hint > 0 ? static_cast<int64_t>(hint - 1)
                                : static_cast<int64_t>(p.cap_tiles) * kTile;
    int g0, g1;
    wave_range(split, S, static_cast<int>((wave_clamp_len(p, ng) + kTile - 1) / kTile), g0, g1);
    auto bt_entry = [&](int64_t lb) -> int {
      return lb < p.max_blocks
                 ? static_cast<int>(load_index(p.bt, p.bt64,
                                               static_cast<int64_t>(b) * p.bts0 + lb * p.bts1))
                 : -1;
    };
    int64_t wb = static_cast<int64_t>(g0) << ppt_shift;
    int win = bt_entry(wb + lane);
    int win_next = bt_entry(wb + 32 + lane);
    const int ppt = 1 << ppt_shift;
    const uint32_t tile_bits = (1u << ppt) - 1u;
    const uint32_t page_bytes = static_cast<uint32_t>(bs * D * 2 * 2);  // K and V of one page

    // Issue the TMA boxes of tiles [i0, i0 + np / ppt): lane j's block id
    // `blk` is page j of the group, `pages` the pages to load, each tile's
    // bytes counted on bars[tile].  One box per (page, plane) -- a page's
    // tokens x all of head_dim (the head_dim 128 map carries the 64-dim half
    // axis), [half][tokens][64] in the stage -- or, with the K + V pair map,
    // one box per page for both planes.  Every box of a group is issued by
    // one warp instruction (lane = box): each TMA operation costs issue time
    // on the SM, and an instruction issuing many costs far less per operation
    // than one issuing a few.
    auto issue = [&](int i0, int np, uint32_t pages, int blk, uint64_t* bars) {
      if (D == 128 && (kPageRows == 0 || kPageRows == 16) && p.kv_box) {
        // one box per page: K and V of the page, [plane][half][bs][64]; the
        // pages of a tile follow one another in the stage (16-token pages:
        // page j at j x 8 KB, see the consumer's page_pair)
        if (lane < np && ((pages >> lane) & 1u)) {
          const int i = i0 + (lane >> ppt_shift);
          const int j = lane & (ppt - 1);  // page of the tile
          tma_load_5d(smem_u32(stages + (i % NST) * SM::kStageBytes) + j * (bs * 512), &tmap_k,
                      smem_u32(&bars[i % kWaveTileBars]), 0, 0, 0,
                      blk * p.pair_m[0] + kv_head * p.pair_m[1], blk * p.pair_m[2], policy);
        }
        return;
      }
      const int nops = np * 2;
      for (int base = 0; base < nops; base += 32) {
        const int op = base + lane;
        const int page = op >> 1;  // page of the group
        const int pblk = __shfl_sync(0xffffffffu, blk, page & 31);
        if (op < nops && ((pages >> page) & 1u)) {
          const int plane = op & 1;  // 0: K, 1: V
          const int i = i0 + (page >> ppt_shift);
          const int j = page & (ppt - 1);  // page of the tile
          const uint32_t sbase = smem_u32(stages + (i % NST) * SM::kStageBytes) +
                                 plane * (SM::kHalves * SM::kHalfBytes);
          const uint32_t fbar = smem_u32(&bars[i % kWaveTileBars]);
          const int* perm = plane ? p.vperm : p.kperm;
          const CUtensorMap* map = plane ? &tmap_v : &tmap_k;
          if constexpr (D == 128) {
            tma_load_5d(sbase + j * (bs * 256), map, fbar, 0, tmap_coord(perm[0], kv_head, pblk),
                        tmap_coord(perm[1], kv_head, pblk), tmap_coord(perm[2], kv_head, pblk),
                        tmap_coord(perm[3], kv_head, pblk), policy);
          } else {
            tma_load_4d(sbase + ((j * bs) << 7), map, fbar, 0, tmap_coord(perm[0], kv_head, pblk),
                        tmap_coord(perm[1], kv_head, pblk), tmap_coord(perm[2], kv_head, pblk),
                        policy);
          }
        }
      }
    };

    // ---- speculative first group ----------------------------------------
    // When the prefetch warp has published the block-table window it read
    // before griddepcontrol.wait, the first group goes out from it now,
    // while the real reads above are in flight.  Only the choice of pages is
    // speculative: the bytes are read after the wait.  Below, each tile is
    // checked against the real block table and either confirmed on its
    // "verified" barrier or, once the speculative copy has landed, loaded
    // again from the right pages onto that barrier.
    int spec_ng = 0;          // tiles issued from the speculative window
    uint32_t spec_pages = 0;  // bit j: page j of that group was loaded
    int spec_blk = -1;        // lane j: its block id
    if (abort_flag[8]) {
      const int64_t ns = abort_flag[7] - 1;
      int s0, s1;
      wave_range(split, S, static_cast<int>((ns + kTile - 1) / kTile), s0, s1);
      const int64_t nlb_s = ((kAppend && ns > 0 ? ns - 1 : ns) + bs - 1) >> bs_shift;
      const int64_t pgs = static_cast<int64_t>(s0) << ppt_shift;
      spec_ng = min(min(s1 - s0, NST), 32 >> ppt_shift);
      const int nps = spec_ng << ppt_shift;
      spec_blk = spec_win[lane];
      const bool pv = lane < nps && (pgs + lane) < nlb_s && spec_blk >= 0 && spec_blk < p.num_blocks;
      spec_pages = __ballot_sync(0xffffffffu, pv);
      if (lane < spec_ng) {
        const uint32_t tmask = (spec_pages >> (lane << ppt_shift)) & tile_bits;
        tile_mask[lane] = tmask;
        mbar_arrive_expect_tx(smem_u32(&full_bar[lane]), static_cast<uint32_t>(__popc(tmask)) * page_bytes);
      }
      __syncwarp();
      issue(0, nps, spec_pages, spec_blk, full_bar);
    }

    n = wave_clamp_len(p, __shfl_sync(0xffffffffu, n, 0));
    // reference MASK_INVALID_SLOT: a negative slot attends to nothing
    if (kAppend && __shfl_sync(0xffffffffu, slotv, 0) < 0) n = 0;
    const int tiles = static_cast<int>((n + kTile - 1) / kTile);
    int t0, t1;
    wave_range(split, S, tiles, t0, t1);
    // pages holding cache tokens (with a fused append the last token comes
    // from the call, not the cache)
    const int64_t nlb = ((kAppend && n > 0 ? n - 1 : n) + bs - 1) >> bs_shift;
    const int ntile = t1 - t0;
    bool bad = false;
    bool alive = true;

    // ---- check the speculative group against the real block table -------
    int i_start = 0;
    if (spec_ng > 0) {
      const int nv = min(spec_ng, ntile);
      const int64_t pg0 = static_cast<int64_t>(t0) << ppt_shift;
      if (pg0 != wb) {
        wb = pg0;
        win = bt_entry(wb + lane);
        win_next = bt_entry(wb + 32 + lane);
      }
      const int npv = nv << ppt_shift;
      const int blk_r = win;  // lane j: page pg0 + j
      const bool hr = lane < npv && (pg0 + lane) < nlb;
      const bool pr = hr && blk_r >= 0 && blk_r < p.num_blocks;
      bad = bad || (hr && !pr);
      const uint32_t real_pages = __ballot_sync(0xffffffffu, pr);
      const bool ps = (spec_pages >> lane) & 1u;
      const bool same = lane >= npv || (pr == ps && (!pr || blk_r == spec_blk));
      const uint32_t diff = __ballot_sync(0xffffffffu, !same);
      const bool redo = lane < nv && ((diff >> (lane << ppt_shift)) & tile_bits) != 0;
      const uint32_t redo_tiles = __ballot_sync(0xffffffffu, redo);
      bool ok = true;
      if (lane < nv) {
        if (!redo) {
          mbar_arrive(smem_u32(&ver_bar[lane]));
        } else {
          // the speculative copy lands before the right pages overwrite the stage
          ok = mbar_wait(smem_u32(&full_bar[lane]), 0u, p.status, abort_flag);
          if (ok) {
            const uint32_t tmask = (real_pages >> (lane << ppt_shift)) & tile_bits;
            tile_mask[lane] = tmask;
            mbar_arrive_expect_tx(smem_u32(&ver_bar[lane]),
                                  static_cast<uint32_t>(__popc(tmask)) * page_bytes);
          }
        }
      }
      alive = __all_sync(0xffffffffu, ok);
      if (alive && redo_tiles) {
        const uint32_t redo_pages =
            __ballot_sync(0xffffffffu, pr && ((redo_tiles >> (lane >> ppt_shift)) & 1u));
        issue(0, npv, redo_pages, blk_r, ver_bar);
      }
      i_start = nv;
    }

    // ---- the remaining tiles, in groups ---------------------------------
    // Lane l of the warp does the bookkeeping of tile i0 + l (its stage's
    // "empty" wait, its page mask, the byte count on its "full" barrier and
    // the arrival on its "verified" one).  The first group fills every free
    // stage; later groups take at most half the ring.
    for (int i0 = i_start; alive && i0 < ntile;) {
      const int64_t pg0 = static_cast<int64_t>(t0 + i0) << ppt_shift;
      if (pg0 < wb || pg0 >= wb + 64) {
        wb = pg0;  // (re)load the window at this group
        win = bt_entry(wb + lane);
        win_next = bt_entry(wb + 32 + lane);
      } else if (pg0 >= wb + 32) {
        wb += 32;  // slide by one window; prefetch the following one
        win = win_next;
        win_next = bt_entry(wb + 32 + lane);
      }
      const int room = static_cast<int>((wb + 32 - pg0) >> ppt_shift);  // tiles left in the window
      const int cap = i0 < NST ? NST - i0 : max(1, NST / 2);
      const int ng = min(min(ntile - i0, cap), room);
      const int np = ng << ppt_shift;  // pages of the group (<= 32)
      const int blk_l = __shfl_sync(0xffffffffu, win, static_cast<int>(pg0 - wb + lane) & 31);
      const bool has_tokens = lane < np && (pg0 + lane) < nlb;
      const bool pvalid = has_tokens && blk_l >= 0 && blk_l < p.num_blocks;
      bad = bad || (has_tokens && !pvalid);
      const uint32_t pages = __ballot_sync(0xffffffffu, pvalid);
      bool ok = true;
      if (lane < ng) {
        const int i = i0 + lane;
        if (i >= NST) {
          ok = mbar_wait(smem_u32(&empty_bar[i % NST]), static_cast<uint32_t>((i / NST) - 1) & 1u,
                         p.status, abort_flag);
        }
        if (ok) {
          const uint32_t tmask = (pages >> (lane << ppt_shift)) & tile_bits;
          tile_mask[i % kWaveTileBars] = tmask;
          mbar_arrive_expect_tx(smem_u32(&full_bar[i % kWaveTileBars]),
                                static_cast<uint32_t>(__popc(tmask)) * page_bytes);
          mbar_arrive(smem_u32(&ver_bar[i % kWaveTileBars]));
        }
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      issue(i0, np, pages, blk_l, full_bar);
      i0 += ng;
    }
    // speculative tiles this CTA turned out not to need still land in its
    // shared memory: the CTA waits for them before it may exit
    if (lane < spec_ng && lane >= ntile) {
      mbar_wait(smem_u32(&full_bar[lane]), 0u, p.status, abort_flag);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
    return;
  }

  // =========================================================================
  // consumer warps 0-3: tile i belongs to warp i % 4
  // =========================================================================
  const int g8 = lane >> 2;
  const int t4 = lane & 3;
  const int mi = lane >> 3;
  const int r8 = lane & 7;
  int64_t n = wave_clamp_len(p, load_index(p.sl, p.sl64, static_cast<int64_t>(b) * p.sls));
  if constexpr (kAppend) {
    if (load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots) < 0) n = 0;
  }
  const int tiles = static_cast<int>((n + kTile - 1) / kTile);
  int t0, t1;
  wave_range(split, S, tiles, t0, t1);
  const int ntile = t1 - t0;

  // ---- q rows -> shared (tile layout) -> B fragments of Q^T ---------------
  for (int c = tid; c < 16 * (D / 8); c += kWaveConsumerThreads) {
    const int row = c / (D / 8);
    const int ch = c - row * (D / 8);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < nrows) {
      const T* src = static_cast<const T*>(p.q) + b * p.qs0 + (head0 + row) * p.qs1 + ch * 8 * p.qs2;
      if (p.qs2 == 1 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        __align__(16) T e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = src[i * p.qs2];
        v = *reinterpret_cast<const uint4*>(e);
      }
    }
    *reinterpret_cast<uint4*>(qbuf + chunk_offset(row, ch)) = v;
  }
  if constexpr (kAppend) {
    // this sequence's new K / V row and its slot are staged with q (same
    // memory round trip), so the tile that receives the row reads shared
    // memory only
    for (int e = tid; e < 2 * D; e += kWaveConsumerThreads) {
      const int plane = e / D;
      const int d = e - plane * D;
      app_row[e] = plane ? static_cast<const T*>(p.av)[b * p.avs0 + kv_head * p.avs1 + d * p.avs2]
                         : static_cast<const T*>(p.ak)[b * p.aks0 + kv_head * p.aks1 + d * p.aks2];
    }
    if (tid == 0) *app_slot = load_index(p.slot, p.slot64, static_cast<int64_t>(b) * p.slots);
    if (tid < (p.rope_dim >> 1)) {
      // cos / sin of this sequence's angles, once per pair index (the same
      // for every q row and the K row; the RoPE + append kernel evaluates the
      // same expression)
      const float posf = static_cast<float>(
          load_index(p.rope_pos, p.rope_pos64, static_cast<int64_t>(b) * p.rope_pos_stride));
      float sn, cs;
      sincosf(__fmul_rn(posf, p.rope_inv_freq[tid]), &sn, &cs);
      rope_tab[tid] = cs;
      rope_tab[64 + tid] = sn;
    }
  }
  named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
  if (kAppend && p.rope_dim > 0) {
    // RoPE in place of the staged q rows and (row nrows) the appended K row:
    // pair (i, i + rope_dim / 2)
    const int half = p.rope_dim >> 1;
    for (int e = tid; e < (nrows + 1) * half; e += kWaveConsumerThreads) {
      const int row = e / half;
      const int i = e - row * half;
      T* x1p = row < nrows ? reinterpret_cast<T*>(qbuf + tile_offset(row, i)) : app_row + i;
      T* x2p = row < nrows ? reinterpret_cast<T*>(qbuf + tile_offset(row, i + half)) : app_row + i + half;
      float y1, y2;
      rope_rotate_pair_cs(to_f32<T>(*x1p), to_f32<T>(*x2p), rope_tab[i], rope_tab[64 + i], y1, y2);
      *x1p = from_f32<T>(y1);
      *x2p = from_f32<T>(y2);
    }
    named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
  }
  // qf[nt][ks]: B fragment (k16 dims x n8 heads) of query heads nt * 8 + ..
  uint32_t qf[kNT][kKS][2];
  {
    const uint32_t qb = smem_u32(qbuf);
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int kp = 0; kp < kKS / 2; ++kp) {
        ldsm_x4(qb + chunk_offset(nt * 8 + r8, 4 * kp + mi), qf[nt][2 * kp][0], qf[nt][2 * kp][1],
                qf[nt][2 * kp + 1][0], qf[nt][2 * kp + 1][1]);
      }
    }
  }

  // Every CTA of the cluster arrived on the cluster barrier at its start, so
  // this wait costs nothing here; it makes the peers' merge barriers (and
  // receive areas) safe targets for the pushes at the end.
  if constexpr (kCluster) cluster_wait();

  // Per-lane ldmatrix offsets in a stage (the same for every tile).  K as
  // the A operand (tokens x dims): row (mi & 1) * 8 + r8 (+16 per m tile),
  // chunk 2 (ks % 4) + (mi >> 1) of half ks / 4.  V^T as the A operand
  // (dims x tokens, ldmatrix.trans of V rows): row (mi >> 1) * 8 + r8 (+16
  // per token k step), chunk 2 (mt % 4) + (mi & 1) of half mt / 4.
  const uint32_t k_row = stage_row_base<kPageRows>((mi & 1) * 8 + r8, 0);
  const uint32_t v_row = stage_row_base<kPageRows>((mi >> 1) * 8 + r8, 0);
  uint32_t k_sw[4], v_sw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    k_sw[j] = static_cast<uint32_t>((((2 * j) + (mi >> 1)) ^ r8) << 4);
    v_sw[j] = static_cast<uint32_t>((((2 * j) + (mi & 1)) ^ r8) << 4);
  }

  // K and V regions of a stage (swapped when the pair map's first plane is V).
  // Separate planes or 32-token pair boxes: K's [half][32][64] then V's.
  // 16-token pair boxes (page_pair): each page's K then V, [page][plane]
  // [half][16][64], so 16 rows (one page) are 8 KB apart and V sits 4 KB
  // after K.
  const bool page_pair = kPageRows == 16 && p.kv_box;
  const uint32_t kv_span = page_pair ? static_cast<uint32_t>(kPageRows * 256)
                                     : static_cast<uint32_t>(SM::kHalves * SM::kHalfBytes);
  const uint32_t koff = (p.kv_box && p.v_first) ? kv_span : 0u;
  const uint32_t voff = (p.kv_box ? kv_span : static_cast<uint32_t>(SM::kHalves * SM::kHalfBytes)) - koff;
  const uint32_t rows16 = SS::kRows16Bytes + (page_pair ? static_cast<uint32_t>(kPageRows * 256) : 0u);
  // extra bytes before row r's page in the page_pair layout
  auto page_gap = [&](int r) -> uint32_t {
    return page_pair ? static_cast<uint32_t>((r / (kPageRows > 0 ? kPageRows : kTile)) * kPageRows * 256) : 0u;
  };
  float m_run[kNT][2], l_run[kNT][2];
  // o[mt][nt][2 hf + e]: O^T[dim 16 mt + g8 + 8 hf][head nt * 8 + 2 t4 + e]
  float o[kMTD][kNT][4];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < kMTD; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
  }

  for (int i = warp; i < ntile; i += kWaveConsumerWarps) {
    const int t = t0 + i;
    const int stage = i % NST;
    // the tile's bytes have landed, and its pages are the block table's
    // (a speculatively chosen page that turned out wrong is loaded again and
    // lands on the "verified" barrier)
    const uint32_t par = static_cast<uint32_t>(i / kWaveTileBars) & 1u;
    if (!mbar_wait(smem_u32(&full_bar[i % kWaveTileBars]), par, p.status, abort_flag) ||
        !mbar_wait(smem_u32(&ver_bar[i % kWaveTileBars]), par, p.status, abort_flag)) {
      continue;
    }
    uint8_t* sb = stages + stage * SM::kStageBytes;
    const uint32_t kbase = smem_u32(sb) + koff;
    const uint32_t vbase = smem_u32(sb) + voff;
    // tokens of the tile that exist: pages present and position < n
    // cache tokens of the tile that exist: pages present and position below
    // the cache length (n, or n - 1 with a fused append)
    const int64_t rem = (kAppend ? n - 1 : n) - static_cast<int64_t>(t) * kTile;
    const uint32_t len_mask = rem >= 32 ? 0xffffffffu : (rem <= 0 ? 0u : ((1u << rem) - 1u));
    uint32_t vmask = wave_page_rows(tile_mask[i % kWaveTileBars], bs_shift) & len_mask;
    int ra = -1;  // row of the appended token in this tile
    if constexpr (kAppend) {
      const int64_t r = n - 1 - static_cast<int64_t>(t) * kTile;
      if (r >= 0 && r < kTile) {
        ra = static_cast<int>(r);
        vmask |= 1u << ra;
      }
    }
    bool touched = false;
    if (vmask != 0xffffffffu) {
      // rows without data: zero V so that P (0 there) times V stays 0 even
      // if the stale bytes are NaN / Inf
      const uint32_t inv = ~vmask;
      for (int e = lane; e < kTile * (D / 8); e += 32) {
        const int r = e / (D / 8);
        const int c = e - r * (D / 8);
        if ((inv >> r) & 1u) {
          *reinterpret_cast<uint4*>(sb + voff + page_gap(r) + stage_chunk_offset<kPageRows>(r, c)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      __syncwarp();
      touched = true;
    }
    if (kAppend && ra >= 0) {
      // current token: K / V from the call (K rotated with RoPE) patch the
      // tile, and head block 0 stores them into the token's cache slot
      // (reference paged_decode.py:193-221)
      const int64_t slot = *app_slot;
      const int64_t sblk = slot >> bs_shift;
      const int64_t soff = slot - sblk * bs;
      const bool store = jb == 0 && sblk < p.num_blocks;
      T* kc = static_cast<T*>(const_cast<void*>(p.k)) + sblk * p.ks0 + kv_head * p.ks1 + soff * p.ks2;
      T* vc = static_cast<T*>(const_cast<void*>(p.v)) + sblk * p.vs0 + kv_head * p.vs1 + soff * p.vs2;
      for (int d = lane; d < D; d += 32) {
        const T kv = app_row[d];
        const T vv = app_row[D + d];
        *reinterpret_cast<T*>(sb + koff + page_gap(ra) + stage_tile_offset<kPageRows>(ra, d)) = kv;
        *reinterpret_cast<T*>(sb + voff + page_gap(ra) + stage_tile_offset<kPageRows>(ra, d)) = vv;
        if (store) {
          kc[d * p.ks3] = kv;
          vc[d * p.vs3] = vv;
        }
      }
      if (!store && jb == 0 && lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
      __syncwarp();
      touched = true;
    }

    // ---- S^T = K Q^T (32 tokens x 8 kNT heads) ----
    float sa[kQA][2][kNT][4];
#pragma unroll
    for (int qa = 0; qa < kQA; ++qa)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt)
          sa[qa][mt][nt][0] = sa[qa][mt][nt][1] = sa[qa][mt][nt][2] = sa[qa][mt][nt][3] = 0.f;
    // An ldmatrix takes about a hundred cycles to return, an mma a few to
    // issue: K fragments are loaded kKA k steps ahead of their mma (all of
    // them up front for a group of up to 8 heads, where registers allow).
    constexpr int kKA = kNT == 1 ? kKS : 2;
    uint32_t ka[kKA][2][4];
    auto load_k = [&](int ks, uint32_t (&dst)[2][4]) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        ldsm_x4(kbase + k_row + mt * rows16 + (ks >> 2) * SS::kHalfStride + k_sw[ks & 3],
                dst[mt][0], dst[mt][1], dst[mt][2], dst[mt][3]);
      }
    };
#pragma unroll
    for (int ks = 0; ks < kKA; ++ks) load_k(ks, ka[ks]);
#pragma unroll
    for (int ks = 0; ks < kKS; ++ks) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt)
          mma_16816<T>(sa[ks % kQA][mt][nt], ka[ks % kKA][mt], qf[nt][ks][0], qf[nt][ks][1]);
      }
      if (ks + kKA < kKS) load_k(ks + kKA, ka[ks % kKA]);
    }
    // V fragments do not depend on the softmax: the first kVAhead (every one
    // for a group of up to 8 heads) are issued now, under the softmax
    constexpr int kVF = 2 * kMTD;  // V^T fragments of a tile: (token k step, dim m tile)
    constexpr int kVAhead = kNT == 1 ? kVF : 4;
    uint32_t va[kVAhead][4];
    auto load_v = [&](int f, uint32_t (&dst)[4]) {
      const int ks = f / kMTD;
      const int mt = f - ks * kMTD;
      ldsm_x4_t(vbase + v_row + ks * rows16 + (mt >> 2) * SS::kHalfStride + v_sw[mt & 3],
                dst[0], dst[1], dst[2], dst[3]);
    };
#pragma unroll
    for (int f = 0; f < kVAhead; ++f) load_v(f, va[f]);
    float sc[2][kNT][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          float v = sa[0][mt][nt][x];
          if constexpr (kQA == 2) v += sa[1][mt][nt][x];
          sc[mt][nt][x] = v;
        }

    // ---- online softmax per query head (column), base 2 ----
    // sc[mt][nt][2 hf + e]: token 16 mt + g8 + 8 hf, head nt * 8 + 2 t4 + e
    float alpha[kNT][2];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float mx = -INFINITY;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int tok = 16 * mt + g8 + 8 * hf;
            float x = sc[mt][nt][2 * hf + e] * p.scale_log2;
            if (vmask != 0xffffffffu && !((vmask >> tok) & 1u)) x = -INFINITY;
            sc[mt][nt][2 * hf + e] = x;
            mx = fmaxf(mx, x);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m_run[nt][e], mx);
        const float ref = (mn == -INFINITY) ? 0.f : mn;
        alpha[nt][e] = exp2f(m_run[nt][e] - ref);
        float ps = 0.f;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const float pv = exp2f(sc[mt][nt][2 * hf + e] - ref);
            sc[mt][nt][2 * hf + e] = pv;
            ps += pv;
          }
        }
        // the sum stays per lane (8 tokens); the lanes of a head add at the end
        l_run[nt][e] = l_run[nt][e] * alpha[nt][e] + ps;
        m_run[nt][e] = mn;
      }
    }
    bool rescale = false;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) rescale = rescale || alpha[nt][0] != 1.f || alpha[nt][1] != 1.f;
    // once the running maxima settle, alpha is exactly 1 and the rescale
    // would change no bit
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int mt = 0; mt < kMTD; ++mt) {
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
          o[mt][nt][0] *= alpha[nt][0];
          o[mt][nt][1] *= alpha[nt][1];
          o[mt][nt][2] *= alpha[nt][0];
          o[mt][nt][3] *= alpha[nt][1];
        }
      }
    }

    // ---- P^T as B fragments (k16 tokens x n8 heads) ----
    uint32_t pb[2][kNT][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) {
        pb[mt][nt][0] = movmatrix_trans(pack2<T>(sc[mt][nt][0], sc[mt][nt][1]));
        pb[mt][nt][1] = movmatrix_trans(pack2<T>(sc[mt][nt][2], sc[mt][nt][3]));
      }
    }

    // ---- O^T += V^T P^T ----
#pragma unroll
    for (int f = 0; f < kVF; ++f) {
      const int ks = f / kMTD;
      const int mt = f - ks * kMTD;
      uint32_t a[4] = {va[f % kVAhead][0], va[f % kVAhead][1], va[f % kVAhead][2],
                       va[f % kVAhead][3]};
      if (f + kVAhead < kVF) load_v(f + kVAhead, va[f % kVAhead]);
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) mma_16816<T>(o[mt][nt], a, pb[ks][nt][0], pb[ks][nt][1]);
    }
    __syncwarp();
    if (touched) fence_proxy_async_smem();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[stage]));
  }

  // ---- per-head sums over the eight lanes of a head ----
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = l_run[nt][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      l_run[nt][e] = l;
    }
  }

  // ---- the four warps' states -> the idle stage ring ----
  // Every tile was waited on by its warp, so no TMA write is in flight and
  // the producer has nothing left to issue: the ring is free once all warps
  // are past their last tile.
  named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
  float* wbuf = reinterpret_cast<float*>(stages);                            // [4][16][D]
  float2* wml = reinterpret_cast<float2*>(stages + kWaveConsumerWarps * 16 * D * 4);  // [4][16]
#pragma unroll
  for (int mt = 0; mt < kMTD; ++mt) {
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = nt * 8 + 2 * t4 + e;
          const int d = 16 * mt + g8 + 8 * hf;
          wbuf[(warp * 16 + h) * D + wave_col(h, d)] = o[mt][nt][2 * hf + e];
        }
      }
    }
  }
  if (g8 == 0) {
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      wml[warp * 16 + nt * 8 + 2 * t4] = make_float2(m_run[nt][0], l_run[nt][0]);
      wml[warp * 16 + nt * 8 + 2 * t4 + 1] = make_float2(m_run[nt][1], l_run[nt][1]);
    }
  }
  named_barrier(kWaveBarConsumers, kWaveConsumerThreads);

  constexpr int kUnits = D / 4;  // float4 units of a row
  // cluster receive area: slot (source rank * ri + r / S) of owner r % S
  const int ri = (p.rows + S - 1) / S;
  float* recv = reinterpret_cast<float*>(rbuf);
  float2* recv_ml = reinterpret_cast<float2*>(recv + S * ri * D);
  const int crank = kCluster ? static_cast<int>(cluster_ctarank()) : 0;

  for (int u = tid; u < nrows * kUnits; u += kWaveConsumerThreads) {
    const int r = u / kUnits;
    const int d = (u - r * kUnits) * 4;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWaveConsumerWarps; ++w) M = fmaxf(M, wml[w * 16 + r].x);
    float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWaveConsumerWarps; ++w) {
        const float2 ml = wml[w * 16 + r];
        const float wgt = exp2f(ml.x - M);  // 0 for a warp without tiles
        const float4 v = *reinterpret_cast<const float4*>(&wbuf[(w * 16 + r) * D + wave_col(r, d)]);
        L += wgt * ml.y;
        a0 += wgt * v.x;
        a1 += wgt * v.y;
        a2 += wgt * v.z;
        a3 += wgt * v.w;
      }
    }
    if (S == 1) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      wave_store_out4<T>(p, b, head0 + r, d, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
    } else if constexpr (kCluster) {
      const uint32_t owner = static_cast<uint32_t>(r % S);
      const int slot = crank * ri + r / S;
      const uint32_t obar = map_to_rank(smem_u32(merge_bar), owner);
      st_async_v4(map_to_rank(smem_u32(&recv[slot * D + d]), owner), a0, a1, a2, a3, obar);
      if (d == 0) st_async_v2(map_to_rank(smem_u32(&recv_ml[slot]), owner), M, L, obar);
    } else {
      float* ap = p.pacc + b * p.pas0 + (head0 + r) * p.pas1 + split * p.pas2 + d * p.pas3;
      if (p.pas3 == 1 && (reinterpret_cast<uintptr_t>(ap) & 15u) == 0) {
        *reinterpret_cast<float4*>(ap) = make_float4(a0, a1, a2, a3);
      } else {
        ap[0] = a0;
        ap[p.pas3] = a1;
        ap[2 * p.pas3] = a2;
        ap[3 * p.pas3] = a3;
      }
      if (d == 0) {
        const int64_t so = b * p.pss0 + (head0 + r) * p.pss1 + split * p.pss2;
        p.pmax[so] = M;
        p.psum[so] = L;
      }
    }
  }
  if (S == 1) return;

  if constexpr (kCluster) {
    // The merge barrier completes once every byte pushed into this CTA has
    // landed, which also tells it that no peer will touch its shared memory
    // again.  One thread polls it (acquire at cluster scope); the named
    // barrier then extends the acquired view to the other consumer threads.
    if (tid == 0) misc[3] = mbar_wait_cluster(smem_u32(merge_bar), 0u, p.status, abort_flag) ? 1 : 0;
    named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
    if (!misc[3]) return;
    for (int u = tid; u < ri * kUnits; u += kWaveConsumerThreads) {
      const int q = u / kUnits;
      const int r = crank + q * S;
      if (r >= nrows) continue;
      const int d = (u - q * kUnits) * 4;
      float2 ml[kWaveMaxSplits];
      float4 av[kWaveMaxSplits];
#pragma unroll
      for (int s = 0; s < kWaveMaxSplits; ++s) {
        ml[s] = make_float2(-INFINITY, 0.f);
        av[s] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < S) {
          ml[s] = recv_ml[s * ri + q];
          av[s] = *reinterpret_cast<const float4*>(&recv[(s * ri + q) * D + d]);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int s = 0; s < kWaveMaxSplits; ++s) M = fmaxf(M, ml[s].x);
      float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int s = 0; s < kWaveMaxSplits; ++s) {
          const float wgt = exp2f(ml[s].x - M);  // 0 for an empty or absent split
          L += wgt * ml[s].y;
          a0 += wgt * av[s].x;
          a1 += wgt * av[s].y;
          a2 += wgt * av[s].z;
          a3 += wgt * av[s].w;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      wave_store_out4<T>(p, b, head0 + r, d, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
    }
    return;
  } else {
    // The barrier orders every consumer thread's partial stores before
    // thread 0's acq_rel ticket, which releases them at GPU scope and, for
    // the last arriver, acquires the other CTAs' partials; the second barrier
    // extends that to every consumer thread.
    named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
    const int pid = b * static_cast<int>(gridDim.y) + hb;
    if (tid == 0) {
      const int prev = atom_add_acq_rel_gpu(&p.tickets[pid], 1);
      const int last = prev == S - 1;
      if (last) p.tickets[pid] = 0;  // every contributor has arrived: re-arm
      misc[1] = last;
    }
    named_barrier(kWaveBarConsumers, kWaveConsumerThreads);
    if (!misc[1]) return;
    // last CTA of the pair: merge the S partials (reference reducer
    // semantics, paged_decode.py:593-635), all loads in one round trip
    for (int u = tid; u < nrows * kUnits; u += kWaveConsumerThreads) {
      const int r = u / kUnits;
      const int d = (u - r * kUnits) * 4;
      const int64_t sbase = b * p.pss0 + (head0 + r) * p.pss1;
      const float* abase = p.pacc + b * p.pas0 + (head0 + r) * p.pas1 + d * p.pas3;
      float mv[kWaveMaxSplits], lv[kWaveMaxSplits];
      float4 av[kWaveMaxSplits];
#pragma unroll
      for (int s = 0; s < kWaveMaxSplits; ++s) {
        mv[s] = -INFINITY;
        lv[s] = 0.f;
        av[s] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < S) {
          mv[s] = __ldcg(p.pmax + sbase + s * p.pss2);
          lv[s] = __ldcg(p.psum + sbase + s * p.pss2);
          const float* ap = abase + s * p.pas2;
          if (p.pas3 == 1 && (reinterpret_cast<uintptr_t>(ap) & 15u) == 0) {
            av[s] = __ldcg(reinterpret_cast<const float4*>(ap));
          } else {
            av[s] = make_float4(__ldcg(ap), __ldcg(ap + p.pas3), __ldcg(ap + 2 * p.pas3),
                                __ldcg(ap + 3 * p.pas3));
          }
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int s = 0; s < kWaveMaxSplits; ++s) M = fmaxf(M, mv[s]);
      float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int s = 0; s < kWaveMaxSplits; ++s) {
          const float w = exp2f(mv[s] - M);  // 0 for empty or absent splits
          L += w * lv[s];
          a0 += w * av[s].x;
          a1 += w * av[s].y;
          a2 += w * av[s].z;
          a3 += w * av[s].w;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      wave_store_out4<T>(p, b, head0 + r, d, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
    }
  }
}

// Clusters are spread over SMs: two CTAs of one call on one SM would share
// its TMA and load bandwidth (FLASHDEC_B200_WAVE_SPREAD=0 keeps the
// default placement).
cudaClusterSchedulingPolicy wave_cluster_policy() {
  static const cudaClusterSchedulingPolicy pol = [] {
    const char* v = std::getenv("FLASHDEC_B200_WAVE_SPREAD");
    return (v && v[0] == '0') ? cudaClusterSchedulingPolicyDefault
                              : cudaClusterSchedulingPolicySpread;
  }();
  return pol;
}

// Thread-block clusters of S CTAs can merge through distributed shared memory
// only if every pair's cluster is resident at once; the occupancy answer
// depends on the device, the kernel, its shared memory and S (cached).
struct WaveClusterKey {
  int device;
  const void* kern;
  size_t smem;
  int size;
};
std::mutex g_wave_mu;
std::vector<std::pair<WaveClusterKey, int>> g_wave_clusters;

int wave_max_clusters(const void* kern, size_t smem, int size, const DeviceInfo& dev) {
  {
    std::lock_guard<std::mutex> lock(g_wave_mu);
    for (const auto& e : g_wave_clusters) {
      if (e.first.device == dev.device && e.first.kern == kern && e.first.smem == smem &&
          e.first.size == size)
        return e.second;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(size));
  cfg.blockDim = dim3(kWaveThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(size);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
  attr[1].val.clusterSchedulingPolicyPreference = wave_cluster_policy();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();  // not fatal: the launch merges through tickets instead
    n = 0;
  }
  std::lock_guard<std::mutex> lock(g_wave_mu);
  g_wave_clusters.push_back({WaveClusterKey{dev.device, kern, smem, size}, n});
  return n;
}

// Shared memory of one CTA: stages, q rows, cluster receive area, control words.
template <int D>
size_t wave_smem(int stages, int recv_bytes) {
  return 1024 + static_cast<size_t>(stages) * WaveSmem<D>::kStageBytes + WaveSmem<D>::kQBytes +
         recv_bytes + kWaveCtlBytes;
}

template <typename T, int D, int kPageRows, int kNT, bool kCluster, bool kAppend>
int wave_launch(WaveParams p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
                const DeviceInfo& dev, cudaStream_t stream, bool* fits) {
  using SM = WaveSmem<D>;
  auto kern = wave_decode_kernel<T, D, kPageRows, kNT, kCluster, kAppend>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  const int slot = dev.device & 63;
  std::call_once(once[slot], [&] {
    attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kWaveSmemBudget));
    if (attr_err[slot] == cudaSuccess && kCluster) {
      attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    }
  });
  if (attr_err[slot] != cudaSuccess) return cuda_status(attr_err[slot]);
  const int S = static_cast<int>(grid.x);
  int recv = 0;
  if (kCluster) {
    const int ri = (p.rows + S - 1) / S;
    recv = (S * ri * (D * 4 + 8) + 127) & ~127;
  }
  const size_t fixed = wave_smem<D>(0, recv);
  if (fixed + 4 * static_cast<size_t>(SM::kStageBytes) > kWaveSmemBudget) {
    *fits = false;
    return FD_ERR_UNSUPPORTED;
  }
  int stages = static_cast<int>((kWaveSmemBudget - fixed) / SM::kStageBytes);
  stages = std::min(stages, kWaveMaxStages);
  // the merge of the four warps is staged in the stage ring
  if (static_cast<size_t>(stages) * SM::kStageBytes < static_cast<size_t>(SM::kWarpMergeBytes)) {
    *fits = false;
    return FD_ERR_UNSUPPORTED;
  }
  p.num_stages = stages;
  p.recv_bytes = recv;
  const size_t smem = wave_smem<D>(stages, recv);
  if (kCluster) {
    const int64_t clusters = static_cast<int64_t>(grid.y) * grid.z;
    if (wave_max_clusters(reinterpret_cast<const void*>(kern), smem, S, dev) < clusters) {
      *fits = false;
      return FD_ERR_UNSUPPORTED;
    }
  }
  *fits = true;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kWaveThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int nattr = 1;
  if (kCluster) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(S);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    attr[2].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[2].val.clusterSchedulingPolicyPreference = wave_cluster_policy();
    nattr = 3;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p, mk, mv));
}

// Cluster merge when it fits and the tickets are not needed, else the ticket merge.
template <typename T, int D, int kPageRows, int kNT, bool kAppend>
int wave_merge_kind(const WaveParams& p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
                    const DeviceInfo& dev, cudaStream_t stream) {
  bool fits = false;
  if (grid.x >= 2 && cluster_enabled()) {
    const int rc =
        wave_launch<T, D, kPageRows, kNT, true, kAppend>(p, mk, mv, grid, dev, stream, &fits);
    if (fits) return rc;
  }
  if (grid.x >= 2 && (!p.pacc || !p.tickets)) return FD_ERR_UNSUPPORTED;
  return wave_launch<T, D, kPageRows, kNT, false, kAppend>(p, mk, mv, grid, dev, stream, &fits);
}

template <typename T, int D, int kPageRows, int kNT>
int wave_append(const WaveParams& p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
                const DeviceInfo& dev, cudaStream_t stream) {
  // the fused append is its own instantiation: the plain decode carries none of its code
  return p.fused_append ? wave_merge_kind<T, D, kPageRows, kNT, true>(p, mk, mv, grid, dev, stream)
                        : wave_merge_kind<T, D, kPageRows, kNT, false>(p, mk, mv, grid, dev, stream);
}

template <typename T, int D, int kPageRows>
int wave_rows(const WaveParams& p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
              const DeviceInfo& dev, cudaStream_t stream) {
  return p.rows <= 8 ? wave_append<T, D, kPageRows, 1>(p, mk, mv, grid, dev, stream)
                     : wave_append<T, D, kPageRows, 2>(p, mk, mv, grid, dev, stream);
}

template <typename T>
int wave_layout(const WaveParams& p, const CUtensorMap& mk, const CUtensorMap& mv, int head_dim,
                int page_rows, dim3 grid, const DeviceInfo& dev, cudaStream_t stream) {
  if (head_dim == 64) return wave_rows<T, 64, 0>(p, mk, mv, grid, dev, stream);
  if (page_rows == 16) return wave_rows<T, 128, 16>(p, mk, mv, grid, dev, stream);
  if (page_rows == 8) return wave_rows<T, 128, 8>(p, mk, mv, grid, dev, stream);
  return wave_rows<T, 128, 0>(p, mk, mv, grid, dev, stream);
}

}  // namespace

int wave_spec_skew() {
  static const int skew = [] {
    const char* v = std::getenv("FLASHDEC_B200_TEST_SPEC_SKEW");
    return v ? std::atoi(v) : 0;
  }();
  return skew;
}

int wave_splits_override() {
  static const int s = [] {
    const char* v = std::getenv("FLASHDEC_B200_WAVE_SPLITS");
    const int n = v ? std::atoi(v) : 0;
    return n >= 1 && n <= kWaveMaxSplits ? n : 0;
  }();
  return s;
}

bool wave_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_WAVE");
    return !(v && v[0] == '0');
  }();
  return on;
}

int wave_decode(WaveParams p, const CUtensorMap& mk, const CUtensorMap& mv, bool bf16,
                int head_dim, int page_rows, dim3 grid, const DeviceInfo& dev,
                cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return FD_ERR_UNSUPPORTED;
  if (p.rows > 16 || grid.x < 1 || static_cast<int>(grid.x) > kWaveMaxSplits)
    return FD_ERR_UNSUPPORTED;
  return bf16 ? wave_layout<__nv_bfloat16>(p, mk, mv, head_dim, page_rows, grid, dev, stream)
              : wave_layout<__half>(p, mk, mv, head_dim, page_rows, grid, dev, stream);
}

}  // namespace fd
