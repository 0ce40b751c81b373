// Host interface of the one-wave small-batch decode kernel (fd_wave_decode.cu),
// used by fd_paged_decode's planner in fd_attention.cu.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "fd_host.h"

namespace fd {

// Most CTAs one (sequence, head block) pair may be split over by the one-wave
// kernel (its merge loads every split's partial in one round trip).
constexpr int kWaveMaxSplits = 16;

struct WaveParams {
  int num_seqs, num_blocks, max_blocks, block_size;
  int group, hb_per_kv, rows;
  int cap_tiles;    // 32-token tiles of a full block-table row
  int num_stages;   // set by wave_decode
  int recv_bytes;   // set by wave_decode: cluster receive area (0 for the ticket merge)
  float scale_log2;
  const void* q;
  int64_t qs0, qs1, qs2;
  void* out;
  int64_t os0, os1, os2;
  int kperm[4], vperm[4];  // tensor-map axis order (0 token, 1 head, 2 block, 3 half)
  // kv_box: the K map is a K + V pair map (get_kv_pair_tensor_map) and one
  // box moves a page's K and V; v_first: V's plane comes first in the stage;
  // pair_m: page (blk, head) sits at coordinates (blk * pair_m[0] + head *
  // pair_m[1], blk * pair_m[2]) of the map's last two axes
  int kv_box, v_first, num_kv_heads;
  int pair_m[3];
  // test hook: added to every speculatively read block id (mod num_blocks)
  // so that the check of the speculative first group must re-load it
  // (FLASHDEC_B200_TEST_SPEC_SKEW; 0 in normal use)
  int spec_skew;
  // the caches (unit dim stride) for the L2 prefetch of the next call's pages
  const void* k;
  int64_t ks0, ks1, ks2;
  const void* v;
  int64_t vs0, vs1, vs2;
  const void* bt;
  int bt64;
  int64_t bts0, bts1;
  const void* sl;
  int sl64;
  int64_t sls;
  // split partials [seq, q_head, split, dim] and [seq, q_head, split]
  // (max in base-2 units) of the ticket merge; unused with one split per
  // pair or when the splits of a pair merge inside a thread-block cluster
  float* pacc;
  int64_t pas0, pas1, pas2, pas3;
  float* pmax;
  float* psum;
  int64_t pss0, pss1, pss2;
  int* tickets;  // one per (sequence, head block) pair, zero between calls
  int* status;
  // fused current-token append (the reference vLLM launcher's
  // paged_decode.py:193-221): token seq_len - 1 of every sequence comes from
  // append_k / append_v [seq, kv_head, dim] instead of the cache and is
  // stored at slot_mapping[seq]; a negative slot gives a zero output and no
  // store.  With rope_dim > 0 the q rows and the appended K row are rotated
  // by rope_positions[seq] with the fp32 table rope_inv_freq[rope_dim / 2].
  int fused_append;
  int64_t ks3, vs3;  // dim strides of the caches (stores)
  const void* ak;
  int64_t aks0, aks1, aks2;
  const void* av;
  int64_t avs0, avs1, avs2;
  const void* slot;
  int slot64;
  int64_t slots;
  int rope_dim;
  const float* rope_inv_freq;
  const void* rope_pos;
  int rope_pos64;
  int64_t rope_pos_stride;
};

// FLASHDEC_B200_TEST_SPEC_SKEW (read once; 0 when unset).
int wave_spec_skew();

// Whether fd_paged_decode may use the one-wave kernel for small batches
// (default on; FLASHDEC_B200_WAVE=0 keeps the older split schedule).
bool wave_enabled();
// FLASHDEC_B200_WAVE_SPLITS=S (1..16): split count of the length-balanced
// small-batch plan, for tuning sweeps (0: the built-in rule)
int wave_splits_override();

// Launch the one-wave kernel over grid (splits, head blocks, sequences),
// splits <= kWaveMaxSplits.  The tensor maps move one page plane per box:
// head_dim 128 maps carry the 64-dim half axis (CacheDesc::plane_box).
// `page_rows` is the stage layout: 0 for [half][32 rows][64] tiles (32-token
// pages, or head_dim 64), 8 / 16 for [page][half][rows][64].  The splits of a pair merge through distributed shared
// memory when every pair's cluster fits on the device at once, else through
// the ticket and the partials in `p`.
int wave_decode(WaveParams p, const CUtensorMap& mk, const CUtensorMap& mv, bool bf16,
                int head_dim, int page_rows, dim3 grid, const DeviceInfo& dev,
                cudaStream_t stream);

}  // namespace fd
