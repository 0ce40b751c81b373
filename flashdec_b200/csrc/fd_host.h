// Host-side helpers shared by the FlashDec B200 entry points: per-device
// properties, the tensor-map encoder (driver entry point resolved at run time,
// no link-time libcuda dependency) and a small cache of encoded maps.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fd {

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
  int cc_major = 0;
  int cc_minor = 0;
};

// Cached properties of the current device (thread-safe).
const DeviceInfo* current_device_info();

// Description of one paged cache plane for TMA: logical order
// [block, head, token, dim] with element strides; dim stride must be 1.
struct CacheDesc {
  const void* base;
  int elem_bytes;       // 2
  int is_bf16;          // 1 bf16, 0 fp16
  int head_dim;         // 64 / 128
  int block_size;       // 8 / 16 / 32
  int num_heads;
  int num_blocks;
  int64_t stride[4];    // block, head, token, dim (elements)
  int plane_box = 0;    // head_dim 128: the half axis for every page size, so one
                        // box moves a whole page plane (also 32-token pages)
};

// Encode (or fetch from the cache) a tiled tensor map over `d` with 128B
// swizzle whose box is one page plane: [64 dims x block_size tokens x 1 head
// x 1 block] (4-D), or, for head_dim 128 with 16- or 8-token pages (any page
// size with `plane_box`), the same plus a "64-dim half" axis of box 2 (5-D) so
// one copy moves the whole plane.
// `perm[i]` receives which axis tensor-map dimension i+1 is (0 token, 1 head,
// 2 block, 3 half; -1 unused); outer axes are sorted by ascending stride and
// the half axis follows the token axis.  Returns false when the layout cannot
// be described by a tensor map.
bool get_cache_tensor_map(const CacheDesc& d, CUtensorMap* out, int perm[4]);

// One tensor map over the K and V planes of a cache pair with head_dim 128
// and 16- or 32-token pages, box [64 dims, bs tokens, 2 halves, 1, 2] with the
// 128B swizzle: one copy moves a page's K and V (bs x 512 bytes) as
// [plane][half][bs tokens][64 dims].  Two layouts qualify (unit dim stride,
// equal K and V strides):
//  * planes apart: each allocation's (block, head) planes contiguous and
//    evenly spaced (block stride = heads x head stride); dims [64, bs, 2,
//    blocks * heads, 2] with the last axis spanning the two allocations
//    (stride |v - k|): page (blk, head) at coordinates (blk * heads + head, 0);
//  * planes interleaved per block (vLLM's [block, 2, bs, heads, dim] cache:
//    block stride = 2 |v - k|, a block's K within |v - k|): dims [64, bs, 2,
//    heads, 2 * blocks]: page (blk, head) at (head, 2 * blk).
// The page's coordinates on the last two axes are blk * m[0] + head * m[1]
// and blk * m[2].  *v_first is set when the plane at the lower address is V.
// Returns false when the layout does not qualify.
bool get_kv_pair_tensor_map(const CacheDesc& k, const void* v_base, const int64_t v_stride[4],
                            CUtensorMap* out, int* v_first, int m[3]);

// FD_OK, or FD_ERR_CUDA with the message kept for fd_error_string.
int cuda_status(cudaError_t e);

// Device address of the status word of the current device (cached).
int* device_status_ptr();

// Whether launches opt in to programmatic dependent launch (default on;
// FLASHDEC_B200_PDL=0 turns it off).
bool pdl_enabled();

// Whether the small-batch split schedule may merge through thread-block
// clusters (default on; FLASHDEC_B200_CLUSTER=0 turns it off and keeps the
// global-memory ticket merge).
bool cluster_enabled();

// Whether the one-wave decode may move a page's K and V with one box through
// a K + V pair map (default on; FLASHDEC_B200_KV_PAIR=0 keeps one box per
// plane).
bool kv_pair_enabled();

// Whether the cascade prefix pass runs on tcgen05 UMMA where it can (head_dim
// 128, 32-token pages; default on; FLASHDEC_B200_PREFIX_UMMA=0 keeps the
// mma.sync prefix kernel).
bool prefix_umma_enabled();

// Launch `kern` with the programmatic-stream-serialization attribute (the
// kernel calls griddepcontrol.wait before touching global memory).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The same launch without the attribute, for a kernel whose stream
// predecessor is an event wait (a fork or join between streams) instead of
// a kernel it could overlap.
template <typename... KArgs, typename... Args>
cudaError_t launch_plain(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Whether fd_cascade_decode runs the prefix pass on a second stream beside
// the tail pass (default on; FLASHDEC_B200_CASCADE_CONCURRENT=0 runs prefix
// then tail on the caller's stream, the tail merging through tickets).
bool cascade_concurrent_enabled();

}  // namespace fd
