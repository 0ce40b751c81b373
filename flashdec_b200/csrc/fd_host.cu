// Host helpers: device properties, tensor-map encoding/caching, status word,
// error strings.
#include <algorithm>
#include <array>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/flashdec_b200.h"
#include "fd_host.h"

// Device status word: bits FD_STATUS_* raised by kernels (bounded waits that
// ran out, masked out-of-range block ids).  Read with fd_device_status.
__device__ int fd_g_status_word;

namespace fd {

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];
int* g_status_ptr[kMaxDevices] = {nullptr};

thread_local std::string g_last_cuda_error;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void resolve_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
}

struct MapKey {
  const void* base;
  int elem_bytes, is_bf16, head_dim, block_size, num_heads, num_blocks;
  int64_t stride[4];
  int plane_box;
  bool operator==(const MapKey& o) const {
    return base == o.base && elem_bytes == o.elem_bytes && is_bf16 == o.is_bf16 &&
           head_dim == o.head_dim && plane_box == o.plane_box &&
           block_size == o.block_size && num_heads == o.num_heads &&
           num_blocks == o.num_blocks && std::memcmp(stride, o.stride, sizeof(stride)) == 0;
  }
};

struct MapEntry {
  MapKey key;
  CUtensorMap map;
  int perm[4];
  uint64_t stamp;
};

// K + V pair maps (get_kv_pair_tensor_map)
struct PairKey {
  const void* k;
  const void* v;
  int is_bf16, num_heads, num_blocks, block_size;
  int64_t stride[4];
  bool operator==(const PairKey& o) const {
    return k == o.k && v == o.v && is_bf16 == o.is_bf16 && num_heads == o.num_heads &&
           num_blocks == o.num_blocks && block_size == o.block_size &&
           std::memcmp(stride, o.stride, sizeof(stride)) == 0;
  }
};

struct PairEntry {
  PairKey key;
  CUtensorMap map;
  int v_first;
  int m[3];
  uint64_t stamp;
};

std::mutex g_map_mu;
std::vector<MapEntry> g_maps;
std::vector<PairEntry> g_pairs;
uint64_t g_map_clock = 0;
constexpr size_t kMapCacheSize = 64;

}  // namespace

const DeviceInfo* current_device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.device < 0) {
    int sms = 0, smem = 0, ma = 0, mi = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      return nullptr;
    }
    d.num_sms = sms;
    d.max_smem_optin = smem;
    d.cc_major = ma;
    d.cc_minor = mi;
    d.device = dev;
  }
  return &d;
}

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, fd_g_status_word) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool cascade_concurrent_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_CASCADE_CONCURRENT");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool cluster_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_CLUSTER");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool kv_pair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_KV_PAIR");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool prefix_umma_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLASHDEC_B200_PREFIX_UMMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return FD_OK;
  g_last_cuda_error = cudaGetErrorString(e);
  return FD_ERR_CUDA;
}

bool get_cache_tensor_map(const CacheDesc& d, CUtensorMap* out, int perm[4]) {
  if (d.elem_bytes != 2 || d.stride[3] != 1) return false;
  if (d.head_dim != 64 && d.head_dim != 128) return false;
  if (reinterpret_cast<uintptr_t>(d.base) % 16 != 0) return false;
  for (int i = 0; i < 3; ++i) {
    const int64_t bytes = d.stride[i] * d.elem_bytes;
    if (bytes <= 0 || bytes % 16 != 0 || bytes >= (int64_t(1) << 40)) return false;
  }
  MapKey key{d.base, d.elem_bytes, d.is_bf16, d.head_dim, d.block_size, d.num_heads, d.num_blocks,
             {d.stride[0], d.stride[1], d.stride[2], d.stride[3]}, d.plane_box};
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    for (auto& e : g_maps) {
      if (e.key == key) {
        e.stamp = ++g_map_clock;
        *out = e.map;
        std::copy(e.perm, e.perm + 4, perm);
        return true;
      }
    }
  }
  resolve_encoder();
  if (!g_encode) return false;

  // Outer axes: 0 token (box = block_size), 1 head (box 1), 2 block (box 1),
  // sorted by stride.  With head_dim 128 and 16- or 8-token pages the two
  // 64-dim halves are one more axis (id 3, stride 128 bytes, box 2) right
  // after the token axis, so one box holds a whole page plane
  // ([half][block_size][64] in shared memory) instead of two half-size boxes.
  struct Axis {
    int id;
    uint64_t size;
    uint64_t stride_bytes;
    uint32_t box;
  };
  std::array<Axis, 3> ax = {{
      {0, static_cast<uint64_t>(d.block_size), static_cast<uint64_t>(d.stride[2] * 2),
       static_cast<uint32_t>(d.block_size)},
      {1, static_cast<uint64_t>(d.num_heads), static_cast<uint64_t>(d.stride[1] * 2), 1u},
      {2, static_cast<uint64_t>(d.num_blocks), static_cast<uint64_t>(d.stride[0] * 2), 1u},
  }};
  std::stable_sort(ax.begin(), ax.end(),
                   [](const Axis& a, const Axis& b) { return a.stride_bytes < b.stride_bytes; });
  const bool halves =
      d.head_dim == 128 && (d.block_size == 16 || d.block_size == 8 || d.plane_box != 0);
  std::array<Axis, 4> all;
  int n = 0;
  for (const Axis& a : ax) {
    all[n++] = a;
    if (a.id == 0 && halves) all[n++] = Axis{3, 2u, 128u, 2u};
  }
  const int rank = 1 + n;
  cuuint64_t dims[5] = {halves ? 64u : static_cast<cuuint64_t>(d.head_dim), 0, 0, 0, 0};
  cuuint64_t strides[4] = {0, 0, 0, 0};
  cuuint32_t box[5] = {64u, 1u, 1u, 1u, 1u};
  cuuint32_t estride[5] = {1u, 1u, 1u, 1u, 1u};
  int pm[4] = {-1, -1, -1, -1};
  for (int i = 0; i < n; ++i) {
    dims[i + 1] = all[i].size;
    strides[i] = all[i].stride_bytes;
    box[i + 1] = all[i].box;
    pm[i] = all[i].id;
  }
  CUtensorMap map;
  CUresult r = g_encode(&map,
                        d.is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        static_cast<cuuint32_t>(rank), const_cast<void*>(d.base),
                        dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    if (g_maps.size() >= kMapCacheSize) {
      auto oldest = std::min_element(g_maps.begin(), g_maps.end(),
                                     [](const MapEntry& a, const MapEntry& b) {
                                       return a.stamp < b.stamp;
                                     });
      g_maps.erase(oldest);
    }
    MapEntry e;
    e.key = key;
    e.map = map;
    std::copy(pm, pm + 4, e.perm);
    e.stamp = ++g_map_clock;
    g_maps.push_back(e);
  }
  *out = map;
  std::copy(pm, pm + 4, perm);
  return true;
}

bool get_kv_pair_tensor_map(const CacheDesc& k, const void* v_base, const int64_t v_stride[4],
                            CUtensorMap* out, int* v_first, int m[3]) {
  if (k.elem_bytes != 2 || k.head_dim != 128 || (k.block_size != 32 && k.block_size != 16))
    return false;
  for (int i = 0; i < 4; ++i)
    if (k.stride[i] != v_stride[i]) return false;
  if (k.stride[3] != 1) return false;
  const int64_t tok_bytes = k.stride[2] * 2;
  if (tok_bytes % 16 || tok_bytes <= 0) return false;
  const uintptr_t kb = reinterpret_cast<uintptr_t>(k.base);
  const uintptr_t vb = reinterpret_cast<uintptr_t>(v_base);
  if (kb % 16 || vb % 16 || kb == vb) return false;
  const uintptr_t lo = kb < vb ? kb : vb;
  const uint64_t delta = kb < vb ? vb - kb : kb - vb;
  if (delta % 16 || delta >= (uint64_t(1) << 40)) return false;
  PairKey key{k.base, v_base, k.is_bf16, k.num_heads, k.num_blocks, k.block_size,
              {k.stride[0], k.stride[1], k.stride[2], k.stride[3]}};
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    for (auto& e : g_pairs) {
      if (e.key == key) {
        e.stamp = ++g_map_clock;
        *out = e.map;
        *v_first = e.v_first;
        for (int i = 0; i < 3; ++i) m[i] = e.m[i];
        return true;
      }
    }
  }
  const cuuint64_t bs = static_cast<cuuint64_t>(k.block_size);
  const int64_t head_bytes = k.num_heads == 1 ? 128 : k.stride[1] * 2;
  cuuint64_t dims[5], strides[4];
  int mm[3];
  // planes apart: (block, head) planes evenly spaced in each allocation
  const int64_t plane = k.num_heads == 1 ? k.stride[0] : k.stride[1];
  const int64_t planes = static_cast<int64_t>(k.num_blocks) * k.num_heads;
  const bool apart = (k.num_heads == 1 || k.stride[0] == plane * k.num_heads) && plane > 0 &&
                     (plane * 2) % 16 == 0 && static_cast<uint64_t>(planes) * plane * 2 <= delta;
  // interleaved: block stride twice the K -> V distance, a block's K plane
  // (all heads and tokens) inside that distance
  const int64_t k_extent = ((bs - 1) * k.stride[2] + (k.num_heads - 1) * (k.num_heads > 1 ? k.stride[1] : 0) +
                            k.head_dim) * 2;
  const bool interleaved = !apart && static_cast<uint64_t>(k.stride[0]) * 2 == 2 * delta &&
                           head_bytes % 16 == 0 && head_bytes > 0 &&
                           static_cast<uint64_t>(k_extent) <= delta;
  if (apart) {
    dims[0] = 64u; dims[1] = bs; dims[2] = 2u; dims[3] = static_cast<cuuint64_t>(planes); dims[4] = 2u;
    strides[0] = static_cast<cuuint64_t>(tok_bytes);
    strides[1] = 128u;
    strides[2] = static_cast<cuuint64_t>(plane * 2);
    strides[3] = static_cast<cuuint64_t>(delta);
    mm[0] = k.num_heads; mm[1] = 1; mm[2] = 0;
  } else if (interleaved) {
    dims[0] = 64u; dims[1] = bs; dims[2] = 2u; dims[3] = static_cast<cuuint64_t>(k.num_heads);
    dims[4] = 2u * static_cast<cuuint64_t>(k.num_blocks);
    strides[0] = static_cast<cuuint64_t>(tok_bytes);
    strides[1] = 128u;
    strides[2] = static_cast<cuuint64_t>(head_bytes);
    strides[3] = static_cast<cuuint64_t>(delta);
    mm[0] = 0; mm[1] = 1; mm[2] = 2;
  } else {
    return false;
  }
  resolve_encoder();
  if (!g_encode) return false;
  cuuint32_t box[5] = {64u, static_cast<cuuint32_t>(bs), 2u, 1u, 2u};
  cuuint32_t estride[5] = {1u, 1u, 1u, 1u, 1u};
  CUtensorMap map;
  const CUresult r = g_encode(&map,
                              k.is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              5u, reinterpret_cast<void*>(lo), dims, strides, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  *out = map;
  *v_first = vb < kb ? 1 : 0;
  for (int i = 0; i < 3; ++i) m[i] = mm[i];
  std::lock_guard<std::mutex> lock(g_map_mu);
  if (g_pairs.size() >= kMapCacheSize) {
    auto oldest = std::min_element(g_pairs.begin(), g_pairs.end(),
                                   [](const PairEntry& a, const PairEntry& b) {
                                     return a.stamp < b.stamp;
                                   });
    g_pairs.erase(oldest);
  }
  g_pairs.push_back(PairEntry{key, map, *v_first, {mm[0], mm[1], mm[2]}, ++g_map_clock});
  return true;
}

}  // namespace fd

extern "C" {

const char* fd_error_string(int code) {
  switch (code) {
    case FD_OK:
      return "ok";
    case FD_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case FD_ERR_UNSUPPORTED:
      return "unsupported configuration";
    case FD_ERR_WORKSPACE:
      return "workspace missing or too small";
    case FD_ERR_CUDA:
      return fd::g_last_cuda_error.empty() ? "CUDA error" : fd::g_last_cuda_error.c_str();
    case FD_ERR_ALIGNMENT:
      return "misaligned pointer or stride";
    case FD_ERR_CAPACITY:
      return "request needs more workspace than fd_paged_decode_static's static storage "
             "(8 MiB scratch, 4096 tickets)";
    default:
      return "unknown error";
  }
}

int fd_version(void) { return 1; }

int fd_num_sms(void) {
  const fd::DeviceInfo* d = fd::current_device_info();
  return d ? d->num_sms : 0;
}

int fd_device_status(int clear, int* status_out) {
  int* p = fd::device_status_ptr();
  if (!p || !status_out) return FD_ERR_INVALID_ARGUMENT;
  int v = 0;
  int rc = fd::cuda_status(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (rc) return rc;
  *status_out = v;
  if (clear) {
    const int zero = 0;
    rc = fd::cuda_status(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
  }
  return rc;
}

}  // extern "C"
