// Fused split-half RoPE + one-token paged K/V append for B200 (sm_100a).
//
// Replaces flashdec/csrc/fused_rope_kv_append_kernel.cu:38-139 (and, with
// rotary_dim == 0 and no q, flashdec/csrc/kv_append_kernel.cu:10-84).
//
// Semantics (reference .cu:63-81 and flashdec/rope.py:66-85):
//   q_out[b, h]                      = rope(q[b, h], positions[b])
//   k_cache[blk, h, off, :]          = rope(k[b, h], positions[b])
//   v_cache[blk, h, off, :]          = v[b, h]              (bit copy)
// with blk = block_ids[b], off = block_offsets[b] and
//   rope(x)[i]        = x[i] cos(a_i) - x[i + rd/2] sin(a_i)   i <  rd/2
//   rope(x)[i + rd/2] = x[i + rd/2] cos(a_i) + x[i] sin(a_i)
//   rope(x)[i]        = x[i]                                   i >= rd
//   a_i = float(pos) * inv_freq[i]   (fp32, inv_freq passed in by the host)
// The products and the sum are rounded separately (no FMA contraction), as
// torch evaluates `x1 * cos - x2 * sin` in rope.py:76-79, and sin/cos are the
// accurate CUDA library functions (no fast-math), so results differ from the
// reference's fp32 math only by the last-ulp differences of sin/cos.
//
// Layout: one warp per (token, head) row; rows of q come first, then the
// K/V rows.  The integer placement (blk, off) is used exactly as given.
#include <cstring>

#include "fd_host.h"
#include "fd_ptx.cuh"

namespace fd {

struct RopeParams {
  int batch, hq, hkv, head_dim, rotary_dim, block_size, num_blocks;
  const float* inv_freq;
  const void* q;
  int64_t qs0, qs1, qs2;
  void* q_out;
  int64_t qos0, qos1, qos2;
  const void* k;
  int64_t kis0, kis1, kis2;
  const void* v;
  int64_t vis0, vis1, vis2;
  void* kc;
  int64_t kcs0, kcs1, kcs2, kcs3;
  void* vc;
  int64_t vcs0, vcs1, vcs2, vcs3;
  const void* blk;
  const void* off;
  const void* pos;
  int blk64, off64, pos64;
  int* status;
};

template <typename T>
__device__ __forceinline__ void rotate_row(const T* x, int64_t xs, T* y, int64_t ys, int head_dim,
                                           int rotary_dim, float posf, const float* inv_freq,
                                           int lane) {
  const int half = rotary_dim >> 1;
  for (int i = lane; i < half; i += 32) {
    float y1, y2;
    rope_rotate_pair(to_f32<T>(x[i * xs]), to_f32<T>(x[(i + half) * xs]), posf, inv_freq[i], y1,
                     y2);
    y[i * ys] = from_f32<T>(y1);
    y[(i + half) * ys] = from_f32<T>(y2);
  }
  for (int i = rotary_dim + lane; i < head_dim; i += 32) y[i * ys] = x[i * xs];
}

template <typename T>
__global__ void rope_kv_append_kernel(const __grid_constant__ RopeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int warps_per_cta = blockDim.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t q_rows = static_cast<int64_t>(p.batch) * p.hq;
  const int64_t kv_rows = static_cast<int64_t>(p.batch) * p.hkv;
  if (row < q_rows) {
    const int b = static_cast<int>(row / p.hq);
    const int h = static_cast<int>(row - static_cast<int64_t>(b) * p.hq);
    const float posf = static_cast<float>(load_index(p.pos, p.pos64, b));
    const T* x = static_cast<const T*>(p.q) + b * p.qs0 + h * p.qs1;
    T* y = static_cast<T*>(p.q_out) + b * p.qos0 + h * p.qos1;
    rotate_row<T>(x, p.qs2, y, p.qos2, p.head_dim, p.rotary_dim, posf, p.inv_freq, lane);
    return;
  }
  const int64_t r = row - q_rows;
  if (r >= kv_rows) return;
  const int b = static_cast<int>(r / p.hkv);
  const int h = static_cast<int>(r - static_cast<int64_t>(b) * p.hkv);
  const int64_t blk = load_index(p.blk, p.blk64, b);
  const int64_t off = load_index(p.off, p.off64, b);
  if (blk < 0 || blk >= p.num_blocks || off < 0 || off >= p.block_size) {
    // Out-of-range placement: the checked Python entry point rejects these
    // before launch; a trusted caller that passes one gets no write.
    if (lane == 0) atomicOr(p.status, FD_STATUS_BAD_BLOCK_ID);
    return;
  }
  const float posf = static_cast<float>(load_index(p.pos, p.pos64, b));
  const T* kx = static_cast<const T*>(p.k) + b * p.kis0 + h * p.kis1;
  T* ky = static_cast<T*>(p.kc) + blk * p.kcs0 + h * p.kcs1 + off * p.kcs2;
  rotate_row<T>(kx, p.kis2, ky, p.kcs3, p.head_dim, p.rotary_dim, posf, p.inv_freq, lane);
  const T* vx = static_cast<const T*>(p.v) + b * p.vis0 + h * p.vis1;
  T* vy = static_cast<T*>(p.vc) + blk * p.vcs0 + h * p.vcs1 + off * p.vcs2;
  for (int i = lane; i < p.head_dim; i += 32) vy[i * p.vcs3] = vx[i * p.vis2];
}

}  // namespace fd

using namespace fd;

extern "C" int fd_rope_kv_append(const fd_rope_kv_append_args* a, void* cuda_stream) {
  if (!a || a->struct_size != static_cast<int32_t>(sizeof(fd_rope_kv_append_args)))
    return FD_ERR_INVALID_ARGUMENT;
  if (a->dtype != FD_DTYPE_F32 && a->dtype != FD_DTYPE_F16 && a->dtype != FD_DTYPE_BF16)
    return FD_ERR_UNSUPPORTED;
  const bool has_q = a->q != nullptr;
  const bool has_kv = a->num_kv_heads > 0;  // 0: rotate q only (no cache write)
  if (a->batch < 0 || a->num_kv_heads < 0 || a->head_dim <= 0) return FD_ERR_INVALID_ARGUMENT;
  if (!has_kv && !has_q) return FD_ERR_INVALID_ARGUMENT;
  if (has_kv && (a->block_size <= 0 || a->num_blocks <= 0)) return FD_ERR_INVALID_ARGUMENT;
  if (a->rotary_dim < 0 || a->rotary_dim > a->head_dim || (a->rotary_dim & 1))
    return FD_ERR_INVALID_ARGUMENT;
  if (a->rotary_dim > 0 && !a->inv_freq) return FD_ERR_INVALID_ARGUMENT;
  if (has_kv &&
      (!a->k || !a->v || !a->k_cache || !a->v_cache || !a->block_ids || !a->block_offsets))
    return FD_ERR_INVALID_ARGUMENT;
  if ((a->rotary_dim > 0 || has_q) && !a->positions) return FD_ERR_INVALID_ARGUMENT;
  if (has_q && (!a->q_out || a->num_q_heads <= 0)) return FD_ERR_INVALID_ARGUMENT;
  if (a->batch == 0) return FD_OK;

  RopeParams p;
  std::memset(&p, 0, sizeof(p));
  p.batch = a->batch;
  p.hq = has_q ? a->num_q_heads : 0;
  p.hkv = a->num_kv_heads;
  p.head_dim = a->head_dim;
  p.rotary_dim = a->rotary_dim;
  p.block_size = a->block_size;
  p.num_blocks = a->num_blocks;
  p.inv_freq = a->inv_freq;
  p.q = a->q;
  p.qs0 = a->q_stride[0];
  p.qs1 = a->q_stride[1];
  p.qs2 = a->q_stride[2];
  p.q_out = a->q_out;
  p.qos0 = a->q_out_stride[0];
  p.qos1 = a->q_out_stride[1];
  p.qos2 = a->q_out_stride[2];
  p.k = a->k;
  p.kis0 = a->k_stride[0];
  p.kis1 = a->k_stride[1];
  p.kis2 = a->k_stride[2];
  p.v = a->v;
  p.vis0 = a->v_stride[0];
  p.vis1 = a->v_stride[1];
  p.vis2 = a->v_stride[2];
  p.kc = a->k_cache;
  p.kcs0 = a->k_cache_stride[0];
  p.kcs1 = a->k_cache_stride[1];
  p.kcs2 = a->k_cache_stride[2];
  p.kcs3 = a->k_cache_stride[3];
  p.vc = a->v_cache;
  p.vcs0 = a->v_cache_stride[0];
  p.vcs1 = a->v_cache_stride[1];
  p.vcs2 = a->v_cache_stride[2];
  p.vcs3 = a->v_cache_stride[3];
  p.blk = a->block_ids;
  p.off = a->block_offsets;
  p.pos = a->positions ? a->positions : a->block_ids;  // unused when rotary_dim == 0
  p.blk64 = a->block_ids_index == FD_INDEX_I64;
  p.off64 = a->block_offsets_index == FD_INDEX_I64;
  p.pos64 = a->positions ? (a->positions_index == FD_INDEX_I64) : p.blk64;
  p.status = device_status_ptr();
  if (!p.status) return FD_ERR_CUDA;

  const int64_t rows = static_cast<int64_t>(a->batch) * (p.hq + p.hkv);
  constexpr int kWarps = 8;
  const int64_t grid = (rows + kWarps - 1) / kWarps;
  if (grid > 0x7fffffff) return FD_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  const dim3 g(static_cast<unsigned>(grid)), blk(32 * kWarps);
  switch (a->dtype) {
    case FD_DTYPE_BF16:
      return cuda_status(launch_pdl(rope_kv_append_kernel<__nv_bfloat16>, g, blk, 0, stream, p));
    case FD_DTYPE_F16:
      return cuda_status(launch_pdl(rope_kv_append_kernel<__half>, g, blk, 0, stream, p));
    default:
      return cuda_status(launch_pdl(rope_kv_append_kernel<float>, g, blk, 0, stream, p));
  }
}
