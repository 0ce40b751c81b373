// Native host path of the Python API (module flashdec_b200._hostpath).
//
// The C-ABI launch of fd_paged_decode costs about as much host time as the
// kernel launch itself; what a Python call adds on top (a signature of six
// tensors, ctypes marshalling, the current-stream lookup) is larger than
// that.  This module does the repeated part of two calls in C++ and leaves
// everything else -- the first call of a signature, every check and error
// message, workspace allocation -- to the Python code:
//
//  * decode_into(q, k, v, block_tables, seq_lens, out): the prepared call of
//    paged_decode_attention_into with default scalar arguments.  A table maps
//    (shape, stride, dtype, device of all six tensors, current stream) to an
//    fd_paged_decode_args struct that the Python path prepared, checked and
//    bound to that stream's workspace (register_decode copies it); a hit only
//    sets the six data pointers and calls fd_paged_decode.  Returns 0, a
//    negative FD_ERR_* code, or kMiss (Python then takes its own path).
//
//  * layer_run(args, cascade, q, k, v, k_layer, v_layer): one engine layer
//    (fused RoPE + K/V store + decode) on a transaction's prepared struct:
//    shape checks, the output allocation and one fd_paged_decode (or
//    fd_cascade_decode) on the current stream.
//
//  * vllm_into / register_vllm: the same for the vLLM launcher
//    (_vllm_paged_decode_attention_into) with the auto plan.
//
//  * staging_wait / staging_copy / unpack_meta: the engine's per-token
//    metadata upload (one copy from a reused pinned slot, one event per slot)
//    and its split into typed views, each one call instead of several torch
//    operations.
//
//  * copy_async(dst, src): the public flashdec_b200.copy_async, one
//    stream-ordered cudaMemcpyAsync between a host tensor and a device
//    tensor (or two device tensors) on the device's current stream.
//
// The entry points are taken as addresses from the already-loaded
// libflashdec_b200.so (set_entry_points), so both paths call the same
// library.  Every function runs with the GIL held, which serialises the
// table and the structs it hands to the library.
#include <torch/extension.h>

#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAStream.h>

#include <array>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <unordered_map>
#include <vector>

#include "flashdec_b200.h"

namespace {

using DecodeFn = int (*)(const fd_paged_decode_args*, void*);
using CascadeFn = int (*)(const fd_paged_decode_args*, const fd_cascade_args*, void*);

DecodeFn g_decode = nullptr;
CascadeFn g_cascade = nullptr;

constexpr int kMiss = 1;
constexpr int kTensors = 6;
constexpr int kMaxRank = 4;
constexpr int kPerTensor = 2 + 2 * kMaxRank;  // rank | dtype+device, sizes, strides
constexpr size_t kTableLimit = 256;

struct Signature {
  std::array<int64_t, kTensors * kPerTensor + 1> v{};
  bool operator==(const Signature& o) const { return v == o.v; }
};

struct SignatureHash {
  size_t operator()(const Signature& s) const {
    uint64_t h = 1469598103934665603ull;
    for (int64_t x : s.v) {
      h ^= static_cast<uint64_t>(x) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    }
    return static_cast<size_t>(h);
  }
};

std::unordered_map<Signature, fd_paged_decode_args, SignatureHash> g_table;

// false for a tensor the fast path does not describe (rank above four, not
// on a CUDA device); the caller then takes the Python path
bool signature(const at::Tensor* const* ts, cudaStream_t stream, Signature* s) {
  int j = 0;
  for (int i = 0; i < kTensors; ++i) {
    const at::Tensor& t = *ts[i];
    const int64_t r = t.dim();
    if (r > kMaxRank || !t.is_cuda()) return false;
    s->v[j++] = r;
    s->v[j++] = static_cast<int64_t>(t.scalar_type()) * 1024 + t.get_device();
    const auto sz = t.sizes();
    const auto st = t.strides();
    for (int64_t d = 0; d < kMaxRank; ++d) {
      s->v[j++] = d < r ? sz[d] : 0;
      s->v[j++] = d < r ? st[d] : 0;
    }
  }
  s->v[j] = reinterpret_cast<int64_t>(stream);
  return true;
}

void set_entry_points(int64_t decode, int64_t cascade) {
  g_decode = reinterpret_cast<DecodeFn>(decode);
  g_cascade = reinterpret_cast<CascadeFn>(cascade);
}

// Current stream of q's device, or nullptr when q's device is not the
// current device (the Python path switches devices itself).
bool current_stream_of(const at::Tensor& q, cudaStream_t* stream) {
  const int dev = q.get_device();
  if (dev < 0 || c10::cuda::current_device() != dev) return false;
  *stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  return true;
}

int decode_into(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& block_tables, const at::Tensor& seq_lens,
                const at::Tensor& out) {
  if (!g_decode || g_table.empty()) return kMiss;
  cudaStream_t stream;
  if (!current_stream_of(q, &stream)) return kMiss;
  const at::Tensor* ts[kTensors] = {&q, &k, &v, &block_tables, &seq_lens, &out};
  Signature s;
  if (!signature(ts, stream, &s)) return kMiss;
  auto it = g_table.find(s);
  if (it == g_table.end()) return kMiss;
  fd_paged_decode_args& a = it->second;
  a.q = q.data_ptr();
  a.k_cache = k.data_ptr();
  a.v_cache = v.data_ptr();
  a.block_tables = block_tables.data_ptr();
  a.seq_lens = seq_lens.data_ptr();
  a.out = out.data_ptr();
  return g_decode(&a, stream);
}

// Copies the struct at `args` (prepared and bound to the current stream's
// workspace by the caller, who keeps that workspace alive for as long as the
// entry exists) under the signature of these tensors on the current stream.
bool register_decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                     const at::Tensor& block_tables, const at::Tensor& seq_lens,
                     const at::Tensor& out, int64_t args) {
  cudaStream_t stream;
  if (!current_stream_of(q, &stream)) return false;
  const at::Tensor* ts[kTensors] = {&q, &k, &v, &block_tables, &seq_lens, &out};
  Signature s;
  if (!signature(ts, stream, &s)) return false;
  if (g_table.size() >= kTableLimit) g_table.clear();
  fd_paged_decode_args copy;
  std::memcpy(&copy, reinterpret_cast<const void*>(args), sizeof(copy));
  g_table[s] = copy;
  return true;
}

void clear() { g_table.clear(); }

int64_t table_size() { return static_cast<int64_t>(g_table.size()); }

bool contiguous_shape(const at::Tensor& t, int64_t d0, int64_t d1, int64_t d2) {
  if (t.dim() != 3 || !t.is_contiguous()) return false;
  const auto s = t.sizes();
  return s[0] == d0 && s[1] == d1 && s[2] == d2;
}

// One engine layer on the transaction's struct at `args` (and cascade
// description at `cascade`, 0: none).  Returns the output tensor, or the
// non-zero status of the library call as an int.
py::object layer_run(int64_t args, int64_t cascade, const at::Tensor& q, const at::Tensor& k,
                     const at::Tensor& v, int64_t k_layer, int64_t v_layer) {
  auto* a = reinterpret_cast<fd_paged_decode_args*>(args);
  if (!contiguous_shape(q, a->num_seqs, a->num_q_heads, a->head_dim)) {
    throw py::value_error(
        "q must be a contiguous [num_requests, num_q_heads, head_dim] tensor matching the "
        "transaction");
  }
  if (!contiguous_shape(k, a->num_seqs, a->num_kv_heads, a->head_dim) ||
      !contiguous_shape(v, a->num_seqs, a->num_kv_heads, a->head_dim)) {
    throw py::value_error(
        "k and v must be contiguous [num_requests, num_kv_heads, head_dim] tensors matching "
        "the transaction");
  }
  cudaStream_t stream;
  if (!current_stream_of(q, &stream)) {
    throw py::value_error("q must be on the current CUDA device");
  }
  at::Tensor out = at::empty(q.sizes(), q.options());
  a->q = q.data_ptr();
  a->out = out.data_ptr();
  a->append_k = k.data_ptr();
  a->append_v = v.data_ptr();
  a->k_cache = reinterpret_cast<void*>(k_layer);
  a->v_cache = reinterpret_cast<void*>(v_layer);
  const int rc = cascade ? g_cascade(a, reinterpret_cast<const fd_cascade_args*>(cascade), stream)
                         : g_decode(a, stream);
  if (rc != FD_OK) return py::int_(rc);
  return py::cast(out);
}

// ---- the vLLM launcher (kernels/paged_decode.py _vllm_paged_decode_attention_into)
// Same scheme as decode_into for the launcher's eight tensors (q, append_k,
// append_v, the 5-D kv_cache, block tables, seq_lens, out, slot_mapping)
// and its scalars; a hit sets the pointers (V's plane is kv_cache plus one
// stride of its K/V axis) and launches.  The caller keeps the registered
// struct's workspace alive.
constexpr int kVllmTensors = 8;
constexpr int kVllmRank = 5;

struct VllmSignature {
  std::array<int64_t, kVllmTensors * (2 + 2 * kVllmRank) + 7> v{};
  bool operator==(const VllmSignature& o) const { return v == o.v; }
};

struct VllmSignatureHash {
  size_t operator()(const VllmSignature& s) const {
    uint64_t h = 1469598103934665603ull;
    for (int64_t x : s.v) h ^= static_cast<uint64_t>(x) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    return static_cast<size_t>(h);
  }
};

std::unordered_map<VllmSignature, fd_paged_decode_args, VllmSignatureHash> g_vllm;

bool vllm_signature(const at::Tensor* const* ts, cudaStream_t stream, int64_t num_reqs,
                    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                    int64_t block_size, double sm_scale, VllmSignature* s) {
  int j = 0;
  for (int i = 0; i < kVllmTensors; ++i) {
    const at::Tensor& t = *ts[i];
    const int64_t r = t.dim();
    if (r > kVllmRank || !t.is_cuda()) return false;
    s->v[j++] = r;
    s->v[j++] = static_cast<int64_t>(t.scalar_type()) * 1024 + t.get_device();
    const auto sz = t.sizes();
    const auto st = t.strides();
    for (int64_t d = 0; d < kVllmRank; ++d) {
      s->v[j++] = d < r ? sz[d] : 0;
      s->v[j++] = d < r ? st[d] : 0;
    }
  }
  int64_t scale_bits;
  std::memcpy(&scale_bits, &sm_scale, sizeof(scale_bits));
  s->v[j++] = num_reqs;
  s->v[j++] = num_q_heads;
  s->v[j++] = num_kv_heads;
  s->v[j++] = head_dim;
  s->v[j++] = block_size;
  s->v[j++] = scale_bits;
  s->v[j] = reinterpret_cast<int64_t>(stream);
  return true;
}

int vllm_into(const at::Tensor& q, const at::Tensor& append_k, const at::Tensor& append_v,
              const at::Tensor& kv_cache, const at::Tensor& block_tables,
              const at::Tensor& seq_lens, const at::Tensor& out, const at::Tensor& slot_mapping,
              int64_t num_reqs, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
              int64_t block_size, double sm_scale) {
  if (!g_decode || g_vllm.empty()) return kMiss;
  cudaStream_t stream;
  if (!current_stream_of(q, &stream)) return kMiss;
  const at::Tensor* ts[kVllmTensors] = {&q, &append_k, &append_v, &kv_cache,
                                        &block_tables, &seq_lens, &out, &slot_mapping};
  VllmSignature s;
  if (!vllm_signature(ts, stream, num_reqs, num_q_heads, num_kv_heads, head_dim, block_size,
                      sm_scale, &s))
    return kMiss;
  auto it = g_vllm.find(s);
  if (it == g_vllm.end()) return kMiss;
  fd_paged_decode_args& a = it->second;
  char* kv = static_cast<char*>(kv_cache.data_ptr());
  a.q = q.data_ptr();
  a.out = out.data_ptr();
  a.k_cache = kv;
  a.v_cache = kv + kv_cache.stride(1) * kv_cache.element_size();
  a.append_k = append_k.data_ptr();
  a.append_v = append_v.data_ptr();
  a.block_tables = block_tables.data_ptr();
  a.seq_lens = seq_lens.data_ptr();
  a.slot_mapping = slot_mapping.data_ptr();
  return g_decode(&a, stream);
}

bool register_vllm(const at::Tensor& q, const at::Tensor& append_k, const at::Tensor& append_v,
                   const at::Tensor& kv_cache, const at::Tensor& block_tables,
                   const at::Tensor& seq_lens, const at::Tensor& out,
                   const at::Tensor& slot_mapping, int64_t num_reqs, int64_t num_q_heads,
                   int64_t num_kv_heads, int64_t head_dim, int64_t block_size, double sm_scale,
                   int64_t args) {
  cudaStream_t stream;
  if (!current_stream_of(q, &stream)) return false;
  if (kv_cache.dim() != 5 || kv_cache.size(1) != 2) return false;
  const at::Tensor* ts[kVllmTensors] = {&q, &append_k, &append_v, &kv_cache,
                                        &block_tables, &seq_lens, &out, &slot_mapping};
  VllmSignature s;
  if (!vllm_signature(ts, stream, num_reqs, num_q_heads, num_kv_heads, head_dim, block_size,
                      sm_scale, &s))
    return false;
  if (g_vllm.size() >= kTableLimit) g_vllm.clear();
  fd_paged_decode_args copy;
  std::memcpy(&copy, reinterpret_cast<const void*>(args), sizeof(copy));
  g_vllm[s] = copy;
  return true;
}

void clear_vllm() { g_vllm.clear(); }

// ---- pinned staging of the engine's per-token metadata -------------------
// One event per slot of a Python-owned pinned ring (flashdec_b200.cache):
// staging_wait blocks until the slot's previous copy has completed,
// staging_copy enqueues the slot's bytes to a new device buffer on the current
// stream and records the slot's event.  Rings are numbered by the caller.
struct StagingRing {
  int device = -1;
  std::vector<cudaEvent_t> events;
  std::vector<char> recorded;
};
std::unordered_map<int64_t, StagingRing> g_rings;

StagingRing& ring_of(int64_t ring, int64_t slots, int64_t slot) {
  if (slots <= 0 || slot < 0 || slot >= slots) throw py::value_error("staging slot out of range");
  StagingRing& r = g_rings[ring];
  if (static_cast<int64_t>(r.events.size()) != slots) {
    for (cudaEvent_t e : r.events) cudaEventDestroy(e);
    r.events.assign(static_cast<size_t>(slots), nullptr);
    r.recorded.assign(static_cast<size_t>(slots), 0);
    r.device = c10::cuda::current_device();
  }
  return r;
}

void staging_wait(int64_t ring, int64_t slots, int64_t slot) {
  StagingRing& r = ring_of(ring, slots, slot);
  if (r.recorded[slot]) {
    const cudaError_t e = cudaEventSynchronize(r.events[slot]);
    if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
    r.recorded[slot] = 0;
  }
}

at::Tensor staging_copy(int64_t ring, int64_t slots, int64_t slot, int64_t host_ptr,
                        int64_t nbytes) {
  StagingRing& r = ring_of(ring, slots, slot);
  const int dev = c10::cuda::current_device();
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  at::Tensor out = at::empty({nbytes}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, dev));
  cudaError_t e = cudaMemcpyAsync(out.data_ptr(), reinterpret_cast<const void*>(host_ptr),
                                  static_cast<size_t>(nbytes), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess && !r.events[slot])
    e = cudaEventCreateWithFlags(&r.events[slot], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(r.events[slot], stream);
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
  r.recorded[slot] = 1;
  return out;
}

void staging_release(int64_t ring) {
  auto it = g_rings.find(ring);
  if (it == g_rings.end()) return;
  for (cudaEvent_t e : it->second.events)
    if (e) cudaEventDestroy(e);
  g_rings.erase(it);
}

// (positions, block ids, offsets, slots) int64 and effective lengths int32
// views of a packed uint8 metadata buffer of n rows: [4 n int64 | n int32].
std::vector<at::Tensor> unpack_meta(const at::Tensor& buf, int64_t n) {
  at::Tensor i64 = buf.narrow(0, 0, 32 * n).view(at::kLong);
  std::vector<at::Tensor> out;
  out.reserve(5);
  for (int64_t i = 0; i < 4; ++i) out.push_back(i64.narrow(0, i * n, n));
  out.push_back(buf.narrow(0, 32 * n, 4 * n).view(at::kInt));
  return out;
}

}  // namespace

// copy_async(dst, src): dst <- src, bytes as stored, on the current stream of
// the CUDA side's device.  Unlike Tensor.copy_(non_blocking=True) nothing is
// recorded for the host allocator: the caller keeps both tensors alive (and
// the host side unchanged) until the stream has passed the copy.  A pageable
// host tensor makes the copy synchronous with the host, as cudaMemcpyAsync
// does.  Misuse (sizes, layout, devices, overlapping device ranges) raises
// ValueError before any CUDA call.
void copy_async(const at::Tensor& dst, const at::Tensor& src) {
  if (!dst.defined() || !src.defined()) throw py::value_error("copy_async: undefined tensor");
  const bool dc = dst.is_cuda();
  const bool sc = src.is_cuda();
  if (!dc && !sc) throw py::value_error("copy_async: one of dst and src must be a CUDA tensor");
  if ((!dc && !dst.is_cpu()) || (!sc && !src.is_cpu()))
    throw py::value_error("copy_async: tensors must be on the CPU or a CUDA device");
  if (!dst.is_contiguous() || !src.is_contiguous())
    throw py::value_error("copy_async: dst and src must be contiguous");
  const int64_t nbytes = dst.numel() * static_cast<int64_t>(dst.element_size());
  if (nbytes != src.numel() * static_cast<int64_t>(src.element_size()))
    throw py::value_error("copy_async: dst and src must hold the same number of bytes");
  const int dev = c10::cuda::current_device();
  if ((dc && dst.get_device() != dev) || (sc && src.get_device() != dev))
    throw py::value_error("copy_async: CUDA tensors must be on the current CUDA device");
  if (nbytes == 0) return;
  if (dc && sc) {
    const auto d0 = reinterpret_cast<uintptr_t>(dst.data_ptr());
    const auto s0 = reinterpret_cast<uintptr_t>(src.data_ptr());
    if (d0 < s0 + static_cast<uintptr_t>(nbytes) && s0 < d0 + static_cast<uintptr_t>(nbytes))
      throw py::value_error("copy_async: dst and src overlap");
  }
  const cudaMemcpyKind kind = dc && sc ? cudaMemcpyDeviceToDevice
                              : dc     ? cudaMemcpyHostToDevice
                                       : cudaMemcpyDeviceToHost;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  const cudaError_t e = cudaMemcpyAsync(dst.data_ptr(), src.data_ptr(), static_cast<size_t>(nbytes),
                                        kind, stream);
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ host path of the prepared flashdec_b200 launches";
  m.attr("MISS") = kMiss;
  m.attr("ARGS_BYTES") = static_cast<int64_t>(sizeof(fd_paged_decode_args));
  m.def("set_entry_points", &set_entry_points);
  m.def("decode_into", &decode_into);
  m.def("register_decode", &register_decode);
  m.def("clear", &clear);
  m.def("table_size", &table_size);
  m.def("layer_run", &layer_run);
  m.def("vllm_into", &vllm_into);
  m.def("register_vllm", &register_vllm);
  m.def("clear_vllm", &clear_vllm);
  m.def("staging_wait", &staging_wait);
  m.def("staging_copy", &staging_copy);
  m.def("staging_release", &staging_release);
  m.def("unpack_meta", &unpack_meta);
  m.def("copy_async", &copy_async, py::arg("dst"), py::arg("src"),
        "dst <- src on the current stream of the CUDA side's device (one cudaMemcpyAsync); "
        "keep both tensors alive until the stream has passed the copy");
}
