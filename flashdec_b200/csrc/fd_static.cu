// fd_paged_decode_static: paged decode for callers that cannot allocate.
//
// fd_paged_decode needs two caller-owned buffers (an int32 ticket array and
// fp32 partial slots).  Some callers have no way to provide them at call
// time: a plain C or C++ host without a caching allocator, where cudaMalloc
// inside the decode loop would synchronise the whole device and could fail
// under memory pressure in the middle of serving; or a plugin host that gives
// its plugins no device scratch at all.  This entry point takes both buffers
// from storage that belongs to the library's own device image instead, so a
// call makes no allocation of any kind.
//
// Storage: kStaticScratchBytes (8 MiB) of fp32 partials and kStaticTickets
// (4096) int32 tickets in file-scope __device__ arrays.  They exist once per
// device, as soon as the library's module is loaded on that device.
//
// What must start at zero: the tickets must read zero when a call starts.
// The module loader zero-fills them, and every call that completes returns
// each ticket it used to zero.  A call that ends with FD_STATUS_WAIT_TIMEOUT
// in the device status word may leave tickets non-zero; after that this
// entry point must not be used again in the process.  The scratch needs no
// initial value.
//
// Set-up: the first call on a device, with that device current, looks up the
// arrays' device addresses (cudaGetSymbolAddress) and caches them per device
// together with the id of the device's current context; a call that finds a
// different context (after cudaDeviceReset, which reloads the module and may
// move the arrays) looks them up again.  Make the first call on a device, and
// the first call after a reset, before any stream capture.
//
// Partials: with FD_EPILOGUE_PARTIALS the split partials must go to the
// caller's part_acc / part_max / part_sum (the static scratch is private, so
// the caller could not read them): a NULL part_acc is rejected with
// FD_ERR_INVALID_ARGUMENT before anything else happens.
//
// Overlap: every call on a device shares the same storage.  Calls whose
// execution overlaps on the GPU (different streams, or threads without an
// ordering between them) race on it and produce wrong results; order them,
// for example on one stream.
//
// Limit: a call whose need (as fd_paged_decode_workspace reports it) is larger
// than the static storage returns FD_ERR_CAPACITY and launches nothing.  The
// tickets/scratch fields of the caller's arguments are ignored.
#include <cstdint>
#include <mutex>

#include <cudaTypedefs.h>

#include "../../include/flashdec_b200.h"
#include "fd_host.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int64_t kStaticTickets = 4096;
constexpr int kMaxDevices = 64;

}  // namespace

static __device__ __align__(256) float fd_static_scratch[kStaticScratchBytes / sizeof(float)];
static __device__ __align__(256) int32_t fd_static_tickets[kStaticTickets];

namespace {

struct StaticStorage {
  float* scratch = nullptr;
  int32_t* tickets = nullptr;
  unsigned long long ctx_id = 0;  // context the addresses belong to
};

std::mutex g_static_mu;
StaticStorage g_static[kMaxDevices];

// Id of the calling thread's current context (driver entry points resolved at
// run time, no link-time libcuda dependency); 0 if it cannot be read.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device addresses of the static arrays on the current device (looked up on
// the first call per device).
int static_storage(StaticStorage* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fd::cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return FD_ERR_UNSUPPORTED;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_static_mu);
  StaticStorage& s = g_static[dev];
  if (!s.scratch || s.ctx_id != ctx) {
    void* scratch = nullptr;
    void* tickets = nullptr;
    e = cudaGetSymbolAddress(&scratch, fd_static_scratch);
    if (e != cudaSuccess) return fd::cuda_status(e);
    e = cudaGetSymbolAddress(&tickets, fd_static_tickets);
    if (e != cudaSuccess) return fd::cuda_status(e);
    s.tickets = static_cast<int32_t*>(tickets);
    s.scratch = static_cast<float*>(scratch);
    s.ctx_id = ctx;
  }
  *out = s;
  return FD_OK;
}

}  // namespace

extern "C" int fd_paged_decode_static(const fd_paged_decode_args* a, void* cuda_stream) {
  // partials the caller asked for must land in the caller's buffers
  if (a && a->epilogue == FD_EPILOGUE_PARTIALS && !a->part_acc) return FD_ERR_INVALID_ARGUMENT;
  size_t need_scratch = 0;
  int64_t need_tickets = 0;
  int rc = fd_paged_decode_workspace(a, &need_scratch, &need_tickets);
  if (rc) return rc;
  if (need_scratch > kStaticScratchBytes || need_tickets > kStaticTickets) return FD_ERR_CAPACITY;
  StaticStorage s;
  rc = static_storage(&s);
  if (rc) return rc;
  fd_paged_decode_args local = *a;
  local.scratch = s.scratch;
  local.scratch_bytes = kStaticScratchBytes;
  local.tickets = s.tickets;
  local.tickets_capacity = kStaticTickets;
  return fd_paged_decode(&local, cuda_stream);
}
