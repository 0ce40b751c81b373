// Self-test of the failure path shared by every kernel of the library: a
// bounded mbarrier wait that runs out records FD_STATUS_WAIT_TIMEOUT in the
// device status word and returns, leaving the context usable.
//
// One warp waits on a shared-memory mbarrier that nothing ever arrives on,
// through the same mbar_wait the decode kernel uses, with a caller-given
// limit instead of the two-second production limit.  No memory outside the
// CTA is touched except the status word; nothing faults, traps or hangs.
#include "fd_host.h"
#include "fd_ptx.cuh"

namespace fd {

__global__ void wait_timeout_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    mbar_wait(smem_u32(&bar), 0u, status, &abort_flag, limit_ns);  // never completes
  }
}

}  // namespace fd

extern "C" int fd_selftest_wait_timeout(int64_t limit_ns, void* cuda_stream) {
  if (limit_ns <= 0 || limit_ns > 5000000000ll) return FD_ERR_INVALID_ARGUMENT;
  int* status = fd::device_status_ptr();
  if (!status) return FD_ERR_CUDA;
  fd::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(cuda_stream)>>>(
      status, static_cast<uint64_t>(limit_ns));
  return fd::cuda_status(cudaGetLastError());
}
