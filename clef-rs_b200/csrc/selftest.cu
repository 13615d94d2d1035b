// selftest.cu — exercises the bounded-wait failure path on the device.
//
// Every kernel that waits on an mbarrier (GEMM, attention, scan prep) gives up
// after a bounded time, records a code in its device error flag, unwinds and
// releases what it holds; the host turns the flag into
// CLEF_ERR_DEVICE_TIMEOUT. This entry point runs that path on purpose with a
// barrier nothing arrives on and a short limit, so a caller (or a test) can
// check on real hardware that a stuck wait ends as a status, not a hang, and
// that the context stays usable. Nothing faults or traps.
#include "kernels.cuh"
#include "sm100.cuh"

namespace clef {
namespace {

__global__ void wait_probe_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait runs out after limit_ns.
  if (threadIdx.x == 0 && !sm100::mbar_wait(&bar, 0, limit_ns)) raise_device_error(kDevProbeTimeout);
}

}  // namespace
}  // namespace clef

using namespace clef;

extern "C" {

int clef_selftest_wait_timeout(int32_t limit_ms, void* stream) {
  CLEF_CHECK(limit_ms >= 1 && limit_ms <= 2000, CLEF_ERR_INVALID,
             "selftest_wait_timeout: limit_ms must be in [1, 2000]");
  cudaStream_t s = as_stream(stream);
  int code = 0;
  CLEF_CUDA(cudaStreamSynchronize(s));
  if (read_device_error(&code)) return fail(CLEF_ERR_CUDA, "selftest_wait_timeout: flag read");
  wait_probe_kernel<<<1, 32, 0, s>>>((uint64_t)limit_ms * 1000000ull);
  int rc = launch_status("wait_probe");
  if (rc) return rc;
  CLEF_CUDA(cudaStreamSynchronize(s));
  if (read_device_error(&code)) return fail(CLEF_ERR_CUDA, "selftest_wait_timeout: flag read");
  if (code == kDevProbeTimeout)
    return fail(CLEF_ERR_DEVICE_TIMEOUT, "selftest_wait_timeout: the device wait gave up after " +
                                             std::to_string(limit_ms) + " ms and reported it");
  return fail(CLEF_ERR_CUDA, "selftest_wait_timeout: the bounded wait did not report its timeout");
}

}  // extern "C"
