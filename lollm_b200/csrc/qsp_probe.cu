// Failure-detection probe: one CTA waits on an mbarrier that nothing ever signals, through
// the same bounded wait the tensor-core kernels use (qsp_tc.cuh, mbar_wait_limit), so a test
// can watch a wait run out on the GPU: the kernel records QSP_DEV_WAIT_PROBE in the device
// status and returns, and the context stays usable. No copy is in flight and no TMEM is held
// while it waits, so giving up is always safe.
#include "qsp_tc.cuh"

namespace qsp {

__device__ int g_probe_error = 0;

__global__ void wait_probe_kernel(uint32_t polls, uint32_t* polled_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  tc::mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  uint64_t t0, t1;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  // phase 0 never completes: the single expected arrival never comes
  const bool ok = tc::mbar_wait_limit(&bar, 0, QSP_DEV_WAIT_PROBE, &g_probe_error, &abort_flag, polls);
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
  const uint64_t dt_ns = t1 - t0;
  if (polled_ns != nullptr) *polled_ns = ok ? 0u : (uint32_t)(dt_ns > 0xffffffffull ? 0xffffffffull : dt_ns);
}

int probe_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_probe_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_probe_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace qsp

extern "C" int qsp_wait_probe(uint32_t polls, uint32_t* waited_ns, void* stream) {
  QSP_REQUIRE(polls > 0 && polls <= qsp::tc::WAIT_LIMIT, "qsp_wait_probe: polls must be in [1, %u]",
              qsp::tc::WAIT_LIMIT);
  qsp::wait_probe_kernel<<<1, 32, 0, qsp::as_stream(stream)>>>(polls, waited_ns);
  return qsp::check_launch("qsp_wait_probe");
}
