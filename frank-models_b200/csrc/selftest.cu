// Self-test of the bounded device-side waits (failure detection without a
// GPU fault): one thread waits on an mbarrier that nothing ever completes,
// through the same mbar_wait the GEMM and decode kernels use, with a short
// limit.  The wait gives up, records FRANK_ETIMEOUT in the device error word
// and the kernel returns normally; the host reads the status.
#include "common.cuh"
#include "mbarrier.cuh"

__device__ int32_t frank_selftest_result = -1;

namespace {

__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, int32_t* err, int32_t* result) {
  using namespace frank_mbar;
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  mbar_init(smem_u32(&bar), 1);  // expects one arrival that never comes
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, err, limit_ns);
  *result = ok ? 1 : 0;
}

}  // namespace

extern "C" int frank_selftest_bounded_wait(int64_t limit_ns, int32_t* completed, void* stream) {
  if (limit_ns <= 0 || limit_ns > 5000000000LL) {
    frank::set_error("selftest_bounded_wait: limit_ns=%lld outside (0, 5e9]", (long long)limit_ns);
    return FRANK_EINVAL;
  }
  int32_t* err = frank::device_error_word();
  if (!err) {
    frank::set_error("device error word unavailable");
    return FRANK_ECUDA;
  }
  cudaStream_t st = frank::as_stream(stream);
  int32_t* dres = nullptr;  // device word receiving 1 (wait completed) or 0 (gave up)
  FRANK_CUDA_TRY(cudaGetSymbolAddress((void**)&dres, frank_selftest_result));
  bounded_wait_selftest_kernel<<<1, 32, 0, st>>>((uint64_t)limit_ns, err, dres);
  FRANK_LAUNCH_CHECK();
  int32_t h = -1;
  FRANK_CUDA_TRY(cudaMemcpyAsync(&h, dres, sizeof(h), cudaMemcpyDeviceToHost, st));
  FRANK_CUDA_TRY(cudaStreamSynchronize(st));
  if (completed) *completed = h;
  return FRANK_OK;
}
