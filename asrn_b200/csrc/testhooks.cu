// Test hooks of the C ABI (asrn_test_*): switches and probes the parity and failure-detection tests use. They are no
// part of the reference's interface and the layer forward never calls them.
//
// asrn_test_bounded_wait runs the bounded mbarrier wait every tcgen05 kernel of this library uses (umma::mbar_wait)
// on a barrier that nothing arrives on, with a caller-given limit, inside a kernel that holds TMEM: the wait must give
// up, record ASRN_ERR_TIMEOUT in the status word and let the kernel free its TMEM and return, so the context stays
// usable. Nothing is in flight while it waits (no copy, no MMA), so giving up leaves nothing behind.
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

__global__ void __launch_bounds__(32) k_test_bounded_wait(uint64_t limit_ns, int* status, int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  if (threadIdx.x == 0) {
    umma::mbar_init(&bar, 1);
    umma::fence_mbar_init();
  }
  umma::tmem_alloc(&tmem_base, 32);
  umma::tmem_relinquish();
  __syncwarp();
  umma::tc_fence_after();
  bool ok = true;
  if (threadIdx.x == 0) ok = umma::mbar_wait_limit(&bar, 0, status, limit_ns);   // nothing ever arrives
  __syncwarp();
  umma::tc_fence_before();
  umma::tmem_dealloc(tmem_base, 32);
  if (threadIdx.x == 0) result[0] = ok ? 1 : 0;
}

}  // namespace asrn

extern "C" {

int asrn_test_force_cuda_core(int on) { return asrn::set_force_cuda_core(on); }

int asrn_test_bounded_wait(uint64_t limit_ns, int* status, int* result, void* stream) {
  if (!status || !result) return ASRN_ERR_ARG;
  asrn::k_test_bounded_wait<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, status, result);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // extern "C"
