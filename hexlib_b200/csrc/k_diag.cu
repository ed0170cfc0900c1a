// k_diag.cu -- a diagnostic kernel for the bounded-wait failure path.
//
// It initialises an mbarrier that nothing will ever arrive on and waits for
// it with the same bounded wait every pipelined kernel here uses, with a
// caller-chosen limit. The wait gives up, records HB_DEVERR_WAIT_TIMEOUT in
// the session's error word and the kernel returns normally: no trap, no
// fault, no hang. The host then reports HEXLIB_B200_ERR_TIMEOUT and the CUDA
// context remains usable, which is what the failure-detection test checks.
#include <cuda_runtime.h>

#include "hb_device.cuh"
#include "hb_kernels.h"

namespace hb {
namespace {

__global__ void wait_never_arrives(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_wait_limit(&bar, 0, &abort_flag, err, limit_ns);
  }
  __syncthreads();
}

}  // namespace

int diag_kernels_init() {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, wait_never_arrives) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int launch_wait_timeout_probe(int* err, uint32_t limit_us, cudaStream_t s) {
  if (limit_us == 0 || limit_us > 1000000) return HEXLIB_B200_ERR_INVAL_PARAMS;
  wait_never_arrives<<<1, 32, 0, s>>>(err, (uint64_t)limit_us * 1000ull);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

}  // namespace hb
