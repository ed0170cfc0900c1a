// k_attention.cu -- fused attention (placeholder until the tcgen05 kernel
// lands): refuses every call with ERR_NO_KERNEL, so the dispatcher reports the
// op as unserved instead of computing anything.
#include <cuda_runtime.h>

#include "hb_kernels.h"

namespace hb {

int attention_kernels_init() { return HEXLIB_B200_OK; }

int launch_attention(const void*, const void*, const void*, void*, int64_t,
                     int, int, float, int*, cudaStream_t) {
  return HEXLIB_B200_ERR_NO_KERNEL;
}

}  // namespace hb
