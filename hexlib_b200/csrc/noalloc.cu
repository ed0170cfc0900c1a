// noalloc.cu -- hexlib_b200_matmul_epilogue_q4_0_noalloc: the q4_0
// matmul_epilogue with its scratch in a fixed device array, for callers that
// cannot allocate device memory or hand the library a workspace.
//
// The scratch (the fp16 copy of the dequantized weight) is the file-scope
// array below, sized for K * N <= 4 Mi weights (8 MiB: every per-block
// weight of the encoder, up to 768 x 3072 and 3072 x 768); a larger weight
// is refused with HEXLIB_B200_ERR_VTCM_TOO_SMALL. The device addresses of the
// array and of the error word are looked up once per device, with that device
// current, by cudaGetSymbolAddress; nothing here calls cudaMalloc, cudaFree or
// any other allocating API, and the shared library initialisation that maps a
// host error word is not used.
//
// What must start at zero: only the error word, which the module load zeroes
// and which a device-side bounded wait sets to 1 if it ever expires; the
// caller learns of it, and the word is cleared, through
// hexlib_b200_stream_status after the stream has drained (the call itself
// returns as soon as the work is queued, so it cannot report it). The weight
// scratch needs no initial value: each call's dequantization writes every
// byte its GEMM then reads.
//
// Calls share the one scratch per device: two calls that overlap in time (on
// different streams, or from different host threads without ordering) race
// on it and may corrupt each other's weight, so callers serialise them, e.g.
// by issuing them on one stream. The first call on a device performs the
// lookup above; make it before beginning any stream capture.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/hexlib_b200.h"
#include "hb_kernels.h"

namespace hb {

namespace {

constexpr uint64_t kScratchBytes = 8ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_weight_scratch[kScratchBytes];
static __device__ int g_noalloc_err;

struct Slots {
  void* scratch = nullptr;
  int* err = nullptr;
};

std::mutex g_mu;
Slots g_slots[kMaxDevices];

int slots_for_current_device(Slots* out) {
  const int init = kernels_init_device();
  if (init != HEXLIB_B200_OK) return init;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  Slots& s = g_slots[dev];
  if (!s.scratch) {
    void* p = nullptr;
    void* e = nullptr;
    if (cudaGetSymbolAddress(&p, g_weight_scratch) != cudaSuccess ||
        cudaGetSymbolAddress(&e, g_noalloc_err) != cudaSuccess || !p || !e) {
      cudaGetLastError();
      return HEXLIB_B200_ERR_CUDA;
    }
    s.scratch = p;
    s.err = static_cast<int*>(e);
  }
  *out = s;
  return HEXLIB_B200_OK;
}

}  // namespace

int noalloc_take_error(bool* set) {
  *set = false;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_slots[dev].err) return HEXLIB_B200_OK;
  }
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  if (v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return HEXLIB_B200_ERR_CUDA;
    }
    *set = true;
  }
  return HEXLIB_B200_OK;
}

}  // namespace hb

extern "C" int hexlib_b200_matmul_epilogue_q4_0_noalloc(const void* a, const void* w,
                                                       const float* bias, void* out, int M,
                                                       int K, int N, int act, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || N % 32 || act < 0 || act > 2 || !bias || !w)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if ((uint64_t)K * (uint64_t)N * 2u > hb::kScratchBytes) return HEXLIB_B200_ERR_VTCM_TOO_SMALL;
  hb::Slots slots;
  const int rc = hb::slots_for_current_device(&slots);
  if (rc != HEXLIB_B200_OK) return rc;
  hb::GemmDesc g{};
  g.A = a;
  g.B = w;
  g.bias = bias;
  g.out = out;
  g.batch = 1;
  g.M = M;
  g.K = K;
  g.N = N;
  g.b_shared = true;
  g.act = act;
  return hb::launch_gemm_quant(g, hb::QTYPE_Q4_0, slots.scratch, hb::kScratchBytes, slots.err,
                               static_cast<cudaStream_t>(stream));
}
