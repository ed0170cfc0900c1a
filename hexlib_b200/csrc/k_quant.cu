// k_quant.cu -- block-quantized weights for matmul_epilogue: q4_0 and q8_0
// (the ggml block formats; hexlib/exec/quant.py, hexlib/graph/ir.py:23-41).
//
// A weight of logical shape [K, N] is stored row-major with its blocks of 32
// running along N: row k holds N/32 blocks, each a fp16 scale d followed by
//   q4_0: 16 bytes, byte j = element j (low nibble) | element j+16 (high),
//         value (nibble - 8) * d                                  (18 bytes)
//   q8_0: 32 int8, value q * d                                    (34 bytes)
//
// The reference's kernel (kernels/matmul_epilogue_fp16/kernel_api.h:188-190,
// baseline.c:36-47) rounds every dequantized weight to fp16 before it is
// multiplied, with fp32 accumulation. Here the weight is dequantized once per
// GEMM into an fp16 [K, N] copy with exactly that rounding (d * q is exact in
// fp32 -- at most 11 + 8 significant bits -- so the one rounding is the fp16
// narrowing, round to nearest even) and the tcgen05 GEMM runs on the copy:
// the encoder's GEMMs are compute-bound at their M, so the weight's bytes do
// not set their speed, and a bit-identical fp16 weight makes the quantized
// path inherit the fp16 path's parity.
//
// One thread per block: 9 (q4_0) or 17 (q8_0) 16-bit loads (blocks are only
// 2-byte aligned), four 16-byte stores of the 32 fp16 results; consecutive
// threads take consecutive blocks, so a warp reads 576 / 1088 contiguous
// bytes and writes 2 KiB contiguous.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hb_kernels.h"

namespace hb {
namespace {

constexpr int kQThreads = 256;

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void dequant_q4_0(const uint16_t* __restrict__ w, uint4* __restrict__ out,
                             int64_t nblocks) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < nblocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const uint16_t* p = w + blk * 9;
    const float d = half_bits_to_float(__ldg(p));
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint16_t two = __ldg(p + 1 + i);          // bytes 2i and 2i+1 of qs
      const int b0 = two & 0xFF, b1 = two >> 8;
      lo[i] = pack2(d * (float)((b0 & 15) - 8), d * (float)((b1 & 15) - 8));
      hi[i] = pack2(d * (float)((b0 >> 4) - 8), d * (float)((b1 >> 4) - 8));
    }
    uint4* o = out + blk * 4;                          // 32 fp16 = 4 x 16 bytes
    o[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);     // elements 0..7
    o[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);     // 8..15
    o[2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);     // 16..23
    o[3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);     // 24..31
  }
}

__global__ void dequant_q8_0(const uint16_t* __restrict__ w, uint4* __restrict__ out,
                             int64_t nblocks) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < nblocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const uint16_t* p = w + blk * 17;
    const float d = half_bits_to_float(__ldg(p));
    uint32_t v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint16_t two = __ldg(p + 1 + i);
      const int8_t q0 = (int8_t)(two & 0xFF), q1 = (int8_t)(two >> 8);
      v[i] = pack2(d * (float)q0, d * (float)q1);
    }
    uint4* o = out + blk * 4;
#pragma unroll
    for (int g = 0; g < 4; ++g) o[g] = make_uint4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
  }
}

int qgrid(int64_t nblocks) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  int64_t g = (nblocks + kQThreads - 1) / kQThreads;
  const int64_t cap = (int64_t)sms * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

int quant_kernels_init() {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, dequant_q4_0) != cudaSuccess ||
      cudaFuncGetAttributes(&a, dequant_q8_0) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int quant_block_bytes(int qtype) {
  return qtype == QTYPE_Q4_0 ? 18 : qtype == QTYPE_Q8_0 ? 34 : 0;
}

int launch_dequant_f16(int qtype, const void* w, void* out, int64_t K, int64_t N,
                       cudaStream_t s) {
  if (K < 0 || N < 0 || N % 32 || quant_block_bytes(qtype) == 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  const int64_t nblocks = K * (N / 32);
  if (nblocks == 0) return HEXLIB_B200_OK;
  if (!w || !out || (reinterpret_cast<uintptr_t>(w) & 1u) ||
      (reinterpret_cast<uintptr_t>(out) & 15u))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (qtype == QTYPE_Q4_0)
    dequant_q4_0<<<qgrid(nblocks), kQThreads, 0, s>>>((const uint16_t*)w, (uint4*)out, nblocks);
  else
    dequant_q8_0<<<qgrid(nblocks), kQThreads, 0, s>>>((const uint16_t*)w, (uint4*)out, nblocks);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int launch_gemm_quant(const GemmDesc& g, int qtype, void* workspace, uint64_t ws_bytes,
                      int* err, cudaStream_t s) {
  if (g.K <= 0 || g.N <= 0 || g.N % 32 || quant_block_bytes(qtype) == 0 || !g.b_shared ||
      g.batch != 1)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  const uint64_t need = (uint64_t)g.K * (uint64_t)g.N * 2u;
  if (!workspace || ws_bytes < need) return HEXLIB_B200_ERR_INVAL_PARAMS;
  const int rc = launch_dequant_f16(qtype, g.B, workspace, g.K, g.N, s);
  if (rc != HEXLIB_B200_OK) return rc;
  GemmDesc d = g;
  d.B = workspace;
  return launch_gemm(d, err, s);
}

}  // namespace hb
