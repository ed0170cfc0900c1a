// k_memory.cu -- the memory-bound kernels: elementwise (add, scale, cast),
// row reductions (layernorm, rmsnorm, softmax), rope_2d, both transposes and
// patchify.
//
// Each one is HBM-bound: it reads every input once and writes every output
// once, so the target is the copy bandwidth of the part. The common shape is
// 16-byte vector loads and stores, grid-stride loops over a grid sized in
// multiples of the SM count, and warp-shuffle reductions with the row held in
// registers. Arithmetic is fp32 with one rounding to fp16 per output, which
// is the contract every kernels/<k>/kernel_api.h states.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <unordered_map>

#include "hb_kernels.h"

namespace hb {
namespace {

constexpr int kThreads = 256;

int sm_count_cached() {
  static int sm_count = 0;
  if (sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (sm_count <= 0) sm_count = 148;
  }
  return sm_count;
}

int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count_cached()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// CTAs of each row kernel that stay resident on the whole device, filled
// once by memory_kernels_init (read-only afterwards).
std::unordered_map<const void*, int> g_resident;

union H8 {
  uint4 u;
  __half2 h2[4];
};

// ---- add -------------------------------------------------------------------
// y[i] = fp16(float(a[i]) + float(b[i % nb]))   (kernels/add_fp16/kernel_api.h)

__global__ void add_f16_vec(const uint4* __restrict__ a,
                            const uint4* __restrict__ b, uint4* __restrict__ y,
                            int64_t nvec, int64_t nbvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    H8 va, vb, vy;
    va.u = __ldg(a + i);
    vb.u = __ldg(b + (nbvec == nvec ? i : i % nbvec));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 fa = __half22float2(va.h2[j]);
      float2 fb = __half22float2(vb.h2[j]);
      vy.h2[j] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
    }
    y[i] = vy.u;
  }
}

__global__ void add_f16_scalar(const __half* __restrict__ a,
                               const __half* __restrict__ b,
                               __half* __restrict__ y, int64_t n, int64_t nb) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i % nb]));
  }
}

// fp16 + fp32 -> fp16, one rounding.
__global__ void add_f16_f32_vec(const uint4* __restrict__ a,
                                const float4* __restrict__ b,
                                uint4* __restrict__ y, int64_t nvec,
                                int64_t nbvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    H8 va, vy;
    va.u = __ldg(a + i);
    const int64_t bi = (nbvec == nvec ? i : i % nbvec);
    float4 b0 = __ldg(b + 2 * bi);
    float4 b1 = __ldg(b + 2 * bi + 1);
    float fb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 fa = __half22float2(va.h2[j]);
      vy.h2[j] = __floats2half2_rn(fa.x + fb[2 * j], fa.y + fb[2 * j + 1]);
    }
    y[i] = vy.u;
  }
}

__global__ void add_f16_f32_scalar(const __half* __restrict__ a,
                                   const float* __restrict__ b,
                                   __half* __restrict__ y, int64_t n,
                                   int64_t nb) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = __float2half_rn(__half2float(a[i]) + b[i % nb]);
  }
}

// ---- scale -----------------------------------------------------------------
// y[i] = fp16(float(x[i]) * factor)   (kernels/scale_fp16/kernel_api.h)

__global__ void scale_f16_vec(const uint4* __restrict__ x,
                              uint4* __restrict__ y, int64_t nvec,
                              float factor) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    H8 v, o;
    v.u = __ldg(x + i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(v.h2[j]);
      o.h2[j] = __floats2half2_rn(__fmul_rn(f.x, factor),
                                  __fmul_rn(f.y, factor));
    }
    y[i] = o.u;
  }
}

__global__ void scale_f16_scalar(const __half* __restrict__ x,
                                 __half* __restrict__ y, int64_t n,
                                 float factor) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = __float2half_rn(__fmul_rn(__half2float(x[i]), factor));
  }
}

// ---- cast ------------------------------------------------------------------
// y[i] = fp16(x[i]), round to nearest even (kernels/cast_f32_f16/kernel_api.h)

__global__ void cast_f32_f16_vec(const float4* __restrict__ x,
                                 uint4* __restrict__ y, int64_t nvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = __ldg(x + 2 * i);
    float4 b = __ldg(x + 2 * i + 1);
    H8 o;
    o.h2[0] = __floats2half2_rn(a.x, a.y);
    o.h2[1] = __floats2half2_rn(a.z, a.w);
    o.h2[2] = __floats2half2_rn(b.x, b.y);
    o.h2[3] = __floats2half2_rn(b.z, b.w);
    y[i] = o.u;
  }
}

__global__ void cast_f32_f16_scalar(const float* __restrict__ x,
                                    __half* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = __float2half_rn(x[i]);
  }
}

__global__ void copy_vec(const uint4* __restrict__ x, uint4* __restrict__ y,
                         int64_t nvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = __ldg(x + i);
  }
}

__global__ void copy_bytes(const uint8_t* __restrict__ x,
                           uint8_t* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = x[i];
  }
}

// ---- warp reductions ---------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- row kernels: layernorm, rmsnorm, softmax --------------------------------------
// ROW LAYOUT. A row of C = G * V * 8 fp16 is owned by G threads and held in
// their registers as V 16-byte vectors each: vector j*G + g of the row is
// thread g's j-th, so the G threads read G consecutive vectors per access.
// G = 8, 16 or 32 are lanes of one warp (32 / G rows per warp, shuffles of
// width G); G = 256 is a whole CTA (one row per CTA, a shared-memory combine
// across its 8 warps) for rows of 2048 and more. Each warp or CTA walks its
// rows with the next row's loads in flight while the current one is reduced,
// and the launcher sizes the grid to the CTAs that stay resident.

template <int G>
__device__ __forceinline__ float row_sum(float v, float* red) {
  if constexpr (G <= 32) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  } else {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < G / 32; ++i) t += red[i];
    __syncthreads();  // red is reused by the next reduction
    return t;
  }
}

template <int G>
__device__ __forceinline__ float row_max(float v, float* red) {
  if constexpr (G <= 32) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  } else {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = -INFINITY;
#pragma unroll
    for (int i = 0; i < G / 32; ++i) t = fmaxf(t, red[i]);
    __syncthreads();
    return t;
  }
}

// Which rows a thread walks: rows base + sub for base = first, first + step,
// ... while base < R (uniform across the warp or CTA that shares a row), and
// its index g within the row's G threads.
template <int G>
struct RowWalk {
  int g, sub;
  int64_t first, step;
  __device__ RowWalk() {
    if constexpr (G <= 32) {
      const int lane = threadIdx.x & 31;
      g = lane % G;
      sub = lane / G;
      const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
      first = warp * (32 / G);
      step = (((int64_t)gridDim.x * blockDim.x) >> 5) * (32 / G);
    } else {
      g = threadIdx.x;
      sub = 0;
      first = blockIdx.x;
      step = gridDim.x;
    }
  }
};

template <int G, int V>
__device__ __forceinline__ void row_load(uint4 (&d)[V], const uint4* __restrict__ x,
                                         int64_t r, int g) {
  constexpr int C8 = G * V;
#pragma unroll
  for (int j = 0; j < V; ++j) d[j] = __ldg(x + r * C8 + j * G + g);
}

template <int V>
__device__ __forceinline__ void unpack_rows(float (&v)[V][8], const uint4 (&d)[V]) {
#pragma unroll
  for (int j = 0; j < V; ++j) {
    H8 h;
    h.u = d[j];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(h.h2[q]);
      v[j][2 * q] = f.x;
      v[j][2 * q + 1] = f.y;
    }
  }
}

// Sum and max of a thread's V x 8 values of a row in four independent chains
// (two-wide adds, three-input maxima), so no operation waits on the one
// before it the way a single running sum would.
template <int V>
__device__ __forceinline__ float frag_sum(const float (&v)[V][8]) {
  float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 8; q += 4) {
      a = __fadd2_rn(a, make_float2(v[j][q], v[j][q + 1]));
      b = __fadd2_rn(b, make_float2(v[j][q + 2], v[j][q + 3]));
    }
  return (a.x + a.y) + (b.x + b.y);
}

template <int V>
__device__ __forceinline__ float frag_max(const float (&v)[V][8]) {
  float m[4] = {v[0][0], v[0][1], v[0][2], v[0][3]};
#pragma unroll
  for (int q = 0; q < 4; ++q) m[q] = fmaxf(m[q], v[0][4 + q]);
#pragma unroll
  for (int j = 1; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float d;
      asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(m[q]), "f"(v[j][q]), "f"(v[j][4 + q]));
      m[q] = d;
    }
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// A row's mean and 1/sqrt(biased variance + eps), the variance taken over
// the centred values (two passes over the row in registers). Shared by
// layernorm_rows, layernorm_rows_wb and ln_stats_rows, which lay a row out the
// same way for a given width, so the statistics a folded-layernorm GEMM
// applies are exactly the ones the unfolded layernorm uses. (Running sums in one
// chain: with four chains and two-wide arithmetic the 768-wide variant
// needs 130 registers, halving its residency, and measured 7-9% slower.)
template <int G, int V>
__device__ __forceinline__ void row_moments(const float (&v)[V][8], float* red, float eps,
                                            float& mean, float& inv) {
  constexpr int C = G * V * 8;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 8; ++q) s += v[j][q];
  mean = row_sum<G>(s, red) * (1.0f / C);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float d = v[j][q] - mean;
      ss += d * d;
    }
  const float var = row_sum<G>(ss, red) * (1.0f / C);
  inv = 1.0f / sqrtf(var + eps);
}

// layernorm: the mean, then the biased variance of the centred values
// (kernels/layernorm_fp16/kernel_api.h:7-29).
template <int G, int V>
__global__ void __launch_bounds__(kThreads) layernorm_rows(const uint4* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ b,
                                                           uint4* __restrict__ y, int64_t R,
                                                           float eps, int rev) {
  __shared__ float red[kThreads / 32];
  const RowWalk<G> rw;
  // the k-th row walked is row k, or row R - 1 - k when rev
  auto at = [&](int64_t k) { return rev ? R - 1 - k : k; };
  uint4 nxt[V];
  if (rw.first + rw.sub < R) row_load<G, V>(nxt, x, at(rw.first + rw.sub), rw.g);
  for (int64_t base = rw.first; base < R; base += rw.step) {
    const int64_t r = base + rw.sub;
    float v[V][8];
    unpack_rows<V>(v, nxt);
    if (r + rw.step < R) row_load<G, V>(nxt, x, at(r + rw.step), rw.g);
    float mean, inv;
    row_moments<G, V>(v, red, eps, mean, inv);
    if (r < R) {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int c0 = (j * G + rw.g) * 8;
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + c0));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + c0 + 4));
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(b + c0));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(b + c0 + 4));
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        H8 o;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          o.h2[q] = __floats2half2_rn((v[j][2 * q] - mean) * inv * ww[2 * q] + bb[2 * q],
                                      (v[j][2 * q + 1] - mean) * inv * ww[2 * q + 1] +
                                          bb[2 * q + 1]);
        y[at(r) * (G * V) + j * G + rw.g] = o.u;
      }
    }
  }
}

// layernorm with one row per warp (32 lanes x V vectors) and the affine
// weight and bias in registers: a lane meets the same V * 8 columns in every
// row it walks, so it loads their weight and bias once per launch instead of
// four 16-byte loads per 8 outputs per row, which for fp32 weights is four
// times the row's own bytes in L1 traffic. D rows of each warp are in flight
// ahead of the one being reduced (D = 1 and 2 measured alike in the encoder).
#ifndef HB_LN_DEPTH
#define HB_LN_DEPTH 1
#endif
template <int V, int D>
__global__ void __launch_bounds__(kThreads) layernorm_rows_wb(const uint4* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ b,
                                                              uint4* __restrict__ y, int64_t R,
                                                              float eps, int rev) {
  constexpr int G = 32;
  __shared__ float red[kThreads / 32];
  const RowWalk<G> rw;
  auto at = [&](int64_t k) { return rev ? R - 1 - k : k; };
  float ww[V][8], bb[V][8];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c0 = (j * G + rw.g) * 8;
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + c0));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + c0 + 4));
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(b + c0));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(b + c0 + 4));
    ww[j][0] = w0.x; ww[j][1] = w0.y; ww[j][2] = w0.z; ww[j][3] = w0.w;
    ww[j][4] = w1.x; ww[j][5] = w1.y; ww[j][6] = w1.z; ww[j][7] = w1.w;
    bb[j][0] = b0.x; bb[j][1] = b0.y; bb[j][2] = b0.z; bb[j][3] = b0.w;
    bb[j][4] = b1.x; bb[j][5] = b1.y; bb[j][6] = b1.z; bb[j][7] = b1.w;
  }
  uint4 nxt[D][V];
#pragma unroll
  for (int d = 0; d < D; ++d)
    if (rw.first + d * rw.step < R) row_load<G, V>(nxt[d], x, at(rw.first + d * rw.step), rw.g);
  for (int64_t r = rw.first; r < R; r += rw.step) {
    float v[V][8];
    unpack_rows<V>(v, nxt[0]);
#pragma unroll
    for (int d = 0; d + 1 < D; ++d)
#pragma unroll
      for (int j = 0; j < V; ++j) nxt[d][j] = nxt[d + 1][j];
    if (r + D * rw.step < R) row_load<G, V>(nxt[D - 1], x, at(r + D * rw.step), rw.g);
    float mean, inv;
    row_moments<G, V>(v, red, eps, mean, inv);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      H8 o;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o.h2[q] = __floats2half2_rn((v[j][2 * q] - mean) * inv * ww[j][2 * q] + bb[j][2 * q],
                                    (v[j][2 * q + 1] - mean) * inv * ww[j][2 * q + 1] +
                                        bb[j][2 * q + 1]);
      y[at(r) * (G * V) + j * G + rw.g] = o.u;
    }
  }
}

// The row statistics of layernorm alone: (mean, 1/sqrt(var + eps)) per row,
// computed exactly as layernorm_rows computes them, for a GEMM that applies
// the normalisation in its epilogue (the affine weight folded into its
// matrix). Reads the rows once and writes 8 bytes per row.
template <int G, int V>
__global__ void __launch_bounds__(kThreads) ln_stats_rows(const uint4* __restrict__ x,
                                                          float2* __restrict__ stats, int64_t R,
                                                          float eps) {
  __shared__ float red[kThreads / 32];
  const RowWalk<G> rw;
  uint4 nxt[V];
  if (rw.first + rw.sub < R) row_load<G, V>(nxt, x, rw.first + rw.sub, rw.g);
  for (int64_t base = rw.first; base < R; base += rw.step) {
    const int64_t r = base + rw.sub;
    float v[V][8];
    unpack_rows<V>(v, nxt);
    if (r + rw.step < R) row_load<G, V>(nxt, x, r + rw.step, rw.g);
    float mean, inv;
    row_moments<G, V>(v, red, eps, mean, inv);
    if (r < R && rw.g == 0) stats[r] = make_float2(mean, inv);
  }
}

// rmsnorm: y = fp16(x * (1/sqrt(mean(x^2) + eps)) * w), w fp16
// (kernels/rmsnorm_fp16/kernel_api.h:8-14).
template <int G, int V>
__global__ void __launch_bounds__(kThreads) rmsnorm_rows(const uint4* __restrict__ x,
                                                         const uint4* __restrict__ w,
                                                         uint4* __restrict__ y, int64_t R,
                                                         float eps) {
  constexpr int C = G * V * 8;
  __shared__ float red[kThreads / 32];
  const RowWalk<G> rw;
  uint4 nxt[V];
  if (rw.first + rw.sub < R) row_load<G, V>(nxt, x, rw.first + rw.sub, rw.g);
  for (int64_t base = rw.first; base < R; base += rw.step) {
    const int64_t r = base + rw.sub;
    float v[V][8];
    unpack_rows<V>(v, nxt);
    if (r + rw.step < R) row_load<G, V>(nxt, x, r + rw.step, rw.g);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += v[j][q] * v[j][q];
    const float inv = 1.0f / sqrtf(row_sum<G>(ss, red) * (1.0f / C) + eps);
    if (r < R) {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        H8 hw, o;
        hw.u = __ldg(w + j * G + rw.g);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fw = __half22float2(hw.h2[q]);
          o.h2[q] = __floats2half2_rn(v[j][2 * q] * inv * fw.x, v[j][2 * q + 1] * inv * fw.y);
        }
        y[r * (G * V) + j * G + rw.g] = o.u;
      }
    }
  }
}

// softmax: max, exp of the shifted values, sum, divide; fp32 throughout and
// one rounding (kernels/softmax_fp16/kernel_api.h:9-16).
template <int G, int V>
__global__ void __launch_bounds__(kThreads) softmax_rows(const uint4* __restrict__ x,
                                                         uint4* __restrict__ y, int64_t R) {
  __shared__ float red[kThreads / 32];
  const RowWalk<G> rw;
  uint4 nxt[V];
  if (rw.first + rw.sub < R) row_load<G, V>(nxt, x, rw.first + rw.sub, rw.g);
  for (int64_t base = rw.first; base < R; base += rw.step) {
    const int64_t r = base + rw.sub;
    float v[V][8];
    unpack_rows<V>(v, nxt);
    if (r + rw.step < R) row_load<G, V>(nxt, x, r + rw.step, rw.g);
    // e^(x - max) = 2^(x log2(e) - max log2(e)): one FMA and the hardware's
    // approximate 2^x per value (relative error near 2^-22, far below the
    // fp16 rounding of the result); the row sum in four chains; one division
    // per row, then a multiply per value.
    const float ml = row_max<G>(frag_max<V>(v), red) * 1.4426950408889634f;
    const float2 l2 = make_float2(1.4426950408889634f, 1.4426950408889634f);
    const float2 nml = make_float2(-ml, -ml);
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int q = 0; q < 8; q += 2) {
        const float2 a = __ffma2_rn(make_float2(v[j][q], v[j][q + 1]), l2, nml);
        float e0, e1;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a.x));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a.y));
        v[j][q] = e0;
        v[j][q + 1] = e1;
      }
    const float inv = 1.0f / row_sum<G>(frag_sum<V>(v), red);
    if (r < R) {
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        H8 o;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 pv = __fmul2_rn(make_float2(v[j][2 * q], v[j][2 * q + 1]), inv2);
          o.h2[q] = __floats2half2_rn(pv.x, pv.y);
        }
        y[r * (G * V) + j * G + rw.g] = o.u;
      }
    }
  }
}

// Any C: one warp per row, three passes over global memory.

// Any C: one warp per row, three passes over global memory.
__global__ void layernorm_f16_generic(const __half* __restrict__ x,
                                      const float* __restrict__ w,
                                      const float* __restrict__ b,
                                      __half* __restrict__ y, int64_t R, int C,
                                      float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp0; r < R; r += nwarps) {
    const __half* xr = x + r * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += __half2float(xr[c]);
    const float mean = warp_sum(s) / (float)C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float d = __half2float(xr[c]) - mean;
      ss += d * d;
    }
    const float var = warp_sum(ss) / (float)C;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int c = lane; c < C; c += 32)
      y[r * C + c] =
          __float2half_rn((__half2float(xr[c]) - mean) * inv * w[c] + b[c]);
  }
}

// ln_stats for any C: one warp per row, two passes over global memory.
__global__ void ln_stats_generic(const __half* __restrict__ x, float2* __restrict__ stats,
                                 int64_t R, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp0; r < R; r += nwarps) {
    const __half* xr = x + r * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += __half2float(xr[c]);
    const float mean = warp_sum(s) / (float)C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float d = __half2float(xr[c]) - mean;
      ss += d * d;
    }
    const float var = warp_sum(ss) / (float)C;
    if (lane == 0) stats[r] = make_float2(mean, 1.0f / sqrtf(var + eps));
  }
}

__global__ void rmsnorm_f16_generic(const __half* __restrict__ x,
                                    const __half* __restrict__ w,
                                    __half* __restrict__ y, int64_t R, int C,
                                    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp0; r < R; r += nwarps) {
    const __half* xr = x + r * C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float f = __half2float(xr[c]);
      ss += f * f;
    }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / (float)C + eps);
    for (int c = lane; c < C; c += 32)
      y[r * C + c] =
          __float2half_rn(__half2float(xr[c]) * inv * __half2float(w[c]));
  }
}

__global__ void softmax_f16_generic(const __half* __restrict__ x,
                                    __half* __restrict__ y, int64_t R, int C) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp0; r < R; r += nwarps) {
    const __half* xr = x + r * C;
    float m = -INFINITY;
    for (int c = lane; c < C; c += 32) m = fmaxf(m, __half2float(xr[c]));
    m = warp_max(m);
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += expf(__half2float(xr[c]) - m);
    const float sum = warp_sum(s);
    for (int c = lane; c < C; c += 32)
      y[r * C + c] = __float2half_rn(expf(__half2float(xr[c]) - m) / sum);
  }
}

// ---- rope_2d ---------------------------------------------------------------------
// Split-half rotation (kernels/rope_2d_fp16/kernel_api.h:17-26):
//   y[i]      = x[i]      * cos[i]      - x[i+h] * sin[i]
//   y[i + h]  = x[i + h]  * cos[i + h]  + x[i]   * sin[i + h]
// evaluated as the op registry does (structural.py:249-254): the two products
// rounded to fp32 separately, then added, so no fused multiply-add changes a
// rounding. One thread per 8 columns of the first half of one (token, head).

__global__ void rope_f16_vec(const uint4* __restrict__ x,
                             const float* __restrict__ cos_t,
                             const float* __restrict__ sin_t,
                             uint4* __restrict__ y, int64_t rows, int H, int D,
                             int64_t table_rows) {
  const int half = D >> 1;
  const int cpr = half >> 3;  // 8-wide chunks per half
  const int64_t total = rows * H * cpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % cpr);
    const int64_t th = i / cpr;  // token * H + head
    const int64_t t = th / H;
    const int64_t tt = t % table_rows;
    const int64_t base = th * D;  // element offset of this (token, head)
    const int i0 = c * 8;
    H8 lo, hi, olo, ohi;
    lo.u = __ldg(x + (base + i0) / 8);
    hi.u = __ldg(x + (base + half + i0) / 8);
    const float* ct = cos_t + tt * D;
    const float* st = sin_t + tt * D;
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(ct + i0));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(ct + i0 + 4));
    const float4 c2 = __ldg(reinterpret_cast<const float4*>(ct + half + i0));
    const float4 c3 =
        __ldg(reinterpret_cast<const float4*>(ct + half + i0 + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(st + i0));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(st + i0 + 4));
    const float4 s2 = __ldg(reinterpret_cast<const float4*>(st + half + i0));
    const float4 s3 =
        __ldg(reinterpret_cast<const float4*>(st + half + i0 + 4));
    const float cl[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ch[8] = {c2.x, c2.y, c2.z, c2.w, c3.x, c3.y, c3.z, c3.w};
    const float sl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float sh[8] = {s2.x, s2.y, s2.z, s2.w, s3.x, s3.y, s3.z, s3.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = __half22float2(lo.h2[q]);
      const float2 b = __half22float2(hi.h2[q]);
      const float ylo0 = __fadd_rn(__fmul_rn(a.x, cl[2 * q]),
                                   __fmul_rn(-b.x, sl[2 * q]));
      const float ylo1 = __fadd_rn(__fmul_rn(a.y, cl[2 * q + 1]),
                                   __fmul_rn(-b.y, sl[2 * q + 1]));
      const float yhi0 = __fadd_rn(__fmul_rn(b.x, ch[2 * q]),
                                   __fmul_rn(a.x, sh[2 * q]));
      const float yhi1 = __fadd_rn(__fmul_rn(b.y, ch[2 * q + 1]),
                                   __fmul_rn(a.y, sh[2 * q + 1]));
      olo.h2[q] = __floats2half2_rn(ylo0, ylo1);
      ohi.h2[q] = __floats2half2_rn(yhi0, yhi1);
    }
    y[(base + i0) / 8] = olo.u;
    y[(base + half + i0) / 8] = ohi.u;
  }
}

__global__ void rope_f16_scalar(const __half* __restrict__ x,
                                const float* __restrict__ cos_t,
                                const float* __restrict__ sin_t,
                                __half* __restrict__ y, int64_t rows, int H,
                                int D, int64_t table_rows) {
  const int half = D >> 1;
  const int64_t total = rows * H * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int64_t th = i / half;
    const int64_t tt = (th / H) % table_rows;
    const int64_t base = th * D;
    const float a = __half2float(x[base + j]);
    const float b = __half2float(x[base + half + j]);
    const float* ct = cos_t + tt * D;
    const float* st = sin_t + tt * D;
    y[base + j] = __float2half_rn(
        __fadd_rn(__fmul_rn(a, ct[j]), __fmul_rn(-b, st[j])));
    y[base + half + j] = __float2half_rn(
        __fadd_rn(__fmul_rn(b, ct[half + j]), __fmul_rn(a, st[half + j])));
  }
}

// ---- rope over the packed projection, in place -------------------------------------
// qkv is [rows, 3, H, D]; the q and k sections (0 and 1) of every row are
// rotated exactly as rope_f16_vec rotates a [T, H, D] tensor, the v section is
// untouched. Each thread reads the 16 bytes it later writes, so x == y is safe.
__global__ void rope_qk_vec(const uint4* x, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, uint4* y, int64_t rows,
                            int H, int D, int64_t table_rows) {
  const int half = D >> 1;
  const int cpr = half >> 3;                       // 8-wide chunks per half
  const int64_t per_row = 2LL * H * cpr;           // q and k heads
  const int64_t total = rows * per_row;
  const int64_t row_elems = 3LL * H * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row;
    const int rem = (int)(i - row * per_row);
    const int c = rem % cpr;
    const int sh = rem / cpr;                      // section * H + head, section < 2
    const int64_t tt = row % table_rows;
    const int64_t base = row * row_elems + (int64_t)sh * D;
    const int i0 = c * 8;
    H8 lo, hi, olo, ohi;
    lo.u = x[(base + i0) / 8];
    hi.u = x[(base + half + i0) / 8];
    const float* ct = cos_t + tt * D;
    const float* st = sin_t + tt * D;
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(ct + i0));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(ct + i0 + 4));
    const float4 c2 = __ldg(reinterpret_cast<const float4*>(ct + half + i0));
    const float4 c3 = __ldg(reinterpret_cast<const float4*>(ct + half + i0 + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(st + i0));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(st + i0 + 4));
    const float4 s2 = __ldg(reinterpret_cast<const float4*>(st + half + i0));
    const float4 s3 = __ldg(reinterpret_cast<const float4*>(st + half + i0 + 4));
    const float cl[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ch[8] = {c2.x, c2.y, c2.z, c2.w, c3.x, c3.y, c3.z, c3.w};
    const float sl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float sh8[8] = {s2.x, s2.y, s2.z, s2.w, s3.x, s3.y, s3.z, s3.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = __half22float2(lo.h2[q]);
      const float2 b = __half22float2(hi.h2[q]);
      const float ylo0 = __fadd_rn(__fmul_rn(a.x, cl[2 * q]), __fmul_rn(-b.x, sl[2 * q]));
      const float ylo1 = __fadd_rn(__fmul_rn(a.y, cl[2 * q + 1]), __fmul_rn(-b.y, sl[2 * q + 1]));
      const float yhi0 = __fadd_rn(__fmul_rn(b.x, ch[2 * q]), __fmul_rn(a.x, sh8[2 * q]));
      const float yhi1 = __fadd_rn(__fmul_rn(b.y, ch[2 * q + 1]), __fmul_rn(a.y, sh8[2 * q + 1]));
      olo.h2[q] = __floats2half2_rn(ylo0, ylo1);
      ohi.h2[q] = __floats2half2_rn(yhi0, yhi1);
    }
    y[(base + i0) / 8] = olo.u;
    y[(base + half + i0) / 8] = ohi.u;
  }
}

// ---- transpose_th: [T,H,D] -> [H,T,D] per image ----------------------------------
// D is innermost on both sides, so the op moves whole D-runs: one thread per
// 16-byte vector, coalesced on both sides.

__global__ void transpose_th_vec(const uint4* __restrict__ x,
                                 uint4* __restrict__ y, int64_t nimg, int T,
                                 int H, int DV) {
  const int64_t per = (int64_t)T * H * DV;
  const int64_t total = nimg * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t img = i / per;
    int64_t r = i - img * per;  // index in the OUTPUT [H,T,DV]
    const int dv = (int)(r % DV);
    r /= DV;
    const int t = (int)(r % T);
    const int h = (int)(r / T);
    y[i] = __ldg(x + img * per + ((int64_t)t * H + h) * DV + dv);
  }
}

__global__ void transpose_th_scalar(const __half* __restrict__ x,
                                    __half* __restrict__ y, int64_t nimg,
                                    int T, int H, int D) {
  const int64_t per = (int64_t)T * H * D;
  const int64_t total = nimg * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t img = i / per;
    int64_t r = i - img * per;
    const int d = (int)(r % D);
    r /= D;
    const int t = (int)(r % T);
    const int h = (int)(r / T);
    y[i] = x[img * per + ((int64_t)t * H + h) * D + d];
  }
}

// ---- transpose_hd: [B,T,D] -> [B,D,T] ---------------------------------------------
// 64x64 tiles through shared memory (padded against bank conflicts): both
// the read of T x D rows and the write of D x T rows are coalesced.

constexpr int kTile = 64;

__global__ void transpose_hd_tiled(const __half* __restrict__ x,
                                   __half* __restrict__ y, int64_t B, int T,
                                   int D) {
  __shared__ __half tile[kTile][kTile + 2];
  const int tiles_t = (T + kTile - 1) / kTile;
  const int tiles_d = (D + kTile - 1) / kTile;
  const int64_t ntiles = B * tiles_t * tiles_d;
  for (int64_t tid = blockIdx.x; tid < ntiles; tid += gridDim.x) {
    const int64_t b = tid / ((int64_t)tiles_t * tiles_d);
    const int rem = (int)(tid - b * tiles_t * tiles_d);
    const int t0 = (rem / tiles_d) * kTile;
    const int d0 = (rem % tiles_d) * kTile;
    const __half* xb = x + b * (int64_t)T * D;
    __half* yb = y + b * (int64_t)T * D;
    // load: rows t, columns d (d fastest across threads)
    for (int e = threadIdx.x; e < kTile * kTile; e += blockDim.x) {
      const int tr = e / kTile, dc = e % kTile;
      const int t = t0 + tr, d = d0 + dc;
      if (t < T && d < D) tile[tr][dc] = xb[(int64_t)t * D + d];
    }
    __syncthreads();
    // store: rows d, columns t (t fastest across threads)
    for (int e = threadIdx.x; e < kTile * kTile; e += blockDim.x) {
      const int dr = e / kTile, tc = e % kTile;
      const int t = t0 + tc, d = d0 + dr;
      if (t < T && d < D) yb[(int64_t)d * T + t] = tile[tc][dr];
    }
    __syncthreads();
  }
}

// Vector form (T % 8 == 0, D % 8 == 0, 16-byte aligned): 16-byte loads of 8
// consecutive d of one t, 16-byte stores of 8 consecutive t of one d. The
// 64 x 64 tile sits in shared memory as 64 rows of t, its 16-byte chunks
// XOR-swizzled by (t >> 3) & 7: a quarter-warp's row write touches 8
// distinct chunks, and the column gather of eight threads that share d but
// not t >> 3 reads 8 distinct chunks -- no bank conflicts either way.
__global__ void transpose_hd_vec(const uint4* __restrict__ x, uint4* __restrict__ y,
                                 int64_t B, int T, int D) {
  __shared__ __align__(16) __half tile[kTile * kTile];
  const int tiles_t = (T + kTile - 1) / kTile;
  const int tiles_d = (D + kTile - 1) / kTile;
  const int64_t ntiles = B * tiles_t * tiles_d;
  const int dv = D / 8, tv = T / 8;              // uint4 per input row / output row
  for (int64_t tid = blockIdx.x; tid < ntiles; tid += gridDim.x) {
    const int64_t b = tid / ((int64_t)tiles_t * tiles_d);
    const int rem = (int)(tid - b * tiles_t * tiles_d);
    const int t0 = (rem / tiles_d) * kTile;
    const int d0 = (rem % tiles_d) * kTile;
    const uint4* xb = x + b * (int64_t)T * dv;
    uint4* yb = y + b * (int64_t)D * tv;
    // 512 chunks: (row t, chunk c of 8 d)
#pragma unroll
    for (int e = threadIdx.x; e < kTile * 8; e += kThreads) {
      const int tr = e >> 3, c = e & 7;
      const int t = t0 + tr, d = d0 + c * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < T && d < D) v = __ldg(xb + (int64_t)t * dv + d / 8);
      *reinterpret_cast<uint4*>(&tile[tr * kTile + ((c ^ ((tr >> 3) & 7)) * 8)]) = v;
    }
    __syncthreads();
    // 512 outputs: (row d, chunk t8 of 8 t); eight consecutive threads cover
    // one d row's 64 t, so a warp stores four 128-byte row segments
#pragma unroll
    for (int e = threadIdx.x; e < kTile * 8; e += kThreads) {
      const int dr = e >> 3, t8 = e & 7;
      const int d = d0 + dr, t = t0 + t8 * 8;
      const int c = dr >> 3, w = dr & 7;
      __align__(16) __half h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = tile[(t8 * 8 + i) * kTile + ((c ^ t8) * 8) + w];
      if (d < D && t < T) yb[(int64_t)d * tv + t / 8] = *reinterpret_cast<const uint4*>(h);
    }
    __syncthreads();
  }
}

// ---- patchify ---------------------------------------------------------------------
// [C,T,H,W] -> [gh*gw, C*T*p*p] in merge-block token order
// (kernels/patchify_fp32/kernel_api.h:18-38; structural.py:172-207):
//   token = ((bh*Bw + bw)*merge + mh)*merge + mw,  gh = bh*merge + mh, ...
//   feature = ((c*T + t)*p + ph)*p + pw
// One thread per output float4 (4 consecutive pw): a pure, bit-exact move.

__global__ void patchify_vec(const float4* __restrict__ img,
                             float4* __restrict__ out, int64_t nimg, int C,
                             int T, int H, int W, int patch, int merge,
                             int grid_w) {
  const int feat = C * T * patch * patch;
  const int fv = feat / 4;
  const int ntok = (H / patch) * grid_w;
  const int64_t per = (int64_t)ntok * fv;
  const int64_t total = nimg * per;
  const int bw_n = grid_w / merge;
  const int pv = patch / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / per;
    const int64_t r = i - n * per;
    const int tok = (int)(r / fv);
    const int f4 = (int)(r % fv);
    const int pw4 = f4 % pv;
    int q = f4 / pv;
    const int ph = q % patch;
    q /= patch;
    const int t = q % T;
    const int c = q / T;
    const int mw = tok % merge;
    int u = tok / merge;
    const int mh = u % merge;
    u /= merge;
    const int bw = u % bw_n;
    const int bh = u / bw_n;
    const int gh = bh * merge + mh, gw = bw * merge + mw;
    const int h = gh * patch + ph;
    const int64_t src =
        ((((n * C + c) * T + t) * (int64_t)H + h) * W + gw * patch) / 4 + pw4;
    out[i] = __ldg(img + src);
  }
}

// The same move organised by merge block: a CTA takes the merge*merge
// tokens of one merge block (a contiguous span of the output) and first
// tabulates, for each output float4 of a token, its source offset from the
// patch's top-left corner -- so the copy loop has no divisions, which
// otherwise cost more issue slots than the move itself.
// OUT_F16: each float4 is rounded to four fp16 on the way out (round to
// nearest even, as the cast op rounds), so patchify followed by the cast to
// fp16 becomes one pass that writes half the bytes.
template <bool OUT_F16>
__global__ void patchify_blocks(const float4* __restrict__ img, void* __restrict__ out,
                                int64_t n_blocks, int blocks_per_img, int bw_n, int merge,
                                int patch, int C, int T, int H, int W4, int fv) {
  extern __shared__ int src_off[];             // [fv]
  const int pv = patch / 4;
  for (int f = threadIdx.x; f < fv; f += blockDim.x) {
    const int pw4 = f % pv;
    int q = f / pv;
    const int ph = q % patch;
    q /= patch;
    const int t = q % T;
    const int c = q / T;
    src_off[f] = ((c * T + t) * H + ph) * W4 + pw4;
  }
  __syncthreads();
  const int64_t img4 = (int64_t)C * T * H * W4;
  const int mm = merge * merge;
  for (int64_t mb = blockIdx.x; mb < n_blocks; mb += gridDim.x) {
    const int64_t n = mb / blocks_per_img;
    const int rb = (int)(mb - n * blocks_per_img);
    const int bh = rb / bw_n, bw = rb - bh * bw_n;
    const float4* src_n = img + n * img4;
    const int64_t dst0 = mb * mm * (int64_t)fv;     // in float4 units of the output
    for (int m = 0; m < mm; ++m) {
      const int mh = m / merge, mw = m - mh * merge;
      const float4* src =
          src_n + (int64_t)((bh * merge + mh) * patch) * W4 + (bw * merge + mw) * pv;
      const int64_t d0 = dst0 + (int64_t)m * fv;
      if constexpr (OUT_F16) {
        uint2* d = reinterpret_cast<uint2*>(out) + d0;
#pragma unroll 4
        for (int f = threadIdx.x; f < fv; f += blockDim.x) {
          const float4 v = __ldg(src + src_off[f]);
          const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
          d[f] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                            *reinterpret_cast<const uint32_t*>(&hi));
        }
      } else {
        float4* d = reinterpret_cast<float4*>(out) + d0;
#pragma unroll 4
        for (int f = threadIdx.x; f < fv; f += blockDim.x) d[f] = __ldg(src + src_off[f]);
      }
    }
  }
}

__global__ void patchify_scalar(const float* __restrict__ img,
                                float* __restrict__ out, int64_t nimg, int C,
                                int T, int H, int W, int patch, int merge,
                                int grid_w) {
  const int feat = C * T * patch * patch;
  const int ntok = (H / patch) * grid_w;
  const int64_t per = (int64_t)ntok * feat;
  const int64_t total = nimg * per;
  const int bw_n = grid_w / merge;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / per;
    const int64_t r = i - n * per;
    const int tok = (int)(r / feat);
    const int f = (int)(r % feat);
    const int pw = f % patch;
    int q = f / patch;
    const int ph = q % patch;
    q /= patch;
    const int t = q % T;
    const int c = q / T;
    const int mw = tok % merge;
    int u = tok / merge;
    const int mh = u % merge;
    u /= merge;
    const int bw = u % bw_n;
    const int bh = u / bw_n;
    const int gh = bh * merge + mh, gw = bw * merge + mw;
    out[i] = img[(((n * C + c) * T + t) * (int64_t)H + gh * patch + ph) * W +
                 gw * patch + pw];
  }
}

}  // namespace

// ---- launchers ------------------------------------------------------------------

// Load every kernel of this file now, so that no module load happens lazily
// inside a CUDA-graph capture.
int memory_kernels_init() {
  const void* fns[] = {
      (const void*)add_f16_vec,         (const void*)add_f16_scalar,
      (const void*)add_f16_f32_vec,     (const void*)add_f16_f32_scalar,
      (const void*)scale_f16_vec,       (const void*)scale_f16_scalar,
      (const void*)cast_f32_f16_vec,    (const void*)cast_f32_f16_scalar,
      (const void*)copy_vec,            (const void*)copy_bytes,
      (const void*)layernorm_f16_generic, (const void*)rmsnorm_f16_generic,
      (const void*)softmax_f16_generic, (const void*)rope_f16_vec,
      (const void*)rope_f16_scalar,     (const void*)transpose_th_vec,
      (const void*)rope_qk_vec,
      (const void*)transpose_th_scalar, (const void*)transpose_hd_tiled,
      (const void*)transpose_hd_vec,
      (const void*)patchify_vec,        (const void*)patchify_scalar,
  };
  for (const void* f : fns) {
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, f) != cudaSuccess) {
      cudaGetLastError();
      return HEXLIB_B200_ERR_CUDA;
    }
  }
  grid_for(1, kThreads);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto note = [&](const void* f) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, kThreads, 0) != cudaSuccess) {
      cudaGetLastError();
      per_sm = 0;
    }
    g_resident[f] = per_sm * sms;
  };
#define HB_NOTE_ROWS(K)                                                             \
  note((const void*)K<8, 1>); note((const void*)K<16, 1>); note((const void*)K<32, 1>); \
  note((const void*)K<32, 2>); note((const void*)K<32, 3>); note((const void*)K<32, 4>); \
  note((const void*)K<256, 1>); note((const void*)K<256, 2>); note((const void*)K<256, 4>);
  HB_NOTE_ROWS(layernorm_rows)
  note((const void*)layernorm_rows_wb<2, HB_LN_DEPTH>);
  note((const void*)layernorm_rows_wb<3, HB_LN_DEPTH>);
  HB_NOTE_ROWS(ln_stats_rows)
  HB_NOTE_ROWS(rmsnorm_rows)
  HB_NOTE_ROWS(softmax_rows)
#undef HB_NOTE_ROWS
  for (const auto& kv : g_resident)
    if (kv.second <= 0) return HEXLIB_B200_ERR_CUDA;
  return HEXLIB_B200_OK;
}

#define HB_LAUNCH_CHECK()                                           \
  do {                                                                \
    if (cudaPeekAtLastError() != cudaSuccess) {                       \
      cudaGetLastError();                                             \
      return HEXLIB_B200_ERR_CUDA;                                    \
    }                                                                 \
    return HEXLIB_B200_OK;                                            \
  } while (0)

int launch_add_f16(const void* a, const void* b, void* y, int64_t n,
                   int64_t nb, cudaStream_t s) {
  if (n < 0 || nb <= 0 || (n > 0 && n % nb != 0))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (n == 0) return HEXLIB_B200_OK;
  if (n % 8 == 0 && nb % 8 == 0 && aligned16(a) && aligned16(b) &&
      aligned16(y)) {
    const int64_t nv = n / 8;
    add_f16_vec<<<grid_for(nv, kThreads), kThreads, 0, s>>>(
        (const uint4*)a, (const uint4*)b, (uint4*)y, nv, nb / 8);
  } else {
    add_f16_scalar<<<grid_for(n, kThreads), kThreads, 0, s>>>(
        (const __half*)a, (const __half*)b, (__half*)y, n, nb);
  }
  HB_LAUNCH_CHECK();
}

int launch_add_f16_f32(const void* a, const float* b, void* y, int64_t n,
                       int64_t nb, cudaStream_t s) {
  if (n < 0 || nb <= 0 || (n > 0 && n % nb != 0))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (n == 0) return HEXLIB_B200_OK;
  if (n % 8 == 0 && nb % 8 == 0 && aligned16(a) && aligned16(b) &&
      aligned16(y)) {
    const int64_t nv = n / 8;
    add_f16_f32_vec<<<grid_for(nv, kThreads), kThreads, 0, s>>>(
        (const uint4*)a, (const float4*)b, (uint4*)y, nv, nb / 8);
  } else {
    add_f16_f32_scalar<<<grid_for(n, kThreads), kThreads, 0, s>>>(
        (const __half*)a, b, (__half*)y, n, nb);
  }
  HB_LAUNCH_CHECK();
}

int launch_cast_f32_f16(const float* x, void* y, int64_t n, cudaStream_t s) {
  if (n < 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (n == 0) return HEXLIB_B200_OK;
  if (n % 8 == 0 && aligned16(x) && aligned16(y)) {
    const int64_t nv = n / 8;
    cast_f32_f16_vec<<<grid_for(nv, kThreads), kThreads, 0, s>>>(
        (const float4*)x, (uint4*)y, nv);
  } else {
    cast_f32_f16_scalar<<<grid_for(n, kThreads), kThreads, 0, s>>>(
        x, (__half*)y, n);
  }
  HB_LAUNCH_CHECK();
}

int launch_scale_f16(const void* x, void* y, int64_t n, float factor,
                     cudaStream_t s) {
  if (n < 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (n == 0) return HEXLIB_B200_OK;
  if (n % 8 == 0 && aligned16(x) && aligned16(y)) {
    const int64_t nv = n / 8;
    scale_f16_vec<<<grid_for(nv, kThreads), kThreads, 0, s>>>(
        (const uint4*)x, (uint4*)y, nv, factor);
  } else {
    scale_f16_scalar<<<grid_for(n, kThreads), kThreads, 0, s>>>(
        (const __half*)x, (__half*)y, n, factor);
  }
  HB_LAUNCH_CHECK();
}

int launch_copy(const void* x, void* y, int64_t nbytes, cudaStream_t s) {
  if (nbytes < 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (nbytes == 0 || x == y) return HEXLIB_B200_OK;
  if (nbytes % 16 == 0 && aligned16(x) && aligned16(y)) {
    const int64_t nv = nbytes / 16;
    copy_vec<<<grid_for(nv, kThreads), kThreads, 0, s>>>((const uint4*)x,
                                                         (uint4*)y, nv);
  } else {
    copy_bytes<<<grid_for(nbytes, kThreads), kThreads, 0, s>>>(
        (const uint8_t*)x, (uint8_t*)y, nbytes);
  }
  HB_LAUNCH_CHECK();
}

// The (G, V) row layout for a row of C fp16 (C = G * V * 8), or {0, 0}.
struct RowCfg {
  int g, v;
};

RowCfg row_cfg(int C) {
  if (C % 8) return {0, 0};
  switch (C / 8) {
    case 8: return {8, 1};
    case 16: return {16, 1};
    case 32: return {32, 1};
    case 64: return {32, 2};
    case 96: return {32, 3};
    case 128: return {32, 4};
    case 256: return {256, 1};
    case 512: return {256, 2};
    case 1024: return {256, 4};
  }
  return {0, 0};
}

// Launch a row kernel on no more CTAs than stay resident or have rows to do.
template <class F, class... A>
int launch_rows(F* kern, int g, int64_t R, cudaStream_t s, A... args) {
  const int64_t rows_per_cta = g <= 32 ? (kThreads / 32) * (32 / g) : 1;
  const int64_t need = (R + rows_per_cta - 1) / rows_per_cta;
  auto it = g_resident.find((const void*)kern);
  int64_t grid = (it != g_resident.end() && it->second > 0) ? it->second : need;
  if (grid > need) grid = need;
  kern<<<(int)grid, kThreads, 0, s>>>(args...);
  HB_LAUNCH_CHECK();
}

#define HB_ROW_SWITCH(K, cfg, R, s, ...)                                           \
  switch (cfg.g * 16 + cfg.v) {                                                    \
    case 8 * 16 + 1: return launch_rows(K<8, 1>, 8, R, s, __VA_ARGS__);            \
    case 16 * 16 + 1: return launch_rows(K<16, 1>, 16, R, s, __VA_ARGS__);         \
    case 32 * 16 + 1: return launch_rows(K<32, 1>, 32, R, s, __VA_ARGS__);         \
    case 32 * 16 + 2: return launch_rows(K<32, 2>, 32, R, s, __VA_ARGS__);         \
    case 32 * 16 + 3: return launch_rows(K<32, 3>, 32, R, s, __VA_ARGS__);         \
    case 32 * 16 + 4: return launch_rows(K<32, 4>, 32, R, s, __VA_ARGS__);         \
    case 256 * 16 + 1: return launch_rows(K<256, 1>, 256, R, s, __VA_ARGS__);      \
    case 256 * 16 + 2: return launch_rows(K<256, 2>, 256, R, s, __VA_ARGS__);      \
    case 256 * 16 + 4: return launch_rows(K<256, 4>, 256, R, s, __VA_ARGS__);      \
  }

int launch_layernorm_f16(const void* x, const float* w, const float* b,
                         void* y, int64_t R, int C, float eps, cudaStream_t s) {
  if (R < 0 || C <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (R == 0) return HEXLIB_B200_OK;
  const bool al = aligned16(x) && aligned16(y) && aligned16(w) && aligned16(b);
  RowCfg cfg = al ? row_cfg(C) : RowCfg{0, 0};
  // rows of 512 and 768: one row per warp, weight and bias in registers
  // (at 512^2 x 64 in the encoder 48.5 -> 41.7 us against two rows per warp
  // of 16 lanes x 6 vectors that load them per row)
  if (cfg.g == 32 && (cfg.v == 2 || cfg.v == 3)) {
    switch (cfg.v) {
      case 2: return launch_rows(layernorm_rows_wb<2, HB_LN_DEPTH>, 32, R, s, (const uint4*)x,
                                 w, b, (uint4*)y, R, eps, order_next());
      case 3: return launch_rows(layernorm_rows_wb<3, HB_LN_DEPTH>, 32, R, s, (const uint4*)x,
                                 w, b, (uint4*)y, R, eps, order_next());
    }
  }
  HB_ROW_SWITCH(layernorm_rows, cfg, R, s, (const uint4*)x, w, b, (uint4*)y, R, eps,
                order_next())
  layernorm_f16_generic<<<grid_for(R * 32, kThreads), kThreads, 0, s>>>(
      (const __half*)x, w, b, (__half*)y, R, C, eps);
  HB_LAUNCH_CHECK();
}

int launch_patchify_f32_f16(const float* img, void* out, int64_t nimg, int C, int T, int H,
                            int W, int patch, int merge, int grid_h, int grid_w,
                            cudaStream_t s) {
  if (nimg < 0 || C <= 0 || T <= 0 || patch <= 0 || merge <= 0 || grid_h <= 0 ||
      grid_w <= 0 || grid_h * patch != H || grid_w * patch != W || grid_h % merge ||
      grid_w % merge || !img || !out)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (nimg == 0) return HEXLIB_B200_OK;
  const int fv = C * T * patch * patch / 4;
  // the merge-block kernel only: 16-byte image rows, 8-byte output runs
  if ((patch % 4) || !aligned16(img) || (reinterpret_cast<uintptr_t>(out) & 7u) ||
      fv > 8192 || (int64_t)C * T * H * W >= ((int64_t)1 << 31))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  const int bw_n = grid_w / merge;
  const int per_img = (grid_h / merge) * bw_n;
  const int64_t n_blocks = nimg * per_img;
  const int64_t cap = (int64_t)sm_count_cached() * 16;
  patchify_blocks<true><<<(unsigned)(n_blocks < cap ? n_blocks : cap), 128,
                          (size_t)fv * sizeof(int), s>>>(
      (const float4*)img, out, n_blocks, per_img, bw_n, merge, patch, C, T, H, W / 4, fv);
  HB_LAUNCH_CHECK();
}

int launch_ln_stats_f16(const void* x, float* stats, int64_t R, int C, float eps,
                        cudaStream_t s) {
  if (R < 0 || C <= 0 || !x || !stats) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (R == 0) return HEXLIB_B200_OK;
  const bool al = aligned16(x) && (reinterpret_cast<uintptr_t>(stats) & 7u) == 0;
  const RowCfg cfg = al ? row_cfg(C) : RowCfg{0, 0};
  HB_ROW_SWITCH(ln_stats_rows, cfg, R, s, (const uint4*)x, (float2*)stats, R, eps)
  if ((reinterpret_cast<uintptr_t>(stats) & 7u) != 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  ln_stats_generic<<<grid_for(R * 32, kThreads), kThreads, 0, s>>>(
      (const __half*)x, (float2*)stats, R, C, eps);
  HB_LAUNCH_CHECK();
}

int launch_rmsnorm_f16(const void* x, const void* w, void* y, int64_t R, int C,
                       float eps, cudaStream_t s) {
  if (R < 0 || C <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (R == 0) return HEXLIB_B200_OK;
  const bool al = aligned16(x) && aligned16(y) && aligned16(w);
  const RowCfg cfg = al ? row_cfg(C) : RowCfg{0, 0};
  HB_ROW_SWITCH(rmsnorm_rows, cfg, R, s, (const uint4*)x, (const uint4*)w, (uint4*)y, R, eps)
  rmsnorm_f16_generic<<<grid_for(R * 32, kThreads), kThreads, 0, s>>>(
      (const __half*)x, (const __half*)w, (__half*)y, R, C, eps);
  HB_LAUNCH_CHECK();
}

int launch_softmax_f16(const void* x, void* y, int64_t R, int C,
                       cudaStream_t s) {
  if (R < 0 || C <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (R == 0) return HEXLIB_B200_OK;
  const bool al = aligned16(x) && aligned16(y);
  const RowCfg cfg = al ? row_cfg(C) : RowCfg{0, 0};
  HB_ROW_SWITCH(softmax_rows, cfg, R, s, (const uint4*)x, (uint4*)y, R)
  softmax_f16_generic<<<grid_for(R * 32, kThreads), kThreads, 0, s>>>((const __half*)x,
                                                                      (__half*)y, R, C);
  HB_LAUNCH_CHECK();
}

int launch_rope_f16(const void* x, const float* cos_t, const float* sin_t,
                    void* y, int64_t rows, int H, int D, int64_t table_rows,
                    cudaStream_t s) {
  if (rows < 0 || H <= 0 || D <= 0 || (D & 1) || table_rows <= 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (rows == 0) return HEXLIB_B200_OK;
  const bool al = aligned16(x) && aligned16(y) && aligned16(cos_t) &&
                  aligned16(sin_t);
  if (al && (D % 16) == 0) {
    const int64_t total = rows * H * (D / 16);
    rope_f16_vec<<<grid_for(total, kThreads), kThreads, 0, s>>>(
        (const uint4*)x, cos_t, sin_t, (uint4*)y, rows, H, D, table_rows);
  } else {
    const int64_t total = rows * H * (D / 2);
    rope_f16_scalar<<<grid_for(total, kThreads), kThreads, 0, s>>>(
        (const __half*)x, cos_t, sin_t, (__half*)y, rows, H, D, table_rows);
  }
  HB_LAUNCH_CHECK();
}

int launch_rope_qk_f16(const void* qkv, const float* cos_t, const float* sin_t, void* out,
                       int64_t rows, int H, int D, int64_t table_rows, cudaStream_t s) {
  if (rows < 0 || H <= 0 || D <= 0 || (D % 16) || table_rows <= 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (rows == 0) return HEXLIB_B200_OK;
  if (!aligned16(qkv) || !aligned16(out) || !aligned16(cos_t) || !aligned16(sin_t))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (qkv != out) {  // not in place: carry the v section over first
    const int rc = launch_copy(qkv, out, rows * 3LL * H * D * 2, s);
    if (rc != HEXLIB_B200_OK) return rc;
  }
  const int64_t total = rows * 2LL * H * (D / 16);
  rope_qk_vec<<<grid_for(total, kThreads), kThreads, 0, s>>>(
      (const uint4*)out, cos_t, sin_t, (uint4*)out, rows, H, D, table_rows);
  HB_LAUNCH_CHECK();
}

int launch_transpose_th_f16(const void* x, void* y, int64_t nimg, int T, int H,
                            int D, cudaStream_t s) {
  if (nimg < 0 || T <= 0 || H <= 0 || D <= 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (nimg == 0) return HEXLIB_B200_OK;
  const int64_t total = nimg * T * H * (int64_t)D;
  if ((D % 8) == 0 && aligned16(x) && aligned16(y)) {
    transpose_th_vec<<<grid_for(total / 8, kThreads), kThreads, 0, s>>>(
        (const uint4*)x, (uint4*)y, nimg, T, H, D / 8);
  } else {
    transpose_th_scalar<<<grid_for(total, kThreads), kThreads, 0, s>>>(
        (const __half*)x, (__half*)y, nimg, T, H, D);
  }
  HB_LAUNCH_CHECK();
}

int launch_transpose_hd_f16(const void* x, void* y, int64_t B, int T, int D,
                            cudaStream_t s) {
  if (B < 0 || T <= 0 || D <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (B == 0) return HEXLIB_B200_OK;
  const int64_t ntiles =
      B * ((T + kTile - 1) / kTile) * (int64_t)((D + kTile - 1) / kTile);
  int grid = grid_for(ntiles * kThreads, kThreads);
  if (T % 8 == 0 && D % 8 == 0 && aligned16(x) && aligned16(y))
    transpose_hd_vec<<<grid, kThreads, 0, s>>>((const uint4*)x, (uint4*)y, B, T, D);
  else
    transpose_hd_tiled<<<grid, kThreads, 0, s>>>((const __half*)x, (__half*)y, B, T, D);
  HB_LAUNCH_CHECK();
}

int launch_patchify_f32(const float* img, float* out, int64_t nimg, int C,
                        int T, int H, int W, int patch, int merge, int grid_h,
                        int grid_w, cudaStream_t s) {
  if (nimg < 0 || C <= 0 || T <= 0 || patch <= 0 || merge <= 0 ||
      grid_h <= 0 || grid_w <= 0 || grid_h * patch != H ||
      grid_w * patch != W || grid_h % merge || grid_w % merge)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (nimg == 0) return HEXLIB_B200_OK;
  const int64_t total =
      nimg * (int64_t)grid_h * grid_w * C * T * patch * patch;
  const int fv = C * T * patch * patch / 4;
  if ((patch % 4) == 0 && aligned16(img) && aligned16(out) && fv <= 8192 &&
      (int64_t)C * T * H * W < ((int64_t)1 << 31)) {
    const int bw_n = grid_w / merge;
    const int per_img = (grid_h / merge) * bw_n;
    const int64_t n_blocks = nimg * per_img;
    const int64_t cap = (int64_t)sm_count_cached() * 16;
    patchify_blocks<false><<<(unsigned)(n_blocks < cap ? n_blocks : cap), 128,
                             (size_t)fv * sizeof(int), s>>>(
        (const float4*)img, out, n_blocks, per_img, bw_n, merge, patch, C, T, H, W / 4, fv);
  } else if ((patch % 4) == 0 && aligned16(img) && aligned16(out)) {
    patchify_vec<<<grid_for(total / 4, kThreads), kThreads, 0, s>>>(
        (const float4*)img, (float4*)out, nimg, C, T, H, W, patch, merge,
        grid_w);
  } else {
    patchify_scalar<<<grid_for(total, kThreads), kThreads, 0, s>>>(
        img, out, nimg, C, T, H, W, patch, merge, grid_w);
  }
  HB_LAUNCH_CHECK();
}

}  // namespace hb
