// k_attention.cu -- fused attention for the vision encoder on sm_100a:
//   ctx = softmax((q * scale) @ k^T) @ v        per head, q/k/v/ctx [Bn, T, D]
// which the plan writes as five ops per block (hexlib/models/vit.py:183-190:
// scale, transpose_hd, matmul, softmax, matmul) and which, unfused, writes
// and re-reads an [H, T, T] score and probability tensor per image and
// layer. Here the scores live only in tensor memory and registers.
//
// TENSOR-CORE PATH (D = 64). A persistent kernel, one CTA per SM, walking work
// items of 256 queries of one head (two 128-row tiles, a and b) and streaming
// each item's keys in blocks of 128; the next item's Q and keys load while the
// current one finishes, and its first S products run during the current
// item's epilogue:
//   warp 0     TMA: each item's two Q tiles into one of two Q buffers, then
//              its K and V blocks into a 3-stage ring;
//   warp 1     one lane issues tcgen05.mma: S_t = Q_t K^T (M=128, N=128,
//              K=64) into TMEM, and after the softmax has written P_t to
//              TMEM, O_t = P_t V (M=128, N=64, K=128) with A read from TMEM;
//   warps 2-5  softmax of tile a, warps 6-9 softmax of tile b: one query row
//              per thread, the block's scores read from TMEM in one pass,
//              P (fp16) written back to TMEM; the output accumulates in TMEM
//              and is rescaled there only when the running max grows by > 2^8.
// TMEM columns: S_a [0,128), S_b [128,256), O_a [256,320), O_b [320,384),
// P_a [384,448), P_b [448,512).
// While one tile's softmax runs, the tensor core works on the other tile's
// products, so the exp units and the tensor core overlap.
//
// NUMERICS. S and O accumulate in fp32; the running max, exp2 and row sums
// are fp32; P is rounded to fp16 for its MMA (unnormalised, in [0, 1]) and
// the output is divided by the fp32 row sum and rounded to fp16 once. The
// unfused plan instead rounds the scores and the normalised probabilities to
// fp16; the two agree within the fp16 per-op tolerance.
//
// Any other D uses a CUDA-core kernel with the same online softmax.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hb_device.cuh"
#include "hb_kernels.h"
#include "hb_tma.h"

namespace hb {
namespace {

constexpr int AT_BM = 128;      // query rows per tile
constexpr int AT_BN = 128;      // keys per block
constexpr int AT_D = 64;
constexpr int AT_STAGES = 3;
constexpr int AT_THREADS = 320;
constexpr int AT_TILE = AT_BM * AT_D * 2;        // 16 KiB: one Q, K or V tile
constexpr int AT_SMEM = 4 * AT_TILE + AT_STAGES * 2 * AT_TILE + 1024 + 256;
constexpr uint32_t AT_TMEM_COLS = 512;           // S_a, S_b: 128; O_a, O_b, P_a, P_b: 64

struct AttnParams {
  int T;
  int64_t Bn;         // heads in total (images x H)
  int H;              // heads per image: head h of image b is work item b*H + h
  int q_pairs;        // ceil(T / 256)
  int xq, xk, xv;     // x (column) origin of q, k, v in their tensor maps
  float c_log2;       // scale * log2(e)
  __half* out;        // row (b, t) of head h at ((b*T + t)*H + h)*64
  int* err;
  int reverse;        // walk the items last to first (the order only)
};

// 2^x with the hardware's approximate exponential (one MUFU.EX2): the
// softmax feeds it arguments <= 0 and keeps its results in fp32 before they
// are rounded to fp16.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100's three-input form).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    attention_tc(const __grid_constant__ CUtensorMap tmQ,
                 const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // [2 buffers][2 tiles][16 KiB]
  uint8_t* sK = sQ + 4 * AT_TILE;                      // [STAGES][16 KiB]
  uint8_t* sV = sK + AT_STAGES * AT_TILE;              // [STAGES][16 KiB]
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sV + AT_STAGES * AT_TILE);   // [2]
  uint64_t* q_empty = q_full + 2;            // [2]
  uint64_t* kv_full = q_empty + 2;           // [STAGES]
  uint64_t* kv_empty = kv_full + AT_STAGES;  // [STAGES]
  uint64_t* s_full = kv_empty + AT_STAGES;   // [2 tiles]
  uint64_t* s_free = s_full + 2;             // [2]
  uint64_t* p_full = s_free + 2;             // [2]
  uint64_t* o_full = p_full + 2;             // [2]
  uint64_t* o_free = o_full + 2;             // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkv = (p.T + AT_BN - 1) / AT_BN;
  const int64_t items = p.Bn * p.q_pairs;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    for (int s = 0; s < AT_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
      mbar_init(&o_free[t], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, AT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Work item w (this CTA takes w = blockIdx.x, + gridDim.x, ...): with
  // wi = w (or items - 1 - w when p.reverse), the query pair wi % q_pairs of
  // head (wi / q_pairs) % H of image wi / q_pairs / H.
  // Every barrier phase runs on across items: the i-th item of this CTA uses
  // Q buffer i & 1 and key blocks g = i*nkv .. i*nkv + nkv - 1 of the CTA's
  // stream.
  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0;
      int64_t i = 0;
      for (int64_t w = blockIdx.x; w < items; w += gridDim.x, ++i) {
        const int64_t wi = p.reverse ? items - 1 - w : w;
        const int64_t bh = wi / p.q_pairs;
        const int bimg = (int)(bh / p.H), head = (int)(bh % p.H);
        const int q0 = (int)(wi % p.q_pairs) * (2 * AT_BM);
        const int qb = (int)(i & 1);
        // the buffer's previous item (i - 2) has finished its S products
        if (!mbar_wait(&q_empty[qb], ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag, p.err))
          goto done;
        mbar_arrive_expect_tx(&q_full[qb], 2 * AT_TILE);
        uint8_t* qdst = sQ + qb * 2 * AT_TILE;
        tma_load_3d(&tmQ, &q_full[qb], qdst, p.xq + head * AT_D, q0, bimg);
        tma_load_3d(&tmQ, &q_full[qb], qdst + AT_TILE, p.xq + head * AT_D, q0 + AT_BM, bimg);
        for (int j = 0; j < nkv; ++j, ++g) {
          const int st = (int)(g % AT_STAGES);
          const uint32_t ph = (g / AT_STAGES) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag, p.err)) goto done;
          mbar_arrive_expect_tx(&kv_full[st], 2 * AT_TILE);
          tma_load_3d(&tmK, &kv_full[st], sK + st * AT_TILE, p.xk + head * AT_D, j * AT_BN, bimg);
          tma_load_3d(&tmV, &kv_full[st], sV + st * AT_TILE, p.xv + head * AT_D, j * AT_BN, bimg);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(AT_BM, AT_BN, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(AT_BM, AT_D, false, true);
      uint32_t g0 = 0;          // the item's first key block in the CTA's stream
      int64_t i = 0;
      for (int64_t w = blockIdx.x; w < items; w += gridDim.x, ++i, g0 += nkv) {
        const int qb = (int)(i & 1);
        if (!mbar_wait(&q_full[qb], (uint32_t)(i >> 1) & 1u, abort_flag, p.err)) goto done;
        // S_t(j) = Q_t K_j^T, once the softmax has read S_t(j-1) out of TMEM
        // (and K_j, V_j have landed: waited for by the first tile's S(j),
        // which the second tile's S(j) always follows directly)
        auto issue_s = [&](int t, int j) -> bool {
          const uint32_t g = g0 + (uint32_t)j;
          const int st = (int)(g % AT_STAGES);
          if (t == 0 && !mbar_wait(&kv_full[st], (g / AT_STAGES) & 1u, abort_flag, p.err))
            return false;
          if (g > 0 && !mbar_wait(&s_free[t], (g - 1) & 1u, abort_flag, p.err)) return false;
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ + (qb * 2 + t) * AT_TILE);
          const uint32_t kb = smem_u32(sK + st * AT_TILE);
#pragma unroll
          for (int kk = 0; kk < AT_D / 16; ++kk)
            umma_f16(tmem + (uint32_t)(t * AT_BN), sdesc_sw128(qa + kk * 32, 16, 1024),
                     sdesc_sw128(kb + kk * 32, 16, 1024), idesc_s, kk ? 1u : 0u);
          umma_commit(&s_full[t]);
          return true;
        };
        // O_t += P_t(j) V_j, overwriting at the item's first block -- once
        // the previous item's epilogue has read O_t out of TMEM
        auto issue_pv = [&](int t, int j) -> bool {
          const uint32_t g = g0 + (uint32_t)j;
          const int st = (int)(g % AT_STAGES);
          if (!mbar_wait(&p_full[t], g & 1u, abort_flag, p.err)) return false;
          if (j == 0 && i > 0 &&
              !mbar_wait(&o_free[t], (uint32_t)((i - 1) & 1), abort_flag, p.err))
            return false;
          tc_fence_after();
          const uint32_t pa = tmem + 384u + (uint32_t)(t * 64);   // 16 keys = 8 columns
          const uint32_t vb = smem_u32(sV + st * AT_TILE);
#pragma unroll
          for (int kk = 0; kk < AT_BN / 16; ++kk)
            umma_f16_ts(tmem + 256u + (uint32_t)(t * AT_D), pa + (uint32_t)(kk * 8),
                        sdesc_sw128(vb + kk * 2048, 8192, 1024), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&o_full[t]);
          return true;
        };
        if (!issue_s(0, 0) || !issue_s(1, 0)) goto done;
        for (int j = 0; j < nkv; ++j) {
          // Both tiles' S(j+1) go in ahead of their P(j)V(j): each tile's
          // next scores are ready by the time its softmax finishes the
          // current block, and neither tile's scores wait behind the other
          // tile's P V, so the two tiles' softmax phases overlap.
          if (j + 1 < nkv && !issue_s(0, j + 1)) goto done;
          if (j + 1 < nkv && !issue_s(1, j + 1)) goto done;
          if (!issue_pv(0, j)) goto done;
          if (!issue_pv(1, j)) goto done;
          umma_commit(&kv_empty[(g0 + (uint32_t)j) % AT_STAGES]);   // K_j, V_j consumed
        }
        umma_commit(&q_empty[qb]);          // every S of this item has read its Q
      }
    }
  } else {
    // Softmax warpgroups: t = 0 (warps 2-5) or 1 (warps 6-9), one query row
    // per thread. The running output O_t accumulates in TMEM; its scale, the
    // running max m_run, changes only when a block's max exceeds it by more
    // than 2^8 ("lazy" rescaling: between rescales p = 2^(s*c - m_run) stays
    // below 256, exactly representable in range by fp16 P), so most blocks
    // never touch O at all.
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;               // row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + (uint32_t)(t * AT_BN);
    const uint32_t o_col = tmem + lane_off + 256u + (uint32_t)(t * AT_D);
    const uint32_t p_col = tmem + lane_off + 384u + (uint32_t)(t * 64);
    const float c = p.c_log2;
    constexpr float kRescale = 8.0f;
    uint32_t g0 = 0;
    int64_t i = 0;
    for (int64_t w = blockIdx.x; w < items; w += gridDim.x, ++i, g0 += nkv) {
      const int64_t wi = p.reverse ? items - 1 - w : w;
      const int64_t bh = wi / p.q_pairs;
      const int bimg = (int)(bh / p.H), head = (int)(bh % p.H);
      const int q0 = (int)(wi % p.q_pairs) * (2 * AT_BM);
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nkv; ++j) {
        const uint32_t g = g0 + (uint32_t)j;
        const bool ok = mbar_wait(&s_full[t], g & 1u, abort_flag, p.err);
        if (!__all_sync(0xffffffffu, ok)) goto done;
        tc_fence_after();
        uint32_t sv[AT_BN];
#pragma unroll
        for (int cc = 0; cc < AT_BN / 32; ++cc)
          tmem_ld_32x32b_x32(s_col + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[cc * 32]));
        tmem_ld_wait();
        // S is in registers: hand its TMEM back for S(j+1)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);

        const int valid = p.T - j * AT_BN;             // keys of this block that exist
        if (valid < AT_BN) {
#pragma unroll
          for (int e = 0; e < AT_BN; ++e)
            if (e >= valid) sv[e] = __float_as_uint(-INFINITY);
        }
        // row max: four chains of three-input maxima
        float pm[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pm[e] = __uint_as_float(sv[e]);
#pragma unroll
        for (int e = 4; e < AT_BN; e += 8)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            pm[q] = max3f(pm[q], __uint_as_float(sv[e + q]), __uint_as_float(sv[e + 4 + q]));
        // the scale is positive, so max(s)*c is the max of s*c
        const float mx = c * max3f(pm[0], pm[1], fmaxf(pm[2], pm[3]));
        const bool rescale = mx > m_run + kRescale;
        const float m_use = rescale ? mx : m_run;
        const float alpha = rescale ? ex2_approx(m_run - mx) : 1.0f;
        // P V of the previous block must be done: it reads the P buffer this
        // block overwrites, and a rescale (below) must see its contribution
        // in O. (At an item's first block the previous item's epilogue has
        // already waited for its last P V.)
        if (j > 0) {
          const bool ok2 = mbar_wait(&o_full[t], (g - 1) & 1u, abort_flag, p.err);
          if (!__all_sync(0xffffffffu, ok2)) goto done;
          tc_fence_after();
        }
        // p = 2^(s*c - m), 32 keys at a time: one FMA and one MUFU exponential
        // per key, eight partial row sums, and the fp16 pairs stored to this
        // row's lane of P in TMEM (column e holds keys 2e and 2e + 1).
        // (pairs of keys through sm_100's two-wide FMA and add: the same
        // roundings as two scalar operations, half the instructions)
        const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
        float2 ps[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) ps[e] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k32 = 0; k32 < AT_BN / 32; ++k32) {
          uint32_t h2[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int x = k32 * 32 + 2 * e;
            const float2 a = __ffma2_rn(make_float2(__uint_as_float(sv[x]),
                                                    __uint_as_float(sv[x + 1])), c2, nm2);
            const float p0 = ex2_approx(a.x);
            const float p1 = ex2_approx(a.y);
            ps[e & 3].x += p0;
            ps[e & 3].y += p1;
            h2[e] = pack_half2(p0, p1);
          }
          tmem_st_32x32b_x16(p_col + (uint32_t)(k32 * 16), h2);
        }
        const float rs = ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) +
                         ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
        // O *= alpha before P V of this block is issued (rare: the max grew by
        // more than 2^8 since the last rescale)
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int h = 0; h < AT_D / 32; ++h) {
            uint32_t rg[32];
            tmem_ld_32x32b_x32(o_col + h * 32, rg);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              rg[e] = __float_as_uint(__uint_as_float(rg[e]) * alpha);
            tmem_st_32x32b_x32(o_col + h * 32, rg);
          }
          tmem_st_wait();
        }
        tmem_st_wait();                  // P (and a rescaled O) are in TMEM
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        l_run = l_run * alpha + rs;
        m_run = m_use;
      }
      // the item's output: O out of TMEM (then its columns are free for the
      // next item's first P V), divided by the row sum, rounded once
      const bool ok = mbar_wait(&o_full[t], (g0 + (uint32_t)nkv - 1) & 1u, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, ok)) goto done;
      tc_fence_after();
      uint32_t ov[AT_D];
      tmem_ld_32x32b_x32(o_col, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
      tmem_ld_32x32b_x32(o_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[t]);
      const int row = q0 + t * AT_BM + r;
      if (row < p.T) {
        const float inv = 1.0f / l_run;
        uint4* dst = reinterpret_cast<uint4*>(
            p.out + (((int64_t)bimg * p.T + row) * p.H + head) * (int64_t)AT_D);
#pragma unroll
        for (int q = 0; q < AT_D / 8; ++q) {
          const float* o = reinterpret_cast<const float*>(&ov[8 * q]);
          dst[q] = make_uint4(pack_half2(o[0] * inv, o[1] * inv),
                              pack_half2(o[2] * inv, o[3] * inv),
                              pack_half2(o[4] * inv, o[5] * inv),
                              pack_half2(o[6] * inv, o[7] * inv));
        }
      }
    }
  }

done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, AT_TMEM_COLS);
  }
}

// CUDA-core fallback: one thread per query row, online softmax, D <= 256.
template <int DMAX>
__global__ void attention_simt(const __half* __restrict__ q, const __half* __restrict__ k,
                               const __half* __restrict__ v, __half* __restrict__ out,
                               int64_t Bn, int T, int D, float scale) {
  const int64_t rows = Bn * T;
  for (int64_t rr = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; rr < rows;
       rr += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = rr / T;
    const __half* qr = q + rr * D;
    const __half* kb = k + b * (int64_t)T * D;
    const __half* vb = v + b * (int64_t)T * D;
    float qf[DMAX], o[DMAX];
    for (int d = 0; d < D; ++d) {
      qf[d] = __half2float(qr[d]);
      o[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < T; ++j) {
      float s = 0.f;
      for (int d = 0; d < D; ++d) s += qf[d] * __half2float(kb[(int64_t)j * D + d]);
      s *= scale;
      const float mn = fmaxf(m, s);
      const float a = expf(m - mn);
      const float pj = expf(s - mn);
      l = l * a + pj;
      for (int d = 0; d < D; ++d) o[d] = o[d] * a + pj * __half2float(vb[(int64_t)j * D + d]);
      m = mn;
    }
    for (int d = 0; d < D; ++d) out[rr * D + d] = __float2half_rn(o[d] / l);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int g_sms = 0;

}  // namespace

int attention_kernels_init() {
  if (cudaFuncSetAttribute(attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           AT_SMEM) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, attention_simt<256>) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  if (g_sms <= 0) g_sms = 148;
  return HEXLIB_B200_OK;
}

// One CTA per SM (tensor memory holds one CTA's 512 columns), each looping
// over work items; fewer CTAs when there are fewer items.
unsigned persistent_grid(int64_t items) {
  const int64_t sms = g_sms > 0 ? g_sms : 148;
  return (unsigned)(items < sms ? items : sms);
}

int launch_attention(const void* q, const void* k, const void* v, void* ctx, int64_t Bn,
                     int T, int D, float scale, int* err, cudaStream_t s) {
  if (Bn < 0 || T <= 0 || D <= 0 || D > 256) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (Bn == 0) return HEXLIB_B200_OK;
  if (!q || !k || !v || !ctx) return HEXLIB_B200_ERR_INVAL_PARAMS;
  // The tensor-core kernel takes the row max of the raw scores and scales it,
  // which is the max of the scaled scores only for a positive scale.
  if (D == AT_D && scale > 0.f && aligned16(q) && aligned16(k) && aligned16(v) &&
      aligned16(ctx) && Bn < (int64_t)1 << 30 && tma_available()) {
    CUtensorMap mq, mk, mv;
    const bool ok = make_tmap_3d_f16(&mq, q, AT_D, (uint64_t)T, (uint64_t)Bn, 64, AT_BM) &&
                    make_tmap_3d_f16(&mk, k, AT_D, (uint64_t)T, (uint64_t)Bn, 64, AT_BN) &&
                    make_tmap_3d_f16(&mv, v, AT_D, (uint64_t)T, (uint64_t)Bn, 64, AT_BN);
    if (ok) {
      AttnParams p;
      p.T = T;
      p.Bn = Bn;
      p.H = 1;
      p.xq = p.xk = p.xv = 0;
      p.q_pairs = (T + 2 * AT_BM - 1) / (2 * AT_BM);
      p.c_log2 = scale * 1.4426950408889634f;
      p.out = reinterpret_cast<__half*>(ctx);
      p.err = err;
      p.reverse = order_next();
      attention_tc<<<persistent_grid(Bn * p.q_pairs), AT_THREADS, AT_SMEM, s>>>(mq, mk, mv, p);
      if (cudaPeekAtLastError() != cudaSuccess) {
        cudaGetLastError();
        return HEXLIB_B200_ERR_CUDA;
      }
      return HEXLIB_B200_OK;
    }
  }
  const int64_t rows = Bn * T;
  int64_t blocks = (rows + 127) / 128;
  const int64_t cap = (int64_t)(g_sms > 0 ? g_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  attention_simt<256><<<(unsigned)blocks, 128, 0, s>>>(
      reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
      reinterpret_cast<const __half*>(v), reinterpret_cast<__half*>(ctx), Bn, T, D, scale);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int launch_attention_qkv(const void* qkv, void* ctx, int64_t B, int T, int H, int D,
                         float scale, int* err, cudaStream_t s) {
  if (B < 0 || T <= 0 || H <= 0 || D <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (B == 0) return HEXLIB_B200_OK;
  if (!qkv || !ctx) return HEXLIB_B200_ERR_INVAL_PARAMS;
  // The packed layout [B, T, 3, H, D] is served by the tensor-core kernel
  // only: one 3-D map over rows of 3*H*D columns, q/k/v at column offsets.
  if (D != AT_D || scale <= 0.f || !aligned16(qkv) || !aligned16(ctx) || !tma_available() ||
      B * H >= ((int64_t)1 << 30) || B >= ((int64_t)1 << 31))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  const uint64_t W = (uint64_t)3 * H * D;
  CUtensorMap m;
  if (!make_tmap_3d_f16(&m, qkv, W, (uint64_t)T, (uint64_t)B, 64, AT_BM))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  AttnParams p;
  p.T = T;
  p.Bn = B * H;
  p.H = H;
  p.xq = 0;
  p.xk = H * D;
  p.xv = 2 * H * D;
  p.q_pairs = (T + 2 * AT_BM - 1) / (2 * AT_BM);
  p.c_log2 = scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__half*>(ctx);
  p.err = err;
  p.reverse = order_next();
  attention_tc<<<persistent_grid(p.Bn * p.q_pairs), AT_THREADS, AT_SMEM, s>>>(m, m, m, p);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

}  // namespace hb
