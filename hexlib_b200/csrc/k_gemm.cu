// k_gemm.cu -- fp16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA),
// with the matmul_epilogue epilogue fused: out = act(A @ W + bias) (+ resid).
//
// Serves both wire kernels that contract over a dense operand:
//   matmul_epilogue (kernels/matmul_epilogue_fp16/kernel_api.h:188-190, with an
//     fp16 [K, N] weight): A [M, K] per image, W [K, N] shared, bias fp32 [N];
//     the images fold into M, so one launch covers B*T rows.
//   matmul (kernels/matmul_fp16/kernel_api.h:77-78): batched A [Bn, M, K] @
//     B [Bn, K, N], no bias, no activation (attention QK^T and PV).
// Accumulation is fp32 in tensor memory and the output is rounded to fp16
// exactly once, after the bias and the activation (fused.py:44-53).
//
// STRUCTURE. A persistent kernel, one CTA per SM, tiles of 128 x BN, K in
// blocks of 64 (one 128-byte swizzle row of fp16):
//   warp 0      TMA producer: A tile [128 x 64] and BN/64 W tiles [64 x 64]
//               per stage, into a STAGES-deep ring of shared-memory buffers;
//   warp 1      allocates tensor memory, and one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) four times per stage into one of two
//               accumulators, then commits to free the stage;
//   warps 2-9   epilogue: tcgen05.ld the finished accumulator (two warps per
//               32-lane quarter, each taking half of the columns), add bias,
//               apply GELU, round, store; then release the accumulator so the
//               MMA of the tile after next can reuse it.
// Two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//
// A is K-major (row-major [M, K]); W is MN-major (row-major [K, N]) and is
// consumed in place through the descriptor's MN-major mode, so no weight is
// ever transposed.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>

#include "hb_device.cuh"
#include "hb_kernels.h"
#include "hb_tma.h"

namespace hb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + kEpiWarps * 32;  // 320

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;   // 16 KiB
  static constexpr int B_BYTES = BN * BK * 2;   // BN/64 boxes of 8 KiB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;      // two fp32 accumulators
  static constexpr int STAGING = kEpiWarps * 4096;  // one 32x64 fp16 box per warp
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING + 1024 + 256;
};

struct GemmParams {
  int64_t M;        // rows per batch entry
  int K, N;
  int64_t batch;
  int tiles_m, tiles_n;
  int64_t total_tiles;
  int num_kb;
  int b_shared;
  int act;
  const float* bias;
  const __half* resid;
  __half* out;
  int* err;
  // RoPE epilogue (ROPE kernels only): columns [0, rope_cols) are heads of
  // 64; row r is token r % rope_T, whose dims [16s, 16s + 16) and
  // [32 + 16s, 48 + 16s), s = 0, 1, take row rope_idx[2 * token + s] of the
  // [n, 16] segment tables.
  const float* rope_cos;
  const float* rope_sin;
  const int* rope_idx;
  int rope_nseg;
  int rope_stride;   // floats from one segment row to the next (16, or 32 interleaved)
  int rope_T;
  int rope_cols;
  // LayerNorm epilogue (LN kernels only): row r's (mean, rstd) at
  // ln_stats[2 r], the column sums of the folded weight at ln_colsum[n];
  // the value is rstd * (acc - mean * colsum) + bias.
  const float* ln_stats;
  const float* ln_colsum;
  // walk the tiles last to first: tile t of the loop is tile total_tiles-1-t
  // (the order only; every tile is computed the same way)
  int reverse;
};

// One whole 32-byte sector per thread (sm_100's 256-bit load): a residual
// chunk row is two of these, so no half-used sector waits in L1 for its
// other half. `p` 32-byte aligned.
__device__ __forceinline__ void ld_nc_v8(const __half* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y),
                 "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}
// Read-only 16-byte load the L1 keeps in preference to streaming data.
__device__ __forceinline__ float4 ld_nc_evict_last_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::evict_last.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// Split-half rotation of one 64-column head (kernels/rope_2d_fp16/kernel_api.h:
// 17-26) applied to fp16-rounded inputs with separately rounded products, as
// the rope_2d op computes it on the stored q/k. lo holds dims 0..31, hi dims
// 32..63 (two per 32-bit word). The tables are half-symmetric (cos[i] ==
// cos[i + 32], as every rotate-half table built from one frequency list is),
// so rc / rs hold the cos / sin of dims 0..31, which dims 32..63 reuse.
__device__ __forceinline__ void rope_head64(uint32_t (&lo)[16], uint32_t (&hi)[16],
                                            const float (&rc)[32], const float (&rs)[32]) {
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo[q]));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi[q]));
    const float c0 = rc[2 * q], c1 = rc[2 * q + 1], s0 = rs[2 * q], s1 = rs[2 * q + 1];
    const float y0 = __fadd_rn(__fmul_rn(a.x, c0), __fmul_rn(-b.x, s0));
    const float y1 = __fadd_rn(__fmul_rn(a.y, c1), __fmul_rn(-b.y, s1));
    const float z0 = __fadd_rn(__fmul_rn(b.x, c0), __fmul_rn(a.x, s0));
    const float z1 = __fadd_rn(__fmul_rn(b.y, c1), __fmul_rn(a.y, s1));
    lo[q] = pack_half2(y0, y1);
    hi[q] = pack_half2(z0, z1);
  }
}

// The cos / sin of dims 0..31 of token `tok` from the segment tables: two
// 16-float rows each, a few KiB for a whole image, so they stay in L1 while
// every row of every tile reads them.
__device__ __forceinline__ void rope_row(const GemmParams& p, int64_t tok, float (&rc)[32],
                                         float (&rs)[32]) {
  int2 ix = __ldg(reinterpret_cast<const int2*>(p.rope_idx) + tok);
  const int top = p.rope_nseg - 1;                // never read outside the tables
  ix.x = min(max(ix.x, 0), top);
  ix.y = min(max(ix.y, 0), top);
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const float* cp = p.rope_cos + (s ? ix.y : ix.x) * p.rope_stride;
    const float* sp = p.rope_sin + (s ? ix.y : ix.x) * p.rope_stride;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 c = ld_nc_evict_last_f4(cp + 4 * j);
      const float4 n = ld_nc_evict_last_f4(sp + 4 * j);
      rc[16 * s + 4 * j] = c.x; rc[16 * s + 4 * j + 1] = c.y;
      rc[16 * s + 4 * j + 2] = c.z; rc[16 * s + 4 * j + 3] = c.w;
      rs[16 * s + 4 * j] = n.x; rs[16 * s + 4 * j + 1] = n.y;
      rs[16 * s + 4 * j + 2] = n.z; rs[16 * s + 4 * j + 3] = n.w;
    }
  }
}

// One epilogue warp's share of a finished 128-row accumulator tile. TMEM
// lanes [32*quarter, 32*quarter + 32) hold rows row0 + 32*quarter + lane of
// batch entry b; the warp finishes the 64-column groups [g_lo, g_hi) of the
// tile whose first column is n0: each group is read from TMEM 32 columns at a
// time, finished in registers (bias, GELU, residual, rounding), written to
// this warp's 128B-swizzled staging box and stored by one TMA store, which
// also clips the tile's row and column tails.
//
// RES_SMEM: the residual was brought into the warp's staging boxes by TMA
// (one 4 KiB box per group, same swizzle as the output) before the
// accumulator was ready; each group is finished in its own box, in place, so
// no group waits for the previous group's store.
//
// LN: the A operand was the raw row x and the weight diag(gamma) W; the
// accumulator is turned into LayerNorm(x) @ W + bias by the row's (mean,
// rstd) and the weight's column sums: rstd * (acc - mean * colsum) + bias,
// with bias holding beta @ W + the GEMM's own bias.
//
// DBL: two staging boxes per warp (group g - g_lo in box g - g_lo): a box is
// rewritten once the store issued from it one group earlier -- not the
// previous group's store -- has read it.
template <bool ROPE, bool RES_SMEM = false, bool LN = false, bool DBL = false>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const CUtensorMap* tmC,
                                              uint32_t tacc, uint8_t* stage, int quarter,
                                              int lane, int g_lo, int g_hi, int64_t b,
                                              int64_t row0, int n0) {
  const int64_t row = row0 + quarter * 32 + lane;
  const bool row_ok = row < p.M;
  const uint32_t trow = tacc + ((uint32_t)(quarter * 32) << 16);
  // (the RoPE kernels take no residual; RES_SMEM reads it from shared memory)
  const __half* rrow = (!ROPE && !RES_SMEM && p.resid && row_ok)
                           ? p.resid + (b * p.M + row) * (int64_t)p.N
                           : nullptr;
  // the row's cos / sin, loaded once for every head of the tile
  float ln_mean = 0.f, ln_rstd = 0.f;
  if constexpr (LN) {
    if (row_ok) {
      const float2 ms = __ldg(reinterpret_cast<const float2*>(p.ln_stats) + (b * p.M + row));
      ln_mean = ms.x;
      ln_rstd = ms.y;
    }
  }
  float rc[32], rs[32];
  const bool rope_row_ok = ROPE && row_ok && n0 + g_lo * 64 < p.rope_cols;
  if constexpr (ROPE) {
    if (rope_row_ok) rope_row(p, row % p.rope_T, rc, rs);
  }
  const int rl = lane;                                        // row within the slab
  // Residual chunks (32 columns = 64 B of this thread's row) are loaded one
  // chunk ahead into a two-deep register buffer, as two whole 32-byte
  // sectors when the residual is 32-byte aligned (row strides are: N % 8 == 0
  // and 32-column chunks), else as four 16-byte loads.
  uint4 res[2][4];
  const bool res32 = (reinterpret_cast<uintptr_t>(p.resid) & 31u) == 0 && (p.N % 16) == 0;
  auto load_res = [&](int g, int h, uint4 (&r)[4]) {
    const int nc = n0 + g * 64 + h * 32;
    if (res32) {
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        if (nc + 8 * j < p.N) ld_nc_v8(rrow + nc + 8 * j, r[j], r[j + 1]);
        else r[j] = r[j + 1] = make_uint4(0, 0, 0, 0);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = (nc + 8 * j < p.N) ? __ldg(reinterpret_cast<const uint4*>(rrow + nc) + j)
                                  : make_uint4(0, 0, 0, 0);
    }
  };
  if (rrow && g_lo < g_hi) load_res(g_lo, 0, res[0]);
#pragma unroll 1
  for (int g = g_lo; g < g_hi; ++g) {
    uint8_t* box = (RES_SMEM || DBL) ? stage + (g - g_lo) * 4096 : stage;
    uint32_t packed[2][16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c32 = g * 64 + h * 32;          // column within the tile
      const int nc = n0 + c32;                  // global column
      // the next chunk's residual: (g, 1) after (g, 0); (g + 1, 0) after (g, 1)
      if (rrow) {
        if (h == 0) load_res(g, 1, res[1]);
        else if (g + 1 < g_hi) load_res(g + 1, 0, res[0]);
      }
      float bias[32];
      if (LN) {
        // (loaded with the column sums below, next to their use)
      } else if (p.bias && nc < p.N) {
        const float* bp = p.bias + nc;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 bb = (nc + 4 * j < p.N) ? ld_nc_evict_last_f4(bp + 4 * j)
                                               : make_float4(0, 0, 0, 0);
          bias[4 * j] = bb.x; bias[4 * j + 1] = bb.y;
          bias[4 * j + 2] = bb.z; bias[4 * j + 3] = bb.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) bias[j] = 0.f;
      }
      uint32_t rg[32];
      tmem_ld_32x32b_x32(trow + c32, rg);
      tmem_ld_wait();
      float v[32];
      if constexpr (LN) {
        // column sums and bias read four at a time next to their use
        // (both L1-resident)
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const bool in = nc + j < p.N;
          const float4 cs = in ? ld_nc_evict_last_f4(p.ln_colsum + nc + j)
                               : make_float4(0, 0, 0, 0);
          const float4 bb = (in && p.bias) ? ld_nc_evict_last_f4(p.bias + nc + j)
                                           : make_float4(0, 0, 0, 0);
          const float c4[4] = {cs.x, cs.y, cs.z, cs.w};
          const float b4[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            v[j + q] = fmaf(ln_rstd, fmaf(-ln_mean, c4[q], __uint_as_float(rg[j + q])), b4[q]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rg[j]) + bias[j];
      }
      if (p.act == 1) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 g = gelu_tanh_f2(make_float2(v[j], v[j + 1]));
          v[j] = g.x;
          v[j + 1] = g.y;
        }
      } else if (p.act == 2) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_erf_f(v[j]);
      }
      uint32_t hw[16];
      if constexpr (RES_SMEM) {
        // this row's 64 bytes of the chunk, at their swizzled places
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = (h * 4 + j) ^ (rl & 7);
          res[0][j] = *reinterpret_cast<const uint4*>(box + rl * 128 + chunk * 16);
        }
      }
      if (rrow || RES_SMEM) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2* rh = reinterpret_cast<const __half2*>(&res[RES_SMEM ? 0 : h][j]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // The matmul result is an fp16 tensor in the unfused plan:
            // round it, then add the residual in fp32 and round again.
            const float2 fm = __half22float2(
                __floats2half2_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]));
            const float2 fr = __half22float2(rh[q]);
            hw[4 * j + q] = pack_half2(fr.x + fm.x, fr.y + fm.y);
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) hw[q] = pack_half2(v[2 * q], v[2 * q + 1]);
      }
#pragma unroll
      for (int q = 0; q < 16; ++q) packed[h][q] = hw[q];
    }
    if constexpr (ROPE) {
      if (rope_row_ok && n0 + g * 64 < p.rope_cols) rope_head64(packed[0], packed[1], rc, rs);
    }
    if constexpr (!RES_SMEM) {
      // the previous group's store must have finished reading the stage;
      // waited for only now, so that store overlaps this group's TMEM
      // loads and arithmetic
      if (lane == 0) {
        if constexpr (DBL) bulk_wait_read_all_but_1();
        else bulk_wait_read_all();
      }
      __syncwarp();
    }
    // 8 x 16 B into the 128-byte row rl of the stage, swizzled
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int chunk = (h * 4 + j) ^ (rl & 7);
        *reinterpret_cast<uint4*>(box + rl * 128 + chunk * 16) =
            make_uint4(packed[h][4 * j], packed[h][4 * j + 1], packed[h][4 * j + 2],
                       packed[h][4 * j + 3]);
      }
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmC, box, n0 + g * 64, (int)(row0 + quarter * 32), (int)b);
      bulk_commit_group();
    }
  }
}

template <int BN, bool ROPE, bool LN = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_tc(const __grid_constant__ CUtensorMap tmA,
                const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint8_t* sOut = sB + Cfg::STAGES * Cfg::B_BYTES;   // [kEpiWarps][4 KiB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + Cfg::STAGING);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int64_t tiles_per_batch = (int64_t)p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
        const int64_t tt = p.reverse ? p.total_tiles - 1 - t : t;
        const int64_t b = tt / tiles_per_batch;
        const int64_t r = tt - b * tiles_per_batch;
        const int mb = (int)(r / p.tiles_n);
        const int nb = (int)(r % p.tiles_n);
        const int bz = p.b_shared ? 0 : (int)b;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err))
            goto done;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_3d(&tmA, &full[stage], sA + stage * Cfg::A_BYTES, kb * BK,
                      mb * BM, (int)b);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_3d(&tmB, &full[stage],
                        sB + stage * Cfg::B_BYTES + j * (BK * 128),
                        nb * BN + j * 64, kb * BK, bz);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int64_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err))
          goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) goto done;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // A: advance 16 fp16 (32 bytes) along the swizzled row.
            const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
            // W: advance 16 k-rows = two 1024-byte atoms; 64-wide N boxes
            // are BK*128 bytes apart.
            const uint64_t bd = sdesc_sw128(b0 + kk * 2048, BK * 128, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue: warp (quarter, colhalf) owns TMEM lanes [32q, 32q+32) -- rows
    // of the tile -- and half of its 64-column groups.
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int colhalf = ew >> 2;
    constexpr int kGroups = BN / 64;
    const int g_lo = (kGroups >= 2) ? colhalf * (kGroups / 2) : 0;
    const int g_hi = (kGroups >= 2) ? (colhalf + 1) * (kGroups / 2) : (colhalf ? 0 : 1);
    uint8_t* stage = sOut + ew * 4096;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      const int64_t tt = p.reverse ? p.total_tiles - 1 - t : t;
      const int64_t b = tt / tiles_per_batch;
      const int64_t r = tt - b * tiles_per_batch;
      const int mb = (int)(r / p.tiles_n);
      const int nb = (int)(r % p.tiles_n);
      // Every lane waits; the warp proceeds only if all of them saw the
      // phase complete, because tcgen05.ld is warp-collective.
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, ok)) goto done;
      tc_fence_after();
      epilogue_tile<ROPE, false, LN>(p, &tmC, tmem_base + (uint32_t)(acc * BN), stage, quarter, lane,
                          g_lo, g_hi, b, (int64_t)mb * BM, nb * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---- CTA-pair GEMM ---------------------------------------------------------
//
// The same persistent warp-specialised structure run by clusters of two CTAs
// on two SMs that share one 256 x 256 output tile through tcgen05's pair mode
// (cta_group::2). Per 64-deep k-block each CTA lands only its own 128 rows of
// A and its own 128 columns of W (32 KiB), and the leader's single MMA thread
// multiplies the whole 256 x 256 x 64 block across both SMs' tensor cores:
// per SM that is the work of a 128 x 256 tile for two thirds of the shared-
// memory fill traffic, which is what bounds the one-CTA kernel.
//
//   full[s]   leader only: both CTAs' TMA loads count their bytes on it;
//             the leader's producer posts the expected 2 x 32 KiB.
//   empty[s]  in both CTAs: the leader's MMA commit arrives on both when the
//             stage's shared memory has been read.
//   tfull[a]  in both CTAs: accumulator a of this CTA's rows is complete.
//   tempty[a] leader only: all 16 epilogue warps of the pair have drained a.
//
// A wait that gives up raises the abort flag of both CTAs, so the pair
// unwinds together and meets at the closing cluster barrier.
//
// Every mode gives each epilogue warp two 32x64 staging boxes (8 KiB per
// warp, a 5-stage operand ring). Epilogue modes: kPairPlain (bias,
// activation, or a residual read from global memory) and kPairRope write
// their two column groups into alternate boxes; kPairRes: each epilogue warp
// TMA-loads its two residual boxes into the staging as soon as the previous
// tile's stores have read it -- before the accumulator is ready -- so the
// residual's DRAM latency hides under the mainloop instead of stalling the
// epilogue.
// kPairLn / kPairLnRope: the LayerNorm epilogue (see epilogue_tile), without
// or with RoPE.
enum { kPairPlain = 0, kPairRope = 1, kPairRes = 2, kPairLn = 3, kPairLnRope = 4 };

template <int MODE>
struct PairCfg {
  static constexpr int BN = 256;                     // columns of the pair's tile
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = BM * BK * 2;        // 16 KiB: this CTA's 128 rows
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KiB: this CTA's 128 columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;           // two fp32 accumulators
  static constexpr int STAGING = kEpiWarps * 8192;   // two 32x64 fp16 boxes per warp
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING + 1024 + 256;
};

template <int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_pair(const __grid_constant__ CUtensorMap tmA,
                  const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC,
                  const __grid_constant__ CUtensorMap tmR, const GemmParams p) {
  using Cfg = PairCfg<MODE>;
  constexpr int BN = Cfg::BN;
  constexpr bool ROPE = MODE == kPairRope || MODE == kPairLnRope;
  constexpr bool RES = MODE == kPairRes;
  constexpr bool LN = MODE == kPairLn || MODE == kPairLnRope;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint8_t* sOut = sB + Cfg::STAGES * Cfg::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + Cfg::STAGING);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rfull = tempty + 2;                      // [kEpiWarps], kPairRes only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&rfull[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if (RES) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();            // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_lead = cluster_addr(full, 0);
  const uint32_t tempty_lead = cluster_addr(tempty, 0);
  const uint32_t peer_abort = cluster_addr(tmem_slot + 1, rank ^ 1u);

  const int64_t tiles_per_batch = (int64_t)p.tiles_m * p.tiles_n;
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t n_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = pair_id; t < p.total_tiles; t += n_pairs) {
        const int64_t tt = p.reverse ? p.total_tiles - 1 - t : t;
        const int64_t b = tt / tiles_per_batch;
        const int64_t r = tt - b * tiles_per_batch;
        const int mb = (int)(r / p.tiles_n);
        const int nb = (int)(r % p.tiles_n);
        const int bz = p.b_shared ? 0 : (int)b;
        const int row = mb * (2 * BM) + (int)rank * BM;
        const int col = nb * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            st_cluster_u32(peer_abort, 1);
            goto done;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t fb = full_lead + (uint32_t)(stage * 8);
          tma_load_3d_pair(&tmA, fb, sA + stage * Cfg::A_BYTES, kb * BK, row, (int)b);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            tma_load_3d_pair(&tmB, fb, sB + stage * Cfg::B_BYTES + j * (BK * 128),
                             col + j * 64, kb * BK, bz);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int64_t t = pair_id; t < p.total_tiles; t += n_pairs) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err)) {
          st_cluster_u32(peer_abort, 1);
          goto done;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, abort_flag, p.err)) {
            st_cluster_u32(peer_abort, 1);
            goto done;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + kk * 2048, BK * 128, 1024);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int colhalf = ew >> 2;
    constexpr int kGroups = BN / 64;
    const int g_lo = colhalf * (kGroups / 2);
    const int g_hi = (colhalf + 1) * (kGroups / 2);
    uint8_t* stage = sOut + ew * (Cfg::STAGING / kEpiWarps);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t r_phase = 0;
    for (int64_t t = pair_id; t < p.total_tiles; t += n_pairs) {
      const int64_t tt = p.reverse ? p.total_tiles - 1 - t : t;
      const int64_t b = tt / tiles_per_batch;
      const int64_t r = tt - b * tiles_per_batch;
      const int mb = (int)(r / p.tiles_n);
      const int nb = (int)(r % p.tiles_n);
      const int64_t row0 = (int64_t)mb * (2 * BM) + rank * BM;
      if constexpr (RES) {
        if (lane == 0) {
          // the previous tile's stores have read the boxes: refill them
          bulk_wait_read_all();
          mbar_arrive_expect_tx(&rfull[ew], 2 * 4096);
          for (int gi = 0; gi < 2; ++gi)
            tma_load_3d(&tmR, &rfull[ew], stage + gi * 4096, nb * BN + (g_lo + gi) * 64,
                        (int)(row0 + quarter * 32), (int)b);
          // the same boxes of this pair's next tile, into L2 now: their loads
          // are issued only when this tile's epilogue is done with the boxes,
          // and would otherwise wait out a DRAM round trip right then. Only
          // for short K (measured: o-projection K = 768 -3 %; at K = 3072
          // the tile's mainloop already covers the round trip, and the early
          // traffic cost fc2 +1.5 %)
          if (p.num_kb <= 16 && t + n_pairs < p.total_tiles) {
            const int64_t tn = p.reverse ? p.total_tiles - 1 - (t + n_pairs) : t + n_pairs;
            const int64_t bn_ = tn / tiles_per_batch;
            const int64_t rn = tn - bn_ * tiles_per_batch;
            const int64_t row_n = (int64_t)(rn / p.tiles_n) * (2 * BM) + rank * BM;
            for (int gi = 0; gi < 2; ++gi)
              tma_prefetch_l2_3d(&tmR, (int)(rn % p.tiles_n) * BN + (g_lo + gi) * 64,
                                 (int)(row_n + quarter * 32), (int)bn_);
          }
        }
      }
      const bool ok = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) st_cluster_u32(peer_abort, 1);
        goto done;
      }
      tc_fence_after();
      if constexpr (RES) {
        const bool rok = mbar_wait(&rfull[ew], r_phase, abort_flag, p.err);
        r_phase ^= 1u;
        if (!__all_sync(0xffffffffu, rok)) {
          if (lane == 0) st_cluster_u32(peer_abort, 1);
          goto done;
        }
      }
      epilogue_tile<ROPE, RES, LN, !RES>(p, &tmC, tmem_base + (uint32_t)(acc * BN), stage, quarter,
                               lane, g_lo, g_hi, b, row0, nb * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_lead + (uint32_t)(acc * 8));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

done:
  tc_fence_before();
  __syncthreads();
  cluster_sync();            // no CTA leaves while the other may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// CUDA-core fallback for shapes the TMA path cannot describe. 64x64 output
// tiles, K in steps of 16 through shared memory, fp32 accumulate.
__global__ void gemm_f16_simt(const __half* __restrict__ A,
                              const __half* __restrict__ B,
                              const float* __restrict__ bias,
                              const __half* __restrict__ resid,
                              __half* __restrict__ out, int64_t M, int K,
                              int N, int64_t batch, int b_shared, int act) {
  __shared__ float sa[16][65];
  __shared__ float sb[16][65];
  const int tiles_m = (int)((M + 63) / 64), tiles_n = (N + 63) / 64;
  const int64_t total = batch * tiles_m * (int64_t)tiles_n;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t b = t / ((int64_t)tiles_m * tiles_n);
    const int rem = (int)(t - b * tiles_m * (int64_t)tiles_n);
    const int64_t m0 = (int64_t)(rem / tiles_n) * 64;
    const int n0 = (rem % tiles_n) * 64;
    const __half* Ab = A + b * M * K;
    const __half* Bb = B + (b_shared ? 0 : b) * (int64_t)K * N;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
      for (int e = threadIdx.x; e < 16 * 64; e += 256) {
        const int kk = e / 64, mm = e % 64;
        const int64_t gm = m0 + mm;
        const int gk = k0 + kk;
        sa[kk][mm] = (gm < M && gk < K) ? __half2float(Ab[gm * K + gk]) : 0.f;
        const int gn = n0 + mm;
        sb[kk][mm] = (gk < K && gn < N) ? __half2float(Bb[(int64_t)gk * N + gn]) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[i][j] += sa[kk][ty * 4 + i] * sb[kk][tx * 4 + j];
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty * 4 + i;
      if (gm >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int gn = n0 + tx * 4 + j;
        if (gn >= N) continue;
        float v = acc[i][j] + (bias ? bias[gn] : 0.f);
        if (act == 1) v = gelu_tanh_f(v);
        if (act == 2) v = gelu_erf_f(v);
        const int64_t o = (b * M + gm) * N + gn;
        if (resid)
          v = __half2float(resid[o]) + __half2float(__float2half_rn(v));
        out[o] = __float2half_rn(v);
      }
    }
  }
}

int g_sm_count = 0;

int sm_count() {
  if (g_sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  return g_sm_count;
}

template <int BN, bool ROPE, bool LN = false>
int launch_tc(const GemmDesc& g, int* err, cudaStream_t s) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  // A: dims (K, M, batch); box (64, 128, 1).
  if (!make_tmap_3d_f16(&ta, g.A, (uint64_t)g.K, (uint64_t)g.M,
                        (uint64_t)g.batch, BK, BM))
    return -1;
  // W: dims (N, K, batch or 1); box (64, 64, 1).
  if (!make_tmap_3d_f16(&tb, g.B, (uint64_t)g.N, (uint64_t)g.K,
                        (uint64_t)(g.b_shared ? 1 : g.batch), 64, BK))
    return -1;
  // out: dims (N, M, batch); box (64, 32, 1) -- one epilogue warp's slab.
  CUtensorMap tcm;
  if (!make_tmap_3d_f16(&tcm, g.out, (uint64_t)g.N, (uint64_t)g.M,
                        (uint64_t)g.batch, 64, 32))
    return -1;
  GemmParams p;
  p.M = g.M;
  p.K = g.K;
  p.N = g.N;
  p.batch = g.batch;
  p.tiles_m = (int)((g.M + BM - 1) / BM);
  p.tiles_n = (g.N + BN - 1) / BN;
  p.total_tiles = g.batch * (int64_t)p.tiles_m * p.tiles_n;
  p.num_kb = (g.K + BK - 1) / BK;
  p.b_shared = g.b_shared ? 1 : 0;
  p.act = g.act;
  p.bias = g.bias;
  p.resid = reinterpret_cast<const __half*>(g.resid);
  p.out = reinterpret_cast<__half*>(g.out);
  p.err = err;
  p.rope_cos = g.rope_cos;
  p.rope_sin = g.rope_sin;
  p.rope_idx = g.rope_idx;
  p.rope_nseg = g.rope_nseg;
  p.rope_stride = g.rope_stride > 0 ? g.rope_stride : 16;
  p.rope_T = g.rope_T > 0 ? g.rope_T : 1;
  p.rope_cols = ROPE ? g.rope_cols : 0;
  p.ln_stats = g.ln_stats;
  p.ln_colsum = g.ln_colsum;
  p.reverse = g.reverse;
  const int64_t grid64 =
      p.total_tiles < sm_count() ? p.total_tiles : (int64_t)sm_count();
  gemm_f16_tc<BN, ROPE, LN><<<(int)grid64, kGemmThreads, Cfg::SMEM_BYTES, s>>>(ta, tb,
                                                                            tcm, p);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Pairs that fit on the device at once (0: the pair kernel is not used),
// found once by the occupancy calculator for clusters of two.
// Resident CTA-pair clusters per device (0: the pair kernel is unavailable)
// and whether the residual is TMA-staged; published once by
// gemm_kernels_init, read by every launch on any host thread.
std::atomic<int> g_pair_clusters{0};
std::atomic<bool> g_pair_res{false};

template <bool ROPE, bool LN = false>
int launch_pair(const GemmDesc& g, int* err, cudaStream_t s) {
  constexpr int MODE = LN ? (ROPE ? kPairLnRope : kPairLn) : (ROPE ? kPairRope : kPairPlain);
  using Cfg = PairCfg<MODE>;
  CUtensorMap ta, tb, tcm, trm;
  // A: dims (K, M, batch); box (64, 128, 1) -- one CTA's rows.
  if (!make_tmap_3d_f16(&ta, g.A, (uint64_t)g.K, (uint64_t)g.M, (uint64_t)g.batch, BK, BM))
    return -1;
  // W: dims (N, K, batch or 1); box (64, 64, 1); two per CTA per stage.
  if (!make_tmap_3d_f16(&tb, g.B, (uint64_t)g.N, (uint64_t)g.K,
                        (uint64_t)(g.b_shared ? 1 : g.batch), 64, BK))
    return -1;
  if (!make_tmap_3d_f16(&tcm, g.out, (uint64_t)g.N, (uint64_t)g.M, (uint64_t)g.batch, 64, 32))
    return -1;
  // the residual, read through TMA boxes shaped like the output's
  const bool res_tma = !ROPE && !LN && g.resid && g_pair_res.load(std::memory_order_relaxed) &&
                       make_tmap_3d_f16(&trm, g.resid, (uint64_t)g.N, (uint64_t)g.M,
                                        (uint64_t)g.batch, 64, 32);
  if (!res_tma) trm = tcm;
  GemmParams p;
  p.M = g.M;
  p.K = g.K;
  p.N = g.N;
  p.batch = g.batch;
  p.tiles_m = (int)((g.M + 2 * BM - 1) / (2 * BM));   // 256-row pair tiles
  p.tiles_n = (g.N + Cfg::BN - 1) / Cfg::BN;
  p.total_tiles = g.batch * (int64_t)p.tiles_m * p.tiles_n;
  p.num_kb = (g.K + BK - 1) / BK;
  p.b_shared = g.b_shared ? 1 : 0;
  p.act = g.act;
  p.bias = g.bias;
  p.resid = reinterpret_cast<const __half*>(g.resid);
  p.out = reinterpret_cast<__half*>(g.out);
  p.err = err;
  p.rope_cos = g.rope_cos;
  p.rope_sin = g.rope_sin;
  p.rope_idx = g.rope_idx;
  p.rope_nseg = g.rope_nseg;
  p.rope_stride = g.rope_stride > 0 ? g.rope_stride : 16;
  p.rope_T = g.rope_T > 0 ? g.rope_T : 1;
  p.rope_cols = ROPE ? g.rope_cols : 0;
  p.ln_stats = g.ln_stats;
  p.ln_colsum = g.ln_colsum;
  p.reverse = g.reverse;
  const int64_t clusters = g_pair_clusters.load(std::memory_order_relaxed);
  if (clusters <= 0) return -1;
  const int64_t pairs = p.total_tiles < clusters ? p.total_tiles : clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = res_tma ? PairCfg<kPairRes>::SMEM_BYTES : Cfg::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      res_tma ? cudaLaunchKernelEx(&cfg, gemm_f16_pair<kPairRes>, ta, tb, tcm, trm, p)
              : cudaLaunchKernelEx(&cfg, gemm_f16_pair<MODE>, ta, tb, tcm, trm, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

}  // namespace

int gemm_kernels_init() {
  cudaError_t e1 = cudaFuncSetAttribute(
      gemm_f16_tc<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<64>::SMEM_BYTES);
  cudaError_t e2 = cudaFuncSetAttribute(
      gemm_f16_tc<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<128>::SMEM_BYTES);
  cudaError_t e3 = cudaFuncSetAttribute(
      gemm_f16_tc<256, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<256>::SMEM_BYTES);
  cudaError_t e4 = cudaFuncSetAttribute(
      gemm_f16_tc<256, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<256>::SMEM_BYTES);
  cudaError_t e5 = cudaFuncSetAttribute(
      gemm_f16_tc<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<128>::SMEM_BYTES);
  cudaError_t e6 = cudaFuncSetAttribute(
      gemm_f16_tc<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<64>::SMEM_BYTES);
  cudaError_t e8 = cudaFuncSetAttribute(
      gemm_f16_tc<256, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<256>::SMEM_BYTES);
  cudaError_t e9 = cudaFuncSetAttribute(
      gemm_f16_tc<256, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      GemmCfg<256>::SMEM_BYTES);
  cudaFuncAttributes fa;
  cudaError_t e7 = cudaFuncGetAttributes(&fa, gemm_f16_simt);
  sm_count();
  bool pair_on = true, pair_res_on = true;
#ifdef HEXLIB_B200_MEASUREMENT_KNOBS
  // Measurement builds only: HEXLIB_B200_GEMM_PAIR=0 turns the pair kernel
  // off and HEXLIB_B200_GEMM_PAIR_RES=0 its TMA-staged residual.
  {
    const char* env = getenv("HEXLIB_B200_GEMM_PAIR");
    const char* er = getenv("HEXLIB_B200_GEMM_PAIR_RES");
    pair_on = !(env && env[0] == '0');
    pair_res_on = !(er && er[0] == '0');
  }
#endif
  int clusters = 0;
  bool res = false;
  if (pair_on &&
      cudaFuncSetAttribute(gemm_f16_pair<kPairPlain>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           PairCfg<kPairPlain>::SMEM_BYTES) == cudaSuccess &&
      cudaFuncSetAttribute(gemm_f16_pair<kPairRope>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           PairCfg<kPairRope>::SMEM_BYTES) == cudaSuccess) {
    cudaFuncSetAttribute(gemm_f16_pair<kPairLn>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         PairCfg<kPairLn>::SMEM_BYTES);
    cudaFuncSetAttribute(gemm_f16_pair<kPairLnRope>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         PairCfg<kPairLnRope>::SMEM_BYTES);
    res = pair_res_on &&
          cudaFuncSetAttribute(gemm_f16_pair<kPairRes>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               PairCfg<kPairRes>::SMEM_BYTES) == cudaSuccess;
    cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)sm_count(), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = PairCfg<kPairPlain>::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_f16_pair<kPairPlain>, &cfg) == cudaSuccess &&
        n > 0)
      clusters = n;
    cudaGetLastError();
  }
  // Every device of a process is a B200 with the same answer; the values are
  // stored, never cleared, so a launch on another thread reads either the
  // initial "no pair kernel" or the final figures.
  g_pair_res.store(res, std::memory_order_relaxed);
  g_pair_clusters.store(clusters, std::memory_order_relaxed);
  if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess || e4 != cudaSuccess ||
      e5 != cudaSuccess || e6 != cudaSuccess || e7 != cudaSuccess || e8 != cudaSuccess ||
      e9 != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

// Tiling of a GEMM with N % 256 == 0: CTA-pair 256x256
// tiles or single-CTA 128x256 tiles, by the estimate `rounds x per-tile
// cost` -- rounds of tiles over the CTAs that run at once (a tail round
// costs a whole one), per-tile cost in units of one SM's share of a pair
// tile. Fitted to measured encoder shapes at 8K-64K rows on B200: the pair's
// lighter fill traffic pays where the mainloop bounds the tile (cost 1.0,
// 1.03 for a single-CTA tile); with a GELU epilogue the epilogue bounds it
// and the pair's cluster handshakes cost a little (1.05). 128x128 tiles
// were slower at every measured shape of 8K rows and more, and are chosen
// only for GEMMs too small to fill the device once (below). A measurement
// build (HEXLIB_B200_MEASUREMENT_KNOBS) can pin one with HEXLIB_B200_GEMM_TILE
// = pair, 256, 128 or 64; the library as shipped reads no environment.
enum { kTileAuto = 0, kTilePair = 1, kTile256 = 2, kTile128 = 3, kTile64 = 4 };

int tile_pin() {
#ifdef HEXLIB_B200_MEASUREMENT_KNOBS
  static const int pin = [] {
    const char* e = getenv("HEXLIB_B200_GEMM_TILE");
    return !e ? kTileAuto
              : (e[0] == 'p' ? kTilePair
                             : (e[0] == '2' ? kTile256
                                            : (e[0] == '1' ? kTile128
                                                           : (e[0] == '6' ? kTile64 : kTileAuto))));
  }();
  return pin;
#else
  return kTileAuto;
#endif
}

int choose_tiling(const GemmDesc& g) {
  const int pin = tile_pin();
  const int pair_clusters = g_pair_clusters.load(std::memory_order_relaxed);
  const bool pair_ok = pair_clusters > 0 && g.b_shared && g.batch == 1;
  if (pin == kTilePair && pair_ok) return kTilePair;
  if (pin == kTile256) return kTile256;
  if (pin == kTile128) return kTile128;
  if (pin == kTile64) return kTile64;
  if (!pair_ok) return kTile256;
  auto rounds = [](int64_t tiles, int64_t slots) { return (tiles + slots - 1) / slots; };
  // A GEMM whose pair tiles cannot fill the device even once runs on the
  // narrowest single-CTA tiles that still fit in one round: more CTAs, less
  // work each (measured at 256 rows, the 256^2 x 1 encoder: 982 images/s on
  // pair tiles, 1164 on 128x128, 1215 on 128x64). Larger GEMMs keep the
  // model below: at 4096 rows (256^2 x 16) 128x128 tiles everywhere
  // measured 19 % slower.
  const int64_t t_pair = ((g.M + 255) / 256) * (g.N / 256);
  const int64_t t_128 = ((g.M + 127) / 128) * ((g.N + 127) / 128);
  const int64_t t_64 = ((g.M + 127) / 128) * ((g.N + 63) / 64);
  if (t_pair < pair_clusters && t_64 <= sm_count()) return kTile64;
  if (t_pair < pair_clusters && t_128 <= sm_count()) return kTile128;
  const double c_pair = (double)rounds(((g.M + 255) / 256) * (g.N / 256), pair_clusters) *
                        (g.act != 0 ? 1.05 : 1.0);
  const double c_256 = (double)rounds(((g.M + 127) / 128) * (g.N / 256), sm_count()) * 1.03;
  return c_pair <= c_256 ? kTilePair : kTile256;
}

int launch_gemm(const GemmDesc& desc, int* err, cudaStream_t s) {
  GemmDesc g = desc;
  if (g.batch < 0 || g.M < 0 || g.K <= 0 || g.N <= 0 || g.act < 0 ||
      g.act > 2 || !g.A || !g.B || !g.out)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (g.batch == 0 || g.M == 0) return HEXLIB_B200_OK;
  g.reverse = order_next();
  const bool rope = g.rope_cols > 0;
  if (rope && (g.rope_cols % 64 || g.rope_cols > g.N || g.N % 64 || g.rope_T <= 0 ||
               (g.rope_stride != 0 && g.rope_stride != 16 && g.rope_stride != 32) ||
               g.rope_nseg <= 0 || !g.rope_cos || !g.rope_sin || !g.rope_idx ||
               !aligned16(g.rope_cos) ||
               !aligned16(g.rope_sin) || !aligned16(g.rope_idx)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  const bool tma_ok = (g.K % 8) == 0 && (g.N % 8) == 0 && aligned16(g.A) &&
                      aligned16(g.B) && aligned16(g.out) &&
                      (!g.bias || aligned16(g.bias)) &&
                      (!g.resid || aligned16(g.resid)) && tma_available();
  const bool ln = g.ln_stats != nullptr;
  if (ln && (!g.ln_colsum || g.resid || g.N % 256 || !tma_ok ||
             (reinterpret_cast<uintptr_t>(g.ln_stats) & 7u) || !aligned16(g.ln_colsum)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;   // served by the tensor-core kernels only
  if (ln) {
    const int tiling = choose_tiling(g);
    int rc;
    if (tiling == kTilePair)
      rc = rope ? launch_pair<true, true>(g, err, s) : launch_pair<false, true>(g, err, s);
    else
      rc = rope ? launch_tc<256, true, true>(g, err, s) : launch_tc<256, false, true>(g, err, s);
    return rc == -1 ? HEXLIB_B200_ERR_INVAL_PARAMS : rc;
  }
  if (tma_ok) {
    int rc;
    const int tiling = (g.N % 256 == 0) ? choose_tiling(g) : 0;
    if (tiling == kTilePair)
      rc = rope ? launch_pair<true>(g, err, s) : launch_pair<false>(g, err, s);
    else if (tiling == kTile128 && rope)
      rc = launch_tc<128, true>(g, err, s);
    else if (tiling == kTile128)
      rc = launch_tc<128, false>(g, err, s);
    else if (tiling == kTile64)
      rc = rope ? launch_tc<64, true>(g, err, s) : launch_tc<64, false>(g, err, s);
    else if (g.N % 256 == 0)
      rc = rope ? launch_tc<256, true>(g, err, s) : launch_tc<256, false>(g, err, s);
    else if (g.N % 128 == 0)
      rc = rope ? launch_tc<128, true>(g, err, s) : launch_tc<128, false>(g, err, s);
    else
      rc = rope ? launch_tc<64, true>(g, err, s) : launch_tc<64, false>(g, err, s);
    if (rc != -1) return rc;
    if (rope) return HEXLIB_B200_ERR_INVAL_PARAMS;  // no CUDA-core rope path
    // The tensor map was refused on the host: fall through to CUDA cores.
  }
  const int tiles_m = (int)((g.M + 63) / 64), tiles_n = (g.N + 63) / 64;
  int64_t total = g.batch * tiles_m * (int64_t)tiles_n;
  int64_t cap = (int64_t)sm_count() * 4;
  const int grid = (int)(total < cap ? total : cap);
  gemm_f16_simt<<<grid, 256, 0, s>>>(
      reinterpret_cast<const __half*>(g.A), reinterpret_cast<const __half*>(g.B),
      g.bias, reinterpret_cast<const __half*>(g.resid),
      reinterpret_cast<__half*>(g.out), g.M, g.K, g.N, g.batch,
      g.b_shared ? 1 : 0, g.act);
  if (cudaPeekAtLastError() != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

}  // namespace hb
