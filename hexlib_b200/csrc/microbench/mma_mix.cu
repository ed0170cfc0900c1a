// mma_mix -- tcgen05.mma issue throughput on one SM, for the shapes the
// fused attention kernel issues (not part of libhexlib_b200.so).
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -o mma_mix hexlib_b200/csrc/microbench/mma_mix.cu -lcuda && ./mma_mix
//
// Part 1: one thread issues 4096 (or 8192) back-to-back kind::f16 MMAs of
// M=128, K=16 into one accumulator, then one commit; cycles per instruction
// for N = 64 / 128 / 256 with both operands in shared memory, and N = 64 with
// A in tensor memory (the P V product). Rate-proportional cost at the dense
// peak is N / 2 cycles (8192 FLOP per cycle per SM).
//
// Part 2: the attention kernel's per-block MMA mix for two query tiles --
// S_t = Q_t K^T (4 x N=128, SS) and O_t += P_t V (8 x N=64, TS) for t = a, b
// -- issued alternately (S_a, PV_a, S_b, PV_b) or grouped (PV_a, PV_b, S_a,
// S_b), optionally with a commit and an mbarrier wait (on an already
// completed phase) between groups, and optionally with eight warps reading
// 128 and writing 64 TMEM columns per round as the softmax does. Nominal
// tensor time per block is 2 * 4 * 64 + 2 * 8 * 32 = 1024 cycles.
//
// Every shared- and tensor-memory access stays inside the allocation; every
// wait is bounded (mbar_wait); one CTA per SM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../hb_device.cuh"

using namespace hb;

namespace {

constexpr int kSmem = 120 * 1024;   // forces one CTA per SM (tensor memory is 512 columns)

// Part 1. mode 0: SS, K-major A and B; mode 1: TS (A from tensor memory),
// MN-major B; mode 2: SS, MN-major B; mode 3: mode 1 behind a runtime branch.
__global__ void __launch_bounds__(128, 1) single_shape(int N, int mode, int reps,
                                                       long long* out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                 // 16 KiB: 128 rows x 64 fp16
  uint8_t* sB = smem + 16384;         // 32 KiB: 256 rows x 64 fp16
  uint64_t* bar = (uint64_t*)(smem + 49152);
  uint32_t* slot = (uint32_t*)(bar + 1);
  volatile int* abort_flag = (volatile int*)(slot + 1);
  for (int i = threadIdx.x; i < 49152 / 16; i += blockDim.x)
    ((uint4*)smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_shared();
  __syncthreads();
  if (threadIdx.x < 32) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    const long long t0 = clock64();
    if (mode == 0) {
      const uint32_t idesc = idesc_f16_f32(128, N, false, false);
      for (int r = 0; r < reps; ++r)
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem, sdesc_sw128(a0 + kk * 32, 16, 1024), sdesc_sw128(b0 + kk * 32, 16, 1024),
                   idesc, 1u);
    } else if (mode == 1) {
      const uint32_t idesc = idesc_f16_f32(128, N, false, true);
      for (int r = 0; r < reps; ++r)
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ts(tmem, tmem + 256u + (uint32_t)(kk * 8),
                      sdesc_sw128(b0 + kk * 2048, 8192, 1024), idesc, 1u);
    } else if (mode == 2) {
      const uint32_t idesc = idesc_f16_f32(128, N, false, true);
      for (int r = 0; r < reps; ++r)
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem, sdesc_sw128(a0 + (kk & 3) * 32, 16, 1024),
                   sdesc_sw128(b0 + kk * 2048, 8192, 1024), idesc, 1u);
    } else {
      // mode 3: mode 1's instructions, each behind a (uniform, always true)
      // runtime branch -- the cost of control flow between MMAs
      const uint32_t idesc = idesc_f16_f32(128, N, false, true);
      const bool ts = reps > 0;
      for (int r = 0; r < reps; ++r)
        for (int kk = 0; kk < 8; ++kk) {
          if (ts)
            umma_f16_ts(tmem, tmem + 256u + (uint32_t)(kk * 8),
                        sdesc_sw128(b0 + kk * 2048, 8192, 1024), idesc, 1u);
          else
            umma_f16(tmem, sdesc_sw128(a0 + (kk & 3) * 32, 16, 1024),
                     sdesc_sw128(b0 + kk * 2048, 8192, 1024), idesc, 1u);
        }
    }
    umma_commit(bar);
    const bool ok = mbar_wait(bar, 0, abort_flag, err);
    const long long t1 = clock64();
    if (blockIdx.x == 0) {
      out[0] = t1 - t0;
      out[1] = ok;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Part 2. flags: 1 grouped order, 2 commit + wait between groups, 4 TMEM
// traffic from the eight other warps. FLAGS is the same set as a template
// argument (-1: use the runtime one), so the issue loop carries no branch.
template <int FLAGS>
__global__ void __launch_bounds__(352, 1) attention_mix(int flags, int iters, long long* out,
                                                        int* err) {
  if (FLAGS >= 0) flags = FLAGS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;              // two 16 KiB query tiles
  uint8_t* sK = smem + 32768;      // 16 KiB
  uint8_t* sV = smem + 49152;      // 16 KiB
  // [0..3] per-group commits, [4] completed at start, [5] the final commit
  uint64_t* bars = (uint64_t*)(smem + 65536);
  uint32_t* slot = (uint32_t*)(bars + 6);
  volatile int* abort_flag = (volatile int*)(slot + 1);
  volatile int* stop = (volatile int*)(slot + 2);
  for (int i = threadIdx.x; i < 65536 / 16; i += blockDim.x)
    ((uint4*)smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    for (int b = 0; b < 6; ++b) mbar_init(&bars[b], b == 5 && (flags & 128) ? 2 : 1);
    *abort_flag = 0;
    *stop = 0;
    fence_mbar_init();
    mbar_arrive(&bars[4]);
  }
  fence_proxy_async_shared();
  __syncthreads();
  if (threadIdx.x < 32) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool grouped = flags & 1, traffic = flags & 4;
  const bool commits = (flags & 2) || (flags & 8), waits = (flags & 2) || (flags & 16);
  const bool fence = !(flags & 32);
  const bool prefetch = flags & 64;   // test the next group's barrier before this group's MMAs
  const bool two = flags & 128;       // warp 1 issues tile a's MMAs, warp 10 tile b's
  if (warp == 1 || (two && warp == 10)) {
    if (lane == 0) {
      const int only = two ? (warp == 1 ? 0 : 1) : -1;
      const uint32_t idesc_s = idesc_f16_f32(128, 128, false, false);
      const uint32_t idesc_o = idesc_f16_f32(128, 64, false, true);
      bool ready = false;
      auto wait_ready = [&]() -> bool {
        if (!waits) return true;
        if (prefetch && ready) return true;
        return mbar_wait(&bars[4], 0, abort_flag, err);
      };
      auto issue_s = [&](int t) {
        if (!wait_ready()) return;
        if (prefetch) ready = mbar_test_wait(&bars[4], 0);
        if (fence) tc_fence_after();
        const uint32_t qa = smem_u32(sQ + t * 16384), kb = smem_u32(sK);
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + t * 128, sdesc_sw128(qa + kk * 32, 16, 1024),
                   sdesc_sw128(kb + kk * 32, 16, 1024), idesc_s, kk ? 1u : 0u);
        if (commits) umma_commit(&bars[t]);
      };
      auto issue_pv = [&](int t) {
        if (!wait_ready()) return;
        if (prefetch) ready = mbar_test_wait(&bars[4], 0);
        if (fence) tc_fence_after();
        const uint32_t vb = smem_u32(sV);
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ts(tmem + 256 + t * 64, tmem + 384 + t * 64 + kk * 8,
                      sdesc_sw128(vb + kk * 2048, 8192, 1024), idesc_o, 1u);
        if (commits) umma_commit(&bars[2 + t]);
      };
      const long long t0 = clock64();
      for (int it = 0; it < iters; ++it) {
        if (only >= 0) {
          issue_s(only);
          issue_pv(only);
          continue;
        }
        if (grouped) {
          issue_pv(0);
          issue_pv(1);
          issue_s(0);
          issue_s(1);
        } else {
          issue_s(0);
          issue_pv(0);
          issue_s(1);
          issue_pv(1);
        }
      }
      umma_commit(&bars[5]);   // one arrival per issuer, when its MMAs have completed
      mbar_wait(&bars[5], 0, abort_flag, err);
      const long long t1 = clock64();
      if (blockIdx.x == 0 && warp == 1) out[0] = t1 - t0;
      if (blockIdx.x == 0 && warp == 10) out[1] = t1 - t0;
      if (warp == 1) *stop = 1;
    }
  } else if (warp >= 2 && warp < 10 && traffic) {
    // softmax-like traffic in this warp's lane quarter: read a tile's 128
    // score columns, write 64 columns of P
    const int quarter = warp & 3;
    const int t = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t acc = 0;
    int n = 0;
    while (!*stop && n < 1000000) {
      uint32_t v[32];
      for (int c = 0; c < 4; ++c) {
        tmem_ld_32x32b_x32(tmem + lane_off + t * 128 + c * 32, v);
        tmem_ld_wait();
        acc += v[c];
      }
      uint32_t h[16];
      for (int e = 0; e < 16; ++e) h[e] = acc + e;
      for (int c = 0; c < 4; ++c) tmem_st_32x32b_x16(tmem + lane_off + 384 + t * 64 + c * 16, h);
      tmem_st_wait();
      ++n;
      __nanosleep(200);
    }
    if (acc == 0xFFFFFFFFu && blockIdx.x == 0) out[3] = acc;   // keep the loads alive
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int main() {
  long long* d_out;
  int* d_err;
  cudaMalloc(&d_out, 64);
  cudaMalloc(&d_err, 4);
  cudaMemset(d_err, 0, 4);
  cudaFuncSetAttribute(single_shape, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  for (auto k : {attention_mix<0>, attention_mix<2>, attention_mix<6>, attention_mix<66>,
                 attention_mix<70>, attention_mix<130>, attention_mix<134>})
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);

  printf("Part 1: cycles per tcgen05.mma kind::f16, M=128 K=16, all %d SMs busy\n", sms);
  struct Shape { int N, mode, per_rep; const char* name; } shapes[] = {
      {64, 0, 4, "SS K-major  N=64 "}, {128, 0, 4, "SS K-major  N=128"},
      {256, 0, 4, "SS K-major  N=256"}, {64, 1, 8, "TS MN-major N=64 "},
      {64, 2, 8, "SS MN-major N=64 "}, {64, 3, 8, "TS N=64, branch "}};
  for (const Shape& c : shapes) {
    const int reps = 1024;
    single_shape<<<sms, 128, kSmem>>>(c.N, c.mode, reps, d_out, d_err);
    const cudaError_t e = cudaDeviceSynchronize();
    long long h[2] = {0, 0};
    int herr = 0;
    cudaMemcpy(h, d_out, sizeof(h), cudaMemcpyDeviceToHost);
    cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost);
    const double n = (double)reps * c.per_rep;
    printf("  %s  %6.1f cycles (rate-proportional %5.1f)  %s%s\n", c.name, h[0] / n, c.N / 2.0,
           e == cudaSuccess ? "" : cudaGetErrorString(e), herr || !h[1] ? " WAIT FAILED" : "");
  }

  printf("Part 2: cycles per block of the attention MMA mix (nominal 1024)\n");
  const char* names[] = {"alternating", "grouped"};
  for (int v = 0; v < 7; ++v) {
    const int flags = (int[]){0, 2, 66, 6, 70, 130, 134}[v];
    const int iters = 256;
    cudaMemset(d_out, 0, 64);
    switch (flags) {
      case 0: attention_mix<0><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      case 2: attention_mix<2><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      case 66: attention_mix<66><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      case 6: attention_mix<6><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      case 70: attention_mix<70><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      case 130: attention_mix<130><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
      default: attention_mix<134><<<sms, 352, kSmem>>>(flags, iters, d_out, d_err); break;
    }
    const cudaError_t e = cudaDeviceSynchronize();
    long long h = 0;
    int herr = 0;
    cudaMemcpy(&h, d_out, sizeof(h), cudaMemcpyDeviceToHost);
    cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost);
    const char* between = (flags & 128) ? "two issuers, commit+wait"
                          : (flags & 2) ? ((flags & 64) ? "commit+wait, tested ahead" : "commit+wait")
                          : (flags & 8) ? "commit only" : (flags & 16) ? "wait only" : "back-to-back";
    printf("  %-11s %-26s %-13s %7.1f  %s%s\n", names[flags & 1],
           between, (flags & 4) ? "TMEM traffic" : "",
           (double)h / iters, e == cudaSuccess ? "" : cudaGetErrorString(e),
           herr ? " WAIT FAILED" : "");
  }
  return 0;
}
