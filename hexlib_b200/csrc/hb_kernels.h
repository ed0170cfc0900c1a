// hb_kernels.h -- host-side launchers for every kernel in libhexlib_b200.
//
// Each launcher enqueues its kernel(s) on `stream` and returns a status
// (HEXLIB_B200_OK, or HEXLIB_B200_ERR_INVAL_PARAMS for arguments it cannot
// serve); none allocates memory or synchronises, so every one of them can be
// recorded into a CUDA graph. The public kernel_api.h-shaped entry points and
// the batch dispatcher both call these, with the batch dimension the
// dispatcher folds in (images per launch) passed explicitly.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hexlib_b200.h"

namespace hb {

// Walk order of the persistent kernels (GEMM tiles, attention items,
// layernorm rows). Consecutive launches on a host thread alternate between
// ascending and descending order, so that a kernel first reads the rows its
// producer wrote last -- the ones still in L2. Every tile, item and row is
// computed the same way in either order; only the schedule changes.
// order_next() returns 0 (ascending) or 1 (descending) and flips the
// thread's state; order_reset() restarts it at ascending (the dispatcher
// does so before each batch, so a captured plan is the same every time).
// HEXLIB_B200_WALK_ORDER=ascending fixes every launch at ascending.
int order_next();
void order_reset();

// Elementwise. `nb` is the right operand's element count: it is broadcast
// with period nb (nb == n for a plain add; nb < n when a per-image tensor is
// added to one shared by every image).
int launch_add_f16(const void* a, const void* b, void* y, int64_t n,
                   int64_t nb, cudaStream_t s);
int launch_add_f16_f32(const void* a, const float* b, void* y, int64_t n,
                       int64_t nb, cudaStream_t s);
int launch_cast_f32_f16(const float* x, void* y, int64_t n, cudaStream_t s);
int launch_scale_f16(const void* x, void* y, int64_t n, float factor,
                     cudaStream_t s);
int launch_copy(const void* x, void* y, int64_t nbytes, cudaStream_t s);

// Row-wise.
int launch_layernorm_f16(const void* x, const float* w, const float* b,
                         void* y, int64_t R, int C, float eps, cudaStream_t s);
// patchify with its output rounded to fp16 (patchify then cast, in one pass).
int launch_patchify_f32_f16(const float* img, void* out, int64_t nimg, int C, int T, int H,
                            int W, int patch, int merge, int grid_h, int grid_w,
                            cudaStream_t s);
// (mean, 1/sqrt(var + eps)) of each of R rows of C fp16, as float2 pairs.
int launch_ln_stats_f16(const void* x, float* stats, int64_t R, int C, float eps,
                        cudaStream_t s);
int launch_rmsnorm_f16(const void* x, const void* w, void* y, int64_t R, int C,
                       float eps, cudaStream_t s);
int launch_softmax_f16(const void* x, void* y, int64_t R, int C,
                       cudaStream_t s);
// rows = tokens over every image; the cos/sin tables have `table_rows` rows
// and token r uses table row r % table_rows.
int launch_rope_f16(const void* x, const float* cos_t, const float* sin_t,
                    void* y, int64_t rows, int H, int D, int64_t table_rows,
                    cudaStream_t s);

// RoPE on the q and k sections of a packed [rows, 3, H, D] projection; out
// may equal qkv (in place), otherwise the whole tensor is copied first.
int launch_rope_qk_f16(const void* qkv, const float* cos_t, const float* sin_t, void* out,
                       int64_t rows, int H, int D, int64_t table_rows, cudaStream_t s);

// Layout moves. `nimg` independent [T,H,D] -> [H,T,D] permutes.
int launch_transpose_th_f16(const void* x, void* y, int64_t nimg, int T, int H,
                            int D, cudaStream_t s);
// [B,T,D] -> [B,D,T].
int launch_transpose_hd_f16(const void* x, void* y, int64_t B, int T, int D,
                            cudaStream_t s);
int launch_patchify_f32(const float* img, float* out, int64_t nimg, int C,
                        int T, int H, int W, int patch, int merge, int grid_h,
                        int grid_w, cudaStream_t s);

// Tensor-core GEMMs (tcgen05), with a CUDA-core fallback for shapes the TMA
// path cannot describe (K or N not a multiple of 8, misaligned pointers).
//   out[b] = act(A[b] @ W[b or shared] + bias) (+ resid[b])
struct GemmDesc {
  const void* A;       // [batch, M, K] fp16 row-major
  const void* B;       // [batch or 1, K, N] fp16 row-major (MN-major operand)
  const float* bias;   // [N] or nullptr
  const void* resid;   // [batch, M, N] fp16 or nullptr
  void* out;           // [batch, M, N] fp16
  int64_t batch;       // independent products
  int64_t M;
  int K, N;
  bool b_shared;       // B has one copy used by every batch entry
  int act;             // 0 none, 1 gelu_tanh, 2 gelu_erf
  // RoPE epilogue: when rope_cols > 0, columns [0, rope_cols) are 64-wide
  // heads rotated for row r's token t = r % rope_T, after the fp16 rounding
  // of act(A@W + bias) (the rope_2d op on q/k). The [rope_T, 64] cos/sin
  // tables are half-symmetric (dims i and i + 32 share a value) and come as
  // 16-wide segments: dims [16s, 16s + 16) and [32 + 16s, 48 + 16s) of token
  // t are row rope_idx[2t + s] of the [n, 16] fp32 tables rope_cos / rope_sin.
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  const int* rope_idx = nullptr;   // [rope_T, 2]; entries clamped to [0, rope_nseg)
  // floats between consecutive segment rows: 16 for separate cos / sin
  // tables, 32 for one [n, 2, 16] table (rope_sin = rope_cos + 16); 0 = 16
  int rope_stride = 0;
  int rope_nseg = 0;
  int rope_T = 0;
  int rope_cols = 0;
  // LayerNorm epilogue (tensor-core kernels, N % 256 == 0, no residual):
  // when ln_stats is set, A holds the raw rows x and B = diag(gamma) W; row
  // r's (mean, rstd) pair is ln_stats[2r, 2r + 1] (8-byte aligned), the
  // column sums of B are ln_colsum[N] (16-byte aligned), and the result is
  // act(rstd * (A@B - mean * colsum) + bias) = act(LayerNorm(x) @ W + bias)
  // when bias = beta @ W + the original bias.
  const float* ln_stats = nullptr;
  const float* ln_colsum = nullptr;
  // tile walk order, set by launch_gemm from order_next()
  int reverse = 0;
};
int launch_gemm(const GemmDesc& g, int* err, cudaStream_t s);

// Block-quantized weights (k_quant.cu). qtype is the wire dtype id of the
// weight: QTYPE_Q4_0 (18-byte blocks) or QTYPE_Q8_0 (34-byte blocks).
enum : int { QTYPE_Q4_0 = 2, QTYPE_Q8_0 = 4 };
int quant_kernels_init();
int quant_block_bytes(int qtype);  // 0 for anything else
// [K, N] blocks along N (N % 32 == 0) -> fp16 [K, N], out 16-byte aligned.
int launch_dequant_f16(int qtype, const void* w, void* out, int64_t K, int64_t N,
                       cudaStream_t s);
// g with a quantized g.B: dequantize into `workspace` (>= K*N*2 bytes), then
// the fp16 GEMM on it. Weight shared across the batch only (b_shared, batch 1).
int launch_gemm_quant(const GemmDesc& g, int qtype, void* workspace, uint64_t ws_bytes,
                      int* err, cudaStream_t s);

// Fused attention: q, k, v, ctx are [Bn, T, D] fp16.
int launch_attention(const void* q, const void* k, const void* v, void* ctx,
                     int64_t Bn, int T, int D, float scale, int* err,
                     cudaStream_t s);

// Fused attention over a packed projection: qkv is [B, T, 3, H, D] (q, k, v
// sections of each token row), ctx is [B, T, H, D]. D must be 64.
int launch_attention_qkv(const void* qkv, void* ctx, int64_t B, int T, int H, int D,
                         float scale, int* err, cudaStream_t s);

// Diagnostic: a kernel whose bounded wait never completes; it records a
// timeout in `err` after `limit_us` and returns.
int launch_wait_timeout_probe(int* err, uint32_t limit_us, cudaStream_t s);

// Setup of kernel attributes (dynamic shared memory limits) on the current
// device, once per device; allocates nothing. Returns a status.
int kernels_init_device();

// kernels_init_device() plus the one-time allocation of the error word of
// the per-kernel entry points; safe to call repeatedly. Returns a status.
int kernels_init();

// The session-independent device error word that kernels launched through
// the public per-kernel entry points report bounded-wait timeouts in.
int* default_error_word();

// Reads and clears that word (after the caller has drained its stream);
// true if a bounded wait had expired.
bool take_default_error();

// Reads and clears the current device's error word of the non-allocating
// q4_0 entry point (a no-op before that entry has run on the device); sets
// *set when a bounded wait had expired. Returns a status.
int noalloc_take_error(bool* set);

}  // namespace hb
