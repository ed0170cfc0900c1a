// entries.cu -- the kernel_api.h-shaped C entry points of libhexlib_b200.
//
// One function per kernels/<k>/kernel_api.h signature, with a trailing stream
// and an int status. They validate their scalar arguments, then call the same
// launcher the batch dispatcher uses, with one image.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/hexlib_b200.h"
#include "hb_kernels.h"

namespace hb {

int memory_kernels_init();
int gemm_kernels_init();
int quant_kernels_init();
int attention_kernels_init();
int diag_kernels_init();

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_dev_once[kMaxDevices];
int g_dev_status[kMaxDevices];
std::once_flag g_word_once;
int g_word_status = HEXLIB_B200_ERR_INTERNAL;
int* g_err_host = nullptr;
int* g_err_dev = nullptr;
}  // namespace

// Function attributes (the dynamic shared memory each kernel may take) belong
// to the device that is current when they are set, so every device a process
// uses runs this once, with that device current. It allocates nothing.
int kernels_init_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  std::call_once(g_dev_once[dev], [dev] {
    int rc = memory_kernels_init();
    if (rc == HEXLIB_B200_OK) rc = gemm_kernels_init();
    if (rc == HEXLIB_B200_OK) rc = quant_kernels_init();
    if (rc == HEXLIB_B200_OK) rc = attention_kernels_init();
    if (rc == HEXLIB_B200_OK) rc = diag_kernels_init();
    if (rc != HEXLIB_B200_OK) cudaGetLastError();
    g_dev_status[dev] = rc;
  });
  return g_dev_status[dev];
}

// The per-kernel entries' error word: one int of mapped, portable host memory
// that every device can write (a bounded wait that expires sets it to 1) and
// the host reads after the stream has drained (hexlib_b200_stream_status).
int kernels_init() {
  const int rc = kernels_init_device();
  if (rc != HEXLIB_B200_OK) return rc;
  std::call_once(g_word_once, [] {
    int st = HEXLIB_B200_ERR_CUDA;
    int* host = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&host), sizeof(int),
                      cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess) {
      *host = 0;
      if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&g_err_dev), host, 0) ==
          cudaSuccess) {
        g_err_host = host;
        st = HEXLIB_B200_OK;
      }
    }
    if (st != HEXLIB_B200_OK) cudaGetLastError();
    g_word_status = st;
  });
  return g_word_status;
}

// Reads and clears the per-kernel entries' error word; true if it was set.
bool take_default_error() {
  if (!g_err_host) return false;
  volatile int* e = g_err_host;
  const bool set = *e != 0;
  *e = 0;
  return set;
}

int* default_error_word() { return g_err_dev; }

}  // namespace hb

using hb::kernels_init;

#define HB_ENTRY_INIT()                              \
  do {                                               \
    const int _rc = kernels_init();                  \
    if (_rc != HEXLIB_B200_OK) return _rc;           \
  } while (0)

static inline cudaStream_t as_stream(void* s) {
  return reinterpret_cast<cudaStream_t>(s);
}

extern "C" {

int hexlib_b200_add_fp16(const void* a, const void* b, void* y, int n,
                         void* stream) {
  HB_ENTRY_INIT();
  if (n < 0 || (n > 0 && (!a || !b || !y))) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_add_f16(a, b, y, n, n > 0 ? n : 1, as_stream(stream));
}

int hexlib_b200_add_fp16_f32(const void* a, const float* b, void* y, int n,
                             void* stream) {
  HB_ENTRY_INIT();
  if (n < 0 || (n > 0 && (!a || !b || !y))) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_add_f16_f32(a, b, y, n, n > 0 ? n : 1, as_stream(stream));
}

int hexlib_b200_cast_f32_f16(const float* x, void* y, int n, void* stream) {
  HB_ENTRY_INIT();
  if (n < 0 || (n > 0 && (!x || !y))) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_cast_f32_f16(x, y, n, as_stream(stream));
}

int hexlib_b200_scale_fp16(const void* x, void* y, int n, float factor,
                           void* stream) {
  HB_ENTRY_INIT();
  if (n < 0 || (n > 0 && (!x || !y))) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_scale_f16(x, y, n, factor, as_stream(stream));
}

int hexlib_b200_layernorm_fp16(const void* x, const float* w, const float* b,
                               void* y, int R, int C, float eps,
                               void* stream) {
  HB_ENTRY_INIT();
  if (R < 0 || C <= 0 || (R > 0 && (!x || !w || !b || !y)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_layernorm_f16(x, w, b, y, R, C, eps, as_stream(stream));
}

int hexlib_b200_rmsnorm_fp16(const void* x, const void* w, void* y, int R,
                             int C, float eps, void* stream) {
  HB_ENTRY_INIT();
  if (R < 0 || C <= 0 || (R > 0 && (!x || !w || !y)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_rmsnorm_f16(x, w, y, R, C, eps, as_stream(stream));
}

int hexlib_b200_softmax_fp16(const void* x, void* y, int R, int C,
                             void* stream) {
  HB_ENTRY_INIT();
  if (R < 0 || C <= 0 || (R > 0 && (!x || !y)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_softmax_f16(x, y, R, C, as_stream(stream));
}

int hexlib_b200_rope_2d_fp16(const void* x, const float* costab,
                             const float* sintab, void* y, int T, int H, int D,
                             void* stream) {
  HB_ENTRY_INIT();
  if (T < 0 || H <= 0 || D <= 0 || (D & 1) ||
      (T > 0 && (!x || !costab || !sintab || !y)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (T == 0) return HEXLIB_B200_OK;
  return hb::launch_rope_f16(x, costab, sintab, y, T, H, D, T,
                             as_stream(stream));
}

int hexlib_b200_transpose_th_fp16(const void* x, void* y, int T, int H, int D,
                                  void* stream) {
  HB_ENTRY_INIT();
  if (T <= 0 || H <= 0 || D <= 0 || !x || !y)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_transpose_th_f16(x, y, 1, T, H, D, as_stream(stream));
}

int hexlib_b200_transpose_hd_fp16(const void* x, void* y, int B, int T, int D,
                                  void* stream) {
  HB_ENTRY_INIT();
  if (B < 0 || T <= 0 || D <= 0 || (B > 0 && (!x || !y)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_transpose_hd_f16(x, y, B, T, D, as_stream(stream));
}

int hexlib_b200_patchify_fp32(const float* img, float* out, int C, int T,
                              int H, int W, int patch, int merge, int grid_h,
                              int grid_w, void* stream) {
  HB_ENTRY_INIT();
  if (!img || !out) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_patchify_f32(img, out, 1, C, T, H, W, patch, merge, grid_h,
                                 grid_w, as_stream(stream));
}

int hexlib_b200_patchify_fp16(const float* img, void* out, int C, int T, int H, int W,
                              int patch, int merge, int grid_h, int grid_w, void* stream) {
  HB_ENTRY_INIT();
  return hb::launch_patchify_f32_f16(img, out, 1, C, T, H, W, patch, merge, grid_h, grid_w,
                                     as_stream(stream));
}

int hexlib_b200_matmul_fp16(const void* A, const void* B, void* C, int Bn,
                            int M, int K, int N, void* stream) {
  HB_ENTRY_INIT();
  if (Bn < 0 || M < 0 || K <= 0 || N <= 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  hb::GemmDesc g{};
  g.A = A;
  g.B = B;
  g.out = C;
  g.batch = Bn;
  g.M = M;
  g.K = K;
  g.N = N;
  g.b_shared = false;
  g.act = 0;
  return hb::launch_gemm(g, hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_matmul_epilogue_fp16(const void* a, const void* w,
                                     const float* bias, void* out, int M,
                                     int K, int N, int act, void* stream) {
  HB_ENTRY_INIT();
  if (M < 0 || K <= 0 || N <= 0 || act < 0 || act > 2 || !bias)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
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
  return hb::launch_gemm(g, hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_dequant_q4_0_fp16(const void* w, void* out, int K, int N, void* stream) {
  HB_ENTRY_INIT();
  if (K < 0 || N < 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_dequant_f16(hb::QTYPE_Q4_0, w, out, K, N, as_stream(stream));
}

int hexlib_b200_dequant_q8_0_fp16(const void* w, void* out, int K, int N, void* stream) {
  HB_ENTRY_INIT();
  if (K < 0 || N < 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_dequant_f16(hb::QTYPE_Q8_0, w, out, K, N, as_stream(stream));
}

static int matmul_epilogue_quant(int qtype, const void* a, const void* w, const float* bias,
                                 void* out, int M, int K, int N, int act, void* workspace,
                                 uint64_t workspace_bytes, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || N % 32 || act < 0 || act > 2 || !bias || !w)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
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
  return hb::launch_gemm_quant(g, qtype, workspace, workspace_bytes, hb::default_error_word(),
                               as_stream(stream));
}

int hexlib_b200_matmul_epilogue_q4_0(const void* a, const void* w, const float* bias,
                                     void* out, int M, int K, int N, int act, void* workspace,
                                     uint64_t workspace_bytes, void* stream) {
  HB_ENTRY_INIT();
  return matmul_epilogue_quant(hb::QTYPE_Q4_0, a, w, bias, out, M, K, N, act, workspace,
                               workspace_bytes, stream);
}

int hexlib_b200_matmul_epilogue_q8_0(const void* a, const void* w, const float* bias,
                                     void* out, int M, int K, int N, int act, void* workspace,
                                     uint64_t workspace_bytes, void* stream) {
  HB_ENTRY_INIT();
  return matmul_epilogue_quant(hb::QTYPE_Q8_0, a, w, bias, out, M, K, N, act, workspace,
                               workspace_bytes, stream);
}

int hexlib_b200_matmul_epilogue_residual_fp16(const void* a, const void* w,
                                              const float* bias, const void* r,
                                              void* out, int M, int K, int N,
                                              int act, void* stream) {
  HB_ENTRY_INIT();
  if (M < 0 || K <= 0 || N <= 0 || act < 0 || act > 2 || !bias || !r)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  hb::GemmDesc g{};
  g.A = a;
  g.B = w;
  g.bias = bias;
  g.resid = r;
  g.out = out;
  g.batch = 1;
  g.M = M;
  g.K = K;
  g.N = N;
  g.b_shared = true;
  g.act = act;
  return hb::launch_gemm(g, hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_matmul_epilogue_rope_fp16(const void* a, const void* w, const float* bias,
                                          const float* seg_cos, const float* seg_sin,
                                          const int* seg_idx, int n_seg, void* out, int M,
                                          int K, int N, int act, int rope_cols, int T,
                                          void* stream) {
  HB_ENTRY_INIT();
  if (M < 0 || K <= 0 || N <= 0 || act < 0 || act > 2 || !bias || !seg_cos || !seg_sin ||
      !seg_idx || n_seg <= 0 || rope_cols <= 0 || T <= 0 || (M % T) != 0)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
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
  g.rope_cos = seg_cos;
  g.rope_sin = seg_sin;
  g.rope_idx = seg_idx;
  g.rope_nseg = n_seg;
  g.rope_T = T;
  g.rope_cols = rope_cols;
  return hb::launch_gemm(g, hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_ln_stats_fp16(const void* x, float* stats, int R, int C, float eps,
                              void* stream) {
  HB_ENTRY_INIT();
  return hb::launch_ln_stats_f16(x, stats, R, C, eps, as_stream(stream));
}

static int matmul_ln(const void* x, const void* w, const float* cols, const float* stats,
                     const float* segtab, const int* seg_idx, int n_seg, void* out, int M,
                     int K, int N, int act, int rope_cols, int T, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || act < 0 || act > 2 || !cols || !stats)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  hb::GemmDesc g{};
  g.A = x;
  g.B = w;
  g.bias = cols;
  g.ln_colsum = cols + N;
  g.ln_stats = stats;
  g.out = out;
  g.batch = 1;
  g.M = M;
  g.K = K;
  g.N = N;
  g.b_shared = true;
  g.act = act;
  if (segtab) {
    if (!seg_idx || n_seg <= 0 || rope_cols <= 0 || T <= 0 || (M % T) != 0)
      return HEXLIB_B200_ERR_INVAL_PARAMS;
    g.rope_cos = segtab;
    g.rope_sin = segtab + 16;
    g.rope_stride = 32;
    g.rope_idx = seg_idx;
    g.rope_nseg = n_seg;
    g.rope_T = T;
    g.rope_cols = rope_cols;
  }
  return hb::launch_gemm(g, hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_matmul_epilogue_ln_fp16(const void* x, const void* w, const float* cols,
                                        const float* stats, void* out, int M, int K, int N,
                                        int act, void* stream) {
  HB_ENTRY_INIT();
  return matmul_ln(x, w, cols, stats, nullptr, nullptr, 0, out, M, K, N, act, 0, 0, stream);
}

int hexlib_b200_matmul_epilogue_ln_rope_fp16(const void* x, const void* w, const float* cols,
                                             const float* stats, const float* segtab,
                                             const int* seg_idx, int n_seg, void* out, int M,
                                             int K, int N, int act, int rope_cols, int T,
                                             void* stream) {
  HB_ENTRY_INIT();
  if (!segtab) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return matmul_ln(x, w, cols, stats, segtab, seg_idx, n_seg, out, M, K, N, act, rope_cols, T,
                   stream);
}

int hexlib_b200_rope_qk_fp16(const void* qkv, const float* costab, const float* sintab,
                             void* out, int rows, int H, int D, int T, void* stream) {
  HB_ENTRY_INIT();
  if (rows < 0 || T <= 0 || !qkv || !out || !costab || !sintab)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_rope_qk_f16(qkv, costab, sintab, out, rows, H, D, T, as_stream(stream));
}

int hexlib_b200_attention_qkv_fp16(const void* qkv, void* ctx, int B, int T, int H, int D,
                                   float scale, void* stream) {
  HB_ENTRY_INIT();
  return hb::launch_attention_qkv(qkv, ctx, B, T, H, D, scale, hb::default_error_word(),
                                  as_stream(stream));
}

int hexlib_b200_attention_fp16(const void* q, const void* k, const void* v,
                               void* ctx, int Bn, int T, int D, float scale,
                               void* stream) {
  HB_ENTRY_INIT();
  if (Bn < 0 || T <= 0 || D <= 0 || (Bn > 0 && (!q || !k || !v || !ctx)))
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  return hb::launch_attention(q, k, v, ctx, Bn, T, D, scale,
                              hb::default_error_word(), as_stream(stream));
}

int hexlib_b200_stream_status(void* stream) {
  if (cudaStreamSynchronize(as_stream(stream)) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  bool noalloc_set = false;
  const int rc = hb::noalloc_take_error(&noalloc_set);
  const bool default_set = hb::take_default_error();
  if (rc != HEXLIB_B200_OK) return rc;
  return (default_set || noalloc_set) ? HEXLIB_B200_ERR_TIMEOUT : HEXLIB_B200_OK;
}

int hexlib_b200_diag_wait_timeout_stream(uint32_t limit_us, void* stream) {
  HB_ENTRY_INIT();
  return hb::launch_wait_timeout_probe(hb::default_error_word(), limit_us, as_stream(stream));
}

}  // extern "C"
