/* include/hexlib_b200.h -- the C ABI of libhexlib_b200.so, the B200 (sm_100a)
 * execution backend for hexlib's plan executor.
 *
 * Two groups of entry points, both plain C: pointers, sizes and an opaque
 * stream handle, no C++ or torch types.
 *
 *  1. THE BATCH PATH. A session owns a CUDA stream and a set of device buffers
 *     registered by `fd` (the analogue of the rpcmem fds the DSP maps), and runs
 *     one hexlib batch blob -- the byte format of hexlib/runtime/wire.py:135-208
 *     and hexlib/runtime/skel/hexlib_dsp.h:109-182, unchanged -- per `invoke`.
 *     The first invoke of a blob validates it on the host, resolves every
 *     (bi, offset) to a device address and captures all of its ops into one CUDA
 *     graph; later invokes of the same blob replay that graph with one launch.
 *     Lifecycle mirrors hexlib/runtime/idl/hexlib_iface.idl:28-67
 *     (open/start -> mmap -> invoke -> munmap -> stop/close).
 *
 *  2. ONE FUNCTION PER KERNEL, with the argument list of that kernel's
 *     kernels/<k>/kernel_api.h plus a trailing `void *stream` (a cudaStream_t,
 *     NULL for the legacy default stream). Every pointer is a DEVICE pointer.
 *     `hexlib_hf *` becomes `void *` (IEEE binary16 storage). The kernel_api.h
 *     functions return void; these return a status, because a kernel that
 *     cannot serve a request must say so (hexlib_dsp.h:197-199).
 *
 * STATUS CODES are hexlib_dsp.h's (:31-54) number for number: OK is 1, so a
 * zero-filled response can never read as success. Codes this backend needs and
 * the DSP did not are APPENDED (16, 17, 18), never renumbered.
 *
 * THREADING. A session is single-threaded and `invoke` is not reentrant, the
 * same contract as hexlib_dispatch_batch (skel_dispatch.c:134-147). Use one
 * session per thread and one process per GPU.
 */
#ifndef HEXLIB_B200_H
#define HEXLIB_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: hexlib/runtime/skel/hexlib_dsp.h:31-54 ---------------- */
#define HEXLIB_B200_OK                 1
#define HEXLIB_B200_ERR_INTERNAL       2
#define HEXLIB_B200_ERR_BAD_MAGIC      3
#define HEXLIB_B200_ERR_BAD_VERSION    4
#define HEXLIB_B200_ERR_TRUNCATED      5
#define HEXLIB_B200_ERR_INVAL_PARAMS   6
#define HEXLIB_B200_ERR_UNMAPPED       7
#define HEXLIB_B200_ERR_NO_MMAP_SLOT   8
#define HEXLIB_B200_ERR_MMAP_FAILED    9
#define HEXLIB_B200_ERR_NO_KERNEL      10
#define HEXLIB_B200_ERR_VTCM_TOO_SMALL 11
#define HEXLIB_B200_ERR_VTCM_RECLAIMED 12
#define HEXLIB_B200_ERR_REQUIRES       13
#define HEXLIB_B200_ERR_NOT_STARTED    14
#define HEXLIB_B200_ERR_CACHE          15
/* Appended for this backend. */
#define HEXLIB_B200_ERR_CUDA           16  /* a CUDA runtime call failed        */
#define HEXLIB_B200_ERR_TIMEOUT        17  /* a device-side bounded wait expired */
#define HEXLIB_B200_ERR_COMM           18  /* a collective failed or a peer left  */

/* ---- wire constants: hexlib/runtime/wire.py:24-31, hexlib_dsp.h:23-30 ---- */
#define HEXLIB_B200_BATCH_MAGIC   0x424C5848u  /* 'HXLB' */
#define HEXLIB_B200_BATCH_VERSION 1u
#define HEXLIB_B200_MAX_BUFS      8
#define HEXLIB_B200_MAX_SRC       6
#define HEXLIB_B200_MAX_DST       4
#define HEXLIB_B200_MAX_PARAMS    16
#define HEXLIB_B200_MAX_TENSORS   512

/* Buffer flag (hexlib_buf_desc.flags, which the reference always writes 0):
 * every tensor in a buffer carrying this flag is PER IMAGE. With n_images = B,
 * such a tensor at per-image offset `o` of `nbytes` bytes occupies the B
 * contiguous copies [B*o, B*o + B*nbytes) of the registered allocation, image
 * b at B*o + b*nbytes -- so each kernel sees one contiguous [B, ...] array and
 * a GEMM folds the images into its M dimension. With B = 1 the blob means
 * exactly what it means to the DSP. */
#define HEXLIB_B200_BUF_PER_IMAGE 1u

/* Kernel ids on the wire: hexlib/runtime/genentry.py:67-88 (1..12 unchanged),
 * then ids appended for kernels the DSP does not have. */
#define HEXLIB_B200_KIND_ADD              1
#define HEXLIB_B200_KIND_CAST             2
#define HEXLIB_B200_KIND_LAYERNORM        3
#define HEXLIB_B200_KIND_MATMUL           4
#define HEXLIB_B200_KIND_MATMUL_EPILOGUE  5
#define HEXLIB_B200_KIND_PATCHIFY         6
#define HEXLIB_B200_KIND_RESHAPE          7
#define HEXLIB_B200_KIND_ROPE_2D          8
#define HEXLIB_B200_KIND_SCALE            9
#define HEXLIB_B200_KIND_SOFTMAX          10
#define HEXLIB_B200_KIND_TRANSPOSE        11  /* perm (1,0,2) */
#define HEXLIB_B200_KIND_TRANSPOSE_HD     12  /* perm (0,2,1) */
#define HEXLIB_B200_KIND_ATTENTION        13  /* scale->QK^T->softmax->PV, fused */
#define HEXLIB_B200_KIND_RMSNORM          14
#define HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL 15 /* act(a@w+b) + r */
#define HEXLIB_B200_KIND_MATMUL_EPILOGUE_ROPE 16 /* act(a@w+b), RoPE on heads */
#define HEXLIB_B200_KIND_ATTENTION_QKV    17  /* attention over packed q|k|v */
#define HEXLIB_B200_KIND_ROPE_QK          18  /* rope_2d of the q, k sections */
#define HEXLIB_B200_KIND_LN_STATS         19  /* layernorm's (mean, rstd) per row */
#define HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN 20 /* act(layernorm(x) @ w + b), folded */
#define HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN_ROPE 21 /* the same, RoPE on heads */
#define HEXLIB_B200_KIND_PATCHIFY_CAST    22  /* patchify, then cast to fp16 */

/* Invoke modes. */
#define HEXLIB_B200_MODE_GRAPH   0u  /* capture once per blob, replay one graph  */
#define HEXLIB_B200_MODE_EAGER   1u  /* launch op by op, time each with events   */

#if defined(__GNUC__)
#define HEXLIB_B200_API __attribute__((visibility("default")))
#else
#define HEXLIB_B200_API
#endif

typedef struct hexlib_b200_ctx hexlib_b200_ctx;

/* ---- session: hexlib_iface.idl open/start (:32-35) and stop/close ------- */

/* Open a session on CUDA device `device`: create its stream, load every
 * kernel, and set their shared-memory limits, so nothing is loaded lazily
 * inside a graph capture. */
HEXLIB_B200_API int hexlib_b200_open(int device, hexlib_b200_ctx **out);
/* Free every mapped buffer and cached graph, destroy the stream. */
HEXLIB_B200_API int hexlib_b200_close(hexlib_b200_ctx *ctx);

/* hexlib_iface.idl hwinfo (:59-60). Unlike the DSP's, every value is queried:
 * arch is the device's compute capability as major*10+minor (100 on B200). */
HEXLIB_B200_API int hexlib_b200_hwinfo(hexlib_b200_ctx *ctx, uint32_t *arch,
                       uint32_t *sm_count, uint64_t *hbm_bytes,
                       uint64_t *mapped_bytes);

/* ---- buffers: hexlib_iface.idl mmap/munmap (:41-42) ---------------------- */

/* Register buffer `fd` with `size` bytes, backed by one device allocation of
 * size * replicas bytes (replicas >= 1; a per-image buffer needs one replica
 * per image a later invoke names). Re-registering an fd is an error. */
HEXLIB_B200_API int hexlib_b200_mmap(hexlib_b200_ctx *ctx, uint32_t fd, uint64_t size,
                     uint32_t replicas);
HEXLIB_B200_API int hexlib_b200_munmap(hexlib_b200_ctx *ctx, uint32_t fd);
/* Host <-> device copies into a registered buffer at a BYTE offset of its
 * allocation, ordered on the session stream and complete on return. */
HEXLIB_B200_API int hexlib_b200_buf_write(hexlib_b200_ctx *ctx, uint32_t fd, uint64_t offset,
                          const void *src, uint64_t nbytes);
HEXLIB_B200_API int hexlib_b200_buf_read(hexlib_b200_ctx *ctx, uint32_t fd, uint64_t offset,
                         void *dst, uint64_t nbytes);
/* The same copies, returning once they are enqueued on the session stream
 * (no reference counterpart: the reference's buffers are host-mapped memory
 * the DSP reads in place, so its writes need no copy at all). Ordered with
 * the session's invokes; `src`/`dst` must stay valid and unmodified until a
 * later hexlib_b200_sync() returns, and must be page-locked (cudaHostAlloc /
 * cudaHostRegister) for the copy to overlap kernels of another stream. */
HEXLIB_B200_API int hexlib_b200_buf_write_async(hexlib_b200_ctx *ctx, uint32_t fd,
                                                uint64_t offset, const void *src,
                                                uint64_t nbytes);
HEXLIB_B200_API int hexlib_b200_buf_read_async(hexlib_b200_ctx *ctx, uint32_t fd,
                                               uint64_t offset, void *dst, uint64_t nbytes);
/* The device address of a buffer, for callers that hand it to NCCL/torch. */
HEXLIB_B200_API int hexlib_b200_buf_device_ptr(hexlib_b200_ctx *ctx, uint32_t fd,
                               uint64_t *ptr, uint64_t *alloc_bytes);
/* The session's CUDA stream (a cudaStream_t). */
HEXLIB_B200_API int hexlib_b200_stream(hexlib_b200_ctx *ctx, void **stream);

/* ---- batch: hexlib_iface.idl invoke (:64-66) -> skel_dispatch.c:80 ------- */

/* Run one batch blob on one image. Same response layout as the DSP:
 * hexlib_batch_rsp_hdr then one hexlib_op_result per op that was reached.
 * `cycles_total` and `results[i].cycles` carry NANOSECONDS of device time
 * (CUDA events); per-op times are filled only in HEXLIB_B200_MODE_EAGER. */
HEXLIB_B200_API int hexlib_b200_invoke(hexlib_b200_ctx *ctx, const uint8_t *batch,
                       uint32_t len, uint8_t *rsp, uint32_t rsp_cap,
                       uint32_t *rsp_len);
/* The same for `n_images` images (see HEXLIB_B200_BUF_PER_IMAGE), in `mode`.
 * If `sync` is 0 the call returns after enqueueing the work on the session
 * stream (graph mode only); the response then reports only host validation
 * and a later hexlib_b200_sync() reports device-side status. */
HEXLIB_B200_API int hexlib_b200_invoke_images(hexlib_b200_ctx *ctx, const uint8_t *batch,
                              uint32_t len, uint32_t n_images, uint32_t mode,
                              uint32_t sync, uint8_t *rsp, uint32_t rsp_cap,
                              uint32_t *rsp_len);
/* Wait for the session stream; OK, ERR_CUDA or ERR_TIMEOUT. */
HEXLIB_B200_API int hexlib_b200_sync(hexlib_b200_ctx *ctx);

/* Host-only validation of a blob against buffer sizes, with no device and no
 * session: the same checks invoke runs before its first launch, answered in
 * the same response layout (each reached op OK or its error). buf_sizes[i] is
 * the registered size of wire buffer i (in blob order). */
HEXLIB_B200_API int hexlib_b200_check_batch(const uint8_t *batch, uint32_t len,
                            const uint64_t *buf_sizes, uint32_t n_sizes,
                            uint32_t n_images, uint8_t *rsp, uint32_t rsp_cap,
                            uint32_t *rsp_len);

/* Failure-path diagnostic: launch, on the session stream, a kernel whose
 * bounded mbarrier wait is never satisfied; after `limit_us` (1..1e6) it
 * records a timeout and returns. Answers HEXLIB_B200_ERR_TIMEOUT and leaves
 * the session usable -- the same path a lost arrival in any pipelined kernel
 * of this library takes. */
HEXLIB_B200_API int hexlib_b200_diag_wait_timeout(hexlib_b200_ctx *ctx,
                                                  uint32_t limit_us);

/* The per-kernel entry points below return as soon as their work is queued,
 * so a device-side failure cannot be their return value. This waits for
 * `stream` and reports, then clears, what the kernels launched through them
 * recorded since the previous call: HEXLIB_B200_ERR_TIMEOUT if a bounded
 * wait inside one expired (its output is not valid), ERR_CUDA if the stream
 * reported an error, OK otherwise. The record is per process (per device for
 * hexlib_b200_matmul_epilogue_q4_0_noalloc), not per stream. No counterpart
 * in the reference, whose kernel calls are synchronous (skel_dispatch.c:
 * 248-262). */
HEXLIB_B200_API int hexlib_b200_stream_status(void *stream);

/* Failure-path diagnostic for the per-kernel entries: queue on `stream` the
 * kernel of hexlib_b200_diag_wait_timeout, recording into the per-kernel
 * entries' error word; hexlib_b200_stream_status then answers ERR_TIMEOUT. */
HEXLIB_B200_API int hexlib_b200_diag_wait_timeout_stream(uint32_t limit_us, void *stream);

/* The status as text (hexlib_dsp.h:71-91). */
HEXLIB_B200_API const char *hexlib_b200_status_name(int status);

/* ---- kernels: kernels/<k>/kernel_api.h + trailing stream ----------------- */

/* kernels/add_fp16/kernel_api.h:35 */
HEXLIB_B200_API int hexlib_b200_add_fp16(const void *a, const void *b, void *y, int n,
                         void *stream);
/* add with an fp32 right operand, rounded once: the pos_embed add of
 * hexlib/models/vit.py:159-160 exactly as the numpy executor computes it. */
HEXLIB_B200_API int hexlib_b200_add_fp16_f32(const void *a, const float *b, void *y, int n,
                             void *stream);
/* kernels/cast_f32_f16/kernel_api.h:33 */
HEXLIB_B200_API int hexlib_b200_cast_f32_f16(const float *x, void *y, int n, void *stream);
/* kernels/scale_fp16/kernel_api.h:37 */
HEXLIB_B200_API int hexlib_b200_scale_fp16(const void *x, void *y, int n, float factor,
                           void *stream);
/* kernels/layernorm_fp16/kernel_api.h:38-39 */
HEXLIB_B200_API int hexlib_b200_layernorm_fp16(const void *x, const float *w, const float *b,
                               void *y, int R, int C, float eps, void *stream);
/* kernels/rmsnorm_fp16/kernel_api.h:26-27 */
HEXLIB_B200_API int hexlib_b200_rmsnorm_fp16(const void *x, const void *w, void *y, int R,
                             int C, float eps, void *stream);
/* kernels/softmax_fp16/kernel_api.h:69 */
HEXLIB_B200_API int hexlib_b200_softmax_fp16(const void *x, void *y, int R, int C,
                             void *stream);
/* kernels/rope_2d_fp16/kernel_api.h:120-121 */
HEXLIB_B200_API int hexlib_b200_rope_2d_fp16(const void *x, const float *costab,
                             const float *sintab, void *y, int T, int H, int D,
                             void *stream);
/* kernels/transpose_th_fp16/kernel_api.h:38 */
HEXLIB_B200_API int hexlib_b200_transpose_th_fp16(const void *x, void *y, int T, int H, int D,
                                  void *stream);
/* kernels/transpose_hd_fp16/kernel_api.h:67 */
HEXLIB_B200_API int hexlib_b200_transpose_hd_fp16(const void *x, void *y, int B, int T, int D,
                                  void *stream);
/* kernels/patchify_fp32/kernel_api.h:116-118 */
HEXLIB_B200_API int hexlib_b200_patchify_fp32(const float *img, float *out, int C, int T,
                              int H, int W, int patch, int merge, int grid_h,
                              int grid_w, void *stream);
/* patchify followed by the cast of its rows to fp16, in one pass: the
 * arguments of hexlib_b200_patchify_fp32, an fp16 output (8-byte aligned);
 * each value rounded to nearest even exactly as the cast rounds it. patch
 * must be a multiple of 4 and img 16-byte aligned. */
HEXLIB_B200_API int hexlib_b200_patchify_fp16(const float *img, void *out, int C, int T,
                                              int H, int W, int patch, int merge,
                                              int grid_h, int grid_w, void *stream);
/* kernels/matmul_fp16/kernel_api.h:77-78 */
HEXLIB_B200_API int hexlib_b200_matmul_fp16(const void *A, const void *B, void *C, int Bn,
                            int M, int K, int N, void *stream);
/* kernels/matmul_epilogue_fp16/kernel_api.h:188-190, with an fp16 [K, N]
 * row-major weight in place of the q4_0 one; act is MM_ACT_* (0 none,
 * 1 gelu_tanh, 2 gelu_erf, kernel_api.h:181-183). */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_fp16(const void *a, const void *w,
                                     const float *bias, void *out, int M,
                                     int K, int N, int act, void *stream);
/* The reference's own matmul_epilogue (kernels/matmul_epilogue_fp16/
 * kernel_api.h:188-190): w is a q4_0 [K, N] weight, row-major with its
 * 18-byte blocks of 32 along N (K any, N % 32 == 0), dequantized with every
 * weight rounded to fp16 (baseline.c:36-47), fp32 accumulation. The kernel
 * never allocates: the caller hands `workspace` of at least K*N*2 bytes
 * (16-byte aligned) for the fp16 copy of the weight -- the counterpart of the
 * VTCM scratch the reference's entry receives in hexlib_args (vtcm,
 * vtcm_size; hexlib_dsp.h:186-198). ERR_INVAL_PARAMS when it is too small. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_q4_0(const void *a, const void *w,
                                                     const float *bias, void *out, int M,
                                                     int K, int N, int act, void *workspace,
                                                     uint64_t workspace_bytes, void *stream);
/* The same with a q8_0 weight (34-byte blocks: fp16 d, 32 int8; value q*d;
 * hexlib/exec/quant.py, ir.py:26-41). No reference kernel takes q8_0 yet;
 * the contract is q4_0's with the other block format. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_q8_0(const void *a, const void *w,
                                                     const float *bias, void *out, int M,
                                                     int K, int N, int act, void *workspace,
                                                     uint64_t workspace_bytes, void *stream);
/* The q4_0 matmul_epilogue above without a workspace argument and without
 * allocating: its scratch is a fixed 8 MiB device array of the library, so
 * K * N <= 4 Mi (ERR_VTCM_TOO_SMALL otherwise). No counterpart in the
 * reference, whose kernels always receive a scratch from their caller. Calls
 * that overlap in time share that scratch and race; issue them in order (one
 * stream). The first call on a device looks the array up with that device
 * current; make it before any stream capture begins. A bounded wait that
 * expires inside it is reported by hexlib_b200_stream_status. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_q4_0_noalloc(const void *a, const void *w,
                                                             const float *bias, void *out,
                                                             int M, int K, int N, int act,
                                                             void *stream);
/* q4_0 / q8_0 [K, N] -> fp16 [K, N] with the rounding above (w 2-byte
 * aligned, out 16-byte aligned): the dequantization step alone. */
HEXLIB_B200_API int hexlib_b200_dequant_q4_0_fp16(const void *w, void *out, int K, int N,
                                                  void *stream);
HEXLIB_B200_API int hexlib_b200_dequant_q8_0_fp16(const void *w, void *out, int K, int N,
                                                  void *stream);
/* matmul_epilogue followed by the residual add that consumes it
 * (hexlib/models/vit.py:196 and :203): out = act(a@w + bias) + r, with the
 * matmul result rounded to fp16 before the add, as the unfused plan does. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_residual_fp16(const void *a, const void *w,
                                              const float *bias,
                                              const void *r, void *out, int M,
                                              int K, int N, int act,
                                              void *stream);
/* matmul_epilogue whose first `rope_cols` output columns are 64-wide heads
 * rotated by the split-half 2-D RoPE of kernels/rope_2d_fp16/kernel_api.h,
 * applied after the fp16 rounding exactly as rope_2d applies it to a stored
 * q or k. The [T, 64] cos/sin tables must be half-symmetric (dims i and
 * i + 32 share a value, as in every rotate-half table built from one list of
 * frequencies) and come in 16-wide segments: dims [16s, 16s + 16) and
 * [32 + 16s, 48 + 16s) of token t (row r's token is r % T) are row
 * seg_idx[2t + s] of the [n_seg, 16] fp32 tables seg_cos / seg_sin (indices
 * clamped to [0, n_seg)); a 2-D RoPE table deduplicates to a few KiB this
 * way, small enough to stay in L1 while every head reads it. With
 * w = [wq | wk | wv] it is a block's whole q/k/v projection and RoPE
 * (hexlib/models/vit.py:168-180) in one GEMM. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_rope_fp16(
    const void *a, const void *w, const float *bias, const float *seg_cos,
    const float *seg_sin, const int *seg_idx, int n_seg, void *out, int M, int K, int N,
    int act, int rope_cols, int T, void *stream);
/* rope_2d (kernels/rope_2d_fp16/kernel_api.h:120-121) applied to the q and
 * k sections of a packed [rows, 3, H, D] projection, token of row r = r % T
 * of the [T, D] tables; the v section is left as it is. out may equal qkv
 * (in place). */
HEXLIB_B200_API int hexlib_b200_rope_qk_fp16(const void *qkv, const float *costab,
                                             const float *sintab, void *out, int rows,
                                             int H, int D, int T, void *stream);
/* layernorm (kernels/layernorm_fp16/kernel_api.h) without its output: the
 * (mean, 1/sqrt(var + eps)) of each of R rows of C fp16, as R float pairs
 * (stats 8-byte aligned), computed exactly as hexlib_b200_layernorm_fp16
 * computes them. */
HEXLIB_B200_API int hexlib_b200_ln_stats_fp16(const void *x, float *stats, int R, int C,
                                              float eps, void *stream);
/* act(layernorm(x) @ W + b) without materialising layernorm(x): x [M, K] raw
 * rows, w = diag(gamma) W [K, N] fp16 (the layernorm weight folded into the
 * matrix), cols [2, N] fp32 = (beta @ W + b; the column sums of w), stats
 * [M, 2] from hexlib_b200_ln_stats_fp16. The epilogue forms
 * act(rstd * (x @ w - mean * colsum) + bias). N must be a multiple of 256;
 * act: 0 none, 1 gelu_tanh, 2 gelu_erf. */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_ln_fp16(const void *x, const void *w,
                                                        const float *cols, const float *stats,
                                                        void *out, int M, int K, int N,
                                                        int act, void *stream);
/* The same with the RoPE epilogue of hexlib_b200_matmul_epilogue_rope_fp16;
 * the cos and sin segment tables interleaved as one [n_seg, 2, 16] table
 * (segment s: 16 cos values, then 16 sin values). */
HEXLIB_B200_API int hexlib_b200_matmul_epilogue_ln_rope_fp16(
    const void *x, const void *w, const float *cols, const float *stats, const float *segtab,
    const int *seg_idx, int n_seg, void *out, int M, int K, int N, int act, int rope_cols,
    int T, void *stream);
/* Fused attention over a packed projection: qkv [B, T, 3, H, D] (the output
 * of the call above), ctx [B, T, H, D] -- the layout the o-projection reads,
 * so none of the block's four transposes is needed. D must be 64. */
HEXLIB_B200_API int hexlib_b200_attention_qkv_fp16(const void *qkv, void *ctx,
                                                   int B, int T, int H, int D,
                                                   float scale, void *stream);
/* Fused attention over Bn independent heads, q/k/v/ctx [Bn, T, D] fp16:
 * ctx = softmax((q*scale) @ k^T) @ v, the chain hexlib/models/vit.py:183-190
 * writes as five ops, without materialising the [Bn, T, T] scores. */
HEXLIB_B200_API int hexlib_b200_attention_fp16(const void *q, const void *k, const void *v,
                               void *ctx, int Bn, int T, int D, float scale,
                               void *stream);

/* ---- the embedding gather across GPUs (NCCL, with deadlines) --------------
 * The image-sharded encoder's one exchange: an all-gather of every rank's fp16
 * embeddings. No counterpart in the reference, which runs one image at a time
 * on one DSP (skel_dispatch.c:248); the session lifecycle mirrors
 * hexlib_iface.idl:28-67 (open -> work -> close) and, like every entry here,
 * fails by default rather than hang: every wait has a deadline, after which
 * the communicator is aborted and the call answers ERR_TIMEOUT (a peer that
 * stopped answering) or ERR_COMM (NCCL reported an error, e.g. a peer that
 * left). An aborted communicator answers ERR_COMM to any further work;
 * close it and open a new one. NCCL is loaded at run time. */
#define HEXLIB_B200_NCCL_ID_BYTES 128
typedef struct hexlib_b200_comm hexlib_b200_comm;

/* 1 when NCCL could be loaded, else 0. */
HEXLIB_B200_API int hexlib_b200_nccl_available(void);
/* Rank 0's rendezvous id (128 bytes), to be shared with every rank. */
HEXLIB_B200_API int hexlib_b200_nccl_unique_id(uint8_t *id_out);
/* Join the communicator `id` as `rank` of `nranks` on CUDA device `device`,
 * non-blocking, waiting at most timeout_ms for every rank to join. This and
 * the calls below on the communicator make `device` the calling thread's
 * current CUDA device and leave it so (one process per GPU is the use they
 * serve, where it already is). */
HEXLIB_B200_API int hexlib_b200_nccl_open(const uint8_t *id, int nranks, int rank,
                                          int device, uint32_t timeout_ms,
                                          hexlib_b200_comm **out);
/* Enqueue on `stream` the all-gather of `count` fp16 values from every rank:
 * recv holds nranks * count values in rank order. Returns once NCCL has
 * enqueued it (at most timeout_ms); completion is hexlib_b200_nccl_wait's. */
HEXLIB_B200_API int hexlib_b200_nccl_allgather_f16(hexlib_b200_comm *comm, const void *send,
                                                   void *recv, uint64_t count, void *stream,
                                                   uint32_t timeout_ms);
/* Wait at most timeout_ms for `stream` (and the gathers on it) to drain. */
HEXLIB_B200_API int hexlib_b200_nccl_wait(hexlib_b200_comm *comm, void *stream,
                                          uint32_t timeout_ms);
/* Abort the communicator now (its kernels return; later calls answer ERR_COMM). */
HEXLIB_B200_API int hexlib_b200_nccl_abort(hexlib_b200_comm *comm);
/* Finalize (at most timeout_ms; 0 means 10 s) and free the communicator. */
HEXLIB_B200_API int hexlib_b200_nccl_close(hexlib_b200_comm *comm, uint32_t timeout_ms);

#ifdef __cplusplus
}
#endif

#endif /* HEXLIB_B200_H */
