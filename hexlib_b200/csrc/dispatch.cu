// dispatch.cu -- the batch path: session, fd-registered device buffers, and
// `invoke`, which validates one hexlib batch blob on the host and runs its ops
// as one CUDA graph.
//
// What hexlib_dispatch_batch (hexlib/runtime/skel/skel_dispatch.c:80-302)
// does per invoke on the DSP -- validate the header and every section in
// 64-bit arithmetic, map buffers, resolve tensors, look up each op's kernel,
// fill its arguments src-then-dst, run it, stop at the first failure -- this
// does ONCE per distinct blob on the host; the per-op argument guards of the
// generated entries (hexlib/runtime/genentry.py:159-219, 280-348: buffer count,
// null, dtype, layout) are applied at the same time, together with shape
// checks the DSP never needed (element counts against byte counts), because a
// kernel reading past a tensor here is a GPU fault rather than a wrong number.
// The validated op list is captured into a CUDA graph keyed by the blob bytes
// and the image count; every later invoke of that blob is one graph launch.
//
// The response is the DSP's byte for byte (hexlib_dsp.h:160-182): the header
// is written first as ERR_INTERNAL, each reached op gets its kind echoed and
// a status, and the batch status is the first failure or OK. `cycles` fields
// carry nanoseconds of device time measured with CUDA events.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/hexlib_b200.h"
#include "hb_kernels.h"

namespace hb {
namespace {
thread_local int t_walk = 0;
bool walk_alternates() {
#ifdef HEXLIB_B200_MEASUREMENT_KNOBS
  // Measurement builds only: HEXLIB_B200_WALK_ORDER=ascending keeps every
  // launch walking its work in ascending order.
  static const bool alt = [] {
    const char* e = getenv("HEXLIB_B200_WALK_ORDER");
    return !(e && strcmp(e, "ascending") == 0);
  }();
  return alt;
#else
  return true;
#endif
}
}  // namespace

int order_next() {
  if (!walk_alternates()) return 0;
  const int o = t_walk;
  t_walk ^= 1;
  return o;
}

void order_reset() { t_walk = 0; }
}  // namespace hb

namespace {

// ---- wire structs: hexlib/runtime/skel/hexlib_dsp.h:109-182 -----------------
#pragma pack(push, 1)
struct WireHdr {
  uint32_t magic, version, total_size, n_bufs, n_tensors, n_ops, off_bufs,
      off_tensors, off_ops, flags;
};
struct WireBuf {
  uint64_t base, size;
  uint32_t fd, flags;
};
struct WireTensor {
  uint32_t bi, offset, nbytes, dtype, layout, ne[4], data, pad;
};
struct WireOp {
  uint32_t kind, flags;
  int32_t params[HEXLIB_B200_MAX_PARAMS];
  uint16_t src[HEXLIB_B200_MAX_SRC];
  uint16_t dst[HEXLIB_B200_MAX_DST];
};
struct WireRspHdr {
  uint32_t magic, version, status, n_ops;
  uint64_t cycles_total;
  uint32_t arch, pad;
};
struct WireResult {
  uint32_t kind, status;
  uint64_t cycles;
};
#pragma pack(pop)
static_assert(sizeof(WireHdr) == 40, "hexlib_batch_hdr is 40 bytes");
static_assert(sizeof(WireBuf) == 24, "hexlib_buf_desc is 24 bytes");
static_assert(sizeof(WireTensor) == 44, "hexlib_tensor is 44 bytes");
static_assert(sizeof(WireOp) == 92, "hexlib_op_desc is 92 bytes");
static_assert(sizeof(WireRspHdr) == 32, "hexlib_batch_rsp_hdr is 32 bytes");
static_assert(sizeof(WireResult) == 16, "hexlib_op_result is 16 bytes");

// DTYPE_ID / LAYOUT_ID, hexlib/runtime/wire.py:56-57.
enum : uint32_t { DT_FP32 = 0, DT_FP16 = 1, DT_Q4_0 = 2, DT_INT32 = 3, DT_Q8_0 = 4 };
enum : uint32_t { LAYOUT_ROW_MAJOR = 0 };

constexpr uint32_t kArch = 100;

// One resolved buffer argument of an op.
struct Arg {
  void* ptr;          // device address of image 0's copy (or the only copy)
  uint32_t ne[4];
  uint32_t dtype, layout;
  uint64_t nbytes;    // per image
  bool per_image;
};

struct OpRec {
  uint32_t kind;
  uint32_t nbuf;
  Arg a[HEXLIB_B200_MAX_BUFS];
  int32_t params[HEXLIB_B200_MAX_PARAMS];
};

// Buffer as the validator sees it.
struct BufView {
  char* base;         // nullptr in host-only checking
  uint64_t alloc;     // bytes actually backing it
  uint64_t size;      // size declared on the wire
  bool per_image;
};

uint64_t numel(const uint32_t ne[4]) {
  return (uint64_t)ne[0] * ne[1] * ne[2] * ne[3];
}

int esize(uint32_t dt) {
  switch (dt) {
    case DT_FP32: return 4;
    case DT_FP16: return 2;
    case DT_INT32: return 4;
    default: return 0;
  }
}

float param_f(const OpRec& op, int i) {
  float f;
  memcpy(&f, &op.params[i], 4);
  return f;
}

// ---- per-kind argument contract -----------------------------------------------
// Each returns OK or the status the generated DSP entry would give (n_buf
// mismatch -> INVAL_PARAMS, wrong dtype/layout -> REQUIRES), plus
// INVAL_PARAMS for shapes that disagree with their byte counts.

int need(const OpRec& op, uint32_t nbuf) {
  if (op.nbuf != nbuf) return HEXLIB_B200_ERR_INVAL_PARAMS;
  for (uint32_t i = 0; i < nbuf; ++i) {
    if (op.a[i].layout != LAYOUT_ROW_MAJOR) return HEXLIB_B200_ERR_REQUIRES;
    const int es = esize(op.a[i].dtype);
    if (es == 0) {
      // q4_0 / q8_0: blocks of 32 along the last axis (ir.py nbytes)
      const int bb = hb::quant_block_bytes((int)op.a[i].dtype);
      if (bb == 0) return HEXLIB_B200_ERR_REQUIRES;
      const uint64_t n = numel(op.a[i].ne);
      if (n % 32 || (n / 32) * (uint64_t)bb != op.a[i].nbytes)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      continue;
    }
    if (numel(op.a[i].ne) * (uint64_t)es != op.a[i].nbytes)
      return HEXLIB_B200_ERR_INVAL_PARAMS;
  }
  return HEXLIB_B200_OK;
}

int dt(const OpRec& op, uint32_t i, uint32_t want) {
  return op.a[i].dtype == want ? HEXLIB_B200_OK : HEXLIB_B200_ERR_REQUIRES;
}

#define HB_TRY(x)                         \
  do {                                    \
    const int _r = (x);                   \
    if (_r != HEXLIB_B200_OK) return _r;  \
  } while (0)

// Output batched iff some input is; shared inputs must not be written per
// image and per-image outputs need a per-image source.
int batching(const OpRec& op, uint32_t n_in) {
  bool any = false;
  for (uint32_t i = 0; i < n_in; ++i) any = any || op.a[i].per_image;
  for (uint32_t i = n_in; i < op.nbuf; ++i)
    if (op.a[i].per_image != any) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return HEXLIB_B200_OK;
}

int check_op(const OpRec& op) {
  switch (op.kind) {
    case HEXLIB_B200_KIND_ADD: {
      HB_TRY(need(op, 3));
      HB_TRY(dt(op, 0, DT_FP16));
      if (op.a[1].dtype != DT_FP16 && op.a[1].dtype != DT_FP32)
        return HEXLIB_B200_ERR_REQUIRES;
      HB_TRY(dt(op, 2, DT_FP16));
      HB_TRY(batching(op, 2));
      if (numel(op.a[1].ne) != numel(op.a[0].ne) ||
          numel(op.a[2].ne) != numel(op.a[0].ne))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      // A shared left operand with a per-image right one is served by
      // commuting, which only the fp16 + fp16 kernel can do.
      if (!op.a[0].per_image && op.a[1].per_image && op.a[1].dtype != DT_FP16)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_CAST:
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP32));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      return numel(op.a[0].ne) == numel(op.a[1].ne)
                 ? HEXLIB_B200_OK
                 : HEXLIB_B200_ERR_INVAL_PARAMS;
    case HEXLIB_B200_KIND_SCALE:
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      return numel(op.a[0].ne) == numel(op.a[1].ne)
                 ? HEXLIB_B200_OK
                 : HEXLIB_B200_ERR_INVAL_PARAMS;
    case HEXLIB_B200_KIND_LAYERNORM: {
      HB_TRY(need(op, 4));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP32));
      HB_TRY(dt(op, 2, DT_FP32));
      HB_TRY(dt(op, 3, DT_FP16));
      HB_TRY(batching(op, 3));
      const uint32_t* x = op.a[0].ne;  // R = dim:0:0, C = dim:0:1
      if (x[2] != 1 || x[3] != 1 || x[1] == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (numel(op.a[1].ne) != x[1] || numel(op.a[2].ne) != x[1] ||
          op.a[1].per_image || op.a[2].per_image ||
          numel(op.a[3].ne) != numel(x))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_RMSNORM: {
      HB_TRY(need(op, 3));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(dt(op, 2, DT_FP16));
      HB_TRY(batching(op, 2));
      const uint32_t* x = op.a[0].ne;
      if (x[2] != 1 || x[3] != 1 || x[1] == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (numel(op.a[1].ne) != x[1] || op.a[1].per_image ||
          numel(op.a[2].ne) != numel(x))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_SOFTMAX: {
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      // rows:0:2 and dim:0:2 (runner.py SPECS["softmax"]): C is axis 2.
      if (op.a[0].ne[2] == 0 || numel(op.a[1].ne) != numel(op.a[0].ne))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_ROPE_2D: {
      HB_TRY(need(op, 4));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP32));
      HB_TRY(dt(op, 2, DT_FP32));
      HB_TRY(dt(op, 3, DT_FP16));
      HB_TRY(batching(op, 3));
      const uint32_t* x = op.a[0].ne;  // T, H, D
      if (x[3] != 1 || x[2] == 0 || (x[2] & 1)) return HEXLIB_B200_ERR_INVAL_PARAMS;
      const uint64_t tab = (uint64_t)x[0] * x[2];
      if (numel(op.a[1].ne) != tab || numel(op.a[2].ne) != tab ||
          op.a[1].per_image || op.a[2].per_image ||
          numel(op.a[3].ne) != numel(x))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_TRANSPOSE: {
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      const uint32_t* x = op.a[0].ne;
      const uint32_t* y = op.a[1].ne;
      if (x[3] != 1 || y[0] != x[1] || y[1] != x[0] || y[2] != x[2] || y[3] != 1 ||
          numel(x) == 0)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_TRANSPOSE_HD: {
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      const uint32_t* x = op.a[0].ne;
      const uint32_t* y = op.a[1].ne;
      if (x[3] != 1 || y[0] != x[0] || y[1] != x[2] || y[2] != x[1] || y[3] != 1 ||
          numel(x) == 0)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_PATCHIFY:
    case HEXLIB_B200_KIND_PATCHIFY_CAST: {
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP32));
      HB_TRY(dt(op, 1, op.kind == HEXLIB_B200_KIND_PATCHIFY ? DT_FP32 : DT_FP16));
      HB_TRY(batching(op, 1));
      const uint32_t* x = op.a[0].ne;  // C, T, H, W
      const int64_t patch = op.params[0], merge = op.params[1];
      const int64_t gh = op.params[2], gw = op.params[3];
      if (patch <= 0 || merge <= 0 || gh <= 0 || gw <= 0 ||
          gh * patch != (int64_t)x[2] || gw * patch != (int64_t)x[3] ||
          gh % merge || gw % merge)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      const uint64_t want = (uint64_t)gh * gw * x[0] * x[1] * patch * patch;
      if (numel(op.a[1].ne) != want) return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_RESHAPE: {
      HB_TRY(need(op, 2));
      HB_TRY(batching(op, 1));
      if (op.a[0].dtype != op.a[1].dtype || op.a[0].nbytes != op.a[1].nbytes)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_MATMUL: {
      HB_TRY(need(op, 3));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(dt(op, 2, DT_FP16));
      HB_TRY(batching(op, 2));
      // Bn = dim:0:0, M = dim:0:1, K = dim:0:2, N = dim:1:2.
      const uint32_t* a = op.a[0].ne;
      const uint32_t* b = op.a[1].ne;
      if (a[3] != 1 || b[3] != 1 || b[0] != a[0] || b[1] != a[2] || a[2] == 0 ||
          b[2] == 0 || numel(op.a[2].ne) != (uint64_t)a[0] * a[1] * b[2])
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (!op.a[0].per_image && op.a[1].per_image) return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (op.a[0].per_image && !op.a[1].per_image && a[0] != 1)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE:
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL: {
      const bool res = op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL;
      const uint32_t nb = res ? 5 : 4;
      HB_TRY(need(op, nb));
      HB_TRY(dt(op, 0, DT_FP16));
      // the weight: fp16, or the reference's q4_0 (or q8_0), blocks along N
      const uint32_t wdt = op.a[1].dtype;
      if (wdt != DT_FP16 && wdt != DT_Q4_0 && wdt != DT_Q8_0) return HEXLIB_B200_ERR_REQUIRES;
      if (wdt != DT_FP16 && op.a[1].ne[1] % 32) return HEXLIB_B200_ERR_INVAL_PARAMS;
      HB_TRY(dt(op, 2, DT_FP32));
      if (res) HB_TRY(dt(op, 3, DT_FP16));
      HB_TRY(dt(op, nb - 1, DT_FP16));
      HB_TRY(batching(op, nb - 1));
      // M = dim:0:0, K = dim:0:1, N = dim:1:1.
      const uint32_t* a = op.a[0].ne;
      const uint32_t* w = op.a[1].ne;
      if (a[2] != 1 || a[3] != 1 || w[2] != 1 || w[3] != 1 || w[0] != a[1] ||
          a[1] == 0 || w[1] == 0 || numel(op.a[2].ne) != w[1] ||
          op.a[1].per_image || op.a[2].per_image ||
          numel(op.a[nb - 1].ne) != (uint64_t)a[0] * w[1])
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (res && (numel(op.a[3].ne) != (uint64_t)a[0] * w[1] ||
                  op.a[3].per_image != op.a[0].per_image))
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (op.params[0] < 0 || op.params[0] > 2) return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_ROPE: {
      // a, w, bias, seg_cos [n, 16], seg_sin [n, 16], seg_idx [T, 2] int32, out
      HB_TRY(need(op, 7));
      HB_TRY(dt(op, 0, DT_FP16));
      {
        // the weight: fp16, or q4_0 / q8_0 (blocks along N)
        const uint32_t wdt = op.a[1].dtype;
        if (wdt != DT_FP16 && wdt != DT_Q4_0 && wdt != DT_Q8_0) return HEXLIB_B200_ERR_REQUIRES;
        if (wdt != DT_FP16 && op.a[1].ne[1] % 32) return HEXLIB_B200_ERR_INVAL_PARAMS;
      }
      HB_TRY(dt(op, 2, DT_FP32));
      HB_TRY(dt(op, 3, DT_FP32));
      HB_TRY(dt(op, 4, DT_FP32));
      HB_TRY(dt(op, 5, DT_INT32));
      HB_TRY(dt(op, 6, DT_FP16));
      HB_TRY(batching(op, 6));
      const uint32_t* a = op.a[0].ne;   // M, K
      const uint32_t* w = op.a[1].ne;   // K, N
      const uint32_t* c = op.a[3].ne;   // n_seg, 16
      const uint32_t* x = op.a[5].ne;   // T, 2
      if (a[2] != 1 || a[3] != 1 || w[2] != 1 || w[3] != 1 || w[0] != a[1] || a[1] == 0 ||
          w[1] == 0 || numel(op.a[2].ne) != w[1] || op.a[1].per_image ||
          op.a[2].per_image || op.a[3].per_image || op.a[4].per_image || op.a[5].per_image ||
          memcmp(op.a[3].ne, op.a[4].ne, sizeof(uint32_t) * 4) != 0 || c[0] == 0 ||
          c[1] != 16 || c[2] != 1 || c[3] != 1 || x[0] == 0 || x[1] != 2 || x[2] != 1 ||
          x[3] != 1 || a[0] % x[0] != 0 || numel(op.a[6].ne) != (uint64_t)a[0] * w[1])
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (op.params[0] < 0 || op.params[0] > 2 || op.params[1] <= 0 || op.params[1] % 64 ||
          (uint32_t)op.params[1] > w[1] || w[1] % 64)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_LN_STATS: {
      // x [R, C] fp16 -> stats [R, 2] fp32; params: eps
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP32));
      HB_TRY(batching(op, 1));
      const uint32_t* x = op.a[0].ne;
      const uint32_t* y = op.a[1].ne;
      if (x[2] != 1 || x[3] != 1 || x[1] == 0 || y[0] != x[0] || y[1] != 2 || y[2] != 1 ||
          y[3] != 1)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN:
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN_ROPE: {
      // x [M, K], w [K, N] fp16, cols [2, N] fp32 (bias; column sums of w),
      // stats [M, 2] fp32, (RoPE: segtab [n, 2, 16] fp32, seg_idx [T, 2]
      // int32,) out [M, N] fp16; params: act (, rope_cols)
      const bool rope = op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN_ROPE;
      const uint32_t nb = rope ? 7 : 5;
      HB_TRY(need(op, nb));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(dt(op, 2, DT_FP32));
      HB_TRY(dt(op, 3, DT_FP32));
      if (rope) {
        HB_TRY(dt(op, 4, DT_FP32));
        HB_TRY(dt(op, 5, DT_INT32));
      }
      HB_TRY(dt(op, nb - 1, DT_FP16));
      HB_TRY(batching(op, nb - 1));
      const uint32_t* a = op.a[0].ne;
      const uint32_t* w = op.a[1].ne;
      const uint32_t* c = op.a[2].ne;
      const uint32_t* st = op.a[3].ne;
      if (a[2] != 1 || a[3] != 1 || w[2] != 1 || w[3] != 1 || w[0] != a[1] || a[1] == 0 ||
          w[1] == 0 || w[1] % 256 || c[0] != 2 || c[1] != w[1] || c[2] != 1 || c[3] != 1 ||
          st[0] != a[0] || st[1] != 2 || st[2] != 1 || st[3] != 1 || op.a[1].per_image ||
          op.a[2].per_image || op.a[3].per_image != op.a[0].per_image ||
          numel(op.a[nb - 1].ne) != (uint64_t)a[0] * w[1])
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (op.params[0] < 0 || op.params[0] > 2) return HEXLIB_B200_ERR_INVAL_PARAMS;
      if (rope) {
        const uint32_t* t = op.a[4].ne;   // n_seg, 2, 16
        const uint32_t* x = op.a[5].ne;   // T, 2
        if (op.a[4].per_image || op.a[5].per_image || t[0] == 0 || t[1] != 2 ||
            t[2] != 16 || t[3] != 1 || x[0] == 0 || x[1] != 2 || x[2] != 1 || x[3] != 1 ||
            a[0] % x[0] != 0 || op.params[1] <= 0 || op.params[1] % 64 ||
            (uint32_t)op.params[1] > w[1])
          return HEXLIB_B200_ERR_INVAL_PARAMS;
      }
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_ROPE_QK: {
      HB_TRY(need(op, 4));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP32));
      HB_TRY(dt(op, 2, DT_FP32));
      HB_TRY(dt(op, 3, DT_FP16));
      HB_TRY(batching(op, 3));
      const uint32_t* x = op.a[0].ne;   // T, 3, H, D
      const uint32_t* c = op.a[1].ne;   // T, D
      if (x[1] != 3 || x[0] == 0 || x[2] == 0 || x[3] == 0 || x[3] % 16 ||
          memcmp(op.a[3].ne, x, sizeof(uint32_t) * 4) != 0 ||
          memcmp(op.a[2].ne, c, sizeof(uint32_t) * 4) != 0 || c[0] != x[0] ||
          c[1] != x[3] || c[2] != 1 || c[3] != 1 || op.a[1].per_image || op.a[2].per_image)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_ATTENTION_QKV: {
      HB_TRY(need(op, 2));
      HB_TRY(dt(op, 0, DT_FP16));
      HB_TRY(dt(op, 1, DT_FP16));
      HB_TRY(batching(op, 1));
      const uint32_t* x = op.a[0].ne;   // T, 3, H, D
      const uint32_t* y = op.a[1].ne;   // T, H, D
      if (x[1] != 3 || x[3] != 64 || x[0] == 0 || x[2] == 0 || y[0] != x[0] ||
          y[1] != x[2] || y[2] != x[3] || y[3] != 1)
        return HEXLIB_B200_ERR_INVAL_PARAMS;
      float sc;
      memcpy(&sc, &op.params[0], 4);
      if (!(sc > 0.f)) return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    case HEXLIB_B200_KIND_ATTENTION: {
      HB_TRY(need(op, 4));
      for (int i = 0; i < 4; ++i) HB_TRY(dt(op, i, DT_FP16));
      HB_TRY(batching(op, 3));
      const uint32_t* q = op.a[0].ne;  // Bn, T, D
      if (q[3] != 1 || numel(q) == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
      for (int i = 1; i < 4; ++i)
        if (memcmp(op.a[i].ne, q, sizeof(uint32_t) * 4) != 0 ||
            op.a[i].per_image != op.a[0].per_image)
          return HEXLIB_B200_ERR_INVAL_PARAMS;
      return HEXLIB_B200_OK;
    }
    default:
      return HEXLIB_B200_ERR_NO_KERNEL;
  }
}

// Enqueue one validated op for n images. Returns a status.
// `ws`: the session's scratch for dequantized weights (ws_bytes, sized by
// ensure_workspace before any op of the batch is launched or captured).
int run_op(const OpRec& op, uint32_t n_images, int* err, void* ws, uint64_t ws_bytes,
           cudaStream_t s) {
  bool batched = false;
  for (uint32_t i = 0; i < op.nbuf; ++i) batched = batched || op.a[i].per_image;
  const int64_t B = batched ? n_images : 1;
  const Arg* a = op.a;
  switch (op.kind) {
    case HEXLIB_B200_KIND_ADD: {
      const int64_t n = (int64_t)numel(a[0].ne);
      const int64_t total = n * B;
      const Arg* l = &a[0];
      const Arg* r = &a[1];
      if (!l->per_image && r->per_image) std::swap(l, r);
      const int64_t nb = r->per_image ? total : n;
      if (r->dtype == DT_FP32)
        return hb::launch_add_f16_f32(l->ptr, (const float*)r->ptr, a[2].ptr,
                                      total, nb, s);
      return hb::launch_add_f16(l->ptr, r->ptr, a[2].ptr, total, nb, s);
    }
    case HEXLIB_B200_KIND_CAST:
      return hb::launch_cast_f32_f16((const float*)a[0].ptr, a[1].ptr,
                                     (int64_t)numel(a[0].ne) * B, s);
    case HEXLIB_B200_KIND_SCALE:
      return hb::launch_scale_f16(a[0].ptr, a[1].ptr,
                                  (int64_t)numel(a[0].ne) * B, param_f(op, 0), s);
    case HEXLIB_B200_KIND_LAYERNORM:
      return hb::launch_layernorm_f16(a[0].ptr, (const float*)a[1].ptr,
                                      (const float*)a[2].ptr, a[3].ptr,
                                      (int64_t)a[0].ne[0] * B, (int)a[0].ne[1],
                                      param_f(op, 0), s);
    case HEXLIB_B200_KIND_RMSNORM:
      return hb::launch_rmsnorm_f16(a[0].ptr, a[1].ptr, a[2].ptr,
                                    (int64_t)a[0].ne[0] * B, (int)a[0].ne[1],
                                    param_f(op, 0), s);
    case HEXLIB_B200_KIND_SOFTMAX: {
      const int C = (int)a[0].ne[2];
      const int64_t R = (int64_t)(numel(a[0].ne) / a[0].ne[2]) * B;
      return hb::launch_softmax_f16(a[0].ptr, a[1].ptr, R, C, s);
    }
    case HEXLIB_B200_KIND_ROPE_2D:
      return hb::launch_rope_f16(a[0].ptr, (const float*)a[1].ptr,
                                 (const float*)a[2].ptr, a[3].ptr,
                                 (int64_t)a[0].ne[0] * B, (int)a[0].ne[1],
                                 (int)a[0].ne[2], (int64_t)a[0].ne[0], s);
    case HEXLIB_B200_KIND_TRANSPOSE:
      return hb::launch_transpose_th_f16(a[0].ptr, a[1].ptr, B, (int)a[0].ne[0],
                                         (int)a[0].ne[1], (int)a[0].ne[2], s);
    case HEXLIB_B200_KIND_TRANSPOSE_HD:
      return hb::launch_transpose_hd_f16(a[0].ptr, a[1].ptr,
                                         (int64_t)a[0].ne[0] * B,
                                         (int)a[0].ne[1], (int)a[0].ne[2], s);
    case HEXLIB_B200_KIND_PATCHIFY:
      return hb::launch_patchify_f32((const float*)a[0].ptr, (float*)a[1].ptr, B,
                                     (int)a[0].ne[0], (int)a[0].ne[1],
                                     (int)a[0].ne[2], (int)a[0].ne[3],
                                     op.params[0], op.params[1], op.params[2],
                                     op.params[3], s);
    case HEXLIB_B200_KIND_PATCHIFY_CAST:
      return hb::launch_patchify_f32_f16((const float*)a[0].ptr, a[1].ptr, B,
                                         (int)a[0].ne[0], (int)a[0].ne[1], (int)a[0].ne[2],
                                         (int)a[0].ne[3], op.params[0], op.params[1],
                                         op.params[2], op.params[3], s);
    case HEXLIB_B200_KIND_RESHAPE:
      return hb::launch_copy(a[0].ptr, a[1].ptr, (int64_t)a[0].nbytes * B, s);
    case HEXLIB_B200_KIND_MATMUL: {
      hb::GemmDesc g{};
      g.A = a[0].ptr;
      g.B = a[1].ptr;
      g.out = a[2].ptr;
      g.K = (int)a[0].ne[2];
      g.N = (int)a[1].ne[2];
      if (a[0].per_image && !a[1].per_image) {  // Bn == 1: fold images into M
        g.batch = 1;
        g.M = (int64_t)a[0].ne[1] * B;
        g.b_shared = true;
      } else {
        g.batch = (int64_t)a[0].ne[0] * B;
        g.M = a[0].ne[1];
        g.b_shared = false;
      }
      return hb::launch_gemm(g, err, s);
    }
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE:
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL: {
      const bool res = op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL;
      hb::GemmDesc g{};
      g.A = a[0].ptr;
      g.B = a[1].ptr;
      g.bias = (const float*)a[2].ptr;
      g.resid = res ? a[3].ptr : nullptr;
      g.out = a[res ? 4 : 3].ptr;
      g.batch = 1;
      g.M = (int64_t)a[0].ne[0] * B;
      g.K = (int)a[0].ne[1];
      g.N = (int)a[1].ne[1];
      g.b_shared = true;
      g.act = op.params[0];
      if (a[1].dtype != DT_FP16)
        return hb::launch_gemm_quant(g, (int)a[1].dtype, ws, ws_bytes, err, s);
      return hb::launch_gemm(g, err, s);
    }
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_ROPE: {
      hb::GemmDesc g{};
      g.A = a[0].ptr;
      g.B = a[1].ptr;
      g.bias = (const float*)a[2].ptr;
      g.out = a[6].ptr;
      g.batch = 1;
      g.M = (int64_t)a[0].ne[0] * B;
      g.K = (int)a[0].ne[1];
      g.N = (int)a[1].ne[1];
      g.b_shared = true;
      g.act = op.params[0];
      g.rope_cos = (const float*)a[3].ptr;
      g.rope_sin = (const float*)a[4].ptr;
      g.rope_idx = (const int*)a[5].ptr;
      g.rope_nseg = (int)a[3].ne[0];
      g.rope_T = (int)a[5].ne[0];
      g.rope_cols = op.params[1];
      // a quantized weight arrives here already expanded (expand_weights)
      if (a[1].dtype != DT_FP16) return HEXLIB_B200_ERR_REQUIRES;
      return hb::launch_gemm(g, err, s);
    }
    case HEXLIB_B200_KIND_LN_STATS:
      return hb::launch_ln_stats_f16(a[0].ptr, (float*)a[1].ptr, (int64_t)a[0].ne[0] * B,
                                     (int)a[0].ne[1], param_f(op, 0), s);
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN:
    case HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN_ROPE: {
      const bool rope = op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE_LN_ROPE;
      hb::GemmDesc g{};
      g.A = a[0].ptr;
      g.B = a[1].ptr;
      g.N = (int)a[1].ne[1];
      g.bias = (const float*)a[2].ptr;
      g.ln_colsum = (const float*)a[2].ptr + g.N;
      g.ln_stats = (const float*)a[3].ptr;
      g.out = a[rope ? 6 : 4].ptr;
      g.batch = 1;
      g.M = (int64_t)a[0].ne[0] * B;
      g.K = (int)a[0].ne[1];
      g.b_shared = true;
      g.act = op.params[0];
      if (rope) {
        g.rope_cos = (const float*)a[4].ptr;
        g.rope_sin = (const float*)a[4].ptr + 16;
        g.rope_stride = 32;
        g.rope_idx = (const int*)a[5].ptr;
        g.rope_nseg = (int)a[4].ne[0];
        g.rope_T = (int)a[5].ne[0];
        g.rope_cols = op.params[1];
      }
      return hb::launch_gemm(g, err, s);
    }
    case HEXLIB_B200_KIND_ROPE_QK:
      return hb::launch_rope_qk_f16(a[0].ptr, (const float*)a[1].ptr, (const float*)a[2].ptr,
                                    a[3].ptr, (int64_t)a[0].ne[0] * B, (int)a[0].ne[2],
                                    (int)a[0].ne[3], (int64_t)a[1].ne[0], s);
    case HEXLIB_B200_KIND_ATTENTION_QKV:
      return hb::launch_attention_qkv(a[0].ptr, a[1].ptr, B, (int)a[0].ne[0], (int)a[0].ne[2],
                                      (int)a[0].ne[3], param_f(op, 0), err, s);
    case HEXLIB_B200_KIND_ATTENTION:
      return hb::launch_attention(a[0].ptr, a[1].ptr, a[2].ptr, a[3].ptr,
                                  (int64_t)a[0].ne[0] * B, (int)a[0].ne[1],
                                  (int)a[0].ne[2], param_f(op, 0), err, s);
    default:
      return HEXLIB_B200_ERR_NO_KERNEL;
  }
}

// ---- blob parsing -------------------------------------------------------------

void write_rsp_hdr(uint8_t* rsp, uint32_t status, uint32_t n_ops,
                   uint64_t ns) {
  WireRspHdr h;
  memset(&h, 0, sizeof(h));
  h.magic = HEXLIB_B200_BATCH_MAGIC;
  h.version = HEXLIB_B200_BATCH_VERSION;
  h.status = status;
  h.n_ops = n_ops;
  h.cycles_total = ns;
  h.arch = kArch;
  memcpy(rsp, &h, sizeof(h));
}

struct Parsed {
  WireHdr hdr;
  std::vector<OpRec> ops;   // every op whose arguments resolved and checked
  int fail_status = HEXLIB_B200_OK;
  uint32_t fail_index = 0;  // op index that failed (valid if fail_status!=OK)
  std::vector<uint32_t> kinds;  // echoed kinds of ops [0, fail_index]
};

// Validate header and sections; resolve tensors against `bufs` (one view per
// wire buffer, already looked up by fd). Returns a batch-level status; on OK,
// `out` holds the per-op records up to the first failing op.
typedef int (*BufLookup)(void* user, const WireBuf& wb, uint32_t n_images,
                         BufView* view);

int parse_batch(const uint8_t* batch, uint32_t len, uint32_t n_images,
                BufLookup lookup, void* user, uint32_t rsp_cap, Parsed* out) {
  if (len < sizeof(WireHdr)) return HEXLIB_B200_ERR_TRUNCATED;
  WireHdr hdr;
  memcpy(&hdr, batch, sizeof(hdr));
  out->hdr = hdr;
  if (hdr.magic != HEXLIB_B200_BATCH_MAGIC) return HEXLIB_B200_ERR_BAD_MAGIC;
  if (hdr.version != HEXLIB_B200_BATCH_VERSION) return HEXLIB_B200_ERR_BAD_VERSION;
  if (hdr.total_size != len) return HEXLIB_B200_ERR_TRUNCATED;
  if (hdr.n_bufs > HEXLIB_B200_MAX_BUFS || hdr.n_tensors > HEXLIB_B200_MAX_TENSORS)
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  if ((uint64_t)hdr.off_bufs + (uint64_t)hdr.n_bufs * sizeof(WireBuf) > len ||
      (uint64_t)hdr.off_tensors + (uint64_t)hdr.n_tensors * sizeof(WireTensor) > len ||
      (uint64_t)hdr.off_ops + (uint64_t)hdr.n_ops * sizeof(WireOp) > len)
    return HEXLIB_B200_ERR_TRUNCATED;
  if ((uint64_t)sizeof(WireRspHdr) + (uint64_t)hdr.n_ops * sizeof(WireResult) >
      (uint64_t)rsp_cap)
    return HEXLIB_B200_ERR_TRUNCATED;
  if (n_images == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;

  BufView views[HEXLIB_B200_MAX_BUFS];
  for (uint32_t i = 0; i < hdr.n_bufs; ++i) {
    WireBuf wb;
    memcpy(&wb, batch + hdr.off_bufs + (uint64_t)i * sizeof(WireBuf), sizeof(wb));
    const int rc = lookup(user, wb, n_images, &views[i]);
    if (rc != HEXLIB_B200_OK) return rc;
  }

  struct Resolved {
    Arg arg;
    int status;
  };
  std::vector<Resolved> tens(hdr.n_tensors);
  for (uint32_t i = 0; i < hdr.n_tensors; ++i) {
    WireTensor t;
    memcpy(&t, batch + hdr.off_tensors + (uint64_t)i * sizeof(WireTensor), sizeof(t));
    Resolved& r = tens[i];
    r.status = HEXLIB_B200_OK;
    memset(&r.arg, 0, sizeof(r.arg));
    if (t.bi >= hdr.n_bufs) {
      r.status = HEXLIB_B200_ERR_INVAL_PARAMS;
      continue;
    }
    const BufView& v = views[t.bi];
    if ((uint64_t)t.offset + (uint64_t)t.nbytes > v.size) {
      r.status = HEXLIB_B200_ERR_INVAL_PARAMS;
      continue;
    }
    const uint64_t scale = v.per_image ? n_images : 1;
    r.arg.ptr = v.base ? v.base + (uint64_t)t.offset * scale : nullptr;
    memcpy(r.arg.ne, t.ne, sizeof(t.ne));
    r.arg.dtype = t.dtype;
    r.arg.layout = t.layout;
    r.arg.nbytes = t.nbytes;
    r.arg.per_image = v.per_image;
    if (v.base && (reinterpret_cast<uintptr_t>(r.arg.ptr) & 3u)) {
      // every kernel reads at least 4-byte elements' worth of alignment
      if (t.nbytes) r.status = HEXLIB_B200_ERR_INVAL_PARAMS;
    }
  }

  for (uint32_t i = 0; i < hdr.n_ops; ++i) {
    WireOp wop;
    memcpy(&wop, batch + hdr.off_ops + (uint64_t)i * sizeof(WireOp), sizeof(wop));
    out->kinds.push_back(wop.kind);
    OpRec op;
    memset(&op, 0, sizeof(op));
    op.kind = wop.kind;
    memcpy(op.params, wop.params, sizeof(op.params));
    int st = HEXLIB_B200_OK;
    uint32_t nb = 0;
    for (uint32_t s = 0; s < HEXLIB_B200_MAX_SRC && st == HEXLIB_B200_OK; ++s) {
      if (wop.src[s] == 0xFFFF) continue;
      if (wop.src[s] >= hdr.n_tensors || nb >= HEXLIB_B200_MAX_BUFS) {
        st = HEXLIB_B200_ERR_INVAL_PARAMS;
        break;
      }
      if (tens[wop.src[s]].status != HEXLIB_B200_OK) {
        st = tens[wop.src[s]].status;
        break;
      }
      op.a[nb++] = tens[wop.src[s]].arg;
    }
    for (uint32_t d = 0; d < HEXLIB_B200_MAX_DST && st == HEXLIB_B200_OK; ++d) {
      if (wop.dst[d] == 0xFFFF) continue;
      if (wop.dst[d] >= hdr.n_tensors || nb >= HEXLIB_B200_MAX_BUFS) {
        st = HEXLIB_B200_ERR_INVAL_PARAMS;
        break;
      }
      if (tens[wop.dst[d]].status != HEXLIB_B200_OK) {
        st = tens[wop.dst[d]].status;
        break;
      }
      op.a[nb++] = tens[wop.dst[d]].arg;
    }
    op.nbuf = nb;
    if (st == HEXLIB_B200_OK) st = check_op(op);
    if (st != HEXLIB_B200_OK) {
      out->fail_status = st;
      out->fail_index = i;
      return HEXLIB_B200_OK;
    }
    out->ops.push_back(op);
  }
  return HEXLIB_B200_OK;
}

uint64_t fnv1a(const uint8_t* p, size_t n, uint64_t h = 1469598103934665603ull) {
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

struct Graph {
  std::string blob;
  uint32_t n_images = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint32_t n_ops = 0;
  std::vector<uint32_t> kinds;
};

struct DevBuf {
  void* ptr = nullptr;
  uint64_t size = 0;
  uint32_t replicas = 1;
};

// A q4_0 / q8_0 matmul_epilogue weight of a mapped buffer and the fp16 copy
// of it that the session's GEMMs read. `stale` until the copy has been
// (re)computed from the current bytes of `src`.
struct ExpandedWeight {
  const char* src = nullptr;
  uint64_t src_bytes = 0;
  int qtype = 0;
  int64_t K = 0, N = 0;
  void* dst = nullptr;
  bool stale = true;
};

}  // namespace

struct hexlib_b200_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::vector<cudaEvent_t> op_events;
  std::map<uint32_t, DevBuf> bufs;
  std::unordered_map<uint64_t, std::unique_ptr<Graph>> graphs;
  int* err_host = nullptr;
  int* err_dev = nullptr;
  uint64_t mapped = 0;
  // scratch for the fp16 copy of a quantized weight, one op at a time (kept
  // for ops that reach run_op with a quantized weight; expand_weights leaves
  // none in a session's blobs)
  void* ws = nullptr;
  uint64_t ws_bytes = 0;
  // the fp16 copies of the quantized GEMM weights of this session's blobs
  std::vector<ExpandedWeight> expanded;
};

namespace {

int session_lookup(void* user, const WireBuf& wb, uint32_t n_images,
                   BufView* v) {
  hexlib_b200_ctx* ctx = static_cast<hexlib_b200_ctx*>(user);
  auto it = ctx->bufs.find(wb.fd);
  if (it == ctx->bufs.end()) return HEXLIB_B200_ERR_UNMAPPED;
  const DevBuf& d = it->second;
  v->per_image = (wb.flags & HEXLIB_B200_BUF_PER_IMAGE) != 0;
  v->size = wb.size;
  v->alloc = d.size * d.replicas;
  v->base = static_cast<char*>(d.ptr);
  const uint64_t need = v->per_image ? wb.size * (uint64_t)n_images : wb.size;
  if (wb.size > d.size || need > v->alloc) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return HEXLIB_B200_OK;
}

struct SizesUser {
  const uint64_t* sizes;
  uint32_t n;
  uint32_t next;
};

int sizes_lookup(void* user, const WireBuf& wb, uint32_t n_images, BufView* v) {
  SizesUser* u = static_cast<SizesUser*>(user);
  if (u->next >= u->n) return HEXLIB_B200_ERR_UNMAPPED;
  const uint64_t have = u->sizes[u->next++];
  v->per_image = (wb.flags & HEXLIB_B200_BUF_PER_IMAGE) != 0;
  v->size = wb.size;
  v->alloc = have;
  v->base = nullptr;
  const uint64_t need = v->per_image ? wb.size * (uint64_t)n_images : wb.size;
  if (need > have) return HEXLIB_B200_ERR_INVAL_PARAMS;
  return HEXLIB_B200_OK;
}

void write_results(uint8_t* rsp, const Parsed& p, uint32_t n_ok,
                   const std::vector<uint64_t>* per_op_ns) {
  WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
  for (uint32_t i = 0; i < n_ok; ++i) {
    WireResult r;
    r.kind = p.kinds[i];
    r.status = HEXLIB_B200_OK;
    r.cycles = per_op_ns ? (*per_op_ns)[i] : 0;
    memcpy(&res[i], &r, sizeof(r));
  }
}

int check_device_error(hexlib_b200_ctx* ctx) {
  const volatile int* e = ctx->err_host;
  if (*e != 0) {
    *const_cast<int*>(e) = 0;
    return HEXLIB_B200_ERR_TIMEOUT;
  }
  return HEXLIB_B200_OK;
}

// Eager launch of ops[0, n), optionally timing each with events.
int run_eager(hexlib_b200_ctx* ctx, const Parsed& p, uint32_t n,
              uint32_t n_images, std::vector<uint64_t>* per_op_ns,
              uint64_t* total_ns, uint32_t* done, int* fail_status) {
  *done = 0;
  *fail_status = HEXLIB_B200_OK;
  const bool timed = per_op_ns != nullptr;
  if (timed) {
    while (ctx->op_events.size() < n + 1) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return HEXLIB_B200_ERR_CUDA;
      ctx->op_events.push_back(e);
    }
    per_op_ns->assign(n, 0);
  }
  cudaEventRecord(ctx->ev0, ctx->stream);
  if (timed && n) cudaEventRecord(ctx->op_events[0], ctx->stream);
  hb::order_reset();
  for (uint32_t i = 0; i < n; ++i) {
    const int rc = run_op(p.ops[i], n_images, ctx->err_dev, ctx->ws, ctx->ws_bytes,
                          ctx->stream);
    if (rc != HEXLIB_B200_OK) {
      *fail_status = rc;
      break;
    }
    if (timed) cudaEventRecord(ctx->op_events[i + 1], ctx->stream);
    *done = i + 1;
  }
  cudaEventRecord(ctx->ev1, ctx->stream);
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  float ms = 0.f;
  cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
  *total_ns = (uint64_t)(ms * 1.0e6);
  if (timed) {
    for (uint32_t i = 0; i < *done; ++i) {
      float t = 0.f;
      cudaEventElapsedTime(&t, ctx->op_events[i], ctx->op_events[i + 1]);
      (*per_op_ns)[i] = (uint64_t)(t * 1.0e6);
    }
  }
  return check_device_error(ctx);
}

}  // namespace

extern "C" {

const char* hexlib_b200_status_name(int s) {
  switch (s) {
    case HEXLIB_B200_OK: return "OK";
    case HEXLIB_B200_ERR_INTERNAL: return "ERR_INTERNAL";
    case HEXLIB_B200_ERR_BAD_MAGIC: return "ERR_BAD_MAGIC";
    case HEXLIB_B200_ERR_BAD_VERSION: return "ERR_BAD_VERSION";
    case HEXLIB_B200_ERR_TRUNCATED: return "ERR_TRUNCATED";
    case HEXLIB_B200_ERR_INVAL_PARAMS: return "ERR_INVAL_PARAMS";
    case HEXLIB_B200_ERR_UNMAPPED: return "ERR_UNMAPPED";
    case HEXLIB_B200_ERR_NO_MMAP_SLOT: return "ERR_NO_MMAP_SLOT";
    case HEXLIB_B200_ERR_MMAP_FAILED: return "ERR_MMAP_FAILED";
    case HEXLIB_B200_ERR_NO_KERNEL: return "ERR_NO_KERNEL";
    case HEXLIB_B200_ERR_VTCM_TOO_SMALL: return "ERR_VTCM_TOO_SMALL";
    case HEXLIB_B200_ERR_VTCM_RECLAIMED: return "ERR_VTCM_RECLAIMED";
    case HEXLIB_B200_ERR_REQUIRES: return "ERR_REQUIRES";
    case HEXLIB_B200_ERR_NOT_STARTED: return "ERR_NOT_STARTED";
    case HEXLIB_B200_ERR_CACHE: return "ERR_CACHE";
    case HEXLIB_B200_ERR_CUDA: return "ERR_CUDA";
    case HEXLIB_B200_ERR_TIMEOUT: return "ERR_TIMEOUT";
    case HEXLIB_B200_ERR_COMM: return "ERR_COMM";
    default: return "UNKNOWN";
  }
}

int hexlib_b200_open(int device, hexlib_b200_ctx** out) {
  if (!out) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *out = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  const int rc = hb::kernels_init();
  if (rc != HEXLIB_B200_OK) return rc;
  std::unique_ptr<hexlib_b200_ctx> ctx(new hexlib_b200_ctx());
  ctx->device = device;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&ctx->ev0) != cudaSuccess ||
      cudaEventCreate(&ctx->ev1) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void**>(&ctx->err_host), sizeof(int),
                    cudaHostAllocMapped) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  *ctx->err_host = 0;
  if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&ctx->err_dev),
                               ctx->err_host, 0) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  *out = ctx.release();
  return HEXLIB_B200_OK;
}

static void drop_graphs(hexlib_b200_ctx* ctx) {
  for (auto& kv : ctx->graphs) {
    if (kv.second->exec) cudaGraphExecDestroy(kv.second->exec);
    if (kv.second->graph) cudaGraphDestroy(kv.second->graph);
  }
  ctx->graphs.clear();
}

// Grow the quantized-weight scratch to what this batch's ops need. Done on
// the host before any of the batch is launched or captured; growing it frees
// the old block, so every cached graph (which holds its address) is dropped.
static int ensure_workspace(hexlib_b200_ctx* ctx, const Parsed& p) {
  uint64_t need = 0;
  for (const OpRec& op : p.ops) {
    if ((op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE ||
         op.kind == HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL) &&
        op.a[1].dtype != DT_FP16) {
      const uint64_t b = (uint64_t)op.a[1].ne[0] * op.a[1].ne[1] * 2u;
      if (b > need) need = b;
    }
  }
  if (need <= ctx->ws_bytes) return HEXLIB_B200_OK;
  need = (need + 255) & ~uint64_t(255);
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  drop_graphs(ctx);
  if (ctx->ws) cudaFree(ctx->ws);
  ctx->ws = nullptr;
  ctx->ws_bytes = 0;
  if (cudaMalloc(&ctx->ws, need) != cudaSuccess) {
    cudaGetLastError();
    ctx->ws = nullptr;
    return HEXLIB_B200_ERR_CUDA;
  }
  ctx->ws_bytes = need;
  return HEXLIB_B200_OK;
}

// QUANTIZED WEIGHTS. A q4_0 / q8_0 matmul_epilogue weight is dequantized
// ONCE per session into an fp16 copy the session keeps (one per distinct
// weight: its address, format and shape), not once per invoke: the blob's ops
// are rewritten to read the copy as an fp16 weight, so a quantized plan runs
// exactly the kernels -- and, since each value is the same fp16 rounding
// (code * d), exactly the bits -- of the fp16 plan fed the dequantized
// weights, RoPE and residual epilogues included, with no dequantization in
// the replayed graph. The weights of one encoder are a few hundred MB in
// fp16, a small part of the HBM; the quantized bytes stay where the blob put
// them and are the source of truth: a copy is recomputed (before the next
// launch, on the session stream) whenever hexlib_b200_buf_write[_async]
// writes any of its source bytes, and dropped with its buffer.
static int refresh_weights(hexlib_b200_ctx* ctx) {
  for (ExpandedWeight& e : ctx->expanded) {
    if (!e.stale) continue;
    const int rc = hb::launch_dequant_f16(e.qtype, e.src, e.dst, e.K, e.N, ctx->stream);
    if (rc != HEXLIB_B200_OK) return rc;
    e.stale = false;
  }
  return HEXLIB_B200_OK;
}

static int expand_weights(hexlib_b200_ctx* ctx, Parsed& p) {
  for (OpRec& op : p.ops) {
    if (op.kind != HEXLIB_B200_KIND_MATMUL_EPILOGUE &&
        op.kind != HEXLIB_B200_KIND_MATMUL_EPILOGUE_RESIDUAL &&
        op.kind != HEXLIB_B200_KIND_MATMUL_EPILOGUE_ROPE)
      continue;
    Arg& w = op.a[1];
    if (w.dtype != DT_Q4_0 && w.dtype != DT_Q8_0) continue;
    const int64_t K = w.ne[0], N = w.ne[1];
    ExpandedWeight* hit = nullptr;
    for (ExpandedWeight& e : ctx->expanded)
      if (e.src == static_cast<const char*>(w.ptr) && e.qtype == (int)w.dtype && e.K == K &&
          e.N == N)
        hit = &e;
    if (!hit) {
      ExpandedWeight e;
      e.src = static_cast<const char*>(w.ptr);
      e.src_bytes = w.nbytes;
      e.qtype = (int)w.dtype;
      e.K = K;
      e.N = N;
      if (cudaMalloc(&e.dst, (size_t)(K * N * 2)) != cudaSuccess) {
        cudaGetLastError();
        return HEXLIB_B200_ERR_CUDA;
      }
      ctx->expanded.push_back(e);
      hit = &ctx->expanded.back();
    }
    w.ptr = hit->dst;
    w.dtype = DT_FP16;
    w.nbytes = (uint64_t)(K * N * 2);
  }
  return refresh_weights(ctx);
}

// Bytes [lo, lo + n) of a mapped buffer are being rewritten.
static void weights_written(hexlib_b200_ctx* ctx, const char* lo, uint64_t n) {
  for (ExpandedWeight& e : ctx->expanded)
    if (lo < e.src + e.src_bytes && e.src < lo + n) e.stale = true;
}

static void drop_expanded(hexlib_b200_ctx* ctx) {
  for (ExpandedWeight& e : ctx->expanded) cudaFree(e.dst);
  ctx->expanded.clear();
}

int hexlib_b200_close(hexlib_b200_ctx* ctx) {
  if (!ctx) return HEXLIB_B200_ERR_INVAL_PARAMS;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  drop_graphs(ctx);
  for (auto& kv : ctx->bufs) cudaFree(kv.second.ptr);
  ctx->bufs.clear();
  if (ctx->ws) cudaFree(ctx->ws);
  drop_expanded(ctx);
  for (cudaEvent_t e : ctx->op_events) cudaEventDestroy(e);
  if (ctx->ev0) cudaEventDestroy(ctx->ev0);
  if (ctx->ev1) cudaEventDestroy(ctx->ev1);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->err_host) cudaFreeHost(ctx->err_host);
  cudaGetLastError();
  delete ctx;
  return HEXLIB_B200_OK;
}

int hexlib_b200_hwinfo(hexlib_b200_ctx* ctx, uint32_t* arch, uint32_t* sm_count,
                       uint64_t* hbm_bytes, uint64_t* mapped_bytes) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, ctx->device) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  if (arch) *arch = (uint32_t)(prop.major * 10 + prop.minor);
  if (sm_count) *sm_count = (uint32_t)prop.multiProcessorCount;
  if (hbm_bytes) *hbm_bytes = (uint64_t)prop.totalGlobalMem;
  if (mapped_bytes) *mapped_bytes = ctx->mapped;
  return HEXLIB_B200_OK;
}

int hexlib_b200_mmap(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t size,
                     uint32_t replicas) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  if (size == 0 || replicas == 0) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (ctx->bufs.count(fd)) return HEXLIB_B200_ERR_NO_MMAP_SLOT;
  if (ctx->bufs.size() >= 64) return HEXLIB_B200_ERR_NO_MMAP_SLOT;
  cudaSetDevice(ctx->device);
  const uint64_t bytes = size * (uint64_t)replicas;
  if (bytes / replicas != size) return HEXLIB_B200_ERR_INVAL_PARAMS;
  DevBuf d;
  if (cudaMalloc(&d.ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_MMAP_FAILED;
  }
  d.size = size;
  d.replicas = replicas;
  ctx->bufs[fd] = d;
  ctx->mapped += bytes;
  drop_graphs(ctx);
  return HEXLIB_B200_OK;
}

int hexlib_b200_munmap(hexlib_b200_ctx* ctx, uint32_t fd) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  auto it = ctx->bufs.find(fd);
  if (it == ctx->bufs.end()) return HEXLIB_B200_ERR_UNMAPPED;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  drop_graphs(ctx);
  drop_expanded(ctx);     // their sources may live in this buffer
  ctx->mapped -= it->second.size * it->second.replicas;
  cudaFree(it->second.ptr);
  ctx->bufs.erase(it);
  return HEXLIB_B200_OK;
}

static int buf_range(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset,
                     uint64_t nbytes, char** p) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  auto it = ctx->bufs.find(fd);
  if (it == ctx->bufs.end()) return HEXLIB_B200_ERR_UNMAPPED;
  const uint64_t alloc = it->second.size * it->second.replicas;
  if (offset > alloc || nbytes > alloc - offset) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *p = static_cast<char*>(it->second.ptr) + offset;
  return HEXLIB_B200_OK;
}

int hexlib_b200_buf_write(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset,
                          const void* src, uint64_t nbytes) {
  char* p = nullptr;
  const int rc = buf_range(ctx, fd, offset, nbytes, &p);
  if (rc != HEXLIB_B200_OK) return rc;
  if (nbytes == 0) return HEXLIB_B200_OK;
  if (!src) return HEXLIB_B200_ERR_INVAL_PARAMS;
  weights_written(ctx, p, nbytes);
  if (cudaMemcpyAsync(p, src, nbytes, cudaMemcpyHostToDevice, ctx->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int hexlib_b200_buf_read(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset,
                         void* dst, uint64_t nbytes) {
  char* p = nullptr;
  const int rc = buf_range(ctx, fd, offset, nbytes, &p);
  if (rc != HEXLIB_B200_OK) return rc;
  if (nbytes == 0) return HEXLIB_B200_OK;
  if (!dst) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (cudaMemcpyAsync(dst, p, nbytes, cudaMemcpyDeviceToHost, ctx->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

static int buf_copy_async(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset, void* host,
                          uint64_t nbytes, bool to_device) {
  char* p = nullptr;
  const int rc = buf_range(ctx, fd, offset, nbytes, &p);
  if (rc != HEXLIB_B200_OK) return rc;
  if (nbytes == 0) return HEXLIB_B200_OK;
  if (!host) return HEXLIB_B200_ERR_INVAL_PARAMS;
  if (to_device) weights_written(ctx, p, nbytes);
  const cudaError_t e =
      to_device ? cudaMemcpyAsync(p, host, nbytes, cudaMemcpyHostToDevice, ctx->stream)
                : cudaMemcpyAsync(host, p, nbytes, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return HEXLIB_B200_OK;
}

int hexlib_b200_buf_write_async(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset,
                                const void* src, uint64_t nbytes) {
  return buf_copy_async(ctx, fd, offset, const_cast<void*>(src), nbytes, true);
}

int hexlib_b200_buf_read_async(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t offset, void* dst,
                               uint64_t nbytes) {
  return buf_copy_async(ctx, fd, offset, dst, nbytes, false);
}

int hexlib_b200_buf_device_ptr(hexlib_b200_ctx* ctx, uint32_t fd, uint64_t* ptr,
                               uint64_t* alloc_bytes) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  auto it = ctx->bufs.find(fd);
  if (it == ctx->bufs.end()) return HEXLIB_B200_ERR_UNMAPPED;
  if (ptr) *ptr = reinterpret_cast<uint64_t>(it->second.ptr);
  if (alloc_bytes) *alloc_bytes = it->second.size * it->second.replicas;
  return HEXLIB_B200_OK;
}

int hexlib_b200_stream(hexlib_b200_ctx* ctx, void** stream) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  if (!stream) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *stream = ctx->stream;
  return HEXLIB_B200_OK;
}

int hexlib_b200_sync(hexlib_b200_ctx* ctx) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return HEXLIB_B200_ERR_CUDA;
  }
  return check_device_error(ctx);
}

int hexlib_b200_check_batch(const uint8_t* batch, uint32_t len,
                            const uint64_t* buf_sizes, uint32_t n_sizes,
                            uint32_t n_images, uint8_t* rsp, uint32_t rsp_cap,
                            uint32_t* rsp_len) {
  if (!rsp_len) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *rsp_len = 0;
  if (!rsp || rsp_cap < sizeof(WireRspHdr)) return HEXLIB_B200_ERR_TRUNCATED;
  write_rsp_hdr(rsp, HEXLIB_B200_ERR_INTERNAL, 0, 0);
  *rsp_len = sizeof(WireRspHdr);
  if (!batch) {
    write_rsp_hdr(rsp, HEXLIB_B200_ERR_TRUNCATED, 0, 0);
    return HEXLIB_B200_ERR_TRUNCATED;
  }
  SizesUser u{buf_sizes, n_sizes, 0};
  Parsed p;
  const int rc = parse_batch(batch, len, n_images, sizes_lookup, &u, rsp_cap, &p);
  if (rc != HEXLIB_B200_OK) {
    write_rsp_hdr(rsp, rc, 0, 0);
    return rc;
  }
  const uint32_t n_ok = (uint32_t)p.ops.size();
  write_results(rsp, p, n_ok, nullptr);
  uint32_t done = n_ok;
  int status = HEXLIB_B200_OK;
  if (p.fail_status != HEXLIB_B200_OK) {
    WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
    WireResult r{p.kinds[p.fail_index], (uint32_t)p.fail_status, 0};
    memcpy(&res[p.fail_index], &r, sizeof(r));
    done = p.fail_index + 1;
    status = p.fail_status;
  }
  write_rsp_hdr(rsp, (uint32_t)status, done, 0);
  *rsp_len = (uint32_t)(sizeof(WireRspHdr) + done * sizeof(WireResult));
  return status;
}

int hexlib_b200_invoke_images(hexlib_b200_ctx* ctx, const uint8_t* batch,
                              uint32_t len, uint32_t n_images, uint32_t mode,
                              uint32_t sync, uint8_t* rsp, uint32_t rsp_cap,
                              uint32_t* rsp_len) {
  if (!rsp_len) return HEXLIB_B200_ERR_INVAL_PARAMS;
  *rsp_len = 0;
  if (!rsp || rsp_cap < sizeof(WireRspHdr)) return HEXLIB_B200_ERR_TRUNCATED;
  // Failure is the default (skel_dispatch.c:89-92).
  write_rsp_hdr(rsp, HEXLIB_B200_ERR_INTERNAL, 0, 0);
  *rsp_len = sizeof(WireRspHdr);
  if (!ctx) {
    write_rsp_hdr(rsp, HEXLIB_B200_ERR_NOT_STARTED, 0, 0);
    return HEXLIB_B200_ERR_NOT_STARTED;
  }
  if (!batch || mode > HEXLIB_B200_MODE_EAGER) {
    write_rsp_hdr(rsp, HEXLIB_B200_ERR_INVAL_PARAMS, 0, 0);
    return HEXLIB_B200_ERR_INVAL_PARAMS;
  }
  if (len < sizeof(WireHdr)) {
    write_rsp_hdr(rsp, HEXLIB_B200_ERR_TRUNCATED, 0, 0);
    return HEXLIB_B200_ERR_TRUNCATED;
  }
  cudaSetDevice(ctx->device);

  const uint64_t key = fnv1a(batch, len) ^ ((uint64_t)n_images * 0x9E3779B97F4A7C15ull);
  if (mode == HEXLIB_B200_MODE_GRAPH) {
    auto it = ctx->graphs.find(key);
    if (it != ctx->graphs.end() && it->second->n_images == n_images &&
        it->second->blob.size() == len &&
        memcmp(it->second->blob.data(), batch, len) == 0) {
      Graph& g = *it->second;
      const uint64_t need = sizeof(WireRspHdr) + (uint64_t)g.n_ops * sizeof(WireResult);
      if (need > rsp_cap) {
        write_rsp_hdr(rsp, HEXLIB_B200_ERR_TRUNCATED, 0, 0);
        return HEXLIB_B200_ERR_TRUNCATED;
      }
      const int wrc = refresh_weights(ctx);     // copies whose source was rewritten
      if (wrc != HEXLIB_B200_OK) {
        write_rsp_hdr(rsp, (uint32_t)wrc, 0, 0);
        return wrc;
      }
      cudaEventRecord(ctx->ev0, ctx->stream);
      if (cudaGraphLaunch(g.exec, ctx->stream) != cudaSuccess) {
        cudaGetLastError();
        write_rsp_hdr(rsp, HEXLIB_B200_ERR_CUDA, 0, 0);
        return HEXLIB_B200_ERR_CUDA;
      }
      cudaEventRecord(ctx->ev1, ctx->stream);
      int status = HEXLIB_B200_OK;
      uint64_t ns = 0;
      if (sync) {
        if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
          cudaGetLastError();
          status = HEXLIB_B200_ERR_CUDA;
        } else {
          status = check_device_error(ctx);
          float ms = 0.f;
          cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
          ns = (uint64_t)(ms * 1.0e6);
        }
      }
      WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
      for (uint32_t i = 0; i < g.n_ops; ++i) {
        WireResult r{g.kinds[i], (uint32_t)status, 0};
        memcpy(&res[i], &r, sizeof(r));
      }
      write_rsp_hdr(rsp, (uint32_t)status, g.n_ops, ns);
      *rsp_len = (uint32_t)need;
      return status;
    }
  }

  Parsed p;
  int rc = parse_batch(batch, len, n_images, session_lookup, ctx, rsp_cap, &p);
  if (rc != HEXLIB_B200_OK) {
    write_rsp_hdr(rsp, (uint32_t)rc, 0, 0);
    return rc;
  }
  rc = expand_weights(ctx, p);
  if (rc == HEXLIB_B200_OK) rc = ensure_workspace(ctx, p);
  if (rc != HEXLIB_B200_OK) {
    write_rsp_hdr(rsp, (uint32_t)rc, 0, 0);
    return rc;
  }
  const uint32_t n_ok = (uint32_t)p.ops.size();
  const bool complete = p.fail_status == HEXLIB_B200_OK;

  if (mode == HEXLIB_B200_MODE_GRAPH && complete) {
    std::unique_ptr<Graph> g(new Graph());
    g->blob.assign(reinterpret_cast<const char*>(batch), len);
    g->n_images = n_images;
    g->n_ops = n_ok;
    g->kinds = p.kinds;
    int launch_rc = HEXLIB_B200_OK;
    uint32_t failed_at = 0;
    if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) !=
        cudaSuccess) {
      cudaGetLastError();
      write_rsp_hdr(rsp, HEXLIB_B200_ERR_CUDA, 0, 0);
      return HEXLIB_B200_ERR_CUDA;
    }
    hb::order_reset();
    for (uint32_t i = 0; i < n_ok; ++i) {
      launch_rc = run_op(p.ops[i], n_images, ctx->err_dev, ctx->ws, ctx->ws_bytes,
                         ctx->stream);
      if (launch_rc != HEXLIB_B200_OK) {
        failed_at = i;
        break;
      }
    }
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &graph);
    if (launch_rc == HEXLIB_B200_OK && ce == cudaSuccess && graph &&
        cudaGraphInstantiate(&g->exec, graph, 0) == cudaSuccess) {
      g->graph = graph;
      Graph* gp = g.get();
      ctx->graphs[key] = std::move(g);
      if (ctx->graphs.size() > 64) {
        // Bound the cache; evict everything but the graph just built.
        for (auto it = ctx->graphs.begin(); it != ctx->graphs.end();) {
          if (it->second.get() != gp) {
            if (it->second->exec) cudaGraphExecDestroy(it->second->exec);
            if (it->second->graph) cudaGraphDestroy(it->second->graph);
            it = ctx->graphs.erase(it);
          } else {
            ++it;
          }
        }
      }
      // Run it through the cached path.
      return hexlib_b200_invoke_images(ctx, batch, len, n_images, mode, sync,
                                       rsp, rsp_cap, rsp_len);
    }
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    if (launch_rc != HEXLIB_B200_OK) {
      // An op refused its launch: report it like a kernel failure, with the
      // ops before it run eagerly so the arena holds what the DSP's would.
      std::vector<uint64_t> dummy;
      uint64_t ns = 0;
      uint32_t done = 0;
      int fs = HEXLIB_B200_OK;
      run_eager(ctx, p, failed_at, n_images, nullptr, &ns, &done, &fs);
      write_results(rsp, p, failed_at, nullptr);
      WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
      WireResult r{p.kinds[failed_at], (uint32_t)launch_rc, 0};
      memcpy(&res[failed_at], &r, sizeof(r));
      write_rsp_hdr(rsp, (uint32_t)launch_rc, failed_at + 1, ns);
      *rsp_len = (uint32_t)(sizeof(WireRspHdr) + (failed_at + 1) * sizeof(WireResult));
      return launch_rc;
    }
    write_rsp_hdr(rsp, HEXLIB_B200_ERR_CUDA, 0, 0);
    return HEXLIB_B200_ERR_CUDA;
  }

  // Eager mode, or a blob with a failing op: run ops before the failure.
  std::vector<uint64_t> per_op;
  uint64_t ns = 0;
  uint32_t done = 0;
  int fs = HEXLIB_B200_OK;
  rc = run_eager(ctx, p, n_ok, n_images,
                 mode == HEXLIB_B200_MODE_EAGER ? &per_op : nullptr, &ns, &done,
                 &fs);
  write_results(rsp, p, done, mode == HEXLIB_B200_MODE_EAGER ? &per_op : nullptr);
  int status = HEXLIB_B200_OK;
  uint32_t reported = done;
  if (fs != HEXLIB_B200_OK) {
    WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
    WireResult r{p.kinds[done], (uint32_t)fs, 0};
    memcpy(&res[done], &r, sizeof(r));
    reported = done + 1;
    status = fs;
  } else if (!complete) {
    WireResult* res = reinterpret_cast<WireResult*>(rsp + sizeof(WireRspHdr));
    WireResult r{p.kinds[p.fail_index], (uint32_t)p.fail_status, 0};
    memcpy(&res[p.fail_index], &r, sizeof(r));
    reported = p.fail_index + 1;
    status = p.fail_status;
  }
  if (rc != HEXLIB_B200_OK && status == HEXLIB_B200_OK) status = rc;
  write_rsp_hdr(rsp, (uint32_t)status, reported, ns);
  *rsp_len = (uint32_t)(sizeof(WireRspHdr) + reported * sizeof(WireResult));
  return status;
}

int hexlib_b200_diag_wait_timeout(hexlib_b200_ctx* ctx, uint32_t limit_us) {
  if (!ctx) return HEXLIB_B200_ERR_NOT_STARTED;
  cudaSetDevice(ctx->device);
  const int rc = hb::launch_wait_timeout_probe(ctx->err_dev, limit_us, ctx->stream);
  if (rc != HEXLIB_B200_OK) return rc;
  return hexlib_b200_sync(ctx);
}

int hexlib_b200_invoke(hexlib_b200_ctx* ctx, const uint8_t* batch, uint32_t len,
                       uint8_t* rsp, uint32_t rsp_cap, uint32_t* rsp_len) {
  return hexlib_b200_invoke_images(ctx, batch, len, 1, HEXLIB_B200_MODE_GRAPH,
                                   1, rsp, rsp_cap, rsp_len);
}

}  // extern "C"
