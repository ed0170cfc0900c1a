// hb_tma.cu -- TMA tensor-map encoding (see hb_tma.h).
#include "hb_tma.h"

#include <mutex>

namespace hb {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                  void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn g_encode = nullptr;
std::once_flag g_once;

void load_encoder() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                              &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess && fn) {
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  } else {
    cudaGetLastError();
  }
}

}  // namespace

bool tma_available() {
  std::call_once(g_once, load_encoder);
  return g_encode != nullptr;
}

bool make_tmap_3d_f16_strided(CUtensorMap* map, const void* base, uint64_t x,
                              uint64_t y, uint64_t z, uint64_t pitch_y,
                              uint64_t pitch_z, uint32_t box_x,
                              uint32_t box_y) {
  if (!tma_available()) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (x == 0 || y == 0 || z == 0) return false;
  if (pitch_y % 16 || pitch_z % 16) return false;
  if (box_x * 2 > 128 || box_x == 0 || box_y == 0 || box_y > 256) return false;
  const cuuint64_t dims[3] = {x, y, z};
  const cuuint64_t strides[2] = {pitch_y, pitch_z};
  const cuuint32_t box[3] = {box_x, box_y, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                              const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t x,
                      uint64_t y, uint64_t z, uint32_t box_x, uint32_t box_y) {
  return make_tmap_3d_f16_strided(map, base, x, y, z, x * 2, x * y * 2, box_x,
                                  box_y);
}

}  // namespace hb
