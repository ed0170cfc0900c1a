// hb_tma.h -- host-side construction of TMA tensor maps.
//
// cuTensorMapEncodeTiled is a driver-API function; it is fetched once through
// cudaGetDriverEntryPoint so the library links only against the runtime.
// Every map here is 3-D fp16 (x innermost, then y, then a batch z) with the
// 128-byte swizzle, and the host checks the encoder's own preconditions
// (16-byte-aligned base, strides multiple of 16 bytes) before calling it, so a
// shape TMA cannot describe is refused on the host and never reaches a kernel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hb {

bool tma_available();

// Map over a row-major fp16 tensor [z][y][x] of extents (x, y, z), contiguous,
// loaded in boxes of (box_x, box_y, 1). False if the encoder refuses it.
bool make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t x,
                      uint64_t y, uint64_t z, uint32_t box_x, uint32_t box_y);

// Same with explicit byte strides for y and z (row pitch, batch pitch).
bool make_tmap_3d_f16_strided(CUtensorMap* map, const void* base, uint64_t x,
                              uint64_t y, uint64_t z, uint64_t pitch_y,
                              uint64_t pitch_z, uint32_t box_x,
                              uint32_t box_y);

}  // namespace hb
