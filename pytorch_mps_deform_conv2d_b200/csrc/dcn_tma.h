// dcn_tma.h -- host-side construction of TMA tensor maps (driver entry point
// resolved through the runtime, so the library does not link libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace dcn {

// 2-D fp32 tensor map over `rows` rows of `inner` contiguous elements with a
// row pitch of `pitch_elems`; boxes of 32 elements (128 B) x `box_rows` rows,
// 128-byte swizzle, out-of-range elements read as zero.  `base` and the pitch
// in bytes must be multiples of 16.  `atom32` selects the 128-byte swizzle
// with 32-byte atoms (32-byte chunk c of row r lands at chunk c ^ (r % 4)),
// the layout of an MN-major TF32 tensor-core operand.
cudaError_t make_tmap_2d_f32(CUtensorMap* map, const float* base, uint64_t inner, uint64_t rows,
                             uint64_t pitch_elems, uint32_t box_rows, bool atom32 = false);
// The same for 16-bit elements (bf16, or fp16 with `f16`): boxes of 64
// elements (128 B) x `box_rows` rows.
cudaError_t make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                              uint64_t pitch_elems, uint32_t box_rows, bool f16 = false);

// 16-bit tensor map with a box of `box_inner` elements (32: 64-byte rows and
// the 64-byte swizzle; 64: 128-byte rows and the 128-byte swizzle) x
// `box_rows` rows.
cudaError_t make_tmap_2d_h16_box(CUtensorMap* map, const void* base, uint64_t inner,
                                 uint64_t rows, uint64_t pitch_elems, uint32_t box_inner,
                                 uint32_t box_rows, bool f16);

}  // namespace dcn
