// dcn_tma.cu -- TMA tensor-map encoding (see dcn_tma.h).
#include "dcn_tma.h"

#include <mutex>

namespace dcn {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

void resolve_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  g_encode_status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (g_encode_status == cudaSuccess && (q != cudaDriverEntryPointSuccess || fn == nullptr))
    g_encode_status = cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

cudaError_t make_tmap_2d_f32(CUtensorMap* map, const float* base, uint64_t inner, uint64_t rows,
                             uint64_t pitch_elems, uint32_t box_rows, bool atom32) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode_status != cudaSuccess) return g_encode_status;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch_elems * 4) % 16 != 0 ||
      box_rows == 0 || box_rows > 256 || inner == 0 || rows == 0)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {pitch_elems * 4};
  const cuuint32_t box[2] = {32, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                     : CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                              uint64_t pitch_elems, uint32_t box_rows, bool f16) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode_status != cudaSuccess) return g_encode_status;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch_elems * 2) % 16 != 0 ||
      box_rows == 0 || box_rows > 256 || inner == 0 || rows == 0)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {pitch_elems * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                  : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                              2, const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_2d_h16_box(CUtensorMap* map, const void* base, uint64_t inner,
                                 uint64_t rows, uint64_t pitch_elems, uint32_t box_inner,
                                 uint32_t box_rows, bool f16) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode_status != cudaSuccess) return g_encode_status;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch_elems * 2) % 16 != 0 ||
      (box_inner != 32 && box_inner != 64) || box_rows == 0 || box_rows > 256 || inner == 0 ||
      rows == 0)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {pitch_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                  : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                              2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE,
                              box_inner == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace dcn
