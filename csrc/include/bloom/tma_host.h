// Host-side helpers: encode TMA tensor maps through the driver entry point
// (no link-time dependency on libcuda, so the extension also imports on
// machines without a GPU driver) and query device properties once.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace bloom {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      p = nullptr;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) throw std::runtime_error("bloom_b200: cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  return fn;
}

// 2D bf16 tensor map over a row-major matrix [outer, inner] with the given
// row pitch.  The inner box must be 64 elements (128 bytes) for SWIZZLE_128B.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                                uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) throw std::runtime_error("TMA base address not 16-byte aligned");
  if ((row_pitch_bytes & 15u) != 0) throw std::runtime_error("TMA row pitch not a multiple of 16 bytes");
  if ((box_inner * elem_bytes) % 16 != 0) throw std::runtime_error("TMA inner box not a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

inline CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_pitch_bytes,
                                     uint32_t box_inner, uint32_t box_outer,
                                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  return make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, outer, row_pitch_bytes, box_inner, box_outer,
                      swizzle);
}

inline int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (cache[device] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cache[device] = v > 0 ? v : 148;
  }
  return cache[device];
}

}  // namespace bloom
