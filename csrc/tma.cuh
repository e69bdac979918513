// Host-side helpers: build 2-D TMA tensor maps (bf16, 128B swizzle) through the driver
// entry point obtained from the runtime, so the extension does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace mimir {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(err == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// The driver-level encoder needs a current CUDA context.  A host thread that has made no CUDA
// runtime call yet (the autograd engine's worker thread, a Python thread) has none, and
// c10::cuda::CUDAGuard does not create one when the device index already matches; cudaSetDevice
// binds the device's primary context to the calling thread.  Once per thread and device.
inline void bind_device_context() {
  thread_local int bound = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (bound != dev && cudaSetDevice(dev) == cudaSuccess) bound = dev;
}

// Row-major bf16 matrix [rows, cols] with leading dimension `ld` (elements); box is
// {box_cols (inner), box_rows}.  base must be 16-byte aligned, ld*2 a multiple of 16.
inline CUtensorMap make_tmap_bf16_2d(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                                     int box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  bind_device_context();
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

// A batch of row-major bf16 matrices [batch, rows, cols]: leading dimension `ld` and `batch_stride`
// elements between consecutive matrices; box {box_cols, box_rows, 1}.  A single matrix is the
// batch-of-one case (z coordinate 0).
inline CUtensorMap make_tmap_bf16_3d(const void* base, int64_t batch, int64_t rows, int64_t cols, int64_t ld,
                                     int64_t batch_stride, int box_cols, int box_rows,
                                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0 && (batch_stride * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  bind_device_context();
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(batch_stride * 2)};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed with code ", (int)r);
  return map;
}

// Row-major fp32 matrix [rows, cols] (leading dimension `ld` elements), no swizzle; used as
// the destination of TMA reduce-add stores.
inline CUtensorMap make_tmap_f32_2d(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                                    int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 4) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  bind_device_context();
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (f32) failed with code ", (int)r);
  return map;
}

}  // namespace mimir
