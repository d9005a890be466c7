// Host helpers: tensor-map encoding through the driver entry point (no -lcuda
// link needed), SM count cache, argument checks.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

namespace b200 {

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Programmatic dependent launch (PDL).  A kernel launched through launch_pdl
// may start while the previous kernel of the stream is still running; it
// must call pdl_wait() (griddepcontrol.wait: the previous grid has completed
// and its writes are visible) in every CTA before it reads or writes anything
// that kernel touches, and may do independent work (reading weights, barrier
// setup) before.  Kernels call pdl_trigger() early so that their successor
// can be scheduled onto SMs they leave free.  Rule for tensor memory: a
// kernel that allocates TMEM triggers only after its allocation, so a
// successor that allocates before its own wait can never hold TMEM that an
// unfinished predecessor still needs.  Off: plain stream order.
inline bool& pdl_flag() {
  static bool on = true;
  return on;
}
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_flag() ? 1 : 0;
  cuda_check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cuda_check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (!ptr || q != cudaDriverEntryPointSuccess)
      throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Row-major 2-D tensor [rows, cols] of `elem_bytes`-sized elements with row
// pitch `row_stride_bytes`; box = box_cols x box_rows; 128-byte swizzle.
// The tensor map checks base alignment (16 B), pitch (multiple of 16 B) and
// box inner extent (box_cols * elem_bytes <= 128 for SWIZZLE_128B).
inline CUtensorMap make_tma_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                               uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                               uint32_t box_cols, uint32_t box_rows,
                               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (reinterpret_cast<uintptr_t>(base) % 16)
    throw std::invalid_argument("TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16)
    throw std::invalid_argument("TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  (void)elem_bytes;
  return map;
}

// 3-D tensor: dims {d0 (contiguous), d1, d2}, strides in bytes for d1 and d2.
inline CUtensorMap make_tma_3d(const void* base, CUtensorMapDataType dtype, uint64_t d0,
                               uint64_t d1, uint64_t d2, uint64_t stride1, uint64_t stride2,
                               uint32_t b0, uint32_t b1, uint32_t b2,
                               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (reinterpret_cast<uintptr_t>(base) % 16)
    throw std::invalid_argument("TMA base address must be 16-byte aligned");
  if (stride1 % 16 || stride2 % 16)
    throw std::invalid_argument("TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled(3d) failed with code " + std::to_string(int(r)));
  return map;
}

inline int sm_count(int device = -1) {
  static int cached[64] = {0};
  if (device < 0) cuda_check(cudaGetDevice(&device), "cudaGetDevice");
  if (!cached[device]) {
    int n = 0;
    cuda_check(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device), "sm count");
    cached[device] = n;
  }
  return cached[device];
}

}  // namespace b200
