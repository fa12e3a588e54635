// Host-side helpers shared by the cascadia_b200 extension sources.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>

#define CB_CUDA_CHECK(expr)                                                              \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    if (_e != cudaSuccess) {                                                             \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) +   \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));     \
    }                                                                                    \
  } while (0)

namespace cb {

inline int num_sms() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// Programmatic dependent launch (PDL).  A kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may become resident while
// its predecessor in the stream still runs: as soon as every CTA of the
// predecessor has executed griddepcontrol.launch_dependents (or exited).  Its
// set-up (barrier init, TMEM allocation, tensor-map prefetch, the first
// weight copies) then overlaps the predecessor's tail.  Every kernel launched
// this way executes griddepcontrol.wait, in each thread that reads data an
// earlier kernel wrote or writes global memory, and in at least one thread of
// every CTA before it exits, so "predecessor complete" stays transitive along
// the stream.
//
// On by default; CASCADIA_PDL=0 in the environment or set_pdl(false) turns
// the attribute off (the kernels' griddepcontrol instructions are then
// no-ops).  A CUDA graph keeps the setting it was captured with.
inline int& pdl_flag() {
  static int v = [] {
    const char* e = std::getenv("CASCADIA_PDL");
    return e != nullptr ? std::atoi(e) : 1;
  }();
  return v;
}

template <typename... KArgs, typename... Args>
inline void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
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
  CB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// extension does not link libcuda directly.
inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    CB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (p == nullptr || q != cudaDriverEntryPointSuccess)
      throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D bf16 tensor map: inner dimension `inner` (elements), outer `outer` rows,
// row pitch `row_bytes`; box {box_inner, box_outer}.
inline CUtensorMap make_tmap_2d_bf16(void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                                     uint32_t box_inner, uint32_t box_outer,
                                     CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  }
  return m;
}

// X [rows, K] bf16 (row pitch row_bytes) viewed as 3-D {64, rows, K / 64}:
// one load of box {64, box_rows, chunks} brings `chunks` consecutive 64-wide
// K slices, each a [box_rows x 128 B] tile (128B swizzle), back to back in
// shared memory.  The K-slice stride (128 B) is smaller than the row pitch.
inline CUtensorMap make_tmap_kchunks_bf16(void* base, uint64_t K, uint64_t rows,
                                          uint64_t row_bytes, uint32_t box_rows,
                                          uint32_t chunks) {
  CUtensorMap m;
  cuuint64_t dims[3] = {64, rows, K / 64};
  cuuint64_t strides[2] = {row_bytes, 128};
  cuuint32_t box[3] = {64, box_rows, chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("cuTensorMapEncodeTiled (K chunks) failed with code " +
                             std::to_string((int)r));
  }
  return m;
}

}  // namespace cb
