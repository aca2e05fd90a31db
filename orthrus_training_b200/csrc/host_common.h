// Host-side helpers shared by the C ABI wrappers: status macros, TMA tensor-map encoding through
// the driver entry point (no link-time dependency on libcuda), launch checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <utility>
#include <unordered_map>

#include "orthrus_b200.h"

namespace orthrus {

#define ORTHRUS_CHECK_ARG(cond)                                                        \
  do {                                                                                 \
    if (!(cond)) {                                                                     \
      if (getenv("ORTHRUS_DEBUG")) fprintf(stderr, "orthrus: bad argument: %s\n", #cond); \
      return ORTHRUS_EINVAL;                                                           \
    }                                                                                  \
  } while (0)

#define ORTHRUS_CHECK_CUDA(expr)                                                            \
  do {                                                                                      \
    cudaError_t err__ = (expr);                                                             \
    if (err__ != cudaSuccess) {                                                             \
      if (getenv("ORTHRUS_DEBUG"))                                                          \
        fprintf(stderr, "orthrus: %s failed: %s\n", #expr, cudaGetErrorString(err__));      \
      return ORTHRUS_ECUDA;                                                                 \
    }                                                                                       \
  } while (0)

// Kernels launched by this process through the library (diagnostics: every launch site is followed
// by exactly one ORTHRUS_CHECK_LAUNCH).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

#define ORTHRUS_CHECK_LAUNCH()                                                  \
  do {                                                                          \
    orthrus::launch_counter().fetch_add(1, std::memory_order_relaxed);          \
    ORTHRUS_CHECK_CUDA(cudaGetLastError());                                     \
  } while (0)

// Opts a kernel into `bytes` of dynamic shared memory once per process and kernel (the attribute
// persists; repeating it on every launch would also add a driver call inside stream capture).
template <typename Kern>
inline cudaError_t ensure_smem(Kern kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

// Launches `kernel` with the programmatic stream serialization attribute: it may begin (its
// prologue, loads of constant operands) while the previous kernel on the stream finishes. The
// kernel must call griddep_wait() before it touches anything that kernel reads or writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int num_sms() {
  static int cached = 0;
  if (cached == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    if (cached <= 0) cached = 148;
  }
  return cached;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [outer, inner] matrix with row pitch `pitch` elements,
// box = [box_outer rows][box_inner cols], 128-byte swizzle (box_inner * 2 must be 128).
inline bool make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t pitch, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D fp32 tensor map over a row-major [outer, inner] matrix (pitch elements), 128-byte swizzle
// (box_inner * 4 must be 128).
inline bool make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
                             uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D bf16 tensor map over [d2][d1][d0] with element strides s1 (between d1 rows) and s2.
inline bool make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                              uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1 * 2, s2 * 2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// K-blocked view of a row-major bf16 matrix [rows, K] (pitch elements, K a multiple of 64) for
// TMA boxes that carry several 64-column k-blocks at once: dims (64, rows, K / 64) with strides
// (pitch, 64) elements, box (64, box_rows, kblocks), 128-byte swizzle. A box lands in shared
// memory as kblocks consecutive [box_rows][64] K-major tiles, the layout a UMMA operand takes.
// With halves > 1 the rows are split into `halves` groups `half_stride` rows apart (dims (64,
// rows / halves, halves, K / 64)): a box then holds box_rows rows from each group in turn.
inline bool make_tmap_kblocked_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t K, uint64_t pitch,
                                    uint32_t box_rows, uint32_t kblocks, uint32_t halves = 1,
                                    uint64_t half_stride = 0) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr || K % 64 != 0) return false;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r;
  if (halves == 1) {
    cuuint64_t dims[3] = {64, rows, K / 64};
    cuuint64_t strides[2] = {pitch * 2, 128};
    cuuint32_t box[3] = {64, box_rows, kblocks};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[4] = {64, rows / halves, halves, K / 64};
    cuuint64_t strides[3] = {pitch * 2, half_stride * pitch * 2, 128};
    cuuint32_t box[4] = {64, box_rows, halves, kblocks};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

}  // namespace orthrus
