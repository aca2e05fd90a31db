// The C ABI of liborthrus_b200.so (declared in include/orthrus_b200.h). The whole library is one
// translation unit, so device symbols (the error word) need no relocatable device code.
#include <algorithm>
#include <cstdlib>

#include "host_common.h"
#include "sm100.cuh"

#include "attention_simt.cuh"
#include "attention_tc.cuh"
#include "decode.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "lmhead_kl.cuh"
#include "qkv_prep.cuh"

using namespace orthrus;

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int orthrus_version(void) { return 100; }

int orthrus_device_error(int device, unsigned int* word, int clear) {
  ORTHRUS_CHECK_ARG(word != nullptr);
  int prev = 0;
  ORTHRUS_CHECK_CUDA(cudaGetDevice(&prev));
  ORTHRUS_CHECK_CUDA(cudaSetDevice(device));
  ORTHRUS_CHECK_CUDA(cudaDeviceSynchronize());
  unsigned int w = 0;
  ORTHRUS_CHECK_CUDA(cudaMemcpyFromSymbol(&w, g_device_error, sizeof(w)));
  if (clear && w) {
    const unsigned int zero = 0;
    ORTHRUS_CHECK_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
  }
  ORTHRUS_CHECK_CUDA(cudaSetDevice(prev));
  *word = w;
  return w ? ORTHRUS_EDEVICE : ORTHRUS_OK;
}

size_t orthrus_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) { return gemm_ws_bytes(M, N, K); }

int orthrus_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                      int64_t N, int64_t K, int b_kn, int c_f32, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return gemm_bf16_impl(A, lda, B, ldb, C, ldc, M, N, K, b_kn, c_f32, workspace, workspace_bytes,
                        as_stream(stream));
}

size_t orthrus_gemm_simt_workspace_bytes(int64_t M, int64_t N, int64_t K) { return simt_ws_bytes(M, N, K); }

int orthrus_gemm_simt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                      int64_t N, int64_t K, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype == ORTHRUS_F32)
    return gemm_simt_impl<float, false>(static_cast<const float*>(A), lda, static_cast<const float*>(B), ldb,
                                        static_cast<float*>(C), ldc, M, N, K, workspace, workspace_bytes,
                                        as_stream(stream));
  if (dtype == ORTHRUS_BF16)
    return gemm_simt_impl<__nv_bfloat16, false>(
        static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(B), ldb,
        static_cast<__nv_bfloat16*>(C), ldc, M, N, K, workspace, workspace_bytes, as_stream(stream));
  return ORTHRUS_EINVAL;
}

size_t orthrus_lmhead_kl_workspace_bytes(int64_t n, int64_t m, int64_t V, int64_t d, int64_t chunk_rows,
                                         int dtype) {
  return lmhead_plan(n, m, V, d, chunk_rows, dtype).total;
}

int orthrus_lmhead_kl_fwd(const void* student, int64_t n, const void* teacher, int64_t m, const int64_t* index,
                          const void* weight, int64_t V, int64_t d, const float* row_weight,
                          const int64_t* offsets, int num_offsets, float* total, float* kl_rows, uint8_t* agree,
                          void* grad, float* kl_by_offset, int64_t* agree_by_offset, int64_t chunk_rows,
                          void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  if (dtype == ORTHRUS_BF16)
    return lmhead_kl_fwd_impl<__nv_bfloat16>(
        static_cast<const __nv_bfloat16*>(student), n, static_cast<const __nv_bfloat16*>(teacher), m, index,
        static_cast<const __nv_bfloat16*>(weight), V, d, row_weight, offsets, num_offsets, total, kl_rows,
        agree, static_cast<__nv_bfloat16*>(grad), kl_by_offset, agree_by_offset, chunk_rows, workspace,
        workspace_bytes, as_stream(stream));
  if (dtype == ORTHRUS_F32)
    return lmhead_kl_fwd_impl<float>(static_cast<const float*>(student), n, static_cast<const float*>(teacher), m,
                                     index, static_cast<const float*>(weight), V, d, row_weight, offsets,
                                     num_offsets, total, kl_rows, agree, static_cast<float*>(grad), kl_by_offset,
                                     agree_by_offset, chunk_rows, workspace, workspace_bytes, as_stream(stream));
  return ORTHRUS_EINVAL;
}

int orthrus_lmhead_kl_bwd(const void* grad, const float* grad_total, void* grad_student, int64_t count,
                          int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(grad && grad_total && grad_student && count >= 0);
  if (count == 0) return ORTHRUS_OK;
  const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(count, 256), 148 * 8));
  if (dtype == ORTHRUS_BF16)
    scale_by_scalar_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(grad), grad_total, static_cast<__nv_bfloat16*>(grad_student), count);
  else if (dtype == ORTHRUS_F32)
    scale_by_scalar_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const float*>(grad), grad_total, static_cast<float*>(grad_student), count);
  else
    return ORTHRUS_EINVAL;
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // extern "C"
