// Exact fp32 GEMM on CUDA cores (FFMA), for the fp32 path: C[M, N] = A[M, K] @ op(B).
//
// 64 x 64 output tile per CTA, 256 threads with 4 x 4 register micro-tiles, k-slabs of 16 staged
// through shared memory. Each output element accumulates its k products strictly in order with
// fmaf, and the split-K boundaries are a function of (N, K) only, with partials summed in split
// order: the value of an output row never depends on how many rows M the call has. That makes a
// K-token verification pass and a one-token greedy pass bit-identical (lossless decoding).
#pragma once

#include "sm100.cuh"

namespace orthrus {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Accumulates the 64 x 64 tile (rows m0.., cols n0..) over k in [k0, k1) into acc (4 x 4 per
// thread; thread t owns rows (t/16)*4 + i and cols (t%16)*4 + j). B_KN: B is [K, N], else [N, K].
template <typename T, bool B_KN>
__device__ __forceinline__ void simt_tile_accumulate(const T* __restrict__ A, int64_t lda,
                                                     const T* __restrict__ B, int64_t ldb, int M, int N,
                                                     int m0, int n0, int k0, int k1, float (*sA)[64 + 4],
                                                     float (*sB)[64 + 4], float acc[4][4]) {
  const int tid = threadIdx.x;
  const int tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
  for (int kk = k0; kk < k1; kk += 16) {
    // A slab 64 x 16 -> sA[k][m]; B slab -> sB[k][n]
    for (int e = tid; e < 64 * 16; e += 256) {
      const int r = e >> 4, k = e & 15;
      const int gm = m0 + r, gk = kk + k;
      sA[k][r] = (gm < M && gk < k1) ? to_f32(A[static_cast<int64_t>(gm) * lda + gk]) : 0.f;
    }
    if constexpr (B_KN) {
      for (int e = tid; e < 64 * 16; e += 256) {
        const int k = e >> 6, c = e & 63;
        const int gn = n0 + c, gk = kk + k;
        sB[k][c] = (gn < N && gk < k1) ? to_f32(B[static_cast<int64_t>(gk) * ldb + gn]) : 0.f;
      }
    } else {
      for (int e = tid; e < 64 * 16; e += 256) {
        const int c = e >> 4, k = e & 15;
        const int gn = n0 + c, gk = kk + k;
        sB[k][c] = (gn < N && gk < k1) ? to_f32(B[static_cast<int64_t>(gn) * ldb + gk]) : 0.f;
      }
    }
    __syncthreads();
    const int kn = min(16, k1 - kk);
    for (int k = 0; k < kn; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[k][tr + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[k][tc + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
}

template <typename T, bool B_KN>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, int64_t lda,
                                                        const T* __restrict__ B, int64_t ldb,
                                                        T* __restrict__ C, int64_t ldc,
                                                        float* __restrict__ partials, int M, int N,
                                                        int K, int k_per_split) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64, split = blockIdx.z;
  const int k0 = split * k_per_split, k1 = min(K, k0 + k_per_split);
  float acc[4][4] = {};
  simt_tile_accumulate<T, B_KN>(A, lda, B, ldb, M, N, m0, n0, k0, k1, sA, sB, acc);
  const int tid = threadIdx.x;
  const int tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + tr + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tc + j;
      if (c >= N) continue;
      if (partials)
        partials[(static_cast<int64_t>(split) * M + r) * N + c] = acc[i][j];
      else
        C[static_cast<int64_t>(r) * ldc + c] = from_f32<T>(acc[i][j]);
    }
  }
}

template <typename T>
__global__ void simt_splitk_reduce_kernel(const float* __restrict__ ws, T* __restrict__ C, int64_t ldc, int M,
                                          int N, int splits) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[s * total + i];
    C[(i / N) * ldc + (i % N)] = from_f32<T>(acc);
  }
}

inline int simt_splits(int64_t N, int64_t K) {
  const int64_t ntiles = ceil_div(N, 64);
  int splits = 1;
  while (ntiles * splits * 2 <= 2 * num_sms() && K / (splits * 2) >= 256) splits *= 2;
  return splits;
}

inline size_t simt_ws_bytes(int64_t M, int64_t N, int64_t K) {
  const int s = simt_splits(N, K);
  return s > 1 ? static_cast<size_t>(s) * M * N * sizeof(float) : 0;
}

template <typename T, bool B_KN>
int gemm_simt_impl(const T* A, int64_t lda, const T* B, int64_t ldb, T* C, int64_t ldc, int64_t M, int64_t N,
                   int64_t K, void* ws, size_t ws_bytes, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(A && B && C && M > 0 && N > 0 && K > 0 && lda >= K && ldc >= N);
  ORTHRUS_CHECK_ARG(B_KN ? ldb >= N : ldb >= K);
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31));
  const int splits = simt_splits(N, K);
  if (splits > 1 && (ws == nullptr || ws_bytes < simt_ws_bytes(M, N, K))) return ORTHRUS_EWORKSPACE;
  const int kps = static_cast<int>(ceil_div(ceil_div(K, splits), 16) * 16);
  dim3 grid(static_cast<unsigned>(ceil_div(M, 64)), static_cast<unsigned>(ceil_div(N, 64)), splits);
  float* part = splits > 1 ? static_cast<float*>(ws) : nullptr;
  gemm_simt_kernel<T, B_KN><<<grid, 256, 0, stream>>>(A, lda, B, ldb, C, ldc, part, static_cast<int>(M),
                                                       static_cast<int>(N), static_cast<int>(K), kps);
  ORTHRUS_CHECK_LAUNCH();
  if (splits > 1) {
    const int64_t total = M * N;
    const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), 148 * 16));
    simt_splitk_reduce_kernel<T><<<blocks, 256, 0, stream>>>(part, C, ldc, static_cast<int>(M),
                                                              static_cast<int>(N), splits);
    ORTHRUS_CHECK_LAUNCH();
  }
  return ORTHRUS_OK;
}

}  // namespace orthrus
