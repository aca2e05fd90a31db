// Row-wise memory-bound kernels of the decoder layer: RMSNorm forward / backward and the SwiGLU
// activation forward / backward.
//
// Reference math (transformers Qwen3RMSNorm and Qwen3MLP; orthrus/objective.py:128-133,146-149):
//   rmsnorm(x) = w * round(x * rsqrt(mean(x^2) + eps))          (the normalised value is rounded to
//                                                                 the activation dtype first)
//   swiglu(g, u) = round(silu(g)) * u                             (silu rounded, then the product)
// One warp per row for the norm, 16-byte vector accesses, a fixed per-row reduction order (every
// lane sums its own contiguous chunks in order, then a butterfly), so a row's result does not
// depend on how many rows a launch has. The backward of the norm returns dx only: the norm weights
// of the dual-view model are frozen.
#pragma once

#include "gemm_simt.cuh"

namespace orthrus {

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void unpack16(const uint4 raw, float* v) {
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
  } else {
    const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = f[i];
  }
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
  } else {
    const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = f[i];
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  uint4 raw;
  if constexpr (sizeof(T) == 2) {
    raw = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                     pack_bf16x2(v[6], v[7]));
  } else {
    raw = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
  }
  *reinterpret_cast<uint4*>(p) = raw;
}

template <typename T>
__device__ __forceinline__ float round_to_t(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// y = w * round(x * rstd); rstd_out[row] when not null. d % (32 * 16/sizeof(T)) == 0.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_fwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              int64_t rows, int d, float eps, T* __restrict__ y,
                                                              float* __restrict__ rstd_out) {
  constexpr int N = Vec16<T>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (r >= rows) return;
  const T* xr = x + r * d;
  float ss = 0.f;
  for (int c = lane * N; c < d; c += 32 * N) {
    float v[N];
    load16<T>(xr + c, v);
#pragma unroll
    for (int i = 0; i < N; ++i) ss = fmaf(v[i], v[i], ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(ss / static_cast<float>(d) + eps);
  T* yr = y + r * d;
  for (int c = lane * N; c < d; c += 32 * N) {
    float v[N], wv[N];
    load16<T>(xr + c, v);
    load16<T>(w + c, wv);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = wv[i] * round_to_t<T>(v[i] * rstd);
    store16<T>(yr + c, v);
  }
  if (rstd_out != nullptr && lane == 0) rstd_out[r] = rstd;
}

// Same forward with the row held in registers, for d = CH * 32 * N: every lane issues all of its
// 16-byte loads (x and w) before the first use, so a warp has its whole row in flight instead of
// one vector at a time, and x is read once. The per-lane order of the sums and the arithmetic are
// those of rmsnorm_fwd_vec_kernel, so the two give identical bits.
template <typename T, int CH>
__global__ void __launch_bounds__(256) rmsnorm_fwd_reg_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              int64_t rows, float eps, T* __restrict__ y,
                                                              float* __restrict__ rstd_out) {
  constexpr int N = Vec16<T>::N;
  constexpr int D = CH * 32 * N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (r >= rows) return;
  const T* xr = x + r * D;
  uint4 xs[CH], ws[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) xs[c] = *reinterpret_cast<const uint4*>(xr + (c * 32 + lane) * N);
#pragma unroll
  for (int c = 0; c < CH; ++c) ws[c] = *reinterpret_cast<const uint4*>(w + (c * 32 + lane) * N);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float v[N];
    unpack16<T>(xs[c], v);
#pragma unroll
    for (int i = 0; i < N; ++i) ss = fmaf(v[i], v[i], ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(ss / static_cast<float>(D) + eps);
  T* yr = y + r * D;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float v[N], wv[N];
    unpack16<T>(xs[c], v);
    unpack16<T>(ws[c], wv);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = wv[i] * round_to_t<T>(v[i] * rstd);
    store16<T>(yr + (c * 32 + lane) * N, v);
  }
  if (rstd_out != nullptr && lane == 0) rstd_out[r] = rstd;
}

// Same backward with x, dy, w (and dres) held in registers, all loads issued up front; identical
// bits to rmsnorm_bwd_vec_kernel.
template <typename T, int CH, bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_bwd_reg_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              const float* __restrict__ rstd, const T* __restrict__ dy,
                                                              int64_t rows, T* __restrict__ dx,
                                                              const T* __restrict__ dres) {
  constexpr int N = Vec16<T>::N;
  constexpr int D = CH * 32 * N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (r >= rows) return;
  const float rs = rstd[r];
  uint4 xs[CH], gs[CH], ws[CH], as[ADD ? CH : 1];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t off = r * D + (c * 32 + lane) * N;
    xs[c] = *reinterpret_cast<const uint4*>(x + off);
    gs[c] = *reinterpret_cast<const uint4*>(dy + off);
    if constexpr (ADD) as[c] = *reinterpret_cast<const uint4*>(dres + off);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) ws[c] = *reinterpret_cast<const uint4*>(w + (c * 32 + lane) * N);
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float v[N], g[N], wv[N];
    unpack16<T>(xs[c], v);
    unpack16<T>(gs[c], g);
    unpack16<T>(ws[c], wv);
#pragma unroll
    for (int i = 0; i < N; ++i) dot = fmaf(g[i] * wv[i], v[i] * rs, dot);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  const float mean = dot / static_cast<float>(D);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float v[N], g[N], wv[N];
    unpack16<T>(xs[c], v);
    unpack16<T>(gs[c], g);
    unpack16<T>(ws[c], wv);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = rs * (g[i] * wv[i] - v[i] * rs * mean);
    if constexpr (ADD) {
      float a[N];
      unpack16<T>(as[c], a);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] += a[i];
    }
    store16<T>(dx + r * D + (c * 32 + lane) * N, v);
  }
}

// dx = rstd * (w dy - xhat * mean(w dy xhat)), xhat = x * rstd.
// With dres (the gradient arriving at x through the residual path) it is added before the one
// rounding: dx = dres + rstd * (...), the sum autograd would form for a tensor used twice.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              const float* __restrict__ rstd, const T* __restrict__ dy,
                                                              int64_t rows, int d, T* __restrict__ dx,
                                                              const T* __restrict__ dres = nullptr) {
  constexpr int N = Vec16<T>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (r >= rows) return;
  const float rs = rstd[r];
  const T* xr = x + r * d;
  const T* gr = dy + r * d;
  float dot = 0.f;
  for (int c = lane * N; c < d; c += 32 * N) {
    float v[N], g[N], wv[N];
    load16<T>(xr + c, v);
    load16<T>(gr + c, g);
    load16<T>(w + c, wv);
#pragma unroll
    for (int i = 0; i < N; ++i) dot = fmaf(g[i] * wv[i], v[i] * rs, dot);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  const float mean = dot / static_cast<float>(d);
  T* out = dx + r * d;
  for (int c = lane * N; c < d; c += 32 * N) {
    float v[N], g[N], wv[N];
    load16<T>(xr + c, v);
    load16<T>(gr + c, g);
    load16<T>(w + c, wv);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = rs * (g[i] * wv[i] - v[i] * rs * mean);
    if (dres != nullptr) {
      float a[N];
      load16<T>(dres + r * d + c, a);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] += a[i];
    }
    store16<T>(out + c, v);
  }
}

// Same backward for any d (one warp per row, lane-strided scalar accesses).
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          const float* __restrict__ rstd, const T* __restrict__ dy,
                                                          int64_t rows, int d, T* __restrict__ dx) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (r >= rows) return;
  const float rs = rstd[r];
  const T* xr = x + r * d;
  const T* gr = dy + r * d;
  float dot = 0.f;
  for (int e = lane; e < d; e += 32) dot = fmaf(to_f32<T>(gr[e]) * to_f32<T>(w[e]), to_f32<T>(xr[e]) * rs, dot);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  const float mean = dot / static_cast<float>(d);
  T* out = dx + r * d;
  for (int e = lane; e < d; e += 32) {
    const float xh = to_f32<T>(xr[e]) * rs;
    out[e] = from_f32<T>(rs * (to_f32<T>(gr[e]) * to_f32<T>(w[e]) - xh * mean));
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }

// out[r, i] = round(silu(g)) * u with g = gu[r, i], u = gu[r, I + i]. I % (16/sizeof(T)) == 0.
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, int64_t rows, int I, T* __restrict__ out) {
  constexpr int N = Vec16<T>::N;
  const int64_t per_row = I / N;
  const int64_t total = rows * per_row;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / per_row;
    const int c = static_cast<int>(idx % per_row) * N;
    float g[N], u[N];
    load16<T>(gu + r * 2 * I + c, g);
    load16<T>(gu + r * 2 * I + I + c, u);
#pragma unroll
    for (int i = 0; i < N; ++i) g[i] = round_to_t<T>(silu_f(g[i])) * u[i];
    store16<T>(out + r * I + c, g);
  }
}

// dgu[r, i] = d(silu)(g) * round(dout * u), dgu[r, I + i] = dout * round(silu(g)).
template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ gu, const T* __restrict__ dout, int64_t rows, int I,
                                  T* __restrict__ dgu) {
  constexpr int N = Vec16<T>::N;
  const int64_t per_row = I / N;
  const int64_t total = rows * per_row;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / per_row;
    const int c = static_cast<int>(idx % per_row) * N;
    float g[N], u[N], d[N], dg[N], du[N];
    load16<T>(gu + r * 2 * I + c, g);
    load16<T>(gu + r * 2 * I + I + c, u);
    load16<T>(dout + r * I + c, d);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float sg = sigmoid_fast(g[i]);
      const float s = round_to_t<T>(g[i] * sg);
      const float ds = round_to_t<T>(d[i] * u[i]);
      dg[i] = ds * sg * (1.f + g[i] * (1.f - sg));
      du[i] = d[i] * s;
    }
    store16<T>(dgu + r * 2 * I + c, dg);
    store16<T>(dgu + r * 2 * I + I + c, du);
  }
}

}  // namespace orthrus
