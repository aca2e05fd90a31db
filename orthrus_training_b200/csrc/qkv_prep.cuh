// q/k RMSNorm + RoPE + head-major layout, forward and backward.
//
// Reference math (orthrus/objective.py:128-143; transformers Qwen3RMSNorm / apply_rotary_pos_emb):
//   y = w * (x * rsqrt(mean(x^2) + eps)), then rope(y) = y * cos + rotate_half(y) * sin with
//   rotate_half(y) = [-y2, y1], angle(pos, i) = pos * inv_freq[i mod hd/2]. cos / sin are rounded to
//   the activation dtype before use, as the reference's rotary embedding returns them in x.dtype.
// One warp per (token row, head): the warp reads the head's hd values of the fused projection
// output, reduces the sum of squares with shuffles (fixed order), and writes the normalised,
// rotated row into the head-major [B, H, rows, D] buffer (D >= hd, zero padding) that the attention
// kernels read with TMA. Values are also written into a KV cache at a per-sequence row offset.
#pragma once

#include "gemm_simt.cuh"

namespace orthrus {

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// Rounds the N values to T in place; bf16 pairs go through one packed conversion each.
template <typename T, int N>
__device__ __forceinline__ void round_all(float* v) {
  if constexpr (sizeof(T) == 2 && N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const uint32_t p = pack_bf16x2(v[i], v[i + 1]);
      v[i] = __uint_as_float(p << 16);
      v[i + 1] = __uint_as_float(p & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = round_to<T>(v[i]);
  }
}

// kind: 0 = q heads, 1 = k heads, 2 = v heads
template <typename T>
__global__ void __launch_bounds__(256) qkv_prep_fwd_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
    const T* __restrict__ q_norm_w, const T* __restrict__ k_norm_w, int64_t B, int64_t Tn, int Hq, int Hkv,
    int hd, int D, float eps, T* __restrict__ q_out, T* __restrict__ k_out, T* __restrict__ v_out, int64_t cap,
    const int32_t* __restrict__ offset, float* __restrict__ rstd_out) {
  __shared__ float buf[8][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int64_t items = B * Tn * heads;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (item >= items) return;
  const int64_t row = item / heads;
  const int head = static_cast<int>(item % heads);
  const int64_t b = row / Tn, t = row % Tn;
  const int C = heads * hd;
  const T* x = qkv + row * C + static_cast<int64_t>(head) * hd;
  const int half = hd >> 1;
  float* sh = buf[warp];

  if (head >= Hq + Hkv) {  // v: copy into the (cache) layout
    const int hv = head - Hq - Hkv;
    const int64_t orow = (offset ? offset[b] : 0) + t;
    T* dst = v_out + ((b * Hkv + hv) * cap + orow) * D;
    for (int e = lane; e < D; e += 32) dst[e] = e < hd ? x[e] : from_f32<T>(0.f);
    return;
  }
  const bool is_q = head < Hq;
  const T* w = is_q ? q_norm_w : k_norm_w;
  float ss = 0.f;
  for (int e = lane; e < hd; e += 32) {
    const float v = to_f32<T>(x[e]);
    sh[e] = v;
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(ss / static_cast<float>(hd) + eps);
  __syncwarp();
  // normalised and weighted, rounded to the activation dtype as the reference does
  for (int e = lane; e < hd; e += 32) sh[e] = round_to<T>(to_f32<T>(w[e]) * round_to<T>(sh[e] * rstd));
  __syncwarp();
  const float pos = static_cast<float>(positions[row]);
  T* dst;
  if (is_q) {
    dst = q_out + ((b * Hq + head) * Tn + t) * D;
  } else {
    const int64_t orow = (offset ? offset[b] : 0) + t;
    dst = k_out + ((b * Hkv + (head - Hq)) * cap + orow) * D;
  }
  for (int e = lane; e < D; e += 32) {
    float out = 0.f;
    if (e < hd) {
      const int i = e < half ? e : e - half;
      const float ang = pos * inv_freq[i];
      float c, s;
      sincosf(ang, &s, &c);
      c = round_to<T>(c);
      s = round_to<T>(s);
      const float rot = e < half ? -sh[e + half] : sh[e - half];
      out = sh[e] * c + rot * s;
    }
    dst[e] = from_f32<T>(out);
  }
  if (rstd_out && lane == 0) rstd_out[row * (Hq + Hkv) + head] = rstd;
}

// Backward for q (kind 0) or k (kind 1) heads. Fixed work split: grid-stride over (row, head)
// items with a grid that depends only on the problem size; each warp keeps its norm-weight
// gradient partial in registers, the CTA sums its warps in order into part[blockIdx.x][hd].
template <typename T>
__global__ void __launch_bounds__(256) qkv_prep_bwd_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
    const T* __restrict__ norm_w, const float* __restrict__ rstd, const float* __restrict__ dy, int64_t B,
    int64_t Tn, int Hq, int Hkv, int hd, int D, int kind, T* __restrict__ dqkv, float* __restrict__ part) {
  __shared__ float gsh[8][128];
  __shared__ float xsh[8][128];
  __shared__ float wpart[8][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int H = kind == 0 ? Hq : Hkv;
  const int head0 = kind == 0 ? 0 : Hq;
  const int64_t items = B * Tn * H;
  const int C = heads * hd;
  const int half = hd >> 1;
  float wacc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t stride = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + warp; item < items; item += stride) {
    const int64_t row = item / H;
    const int h = static_cast<int>(item % H);
    const int64_t b = row / Tn, t = row % Tn;
    const T* x = qkv + row * C + static_cast<int64_t>(head0 + h) * hd;
    const float* g = dy + ((b * H + h) * Tn + t) * D;
    const float r = rstd[row * (Hq + Hkv) + head0 + h];
    const float pos = static_cast<float>(positions[row]);
    for (int e = lane; e < hd; e += 32) {
      gsh[warp][e] = g[e];
      xsh[warp][e] = to_f32<T>(x[e]) * r;  // xhat
    }
    __syncwarp();
    // undo the rotation: g_j = dy_j c_j + dy_{j+h} s_{j+h} (j < h), dy_j c_j - dy_{j-h} s_{j-h}
    float gn[4];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k;
      gn[k] = 0.f;
      if (e < hd) {
        const int i = e < half ? e : e - half;
        float c, s;
        sincosf(pos * inv_freq[i], &s, &c);
        c = round_to<T>(c);
        s = round_to<T>(s);
        const float other = e < half ? gsh[warp][e + half] : -gsh[warp][e - half];
        const float gr = gsh[warp][e] * c + other * s;
        gn[k] = gr;
        wacc[k] = fmaf(gr, xsh[warp][e], wacc[k]);
        dot = fmaf(gr * to_f32<T>(norm_w[e]), xsh[warp][e], dot);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / static_cast<float>(hd);
    T* out = dqkv + row * C + static_cast<int64_t>(head0 + h) * hd;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = lane + 32 * k;
      if (e < hd) out[e] = from_f32<T>(r * (gn[k] * to_f32<T>(norm_w[e]) - xsh[warp][e] * mean));
    }
    __syncwarp();
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    if (e < 128) wpart[warp][e] = e < hd ? wacc[k] : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < hd; e += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < 8; ++w) acc += wpart[w][e];
    part[static_cast<int64_t>(blockIdx.x) * hd + e] = acc;
  }
}

template <typename T>
__global__ void copy_v_grad_kernel(const float* __restrict__ dv, int64_t B, int64_t Tn, int Hq, int Hkv, int hd,
                                   int D, T* __restrict__ dqkv) {
  const int heads = Hq + 2 * Hkv;
  const int64_t total = B * Tn * Hkv * hd;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i % hd);
    const int64_t rest = i / hd;
    const int h = static_cast<int>(rest % Hkv);
    const int64_t row = rest / Hkv;
    const int64_t b = row / Tn, t = row % Tn;
    const float v = dv ? dv[((b * Hkv + h) * Tn + t) * D + e] : 0.f;
    dqkv[row * heads * hd + static_cast<int64_t>(Hq + Hkv + h) * hd + e] = from_f32<T>(v);
  }
}

template <typename T>
__global__ void zero_heads_kernel(int64_t rows, int heads, int hd, int head0, int nheads, T* __restrict__ dqkv) {
  const int64_t total = rows * nheads * hd;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i % hd);
    const int64_t rest = i / hd;
    const int h = static_cast<int>(rest % nheads);
    const int64_t row = rest / nheads;
    dqkv[row * heads * hd + static_cast<int64_t>(head0 + h) * hd + e] = from_f32<T>(0.f);
  }
}

// out[e] = sum over p of part[p][e]: one warp per element, lane l adds the partials l, l + 32, ...
// in order, then a fixed butterfly (the result does not depend on timing). Grid ceil(hd / 8) x 256.
__global__ void sum_partials_kernel(const float* __restrict__ part, int nparts, int hd, float* __restrict__ out) {
  const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (e >= hd) return;
  float acc = 0.f;
  for (int p = lane; p < nparts; p += 32) acc += part[static_cast<int64_t>(p) * hd + e];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) out[e] = acc;
}

// RMSNorm over rows of length d (the hidden size): y = w * round(x * rsqrt(mean(x^2) + eps)), one
// warp per row with a fixed-order shuffle reduction, so a row's result never depends on the number
// of rows (transformers Qwen3RMSNorm; orthrus/objective.py:128-133).
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t rows,
                                                      int d, float eps, T* __restrict__ y,
                                                      float* __restrict__ rstd_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (r >= rows) return;
  const T* xr = x + r * d;
  float ss = 0.f;
  for (int e = lane; e < d; e += 32) {
    const float v = to_f32<T>(xr[e]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(ss / static_cast<float>(d) + eps);
  T* yr = y + r * d;
  for (int e = lane; e < d; e += 32) yr[e] = from_f32<T>(to_f32<T>(w[e]) * round_to<T>(to_f32<T>(xr[e]) * rstd));
  if (rstd_out != nullptr && lane == 0) rstd_out[r] = rstd;
}

constexpr int kPrepBwdBlocks = 444;  // fixed grid (3 x 148, one wave): a deterministic split of the items

// ------------------------------------------------------------------------------------------------
// Row-parallel prologue for head dims 32 / 64 / 128: one CTA per token row computes the row's
// RoPE cos / sin table once in shared memory (they depend on the position only, not on the head),
// then eight warps handle the row's heads. A lane owns HD/32 contiguous elements of a head; the
// RoPE partner of element e (e +- HD/2) belongs to lane ^ 16 at the same slot.
// ------------------------------------------------------------------------------------------------

// N consecutive elements as one vector access when N * sizeof(T) is 4, 8 or 16 bytes (the address
// aligned to that size), element by element otherwise.
template <typename T, int N>
__device__ __forceinline__ void load_elems(const T* p, float* v) {
  constexpr int BYTES = N * static_cast<int>(sizeof(T));
  if constexpr (BYTES != 4 && BYTES != 8 && BYTES != 16) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = to_f32<T>(p[i]);
  } else {
    uint32_t w[BYTES / 4];
    if constexpr (BYTES == 16) {
      const uint4 r = *reinterpret_cast<const uint4*>(p);
      w[0] = r.x; w[1] = r.y; w[2] = r.z; w[3] = r.w;
    } else if constexpr (BYTES == 8) {
      const uint2 r = *reinterpret_cast<const uint2*>(p);
      w[0] = r.x; w[1] = r.y;
    } else {
      w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
    if constexpr (sizeof(T) == 2) {
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = __uint_as_float(w[i]);
    }
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_elems(T* p, const float* v) {
  constexpr int BYTES = N * static_cast<int>(sizeof(T));
  if constexpr (BYTES != 4 && BYTES != 8 && BYTES != 16) {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f32<T>(v[i]);
  } else {
    uint32_t w[BYTES / 4];
    if constexpr (sizeof(T) == 2) {
#pragma unroll
      for (int i = 0; i < N / 2; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) w[i] = __float_as_uint(v[i]);
    }
    if constexpr (BYTES == 16)
      *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    else if constexpr (BYTES == 8)
      *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    else
      *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}

// This lane's cos / sin of the RoPE angle for its elements e = lane * NE + k (pair index
// e mod HD/2), rounded to the activation dtype as the reference's rotary table is.
template <typename T, int HD>
__device__ __forceinline__ void rope_lane_table(float pos, const float* __restrict__ inv_freq, int lane, float* cs,
                                                float* sn) {
  constexpr int NE = HD / 32;
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    const int i = (lane * NE + k) & (HD / 2 - 1);
    float sv, cv;
    sincosf(pos * inv_freq[i], &sv, &cv);
    cs[k] = round_to<T>(cv);
    sn[k] = round_to<T>(sv);
  }
}

// One warp per token row (8 rows per CTA), no shared memory: every lane builds the RoPE table of
// its own elements, then the warp walks the row's heads PER at a time, all PER head rows loaded
// before any is computed. Lane l holds the elements [l * NE, l * NE + NE) of a head as one vector
// The prologue of one q or k head row in place: lane holds the elements [lane * NE, lane * NE +
// NE) of x; RMSNorm with the fixed-order butterfly (x * rstd rounded, times the q or k norm weight
// wq / wk, rounded), then RoPE
// with this lane's cos / sin (partner element from lane ^ 16). Returns rstd. The forward prologue
// and the decode attention, which runs it on the block rows itself, share this arithmetic, so a
// key or query gets the same bits on either path.
template <typename T, int HD>
__device__ __forceinline__ float prep_head_row(float* x, const float* wq, const float* wk, bool is_q, const float* cs,
                                               const float* sn, float eps, int lane) {
  constexpr int NE = HD / 32;
  constexpr int HALF = HD / 2;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NE; ++k) ss = fmaf(x[k], x[k], ss);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
  for (int k = 0; k < NE; ++k) x[k] *= rstd;
  round_all<T, NE>(x);
#pragma unroll
  for (int k = 0; k < NE; ++k) x[k] *= is_q ? wq[k] : wk[k];
  round_all<T, NE>(x);
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[k], 16);
    const float rot = (lane * NE + k) < HALF ? -partner : partner;
    x[k] = x[k] * cs[k] + rot * sn[k];
  }
  return rstd;
}

// access. Requires 16-byte aligned tensors and D % 8 == 0 (checked by the host).
template <typename T, int HD>
__global__ void __launch_bounds__(256, 4) qkv_prep_fwd_row_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
    const T* __restrict__ q_norm_w, const T* __restrict__ k_norm_w, int64_t rows, int64_t Tn, int Hq, int Hkv,
    int D, float eps, T* __restrict__ q_out, T* __restrict__ k_out, T* __restrict__ v_out, int64_t cap,
    const int32_t* __restrict__ offset, float* __restrict__ rstd_out, int wpr) {
  constexpr int NE = HD / 32;
  constexpr int HALF = HD / 2;
  constexpr int PER = HD == 128 ? 4 : 8;  // head rows in flight per warp within 64 registers
  const int lane = threadIdx.x & 31;
  // wpr warps share a row (few rows: decode); warp `sub` of a row takes the heads sub, sub + wpr,
  // ... with the same per-head arithmetic, so the result does not depend on wpr
  const int warp = threadIdx.x >> 5, sub = warp % wpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (8 / wpr) + warp / wpr;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  if (row >= rows) return;
  const int64_t b = row / Tn, t = row % Tn;
  const int heads = Hq + 2 * Hkv;
  const int nmine = (heads - sub + wpr - 1) / wpr;  // heads of this warp
  const T* xrow = qkv + row * static_cast<int64_t>(heads) * HD;
  float v[PER][NE];
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (j < nmine) load_elems<T, NE>(xrow + (sub + wpr * j) * HD + lane * NE, v[j]);
  float cs[NE], sn[NE], wq[NE], wk[NE];
  rope_lane_table<T, HD>(static_cast<float>(positions[row]), inv_freq, lane, cs, sn);
  load_elems<T, NE>(q_norm_w + lane * NE, wq);
  load_elems<T, NE>(k_norm_w + lane * NE, wk);
  const int64_t orow_kv = (offset ? offset[b] : 0) + t;
  for (int h0 = 0; h0 < nmine; h0 += PER) {
    if (h0 > 0) {
#pragma unroll
      for (int j = 0; j < PER; ++j)
        if (h0 + j < nmine) load_elems<T, NE>(xrow + (sub + wpr * (h0 + j)) * HD + lane * NE, v[j]);
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (h0 + j >= nmine) break;  // warp-uniform
      const int head = sub + wpr * (h0 + j);
      float* x = v[j];
      T* dst;
      if (head >= Hq + Hkv) {
        dst = v_out + ((b * Hkv + (head - Hq - Hkv)) * cap + orow_kv) * D;
      } else {
        const bool is_q = head < Hq;
        const float rstd = prep_head_row<T, HD>(x, wq, wk, is_q, cs, sn, eps, lane);
        if (rstd_out != nullptr && lane == 0) rstd_out[row * (Hq + Hkv) + head] = rstd;
        dst = is_q ? q_out + ((b * Hq + head) * Tn + t) * D
                   : k_out + ((b * Hkv + (head - Hq)) * cap + orow_kv) * D;
      }
      store_elems<T, NE>(dst + lane * NE, x);
      for (int e = HD + lane; e < D; e += 32) dst[e] = from_f32<T>(0.f);
    }
  }
}

// Backward of the row prologue (training layout: offset 0, cap = T). Fixed grid of kPrepBwdBlocks
// CTAs, rows strided over the CTAs, heads over the warps in a fixed order, so the norm-weight
// gradient partials part_q / part_k [block][HD] are deterministic.
template <typename T, int HD>
__global__ void __launch_bounds__(256, 3) qkv_prep_bwd_row_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
    const T* __restrict__ q_norm_w, const T* __restrict__ k_norm_w, const float* __restrict__ rstd,
    const float* __restrict__ dq, const float* __restrict__ dk, const float* __restrict__ dv, int64_t rows,
    int64_t Tn, int Hq, int Hkv, int D, T* __restrict__ dqkv, float* __restrict__ part_q,
    float* __restrict__ part_k) {
  constexpr int NE = HD / 32;
  constexpr int HALF = HD / 2;
  constexpr int PER = HD == 128 ? 2 : 4;  // head rows in flight per warp within 80 registers
  __shared__ float wpart[2][8][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  float wq[NE], wk[NE], nq[NE], nk[NE];
#pragma unroll
  for (int k = 0; k < NE; ++k) wq[k] = wk[k] = 0.f;
  load_elems<T, NE>(q_norm_w + lane * NE, nq);
  load_elems<T, NE>(k_norm_w + lane * NE, nk);
  // one warp per row; rows strided over the fixed grid in a fixed order (deterministic partials)
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows;
       row += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t b = row / Tn, t = row % Tn;
    float cs[NE], sn[NE];
    rope_lane_table<T, HD>(static_cast<float>(positions[row]), inv_freq, lane, cs, sn);
    for (int h0 = 0; h0 < heads; h0 += PER) {
      // loads of up to PER heads first: the incoming gradient and, for q / k, the input row
      float gv[PER][NE], xv[PER][NE], rr[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int head = h0 + j;
        rr[j] = 0.f;
        if (head >= heads) continue;
        const bool is_v = head >= Hq + Hkv, is_q = head < Hq;
        const int h = is_v ? head - Hq - Hkv : is_q ? head : head - Hq;
        const float* gsrc = is_v ? dv : is_q ? dq : dk;
        if (gsrc != nullptr) {
          load_elems<float, NE>(gsrc + ((b * (is_q ? Hq : Hkv) + h) * Tn + t) * D + lane * NE, gv[j]);
        } else {
#pragma unroll
          for (int k = 0; k < NE; ++k) gv[j][k] = 0.f;
        }
        if (!is_v && gsrc != nullptr) {
          load_elems<T, NE>(qkv + row * static_cast<int64_t>(heads) * HD + head * HD + lane * NE, xv[j]);
          rr[j] = rstd[row * (Hq + Hkv) + head];
        }
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int head = h0 + j;  // warp-uniform
        if (head >= heads) break;
        T* out = dqkv + row * static_cast<int64_t>(heads) * HD + head * HD + lane * NE;
        const bool is_v = head >= Hq + Hkv, is_q = head < Hq;
        const float* gsrc = is_v ? dv : is_q ? dq : dk;
        if (is_v || gsrc == nullptr) {
          store_elems<T, NE>(out, gv[j]);  // dV passes through; a missing gradient is zero
          continue;
        }
        const float r = rr[j];
        const float* w = is_q ? nq : nk;
        float xh[NE], gr[NE], o[NE];
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < NE; ++k) {
          xh[k] = xv[j][k] * r;
          const float partner = __shfl_xor_sync(0xffffffffu, gv[j][k], 16);
          const float other = (lane * NE + k) < HALF ? partner : -partner;
          gr[k] = gv[j][k] * cs[k] + other * sn[k];
          dot = fmaf(gr[k] * w[k], xh[k], dot);
          if (is_q)
            wq[k] = fmaf(gr[k], xh[k], wq[k]);
          else
            wk[k] = fmaf(gr[k], xh[k], wk[k]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float mean = dot / static_cast<float>(HD);
#pragma unroll
        for (int k = 0; k < NE; ++k) o[k] = r * (gr[k] * w[k] - xh[k] * mean);
        store_elems<T, NE>(out, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    wpart[0][warp][lane * NE + k] = wq[k];
    wpart[1][warp][lane * NE + k] = wk[k];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < HD; e += blockDim.x) {
    float aq = 0.f, ak = 0.f;
    for (int w = 0; w < 8; ++w) {
      aq += wpart[0][w][e];
      ak += wpart[1][w][e];
    }
    part_q[static_cast<int64_t>(blockIdx.x) * HD + e] = aq;
    part_k[static_cast<int64_t>(blockIdx.x) * HD + e] = ak;
  }
}


// Backward of the row prologue for bf16, head dim 128, with the next group's loads in flight while
// the current group is computed. Same per-element arithmetic as qkv_prep_bwd_row_kernel; the work
// of a warp is its rows (fixed grid, fixed order) split into groups of kPipePer heads of one kind
// (q, k or v; the host checks Hq and Hkv are multiples of kPipePer). Group i + 1's gradient and
// input rows are loaded into a second register set before group i is computed, so each warp keeps
// a group's bytes in flight without a gap between groups and rows. The loaded words are converted
// only when their group is computed, so the loads never stall the warp early.
constexpr int kPipePer = 4;
constexpr int kPipeBlocks = 296;  // 2 x 148: two CTAs of 8 warps per SM, one wave

struct PipeGroup {
  float4 g[kPipePer];   // incoming gradient, 4 fp32 elements of each head for this lane
  uint2 x[kPipePer];    // projection input, 4 bf16 elements of each q / k head
  float r[kPipePer];    // rstd of each q / k head
  float pos;            // the row's position (read for the first group of a row)
};

struct PipeShape {
  const __nv_bfloat16* qkv; const int64_t* positions; const float* rstd;
  const float* dq; const float* dk; const float* dv;
  int64_t rows, Tn, first, stride; int Hq, Hkv, D, heads, groups;
};

__device__ __forceinline__ void pipe_where(const PipeShape& s, int64_t i, int64_t& row, int& head0, int& kind,
                                           int& h) {
  row = s.first + (i / s.groups) * s.stride;
  head0 = static_cast<int>(i % s.groups) * kPipePer;
  kind = head0 < s.Hq ? 0 : head0 < s.Hq + s.Hkv ? 1 : 2;  // q, k, v
  h = kind == 0 ? head0 : kind == 1 ? head0 - s.Hq : head0 - s.Hq - s.Hkv;
}

__device__ __forceinline__ void pipe_load(const PipeShape& s, int64_t i, int lane, PipeGroup& G) {
  int64_t row;
  int head0, kind, h;
  pipe_where(s, i, row, head0, kind, h);
  const int64_t b = row / s.Tn, t = row % s.Tn;
  const float* gsrc = kind == 0 ? s.dq : kind == 1 ? s.dk : s.dv;
  const int H = kind == 0 ? s.Hq : s.Hkv;
#pragma unroll
  for (int j = 0; j < kPipePer; ++j) {
    G.g[j] = gsrc ? __ldg(reinterpret_cast<const float4*>(gsrc + ((b * H + h + j) * s.Tn + t) * s.D) + lane)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    if (kind != 2 && gsrc) {
      G.x[j] = __ldg(reinterpret_cast<const uint2*>(s.qkv + row * static_cast<int64_t>(s.heads) * 128 +
                                                    (head0 + j) * 128) + lane);
      G.r[j] = __ldg(s.rstd + row * (s.Hq + s.Hkv) + head0 + j);
    }
  }
  if (head0 == 0) G.pos = static_cast<float>(__ldg(s.positions + row));
}

__device__ __forceinline__ void pipe_compute(const PipeShape& s, int64_t i, int lane, const PipeGroup& G,
                                             const float* __restrict__ inv_freq, const float* nq, const float* nk,
                                             float* cs, float* sn, float* wq, float* wk,
                                             __nv_bfloat16* __restrict__ dqkv) {
  constexpr int NE = 4, HALF = 64;
  int64_t row;
  int head0, kind, h;
  pipe_where(s, i, row, head0, kind, h);
  if (head0 == 0) rope_lane_table<__nv_bfloat16, 128>(G.pos, inv_freq, lane, cs, sn);
  const float* gsrc = kind == 0 ? s.dq : kind == 1 ? s.dk : s.dv;
#pragma unroll
  for (int j = 0; j < kPipePer; ++j) {
    __nv_bfloat16* out = dqkv + row * static_cast<int64_t>(s.heads) * 128 + (head0 + j) * 128 + lane * NE;
    const float gv[NE] = {G.g[j].x, G.g[j].y, G.g[j].z, G.g[j].w};
    if (kind == 2 || gsrc == nullptr) {
      store_elems<__nv_bfloat16, NE>(out, gv);  // dV passes through; a missing gradient is zero
      continue;
    }
    const float xv[NE] = {__uint_as_float(G.x[j].x << 16), __uint_as_float(G.x[j].x & 0xffff0000u),
                          __uint_as_float(G.x[j].y << 16), __uint_as_float(G.x[j].y & 0xffff0000u)};
    const float r = G.r[j];
    const float* w = kind == 0 ? nq : nk;
    float xh[NE], gr[NE], o[NE];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NE; ++k) {
      xh[k] = xv[k] * r;
      const float partner = __shfl_xor_sync(0xffffffffu, gv[k], 16);
      const float other = (lane * NE + k) < HALF ? partner : -partner;
      gr[k] = gv[k] * cs[k] + other * sn[k];
      dot = fmaf(gr[k] * w[k], xh[k], dot);
      if (kind == 0)
        wq[k] = fmaf(gr[k], xh[k], wq[k]);
      else
        wk[k] = fmaf(gr[k], xh[k], wk[k]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mean = dot / 128.f;
#pragma unroll
    for (int k = 0; k < NE; ++k) o[k] = r * (gr[k] * w[k] - xh[k] * mean);
    store_elems<__nv_bfloat16, NE>(out, o);
  }
}

__global__ void __launch_bounds__(256, 2) qkv_prep_bwd_pipe_kernel(
    const __nv_bfloat16* __restrict__ qkv, const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
    const __nv_bfloat16* __restrict__ q_norm_w, const __nv_bfloat16* __restrict__ k_norm_w,
    const float* __restrict__ rstd, const float* __restrict__ dq, const float* __restrict__ dk,
    const float* __restrict__ dv, int64_t rows, int64_t Tn, int Hq, int Hkv, int D,
    __nv_bfloat16* __restrict__ dqkv, float* __restrict__ part_q, float* __restrict__ part_k) {
  constexpr int NE = 4;
  __shared__ float wpart[2][8][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  PipeShape s{qkv, positions, rstd, dq, dk, dv, rows, Tn, static_cast<int64_t>(blockIdx.x) * 8 + warp,
              static_cast<int64_t>(gridDim.x) * 8, Hq, Hkv, D, Hq + 2 * Hkv, (Hq + 2 * Hkv) / kPipePer};
  const int64_t my_rows = s.first < rows ? (rows - 1 - s.first) / s.stride + 1 : 0;
  const int64_t iters = my_rows * s.groups;
  float wq[NE], wk[NE], nq[NE], nk[NE], cs[NE], sn[NE];
#pragma unroll
  for (int k = 0; k < NE; ++k) wq[k] = wk[k] = cs[k] = sn[k] = 0.f;
  load_elems<__nv_bfloat16, NE>(q_norm_w + lane * NE, nq);
  load_elems<__nv_bfloat16, NE>(k_norm_w + lane * NE, nk);
  PipeGroup A, B;
  if (iters > 0) pipe_load(s, 0, lane, A);
  for (int64_t i = 0; i < iters; i += 2) {
    if (i + 1 < iters) pipe_load(s, i + 1, lane, B);
    pipe_compute(s, i, lane, A, inv_freq, nq, nk, cs, sn, wq, wk, dqkv);
    if (i + 1 < iters) {
      if (i + 2 < iters) pipe_load(s, i + 2, lane, A);
      pipe_compute(s, i + 1, lane, B, inv_freq, nq, nk, cs, sn, wq, wk, dqkv);
    }
  }
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    wpart[0][warp][lane * NE + k] = wq[k];
    wpart[1][warp][lane * NE + k] = wk[k];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 128; e += blockDim.x) {
    float aq = 0.f, ak = 0.f;
    for (int w = 0; w < 8; ++w) {
      aq += wpart[0][w][e];
      ak += wpart[1][w][e];
    }
    part_q[static_cast<int64_t>(blockIdx.x) * 128 + e] = aq;
    part_k[static_cast<int64_t>(blockIdx.x) * 128 + e] = ak;
  }
}

template <typename T>
int qkv_prep_fwd_impl(const T* qkv, const int64_t* positions, const float* inv_freq, const T* qw, const T* kw,
                      int64_t B, int64_t Tn, int Hq, int Hkv, int hd, int D, float eps, T* q_out, T* k_out,
                      T* v_out, int64_t cap, const int32_t* offset, float* rstd, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(qkv && positions && inv_freq && qw && kw && q_out && k_out && v_out);
  ORTHRUS_CHECK_ARG(B > 0 && Tn > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0);
  ORTHRUS_CHECK_ARG(hd >= 2 && hd % 2 == 0 && hd <= 128 && D >= hd && D <= 128 && cap >= Tn);
  // the row kernel makes vector accesses: 16-byte aligned tensors and rows of D % 8 == 0 elements
  const bool vec_ok = D % 8 == 0 && aligned16(qkv) && aligned16(qw) && aligned16(kw) && aligned16(q_out) &&
                      aligned16(k_out) && aligned16(v_out);
  if (vec_ok && (hd == 128 || hd == 64 || hd == 32)) {
    const int64_t rows = B * Tn;
    const int wpr = rows < 4 * 148 * 8 ? 8 : 1;  // few rows: a CTA per row, its 8 warps share the heads
    const unsigned grid = static_cast<unsigned>(ceil_div(rows, 8 / wpr));
    if (hd == 128)
      ORTHRUS_CHECK_CUDA(launch_pdl(qkv_prep_fwd_row_kernel<T, 128>, dim3(grid), dim3(256), 0, stream, qkv, positions,
                                    inv_freq, qw, kw, rows, Tn, Hq, Hkv, D, eps, q_out, k_out, v_out, cap,
                                    offset, rstd, wpr));
    else if (hd == 64)
      ORTHRUS_CHECK_CUDA(launch_pdl(qkv_prep_fwd_row_kernel<T, 64>, dim3(grid), dim3(256), 0, stream, qkv, positions,
                                    inv_freq, qw, kw, rows, Tn, Hq, Hkv, D, eps, q_out, k_out, v_out, cap,
                                    offset, rstd, wpr));
    else
      ORTHRUS_CHECK_CUDA(launch_pdl(qkv_prep_fwd_row_kernel<T, 32>, dim3(grid), dim3(256), 0, stream, qkv, positions,
                                    inv_freq, qw, kw, rows, Tn, Hq, Hkv, D, eps, q_out, k_out, v_out, cap,
                                    offset, rstd, wpr));
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  const int64_t items = B * Tn * (Hq + 2 * Hkv);
  qkv_prep_fwd_kernel<T><<<static_cast<unsigned>(ceil_div(items, 8)), 256, 0, stream>>>(
      qkv, positions, inv_freq, qw, kw, B, Tn, Hq, Hkv, hd, D, eps, q_out, k_out, v_out, cap, offset, rstd);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

inline size_t qkv_prep_bwd_ws(int hd) { return static_cast<size_t>(2) * kPrepBwdBlocks * hd * sizeof(float); }

template <typename T>
int qkv_prep_bwd_impl(const T* qkv, const int64_t* positions, const float* inv_freq, const T* qw, const T* kw,
                      const float* rstd, const float* dq, const float* dk, const float* dv, int64_t B, int64_t Tn,
                      int Hq, int Hkv, int hd, int D, T* dqkv, float* dqw, float* dkw, void* ws, size_t ws_bytes,
                      cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(qkv && positions && inv_freq && qw && kw && rstd && dqkv && dqw && dkw);
  ORTHRUS_CHECK_ARG(B > 0 && Tn > 0 && hd >= 2 && hd % 2 == 0 && hd <= 128 && D >= hd && D <= 128);
  if (ws == nullptr || ws_bytes < qkv_prep_bwd_ws(hd)) return ORTHRUS_EWORKSPACE;
  float* part_q = static_cast<float*>(ws);
  float* part_k = part_q + static_cast<int64_t>(kPrepBwdBlocks) * hd;
  const int heads = Hq + 2 * Hkv;
  const int64_t rows = B * Tn;
  const bool vec_ok = D % 8 == 0 && aligned16(qkv) && aligned16(qw) && aligned16(kw) && aligned16(dqkv) &&
                      (!dq || aligned16(dq)) && (!dk || aligned16(dk)) && (!dv || aligned16(dv));
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    if (vec_ok && hd == 128 && D % 4 == 0 && Hq % kPipePer == 0 && Hkv % kPipePer == 0) {
      ORTHRUS_CHECK_CUDA(launch_pdl(qkv_prep_bwd_pipe_kernel, dim3(kPipeBlocks), dim3(256), 0, stream, qkv, positions,
                                    inv_freq, qw, kw, rstd, dq, dk, dv, rows, Tn, Hq, Hkv, D, dqkv, part_q,
                                    part_k));
      ORTHRUS_CHECK_LAUNCH();
      ORTHRUS_CHECK_CUDA(launch_pdl(sum_partials_kernel, dim3((hd + 7) / 8), dim3(256), 0, stream,
                                    static_cast<const float*>(part_q), kPipeBlocks, hd, dqw));
      ORTHRUS_CHECK_LAUNCH();
      ORTHRUS_CHECK_CUDA(launch_pdl(sum_partials_kernel, dim3((hd + 7) / 8), dim3(256), 0, stream,
                                    static_cast<const float*>(part_k), kPipeBlocks, hd, dkw));
      ORTHRUS_CHECK_LAUNCH();
      return ORTHRUS_OK;
    }
  }
  if (vec_ok && (hd == 128 || hd == 64 || hd == 32)) {
    if (hd == 128)
      qkv_prep_bwd_row_kernel<T, 128><<<kPrepBwdBlocks, 256, 0, stream>>>(qkv, positions, inv_freq, qw, kw, rstd, dq, dk,
                                                                          dv, rows, Tn, Hq, Hkv, D, dqkv, part_q, part_k);
    else if (hd == 64)
      qkv_prep_bwd_row_kernel<T, 64><<<kPrepBwdBlocks, 256, 0, stream>>>(qkv, positions, inv_freq, qw, kw, rstd, dq, dk,
                                                                         dv, rows, Tn, Hq, Hkv, D, dqkv, part_q, part_k);
    else
      qkv_prep_bwd_row_kernel<T, 32><<<kPrepBwdBlocks, 256, 0, stream>>>(qkv, positions, inv_freq, qw, kw, rstd, dq, dk,
                                                                         dv, rows, Tn, Hq, Hkv, D, dqkv, part_q, part_k);
    ORTHRUS_CHECK_LAUNCH();
    sum_partials_kernel<<<(hd + 7) / 8, 256, 0, stream>>>(part_q, kPrepBwdBlocks, hd, dqw);
    ORTHRUS_CHECK_LAUNCH();
    sum_partials_kernel<<<(hd + 7) / 8, 256, 0, stream>>>(part_k, kPrepBwdBlocks, hd, dkw);
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  if (dq) {
    qkv_prep_bwd_kernel<T><<<kPrepBwdBlocks, 256, 0, stream>>>(qkv, positions, inv_freq, qw, rstd, dq, B, Tn, Hq,
                                                               Hkv, hd, D, 0, dqkv, part_q);
    ORTHRUS_CHECK_LAUNCH();
    sum_partials_kernel<<<(hd + 7) / 8, 256, 0, stream>>>(part_q, kPrepBwdBlocks, hd, dqw);
  } else {
    zero_heads_kernel<T><<<592, 256, 0, stream>>>(rows, heads, hd, 0, Hq, dqkv);
    ORTHRUS_CHECK_CUDA(cudaMemsetAsync(dqw, 0, hd * sizeof(float), stream));
  }
  ORTHRUS_CHECK_LAUNCH();
  if (dk) {
    qkv_prep_bwd_kernel<T><<<kPrepBwdBlocks, 256, 0, stream>>>(qkv, positions, inv_freq, kw, rstd, dk, B, Tn, Hq,
                                                               Hkv, hd, D, 1, dqkv, part_k);
    ORTHRUS_CHECK_LAUNCH();
    sum_partials_kernel<<<(hd + 7) / 8, 256, 0, stream>>>(part_k, kPrepBwdBlocks, hd, dkw);
  } else {
    zero_heads_kernel<T><<<592, 256, 0, stream>>>(rows, heads, hd, Hq, Hkv, dqkv);
    ORTHRUS_CHECK_CUDA(cudaMemsetAsync(dkw, 0, hd * sizeof(float), stream));
  }
  ORTHRUS_CHECK_LAUNCH();
  copy_v_grad_kernel<T><<<592, 256, 0, stream>>>(dv, B, Tn, Hq, Hkv, hd, D, dqkv);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // namespace orthrus
