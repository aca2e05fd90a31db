// Exact attention on CUDA cores for the fp32 path and for decoding (any head dim <= 128).
//
// One warp per query row. Keys are visited in tiles of 32 starting at key 0 of source 1, then
// source 2; each tile is staged in shared memory once per CTA and every lane scores one key.
// A query's softmax state (max, sum, output) is updated only by tiles that contain one of its
// visible keys, in tile order, with fixed-order shuffle reductions: the result for a query does not
// depend on which other queries share the launch, so a K-token verification pass reproduces a
// one-token greedy pass bit for bit.
//
// Mask semantics (one rule for training and decoding, see orthrus_b200.h): query t of batch b sees
// source-1 keys [0, e1) and source-2 keys [s2, e2).
//   causal: e1 = t + 1 + offset[b]              (teacher pass, verification over a KV cache)
//   dual:   e1 = min(anchor[b, t / K], L1), [s2, e2) = own block   (orthrus/modeling_orthrus.py:58-74)
//   draft:  e1 = offset[b], [s2, e2) = [0, limit2[b])              (orthrus/modeling_orthrus.py:469-481)
#pragma once

#include "gemm_simt.cuh"

namespace orthrus {

struct MaskParams {
  int mode;
  const int64_t* anchors;
  int64_t A;
  int block;
  const int32_t* offset;
  const int32_t* limit2;
  int64_t L1, L2;
  // opt-in document mask: int32 [B, L1], the first position of each position's document (packed
  // rows of several documents); null keeps the reference's mask over the whole row
  const int32_t* doc_start = nullptr;
};

__device__ __forceinline__ void query_ranges(const MaskParams& mp, int64_t b, int64_t t, int64_t& e1, int64_t& s2,
                                             int64_t& e2) {
  if (mp.mode == ORTHRUS_MASK_CAUSAL) {
    e1 = min(mp.L1, t + 1 + (mp.offset ? mp.offset[b] : 0));
    s2 = 0;
    e2 = 0;
  } else if (mp.mode == ORTHRUS_MASK_DUAL) {
    const int64_t blk = min(t / mp.block, mp.A - 1);
    e1 = min(mp.L1, mp.anchors[b * mp.A + blk]);
    s2 = blk * mp.block;
    e2 = min(mp.L2, s2 + mp.block);
  } else if (mp.mode == ORTHRUS_MASK_TREE) {
    // the new tokens sit in the cache at rows base + t; source 2 is that same buffer
    const int64_t base = mp.offset ? mp.offset[b] : 0;
    e1 = min(mp.L1, base + 1);
    s2 = base + mp.limit2[t];
    e2 = min(mp.L2, base + t + 1);
  } else {
    e1 = min(mp.L1, static_cast<int64_t>(mp.offset ? mp.offset[b] : mp.L1));
    s2 = 0;
    e2 = mp.limit2 ? min(mp.L2, static_cast<int64_t>(mp.limit2[b])) : mp.L2;
  }
  if (e1 < 0) e1 = 0;
}

// First visible source-1 key of query t: 0, or with the document mask the start of the document
// of the query's own position (CAUSAL) or of its block's anchor (DUAL: the AR prefix keeps to the
// anchor's document).
__device__ __forceinline__ int64_t source1_start(const MaskParams& mp, int64_t b, int64_t t) {
  if (mp.doc_start == nullptr || mp.L1 <= 0) return 0;
  int64_t p;
  if (mp.mode == ORTHRUS_MASK_CAUSAL) {
    p = t + (mp.offset ? mp.offset[b] : 0);
  } else if (mp.mode == ORTHRUS_MASK_DUAL) {
    p = mp.anchors[b * mp.A + min(t / mp.block, mp.A - 1)];
  } else {
    return 0;
  }
  p = min(max(p, static_cast<int64_t>(0)), mp.L1 - 1);
  return mp.doc_start[b * mp.L1 + p];
}

constexpr int kSimtQ = 4;  // queries (warps) per CTA

// grid (ceil(Tq / kSimtQ), Hq, B), block 32 * kSimtQ. Source strides in elements.
template <typename T>
__global__ void __launch_bounds__(32 * kSimtQ) attn_fwd_simt_kernel(
    const T* __restrict__ q, const T* __restrict__ k1, const T* __restrict__ v1, int64_t s1h, int64_t s1b,
    const T* __restrict__ k2, const T* __restrict__ v2, int64_t s2h, int64_t s2b, int Hq, int Hkv, int64_t Tq,
    int hd, int D, float scale, MaskParams mp, T* __restrict__ o, float* __restrict__ lse) {
  __shared__ float sk[32][129];
  __shared__ float sv[32][128];
  __shared__ float sq[kSimtQ][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kSimtQ + warp;
  const bool live = t < Tq;
  int64_t e1 = 0, s2 = 0, e2 = 0;
  if (live) query_ranges(mp, b, t, e1, s2, e2);
  const int64_t s1 = live ? source1_start(mp, b, t) : 0;
  const T* qrow = q + ((b * Hq + h) * Tq + (live ? t : 0)) * D;
  for (int e = lane; e < hd; e += 32) sq[warp][e] = live ? to_f32<T>(qrow[e]) : 0.f;
  // CTA-wide key ranges
  __shared__ int64_t r1max, r2min, r2max;
  if (threadIdx.x == 0) {
    r1max = 0;
    r2min = INT64_MAX;
    r2max = 0;
  }
  __syncthreads();
  if (live && lane == 0) {
    atomicMax(reinterpret_cast<unsigned long long*>(&r1max), static_cast<unsigned long long>(e1));
    if (e2 > s2) {
      atomicMin(reinterpret_cast<unsigned long long*>(&r2min), static_cast<unsigned long long>(s2));
      atomicMax(reinterpret_cast<unsigned long long*>(&r2max), static_cast<unsigned long long>(e2));
    }
  }
  __syncthreads();
  float m = -INFINITY, l = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int src = 0; src < 2; ++src) {
    const T* K = src == 0 ? k1 + b * s1b + hk * s1h : k2 + b * s2b + hk * s2h;
    const T* Vv = src == 0 ? v1 + b * s1b + hk * s1h : v2 + b * s2b + hk * s2h;
    const int64_t lo = src == 0 ? 0 : (r2min / 32) * 32;
    const int64_t hi = src == 0 ? r1max : r2max;
    const int64_t my_lo = src == 0 ? s1 : s2, my_hi = src == 0 ? e1 : e2;
    if (src == 1 && (k2 == nullptr || r2max <= r2min)) break;
    for (int64_t k0 = lo; k0 < hi; k0 += 32) {
      __syncthreads();
      for (int i = threadIdx.x; i < 32 * hd; i += blockDim.x) {
        const int r = i / hd, e = i % hd;
        const int64_t key = k0 + r;
        const bool ok = key < hi;
        sk[r][e] = ok ? to_f32<T>(K[key * D + e]) : 0.f;
        sv[r][e] = ok ? to_f32<T>(Vv[key * D + e]) : 0.f;
      }
      __syncthreads();
      // no visible key in this tile (an empty range: a document starting at the block's anchor)
      if (!live || my_hi <= my_lo || k0 + 32 <= my_lo || k0 >= my_hi) continue;
      const int64_t key = k0 + lane;
      const bool vis = key >= my_lo && key < my_hi;
      float s = 0.f;
      for (int e = 0; e < hd; ++e) s = fmaf(sq[warp][e], sk[lane][e], s);
      s = vis ? s * scale : -INFINITY;
      float tm = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
      const float mn = fmaxf(m, tm);
      const float alpha = expf(m - mn);  // m = -inf at first: 0
      const float p = vis ? expf(s - mn) : 0.f;
      float ps = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l = l * alpha + ps;
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] *= alpha;
      for (int j = 0; j < 32; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = lane + 32 * k;
          if (e < hd) acc[k] = fmaf(pj, sv[j][e], acc[k]);
        }
      }
      m = mn;
    }
  }
  if (!live) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* orow = o + ((b * Tq + t) * Hq + h) * hd;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    if (e < hd) orow[e] = from_f32<T>(acc[k] * inv);
  }
  if (lse && lane == 0) lse[(b * Hq + h) * Tq + t] = m + logf(l);
}

// delta[b, h, t] = sum_e dO[b, t, h, e] * O[b, t, h, e] (fp32).
template <typename T>
__global__ void attn_delta_kernel(const T* __restrict__ o, const T* __restrict__ dout, int64_t B, int Hq,
                                  int64_t Tq, int hd, float* __restrict__ delta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp;  // (b, t, h)
  if (item >= B * Tq * Hq) return;
  const int h = static_cast<int>(item % Hq);
  const int64_t bt = item / Hq;
  const int64_t b = bt / Tq, t = bt % Tq;
  float acc = 0.f;
  for (int e = lane; e < hd; e += 32) acc = fmaf(to_f32<T>(o[item * hd + e]), to_f32<T>(dout[item * hd + e]), acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[(b * Hq + h) * Tq + t] = acc;
}

// Same delta for bf16 rows of 128: 16 lanes per (b, t, h) item, one 16-byte load of O and of dO
// per lane, then a fixed butterfly over the 16 lanes. 256 threads = 16 items per block.
__global__ void attn_delta128_bf16_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                          int64_t B, int Hq, int64_t Tq, float* __restrict__ delta) {
  const int sub = threadIdx.x & 15;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 16 + (threadIdx.x >> 4);  // (b, t, h)
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  const bool live = item < B * Tq * Hq;
  const int64_t it = live ? item : 0;
  const uint4 a = *reinterpret_cast<const uint4*>(o + it * 128 + sub * 8);
  const uint4 g = *reinterpret_cast<const uint4*>(dout + it * 128 + sub * 8);
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc = fmaf(__uint_as_float(aw[i] << 16), __uint_as_float(gw[i] << 16), acc);
    acc = fmaf(__uint_as_float(aw[i] & 0xffff0000u), __uint_as_float(gw[i] & 0xffff0000u), acc);
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && sub == 0) {
    const int h = static_cast<int>(item % Hq);
    const int64_t bt = item / Hq;
    delta[(bt / Tq * Hq + h) * Tq + bt % Tq] = acc;
  }
}

// dQ for every query (all visible keys of both sources), fp32 out [B, Hq, Tq, D].
template <typename T>
__global__ void __launch_bounds__(32 * kSimtQ) attn_dq_simt_kernel(
    const T* __restrict__ q, const T* __restrict__ k1, const T* __restrict__ v1, int64_t s1h, int64_t s1b,
    const T* __restrict__ k2, const T* __restrict__ v2, int64_t s2h, int64_t s2b, int Hq, int Hkv, int64_t Tq,
    int hd, int D, float scale, MaskParams mp, const float* __restrict__ lse, const float* __restrict__ delta,
    const T* __restrict__ dout, float* __restrict__ dq) {
  __shared__ float sk[32][129];
  __shared__ float sv[32][129];
  __shared__ float sq[kSimtQ][128];
  __shared__ float sdo[kSimtQ][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kSimtQ + warp;
  const bool live = t < Tq;
  int64_t e1 = 0, s2 = 0, e2 = 0;
  if (live) query_ranges(mp, b, t, e1, s2, e2);
  const int64_t s1 = live ? source1_start(mp, b, t) : 0;
  const int64_t qi = (b * Hq + h) * Tq + (live ? t : 0);
  for (int e = lane; e < hd; e += 32) {
    sq[warp][e] = live ? to_f32<T>(q[qi * D + e]) : 0.f;
    sdo[warp][e] = live ? to_f32<T>(dout[((b * Tq + (live ? t : 0)) * Hq + h) * hd + e]) : 0.f;
  }
  const float L = live ? lse[qi] : 0.f;
  const float dl = live ? delta[qi] : 0.f;
  __shared__ int64_t r1max, r2min, r2max;
  if (threadIdx.x == 0) {
    r1max = 0;
    r2min = INT64_MAX;
    r2max = 0;
  }
  __syncthreads();
  if (live && lane == 0) {
    atomicMax(reinterpret_cast<unsigned long long*>(&r1max), static_cast<unsigned long long>(e1));
    if (e2 > s2) {
      atomicMin(reinterpret_cast<unsigned long long*>(&r2min), static_cast<unsigned long long>(s2));
      atomicMax(reinterpret_cast<unsigned long long*>(&r2max), static_cast<unsigned long long>(e2));
    }
  }
  __syncthreads();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int src = 0; src < 2; ++src) {
    if (src == 1 && (k2 == nullptr || r2max <= r2min)) break;
    const T* K = src == 0 ? k1 + b * s1b + hk * s1h : k2 + b * s2b + hk * s2h;
    const T* Vv = src == 0 ? v1 + b * s1b + hk * s1h : v2 + b * s2b + hk * s2h;
    const int64_t lo = src == 0 ? 0 : (r2min / 32) * 32;
    const int64_t hi = src == 0 ? r1max : r2max;
    const int64_t my_lo = src == 0 ? s1 : s2, my_hi = src == 0 ? e1 : e2;
    for (int64_t k0 = lo; k0 < hi; k0 += 32) {
      __syncthreads();
      for (int i = threadIdx.x; i < 32 * hd; i += blockDim.x) {
        const int r = i / hd, e = i % hd;
        const int64_t key = k0 + r;
        const bool ok = key < hi;
        sk[r][e] = ok ? to_f32<T>(K[key * D + e]) : 0.f;
        sv[r][e] = ok ? to_f32<T>(Vv[key * D + e]) : 0.f;
      }
      __syncthreads();
      if (!live || my_hi <= my_lo || k0 + 32 <= my_lo || k0 >= my_hi) continue;
      const int64_t key = k0 + lane;
      const bool vis = key >= my_lo && key < my_hi;
      float s = 0.f, dp = 0.f;
      for (int e = 0; e < hd; ++e) {
        s = fmaf(sq[warp][e], sk[lane][e], s);
        dp = fmaf(sdo[warp][e], sv[lane][e], dp);
      }
      const float p = vis ? expf(s * scale - L) : 0.f;
      const float ds = p * (dp - dl);
      for (int j = 0; j < 32; ++j) {
        const float dsj = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = lane + 32 * k;
          if (e < hd) acc[k] = fmaf(dsj, sk[j][e], acc[k]);
        }
      }
    }
  }
  if (!live) return;
  float* out = dq + qi * D;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    if (e < D) out[e] = e < hd ? acc[k] * scale : 0.f;
  }
}

// dK / dV of the source-2 (block) keys under the dual mask: one warp per key, looping over the
// block's queries of every head of the group in a fixed order. fp32 out [B, Hkv, L2, D].
template <typename T>
__global__ void __launch_bounds__(256) attn_dkdv_block_simt_kernel(
    const T* __restrict__ q, const T* __restrict__ k2, const T* __restrict__ v2, int64_t s2h, int64_t s2b,
    int Hq, int Hkv, int64_t Tq, int hd, int D, float scale, int block, int64_t L2, const float* __restrict__ lse,
    const float* __restrict__ delta, const T* __restrict__ dout, float* __restrict__ dk, float* __restrict__ dv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t B = gridDim.z;
  const int hk = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t j = static_cast<int64_t>(blockIdx.x) * 8 + warp;  // key index in source 2
  if (j >= L2) return;
  (void)B;
  const T* kr = k2 + b * s2b + hk * s2h + j * D;
  const T* vr = v2 + b * s2b + hk * s2h + j * D;
  float kk[4], vv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    kk[k] = e < hd ? to_f32<T>(kr[e]) : 0.f;
    vv[k] = e < hd ? to_f32<T>(vr[e]) : 0.f;
  }
  const int G = Hq / Hkv;
  const int64_t q0 = (j / block) * block, q1 = min(Tq, q0 + block);
  float adk[4] = {0.f, 0.f, 0.f, 0.f}, adv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int g = 0; g < G; ++g) {
    const int h = hk * G + g;
    for (int64_t t = q0; t < q1; ++t) {
      const int64_t qi = (b * Hq + h) * Tq + t;
      const T* qr = q + qi * D;
      const T* dor = dout + ((b * Tq + t) * Hq + h) * hd;
      float qv[4], dov[4];
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = lane + 32 * k;
        qv[k] = e < hd ? to_f32<T>(qr[e]) : 0.f;
        dov[k] = e < hd ? to_f32<T>(dor[e]) : 0.f;
        s = fmaf(qv[k], kk[k], s);
        dp = fmaf(dov[k], vv[k], dp);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, off);
        dp += __shfl_xor_sync(0xffffffffu, dp, off);
      }
      const float p = expf(s * scale - lse[qi]);
      const float ds = p * (dp - delta[qi]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        adv[k] = fmaf(p, dov[k], adv[k]);
        adk[k] = fmaf(ds, qv[k], adk[k]);
      }
    }
  }
  float* dkr = dk + ((b * Hkv + hk) * L2 + j) * D;
  float* dvr = dv + ((b * Hkv + hk) * L2 + j) * D;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = lane + 32 * k;
    if (e < D) {
      dkr[e] = e < hd ? adk[k] * scale : 0.f;
      dvr[e] = e < hd ? adv[k] : 0.f;
    }
  }
}

}  // namespace orthrus
