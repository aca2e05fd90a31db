// Attention of the decode passes (a block of at most 64 query rows per sequence over its KV
// cache), split over the keys so that a batch of one still spreads over the GPU.
//
// The verify pass (causal over the cache, orthrus/modeling_orthrus.py:489-497) and the draft pass
// (the cache before the block plus the block's own keys, :469-481) read the whole cache for a few
// query rows: the work is the K/V read, and the 128-row tensor-core tiles of the training kernels
// would run one CTA per KV head with three quarters of their rows empty. Here the keys of source 1
// are cut into splits of 128 from key 0 and the draft block's keys form one more split; one CTA of
// 16-row warps takes one (split, KV head, sequence), scores all G * Tq query rows of the KV head's
// G query heads against its keys with warp-level bf16 MMAs (mma.sync m16n8k16, fp32 accumulation;
// Q, K and V staged once by cp.async into padded shared rows), and writes each row's partial
// softmax state (max, sum, unnormalised output). A second kernel merges a row's splits in split
// order.
//
// Everything a row computes depends only on its own visible keys and on key positions (the split
// and 64-key sub-chunk boundaries are multiples of 64 from key 0), never on which other rows share
// the launch: a 32-row verification pass reproduces one-token greedy passes bit for bit, which is
// what makes block decoding lossless.
#pragma once

#include "attention_blockkv.cuh"
#include "attention_simt.cuh"

namespace orthrus {

constexpr int kDecSplit = 128;  // keys per split
constexpr int kDecSub = 64;     // keys per sub-chunk (one QK^T / PV round)
constexpr int kDecRow = 272;    // bytes of a padded [128] bf16 shared row (conflict-free ldmatrix)
constexpr int kDecMaxRows = 128;

__host__ __device__ inline int64_t decode_splits1(int64_t L1) { return (L1 + kDecSplit - 1) / kDecSplit; }

__host__ __device__ inline int decode_smem_bytes(int rows) {
  const int warps_rows = ((rows + 15) / 16) * 16;
  return warps_rows * kDecRow + 4 * kDecSub * kDecRow;  // Q rows, then K0, V0, K1, V1
}

// The end of the visible keys of source `src` over all rows of sequence b (what the CTAs load):
// the largest e1 (or e2) query_ranges gives any of the Tq rows.
__device__ __forceinline__ int64_t decode_source_end(const MaskParams& mp, int64_t b, int src, int64_t Tq) {
  if (src == 0) {
    int64_t e;
    if (mp.mode == ORTHRUS_MASK_CAUSAL) {
      e = min(mp.L1, Tq + (mp.offset ? mp.offset[b] : 0));
    } else {
      e = min(mp.L1, static_cast<int64_t>(mp.offset ? mp.offset[b] : mp.L1));
    }
    return max(e, static_cast<int64_t>(0));
  }
  return mp.limit2 ? min(mp.L2, static_cast<int64_t>(mp.limit2[b])) : mp.L2;
}

// grid (ns1 + has2, Hkv, B), 32 * ceil(G * Tq / 16) threads. part_o fp32 [S, B, Hq, Tq, 128],
// part_ml fp32 [S, B, Hq, Tq, 2] (max in log2 units, sum).
__global__ void __launch_bounds__(256) attn_decode_split_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k1, const __nv_bfloat16* __restrict__ v1,
    int64_t s1h, int64_t s1b, const __nv_bfloat16* __restrict__ k2, const __nv_bfloat16* __restrict__ v2, int64_t s2h,
    int64_t s2b, int Hq, int Hkv, int Tq, float sl2, MaskParams mp, int ns1, float* __restrict__ part_o,
    float* __restrict__ part_ml) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int split = blockIdx.x, g = blockIdx.y;
  const int64_t b = blockIdx.z, B = gridDim.z;
  const int G = Hq / Hkv, rows = G * Tq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nthreads = blockDim.x;
  griddep_launch_dependents();  // launched as a programmatic dependent
  // Before griddep_wait() only what the kernels still running ahead of this one never write: the
  // cycle's positions (offset, limit2) and the cache rows below offset[b], written by earlier
  // passes. Q and this pass's own keys (the block's rows of the cache, or source 2) come after it.
  const int src = split >= ns1 ? 1 : 0;
  const int64_t key0 = src == 0 ? static_cast<int64_t>(split) * kDecSplit : 0;
  const int64_t kend = decode_source_end(mp, b, src, Tq);
  if (key0 >= kend) return;  // no row's visible keys reach this split: nobody reads its partial
  const int nkeys = static_cast<int>(min(static_cast<int64_t>(src == 0 ? kDecSplit : kDecSub), kend - key0));
  // keys [0, nold) of this split are earlier passes' cache rows
  const int64_t prior = src == 0 ? (mp.offset ? static_cast<int64_t>(mp.offset[b]) : 0) : 0;
  const int nold = static_cast<int>(min(static_cast<int64_t>(nkeys), max(prior - key0, static_cast<int64_t>(0))));
  const __nv_bfloat16* K = src == 0 ? k1 + b * s1b + g * s1h : k2 + b * s2b + g * s2h;
  const __nv_bfloat16* V = src == 0 ? v1 + b * s1b + g * s1h : v2 + b * s2b + g * s2h;
  const int qrows = ((rows + 15) / 16) * 16;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = sQ + qrows * kDecRow;  // sub-chunk c: K at sKV + 2c * TILE, V after it
  constexpr int TILE = kDecSub * kDecRow;
  // keys of sub-chunk c in [lo_key, hi_key) of the split: copies, or zeros past the loaded range
  auto stage_keys = [&](int c, int lo_key, int hi_key, bool zero_rest) {
    for (int i = threadIdx.x; i < kDecSub * 16; i += nthreads) {
      const int kk = i >> 4, ch = i & 15;
      const int key = c * kDecSub + kk;
      const uint32_t dk = sKV + (2 * c) * TILE + kk * kDecRow + ch * 16, dv = dk + TILE;
      if (key >= lo_key && key < hi_key) {
        cp_async16(dk, K + (key0 + key) * 128 + ch * 8);
        cp_async16(dv, V + (key0 + key) * 128 + ch * 8);
      } else if (zero_rest && key >= nkeys) {  // masked scores, and P = 0 times a finite V
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dk), "r"(0) : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dv), "r"(0) : "memory");
      }
    }
  };
  // groups 1, 2: the earlier passes' keys of sub-chunks 0 and 1, in flight during the wait
  stage_keys(0, 0, nold, true);
  asm volatile("cp.async.commit_group;" ::: "memory");
  stage_keys(1, 0, nold, true);
  asm volatile("cp.async.commit_group;" ::: "memory");
  griddep_wait();
  // groups 3, 4: Q (zero rows past the last) with this pass's keys of sub-chunk 0, then of sub-chunk 1
  for (int i = threadIdx.x; i < qrows * 16; i += nthreads) {
    const int r = i >> 4, c = i & 15;
    const uint32_t dst = sQ + r * kDecRow + c * 16;
    if (r < rows) {
      const int hh = g * G + r / Tq, t = r % Tq;
      cp_async16(dst, q + ((b * Hq + hh) * static_cast<int64_t>(Tq) + t) * 128 + c * 8);
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
    }
  }
  stage_keys(0, nold, nkeys, false);
  asm volatile("cp.async.commit_group;" ::: "memory");
  stage_keys(1, nold, nkeys, false);
  asm volatile("cp.async.commit_group;" ::: "memory");
  // the two rows of this thread: 16 * warp + lane / 4 (+ 8)
  const int rA = 16 * warp + (lane >> 2), rB = rA + 8;
  int64_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = i == 0 ? rA : rB;
    if (r < rows) {
      int64_t e1, s2, e2;
      query_ranges(mp, b, r % Tq, e1, s2, e2);
      lo[i] = src == 0 ? 0 : s2;
      hi[i] = src == 0 ? e1 : e2;
    }
  }
  uint32_t qa[8][4];
  float o[16][4];
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  const bool active = 16 * warp < rows;
  for (int c = 0; c < 2; ++c) {
    if (c == 0) {  // groups 1-3: sub-chunk 0 complete (group 2, sub-chunk 1's earlier keys, too)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int64_t cbase = key0 + c * kDecSub;
    if (cbase >= kend) break;  // the same for the whole CTA
    if (!active) continue;
    if (c == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int row = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int col = 16 * kk + 8 * (lane >> 4);
        ldsm_x4(sQ + row * kDecRow + col * 2, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    const uint32_t sK = sKV + (2 * c) * TILE, sV = sK + TILE;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // key n-tiles 2jp, 2jp + 1
        const int key = 16 * jp + (lane & 7) + 8 * (lane >> 4);
        const int dim = 16 * kk + 8 * ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK + key * kDecRow + dim * 2, b0, b1, b2, b3);
        mma_bf16_16816(s[2 * jp], qa[kk], b0, b1);
        mma_bf16_16816(s[2 * jp + 1], qa[kk], b2, b3);
      }
    }
    // mask, scale to log2 units, online softmax per row
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e >> 1;
        const int64_t key = cbase + 8 * j + 2 * (lane & 3) + (e & 1);
        const bool vis = key >= lo[i] && key < hi[i];
        s[j][e] = vis ? s[j][e] * sl2 : -INFINITY;
        mx[i] = fmaxf(mx[i], s[j][e]);
      }
    }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mn = fmaxf(m[i], mx[i]);
      alpha[i] = mn == m[i] ? 1.f : ex2_approx(m[i] - mn);  // m = -inf before the first visible key: 0
      m[i] = mn;
    }
    uint32_t pa[4][4];
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e >> 1;
        p[e] = s[j][e] == -INFINITY ? 0.f : ex2_approx(s[j][e] - m[i]);
        ps[i] += p[e];
      }
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) l[i] = l[i] * alpha[i] + ps[i];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // O += P V: A = P (16 rows x 16 keys per step), B = V [key][dim] through ldmatrix.trans
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a[4] = {pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3]};
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {  // dim n-tiles 2jp, 2jp + 1
        const int key = 16 * ks + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int dim = 16 * jp + 8 * (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV + key * kDecRow + dim * 2, b0, b1, b2, b3);
        mma_bf16_16816(o[2 * jp], a, b0, b1);
        mma_bf16_16816(o[2 * jp + 1], a, b2, b3);
      }
    }
  }
  if (!active) return;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
    l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = i == 0 ? rA : rB;
    if (r >= rows) continue;
    const int hh = g * G + r / Tq, t = r % Tq;
    const int64_t idx = ((static_cast<int64_t>(split) * B + b) * Hq + hh) * Tq + t;
    if ((lane & 3) == 0) *reinterpret_cast<float2*>(part_ml + idx * 2) = make_float2(m[i], l[i]);
    float* dst = part_o + idx * 128 + 2 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 16; ++j) *reinterpret_cast<float2*>(dst + 8 * j) = make_float2(o[j][2 * i], o[j][2 * i + 1]);
  }
}

// One warp per (b, head, t) row: merge the row's splits in split order, o bf16 [B, Tq, Hq, 128].
__global__ void __launch_bounds__(256) attn_decode_combine_kernel(const float* __restrict__ part_o,
                                                                  const float* __restrict__ part_ml, int64_t B, int Hq,
                                                                  int Tq, int ns1, MaskParams mp,
                                                                  __nv_bfloat16* __restrict__ o) {
  griddep_launch_dependents();
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (item >= B * Hq * Tq) return;
  const int t = static_cast<int>(item % Tq);
  const int hh = static_cast<int>((item / Tq) % Hq);
  const int64_t b = item / (static_cast<int64_t>(Tq) * Hq);
  int64_t e1, s2, e2;
  query_ranges(mp, b, t, e1, s2, e2);
  const int n1 = static_cast<int>((max(e1, static_cast<int64_t>(0)) + kDecSplit - 1) / kDecSplit);
  const bool has2 = mp.mode == ORTHRUS_MASK_DRAFT && e2 > s2;
  auto part = [&](int s) { return ((static_cast<int64_t>(s) * B + b) * Hq + hh) * Tq + t; };
  float M = -INFINITY;
#pragma unroll 4
  for (int s = 0; s < n1; ++s) M = fmaxf(M, part_ml[part(s) * 2]);
  if (has2) M = fmaxf(M, part_ml[part(ns1) * 2]);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int k = 0; k < n1 + (has2 ? 1 : 0); ++k) {  // unrolled so the loads of several splits are in flight
    const int s = k < n1 ? k : ns1;
    const int64_t idx = part(s);
    const float ms = part_ml[idx * 2], ls = part_ml[idx * 2 + 1];
    const float w = ms == -INFINITY ? 0.f : ex2_approx(ms - M);
    L += ls * w;
    const float4 x = *reinterpret_cast<const float4*>(part_o + idx * 128 + lane * 4);
    acc.x += w * x.x;
    acc.y += w * x.y;
    acc.z += w * x.z;
    acc.w += w * x.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __nv_bfloat16* dst = o + ((b * Tq + t) * Hq + hh) * 128 + lane * 4;
  *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
}

}  // namespace orthrus
