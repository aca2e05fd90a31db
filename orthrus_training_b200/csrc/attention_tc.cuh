// Dual-view attention on the 5th-generation tensor cores (bf16 in, fp32 accumulate in TMEM).
//
// Three kernels, all with the same CTA shape (192 threads: warp 0 = TMA producer, warp 1 = TMEM
// owner and single-thread tcgen05.mma issuer, warps 2-5 = 128 "row" threads, one per TMEM lane):
//
//   attn_fwd_tc      CTA = 128 query rows of one head. Visits only the key tiles the mask can
//                    reach (the per-anchor tile map: source-1 tiles below the largest anchor of
//                    the tile, plus the own-block tile of source 2), S = Q K^T into one of two TMEM
//                    buffers, online softmax in registers, P (bf16) to shared memory,
//                    O_j = P V into one of two TMEM buffers, O += alpha-rescaled O_j in registers.
//   attn_dq_tc       CTA = 128 query rows of one head: S = Q K^T and dP = dO V^T per visible key
//                    tile, dS = P (dP - delta) to shared memory, dQ += dS K accumulated in TMEM.
//   attn_dkdv_tc     CTA = 128 block keys of one KV head: for every query head of the group,
//                    S^T = K Q^T, dP^T = V dO^T, then dV += P^T dO and dK += dS^T Q in TMEM. Only the
//                    own-block keys get gradients: source-1 keys belong to the frozen teacher
//                    (the reference's skip_ar_key_grads, orthrus/objective.py:168-198).
//
// Operand tiles are [128 rows][D] bf16 loaded by TMA as D/64 boxes of [128][64] with 128-byte
// swizzle. The same tile is a K-major UMMA operand when the reduction runs over the head dim
// (Q K^T, dO V^T) and an MN-major operand when it runs over the rows (P V, dS K, P^T dO, dS^T Q).
#pragma once

#include "attention_simt.cuh"

namespace orthrus {

constexpr int kAttnTileBytes = 128 * 64 * 2;  // one [128][64] bf16 box = 16 KB

// K-major descriptor of k-step kk (16 elements) of a [128][D] tile stored as D/64 boxes.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int kk) {
  return umma_desc_sw128(base + (kk >> 2) * kAttnTileBytes + (kk & 3) * 32, 16, 1024);
}
// MN-major descriptor of k-step kk (16 rows) of a [128 rows][D] tile (D along MN).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int kk) {
  return umma_desc_sw128(base + kk * 2048, kAttnTileBytes, 1024);
}

// Writes 32 consecutive bf16 values (columns c0..c0+31 of row r) into a K-major swizzled tile.
__device__ __forceinline__ void store_row32_sw128(uint32_t tile_base, int r, int c0, const float* v) {
  const uint32_t box = tile_base + (c0 >> 6) * kAttnTileBytes;
  const int chunk0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    st_shared_v4(box + sw128_offset(r, chunk0 + q), pack_bf16x2(v[8 * q], v[8 * q + 1]),
                 pack_bf16x2(v[8 * q + 2], v[8 * q + 3]), pack_bf16x2(v[8 * q + 4], v[8 * q + 5]),
                 pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
}

// Same store from 16 words that already hold the 32 values as bf16 pairs.
__device__ __forceinline__ void store_row32_sw128_packed(uint32_t tile_base, int r, int c0, const uint32_t* w) {
  const uint32_t box = tile_base + (c0 >> 6) * kAttnTileBytes;
  const int chunk0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    st_shared_v4(box + sw128_offset(r, chunk0 + q), w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// How the columns [c0, c0 + width) of a score tile meet the visible ranges [lo, hi) of the 32 rows
// of this warp: 0 = no row sees any of them, 1 = every row sees all of them, 2 = mixed. The answer
// is the same in every lane, so a branch on it may hold warp-collective TMEM loads. All 32 lanes
// must call it.
__device__ __forceinline__ int chunk_kind_warp(int64_t lo, int64_t hi, int c0, int width) {
  const bool none = hi <= c0 || lo >= c0 + width || hi <= lo;
  const bool full = lo <= c0 && hi >= c0 + width;
  if (__all_sync(0xffffffffu, none)) return 0;
  if (__all_sync(0xffffffffu, full)) return 1;
  return 2;
}

struct AttnTiles {
  int n1;        // source-1 tiles [0, n1)
  int t2a, n2;   // source-2 tiles [t2a, t2a + n2)
};

// Row-thread part of the tile map: reduce the key ranges of the CTA's rows.
__device__ __forceinline__ void attn_tile_map(const MaskParams& mp, int64_t b, int64_t q0, int64_t Tq, bool has2,
                                              int row_thread, unsigned long long* red, AttnTiles* out) {
  // red[0] = max e1, red[1] = min s2, red[2] = max e2
  if (row_thread >= 0) {
    const int64_t t = q0 + row_thread;
    if (t < Tq) {
      int64_t e1, s2, e2;
      query_ranges(mp, b, t, e1, s2, e2);
      atomicMax(&red[0], static_cast<unsigned long long>(e1));
      if (has2 && e2 > s2) {
        atomicMin(&red[1], static_cast<unsigned long long>(s2));
        atomicMax(&red[2], static_cast<unsigned long long>(e2));
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    out->n1 = static_cast<int>((red[0] + 127) / 128);
    if (red[2] > red[1]) {
      out->t2a = static_cast<int>(red[1] / 128);
      out->n2 = static_cast<int>((red[2] + 127) / 128) - out->t2a;
    } else {
      out->t2a = 0;
      out->n2 = 0;
    }
  }
  __syncthreads();
}

template <int D>
struct FwdSmem {
  static constexpr int BOXES = D / 64;
  static constexpr int TILE = BOXES * kAttnTileBytes;  // [128][D]
  static constexpr int STAGES = 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = TILE;                         // stage s: K at +2s*TILE, V at +(2s+1)*TILE
  static constexpr int OFF_P = OFF_KV + 2 * STAGES * TILE;    // P: [128][128] = 2 boxes
  static constexpr int OFF_BAR = OFF_P + 2 * kAttnTileBytes;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK1,
                       const __grid_constant__ CUtensorMap tmV1, const __grid_constant__ CUtensorMap tmK2,
                       const __grid_constant__ CUtensorMap tmV2, int Hq, int Hkv, int64_t Tq, int hd,
                       float scale_log2, MaskParams mp, bool has2, __nv_bfloat16* __restrict__ o,
                       float* __restrict__ lse) {
  using S = FwdSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* p_empty = bars + 10;
  uint64_t* o_full = bars + 11;   // [2]
  uint64_t* o_empty = bars + 13;  // [2]
  unsigned long long* red = reinterpret_cast<unsigned long long*>(bars + 16);  // [3]
  AttnTiles* tiles = reinterpret_cast<AttnTiles*>(bars + 20);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 128;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int row_thread = warp >= 2 ? (warp & 3) * 32 + lane : -1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(p_full, 128);
    mbar_init(p_empty, 1);
    red[0] = 0;
    red[1] = ~0ull;
    red[2] = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  // a programmatic dependent launch may start this kernel during the previous one: the tile map,
  // the operands and the outputs belong to the stream order only after griddep_wait()
  griddep_launch_dependents();
  griddep_wait();
  attn_tile_map(mp, b, q0, Tq, has2, row_thread, red, tiles);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n1 = tiles->n1, t2a = tiles->t2a;
  const int nt = n1 + tiles->n2;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, S::TILE);
#pragma unroll
      for (int c = 0; c < S::BOXES; ++c)
        tma_load_3d(smem + S::OFF_Q + c * kAttnTileBytes, &tmQ, q_full, c * 64, static_cast<int>(q0),
                    static_cast<int>(b * Hq + h));
      int issued = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        const bool src2 = j >= n1;
        const int key0 = (src2 ? t2a + (j - n1) : j) * 128;
        const CUtensorMap* mk = src2 ? &tmK2 : &tmK1;
        const CUtensorMap* mv = src2 ? &tmV2 : &tmV1;
        uint8_t* kt = smem + S::OFF_KV + (2 * s) * S::TILE;
        uint8_t* vt = kt + S::TILE;
        mbar_arrive_expect_tx(&kv_full[s], 2 * S::TILE);
#pragma unroll
        for (int c = 0; c < S::BOXES; ++c) {
          tma_load_3d(kt + c * kAttnTileBytes, mk, &kv_full[s], c * 64, key0, static_cast<int>(b * Hkv + hk));
          tma_load_3d(vt + c * kAttnTileBytes, mv, &kv_full[s], c * 64, key0, static_cast<int>(b * Hkv + hk));
        }
        issued = j + 1;
      }
      if (*abort_flag) {
        mbar_wait_short(q_full, 0);
        for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait_short(&kv_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, false, true);
      const uint32_t q_base = smem_u32(smem + S::OFF_Q);
      const uint32_t p_base = smem_u32(smem + S::OFF_P);
      bool ok = mbar_wait(q_full, 0);
      auto issue_pv = [&](int j) -> bool {
        // O_j = P_j V_j into O buffer j & 1
        if (!mbar_wait(p_full, j & 1)) return false;
        if (!mbar_wait(&o_empty[j & 1], ((j >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + S::OFF_KV + (2 * (j & 1) + 1) * S::TILE);
        const uint32_t acc = tmem + 256 + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(acc, desc_kmajor(p_base, kk), desc_mnmajor(v_base, kk), idesc_o, kk > 0 ? 1u : 0u);
        umma_commit(&o_full[j & 1]);
        umma_commit(&kv_empty[j & 1]);
        umma_commit(p_empty);
        return true;
      };
      for (int j = 0; ok && j < nt; ++j) {
        if (*abort_flag || !mbar_wait(&kv_full[j & 1], (j >> 1) & 1) ||
            !mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + S::OFF_KV + (2 * (j & 1)) * S::TILE);
        const uint32_t acc = tmem + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(acc, desc_kmajor(q_base, kk), desc_kmajor(k_base, kk), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nt >= 1 && !issue_pv(nt - 1)) ok = false;
      if (!ok) *abort_flag = 1;
      umma_commit(p_empty);  // completes once all issued MMAs are done (drain on every path)
    }
  } else {
    const int r = row_thread;
    const int64_t t = q0 + r;
    const bool live = t < Tq;
    int64_t e1 = 0, s2 = 0, e2 = 0;
    if (live) query_ranges(mp, b, t, e1, s2, e2);
    const int64_t s1 = live ? source1_start(mp, b, t) : 0;
    if (!has2) e2 = s2 = 0;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t p_base = smem_u32(smem + S::OFF_P);
    float m = -INFINITY, l = 0.f;
    float acc[D];
#pragma unroll
    for (int i = 0; i < D; ++i) acc[i] = 0.f;
    float alpha_prev = 0.f;
    bool ok = true;
    auto correction = [&](int j, float alpha) -> bool {
      if (!mbar_wait(&o_full[j & 1], (j >> 1) & 1)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float x[32];
        tmem_ld32(lane_base + 256 + (j & 1) * 128 + c * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[c * 32 + i] = fmaf(acc[c * 32 + i], alpha, x[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[j & 1]);
      return true;
    };
    for (int j = 0; j < nt; ++j) {
      if (*abort_flag || !mbar_wait(&s_full[j & 1], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool src2 = j >= n1;
      const int64_t key0 = (src2 ? t2a + (j - n1) : j) * 128;
      const int64_t lo = src2 ? s2 : s1, hi = src2 ? e2 : e1;
      const uint32_t sb = lane_base + (j & 1) * 128;
      // pass 1: masked row max (log2 units)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32];
        tmem_ld32(sb + c * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int64_t key = key0 + c * 32 + i;
          if (key >= lo && key < hi) tmax = fmaxf(tmax, x[i] * scale_log2);
        }
      }
      const float m_new = fmaxf(m, tmax);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      // pass 2: P = exp2(s - m) to shared memory (after the previous P V has read the buffer)
      if (!mbar_wait(p_empty, (j & 1) ^ 1)) {
        ok = false;
        break;
      }
      float rsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32];
        tmem_ld32(sb + c * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int64_t key = key0 + c * 32 + i;
          const float p = (key >= lo && key < hi) ? exp2f(fmaf(x[i], scale_log2, -m_use)) : 0.f;
          x[i] = p;
          rsum += p;
        }
        store_row32_sw128(p_base, r, c * 32, x);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[j & 1]);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
      l = l * alpha + rsum;
      m = m_new;
      if (j >= 1 && !correction(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && nt >= 1 && !correction(nt - 1, alpha_prev)) ok = false;
    if (!ok) *abort_flag = 1;
    if (ok && live) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = o + ((b * Tq + t) * Hq + h) * hd;
      if (hd == D) {
#pragma unroll
        for (int i = 0; i < D; i += 8) {
          uint4 pk = make_uint4(pack_bf16x2(acc[i] * inv, acc[i + 1] * inv), pack_bf16x2(acc[i + 2] * inv, acc[i + 3] * inv),
                                pack_bf16x2(acc[i + 4] * inv, acc[i + 5] * inv), pack_bf16x2(acc[i + 6] * inv, acc[i + 7] * inv));
          *reinterpret_cast<uint4*>(orow + i) = pk;
        }
      } else {
#pragma unroll
        for (int i = 0; i < D; ++i)
          if (i < hd) orow[i] = __float2bfloat16_rn(acc[i] * inv);
      }
      if (lse) lse[(b * Hq + h) * Tq + t] = (m + log2f(l)) * kLn2;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// Backward: dQ
// ------------------------------------------------------------------------------------------------

template <int D>
struct DqSmem {
  static constexpr int BOXES = D / 64;
  static constexpr int TILE = BOXES * kAttnTileBytes;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = TILE;
  static constexpr int OFF_KV = 2 * TILE;  // 2 stages of (K, V)
  static constexpr int OFF_DS = OFF_KV + 4 * TILE;
  static constexpr int OFF_BAR = OFF_DS + 2 * kAttnTileBytes;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                      const __grid_constant__ CUtensorMap tmK1, const __grid_constant__ CUtensorMap tmV1,
                      const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2, int Hq,
                      int Hkv, int64_t Tq, int hd, float scale, MaskParams mp, bool has2,
                      const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq) {
  using S = DqSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* in_full = bars + 0;   // Q and dO
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // S and dP ready
  uint64_t* s_empty = bars + 6;   // S and dP read (4 warps)
  uint64_t* ds_full = bars + 7;   // dS written (128 threads)
  uint64_t* ds_empty = bars + 8;  // dS consumed by the dQ MMA
  uint64_t* dq_full = bars + 9;
  unsigned long long* red = reinterpret_cast<unsigned long long*>(bars + 16);
  AttnTiles* tiles = reinterpret_cast<AttnTiles*>(bars + 20);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 128;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int row_thread = warp >= 2 ? (warp & 3) * 32 + lane : -1;

  if (threadIdx.x == 0) {
    mbar_init(in_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 4);
    mbar_init(ds_full, 128);
    mbar_init(ds_empty, 1);
    mbar_init(dq_full, 1);
    red[0] = 0;
    red[1] = ~0ull;
    red[2] = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  // a programmatic dependent launch may start this kernel during the previous one: the tile map,
  // the operands and the outputs belong to the stream order only after griddep_wait()
  griddep_launch_dependents();
  griddep_wait();
  attn_tile_map(mp, b, q0, Tq, has2, row_thread, red, tiles);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S: [0,128), dP: [128,256), dQ: [256, 256+D)
  const int n1 = tiles->n1, t2a = tiles->t2a;
  const int nt = n1 + tiles->n2;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(in_full, 2 * S::TILE);
#pragma unroll
      for (int c = 0; c < S::BOXES; ++c) {
        tma_load_3d(smem + S::OFF_Q + c * kAttnTileBytes, &tmQ, in_full, c * 64, static_cast<int>(q0),
                    static_cast<int>(b * Hq + h));
        tma_load_3d(smem + S::OFF_DO + c * kAttnTileBytes, &tmDO, in_full, c * 64 + h * hd, static_cast<int>(q0),
                    static_cast<int>(b));
      }
      int issued = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        const bool src2 = j >= n1;
        const int key0 = (src2 ? t2a + (j - n1) : j) * 128;
        uint8_t* kt = smem + S::OFF_KV + (2 * s) * S::TILE;
        uint8_t* vt = kt + S::TILE;
        mbar_arrive_expect_tx(&kv_full[s], 2 * S::TILE);
#pragma unroll
        for (int c = 0; c < S::BOXES; ++c) {
          tma_load_3d(kt + c * kAttnTileBytes, src2 ? &tmK2 : &tmK1, &kv_full[s], c * 64, key0,
                      static_cast<int>(b * Hkv + hk));
          tma_load_3d(vt + c * kAttnTileBytes, src2 ? &tmV2 : &tmV1, &kv_full[s], c * 64, key0,
                      static_cast<int>(b * Hkv + hk));
        }
        issued = j + 1;
      }
      if (*abort_flag) {
        mbar_wait_short(in_full, 0);
        for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait_short(&kv_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_q = umma_idesc_bf16(128, D, false, true);
      const uint32_t q_base = smem_u32(smem + S::OFF_Q);
      const uint32_t do_base = smem_u32(smem + S::OFF_DO);
      const uint32_t ds_base = smem_u32(smem + S::OFF_DS);
      bool ok = mbar_wait(in_full, 0);
      for (int j = 0; ok && j < nt; ++j) {
        if (*abort_flag || !mbar_wait(&kv_full[j & 1], (j >> 1) & 1) || !mbar_wait(s_empty, (j & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + S::OFF_KV + (2 * (j & 1)) * S::TILE);
        const uint32_t v_base = k_base + S::TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16(tmem, desc_kmajor(q_base, kk), desc_kmajor(k_base, kk), idesc_s, kk > 0 ? 1u : 0u);
          umma_f16(tmem + 128, desc_kmajor(do_base, kk), desc_kmajor(v_base, kk), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        // dQ += dS_j K_j once the row threads wrote dS_j
        if (!mbar_wait(ds_full, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem + 256, desc_kmajor(ds_base, kk), desc_mnmajor(k_base, kk), idesc_q,
                   (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(ds_empty);
        umma_commit(&kv_empty[j & 1]);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(dq_full);
    }
  } else {
    const int r = row_thread;
    const int64_t t = q0 + r;
    const bool live = t < Tq;
    int64_t e1 = 0, s2 = 0, e2 = 0;
    if (live) query_ranges(mp, b, t, e1, s2, e2);
    const int64_t s1 = live ? source1_start(mp, b, t) : 0;
    if (!has2) e2 = s2 = 0;
    const int64_t qi = (b * Hq + h) * Tq + (live ? t : 0);
    const float L2e = live ? lse[qi] * kLog2e : 0.f;
    const float dl = live ? delta[qi] : 0.f;
    const float sl2 = scale * kLog2e;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t ds_base = smem_u32(smem + S::OFF_DS);
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (*abort_flag || !mbar_wait(s_full, j & 1) || !mbar_wait(ds_empty, (j & 1) ^ 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool src2 = j >= n1;
      const int64_t key0 = (src2 ? t2a + (j - n1) : j) * 128;
      const int64_t lo = src2 ? s2 : s1, hi = src2 ? e2 : e1;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32], y[32];
        tmem_ld32(lane_base + c * 32, x);
        tmem_ld32(lane_base + 128 + c * 32, y);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int64_t key = key0 + c * 32 + i;
          const float p = (key >= lo && key < hi) ? exp2f(fmaf(x[i], sl2, -L2e)) : 0.f;
          x[i] = p * (y[i] - dl);
        }
        store_row32_sw128(ds_base, r, c * 32, x);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);
      fence_proxy_async_smem();
      mbar_arrive(ds_full);
    }
    if (!ok) *abort_flag = 1;
    const bool done_ok = mbar_wait(dq_full, 0);
    tc_fence_after();
    float* out = dq + qi * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      float x[32];
      tmem_ld32(lane_base + 256 + c * 32, x);
      tmem_wait_ld();
      if (live && ok && done_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const int e = c * 32 + i;
          float4 v = make_float4(nt > 0 ? x[i] * scale : 0.f, nt > 0 ? x[i + 1] * scale : 0.f,
                                 nt > 0 ? x[i + 2] * scale : 0.f, nt > 0 ? x[i + 3] * scale : 0.f);
          if (e >= hd) v = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(out + e) = v;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// Backward: dK, dV of the own-block (source-2) keys
// ------------------------------------------------------------------------------------------------

template <int D>
struct DkvSmem {
  static constexpr int BOXES = D / 64;
  static constexpr int TILE = BOXES * kAttnTileBytes;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = TILE;
  static constexpr int OFF_Q = 2 * TILE;
  static constexpr int OFF_DO = 3 * TILE;
  static constexpr int OFF_P = 4 * TILE;                     // P^T  [128 keys][128 queries]
  static constexpr int OFF_DS = OFF_P + 2 * kAttnTileBytes;  // dS^T
  static constexpr int MAX_GROUP = 8;  // query heads per KV head
  static constexpr int OFF_STAT = OFF_DS + 2 * kAttnTileBytes;  // [group][lse*log2e | delta][128]
  static constexpr int OFF_BAR = OFF_STAT + MAX_GROUP * 2 * 128 * 4;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
};

// grid (ceil(L2 / 128), Hkv, B). Queries of the block keys [k0, k0 + 128) are rows [k0, k0 + 128).
template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2, int Hq,
                        int Hkv, int64_t Tq, int64_t L2, int hd, int block, float scale,
                        const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dk,
                        float* __restrict__ dv) {
  using S = DkvSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* in_full = bars + 1;    // Q_h, dO_h of the current head
  uint64_t* in_empty = bars + 2;   // Q_h, dO_h consumed
  uint64_t* s_full = bars + 3;     // S^T, dP^T
  uint64_t* s_empty = bars + 4;    // read by the row threads
  uint64_t* p_full = bars + 5;     // P^T, dS^T written (128 arrivals)
  uint64_t* p_empty = bars + 6;    // consumed by the dV / dK MMAs
  uint64_t* acc_full = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13);
  float* s_lse = reinterpret_cast<float*>(smem + S::OFF_STAT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 128;
  const int hk = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = Hq / Hkv;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(in_full, 1);
    mbar_init(in_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_empty, 4);
    mbar_init(p_full, 128);
    mbar_init(p_empty, 1);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp >= 2) {  // per-query statistics of every head of the group, read by all row threads
    const int r = (warp & 3) * 32 + lane;
    const int64_t tq = k0 + r;
    for (int g = 0; g < G; ++g) {
      const int h = hk * G + g;
      const bool qlive = tq < Tq;
      s_lse[g * 256 + r] = qlive ? lse[(b * Hq + h) * Tq + tq] * kLog2e : 0.f;
      s_lse[g * 256 + 128 + r] = qlive ? delta[(b * Hq + h) * Tq + tq] : 0.f;
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S^T [0,128) dP^T [128,256) dV [256,256+D) dK [384, 384+D)

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * S::TILE);
#pragma unroll
      for (int c = 0; c < S::BOXES; ++c) {
        tma_load_3d(smem + S::OFF_K + c * kAttnTileBytes, &tmK2, kv_full, c * 64, static_cast<int>(k0),
                    static_cast<int>(b * Hkv + hk));
        tma_load_3d(smem + S::OFF_V + c * kAttnTileBytes, &tmV2, kv_full, c * 64, static_cast<int>(k0),
                    static_cast<int>(b * Hkv + hk));
      }
      int issued = 0;
      for (int g = 0; g < G; ++g) {
        const int h = hk * G + g;
        if (*abort_flag || !mbar_wait(in_empty, (g & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(in_full, 2 * S::TILE);
#pragma unroll
        for (int c = 0; c < S::BOXES; ++c) {
          tma_load_3d(smem + S::OFF_Q + c * kAttnTileBytes, &tmQ, in_full, c * 64, static_cast<int>(k0),
                      static_cast<int>(b * Hq + h));
          tma_load_3d(smem + S::OFF_DO + c * kAttnTileBytes, &tmDO, in_full, c * 64 + h * hd,
                      static_cast<int>(k0), static_cast<int>(b));
        }
        issued = g + 1;
      }
      if (*abort_flag) {
        mbar_wait_short(kv_full, 0);
        if (issued > 0) mbar_wait_short(in_full, (issued - 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_g = umma_idesc_bf16(128, D, false, true);
      const uint32_t k_base = smem_u32(smem + S::OFF_K), v_base = smem_u32(smem + S::OFF_V);
      const uint32_t q_base = smem_u32(smem + S::OFF_Q), do_base = smem_u32(smem + S::OFF_DO);
      const uint32_t p_base = smem_u32(smem + S::OFF_P), ds_base = smem_u32(smem + S::OFF_DS);
      bool ok = mbar_wait(kv_full, 0);
      for (int g = 0; ok && g < G; ++g) {
        if (*abort_flag || !mbar_wait(in_full, g & 1) || !mbar_wait(s_empty, (g & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16(tmem, desc_kmajor(k_base, kk), desc_kmajor(q_base, kk), idesc_s, kk > 0 ? 1u : 0u);
          umma_f16(tmem + 128, desc_kmajor(v_base, kk), desc_kmajor(do_base, kk), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!mbar_wait(p_full, g & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t acc = (g > 0 || kk > 0) ? 1u : 0u;
          umma_f16(tmem + 256, desc_kmajor(p_base, kk), desc_mnmajor(do_base, kk), idesc_g, acc);
          umma_f16(tmem + 384, desc_kmajor(ds_base, kk), desc_mnmajor(q_base, kk), idesc_g, acc);
        }
        umma_commit(p_empty);
        umma_commit(in_empty);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(acc_full);
    }
  } else {
    const int r = (warp & 3) * 32 + lane;  // key row inside the tile
    const int64_t key = k0 + r;
    const bool live = key < L2;
    const int64_t kblk = key / block;
    // the queries that see this key: its own block, [lo, hi) as columns of the tile
    const int64_t lo = live ? kblk * block - k0 : 0;
    const int64_t hi = live ? min((kblk + 1) * block, Tq) - k0 : 0;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t p_base = smem_u32(smem + S::OFF_P), ds_base = smem_u32(smem + S::OFF_DS);
    const float sl2 = scale * kLog2e;
    bool ok = true;
    for (int g = 0; g < G; ++g) {
      const float* g_lse = s_lse + g * 256;
      const float* g_delta = g_lse + 128;
      // the P^T / dS^T buffers are free once the previous head's dV / dK MMAs completed
      if (*abort_flag || !mbar_wait(p_empty, (g & 1) ^ 1) || !mbar_wait(s_full, g & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32], y[32];
        const int kind = chunk_kind_warp(lo, hi, 32 * c, 32);  // warp-uniform
        if (kind == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = y[i] = 0.f;
        } else {
          tmem_ld32(lane_base + c * 32, x);
          tmem_ld32(lane_base + 128 + c * 32, y);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int qc = c * 32 + i;
            const bool vis = kind == 1 || (qc >= lo && qc < hi);
            const float p = vis ? ex2_approx(fmaf(x[i], sl2, -g_lse[qc])) : 0.f;
            x[i] = p;
            y[i] = p * (y[i] - g_delta[qc]);
          }
        }
        store_row32_sw128(p_base, r, c * 32, x);
        store_row32_sw128(ds_base, r, c * 32, y);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
    }
    if (!ok) *abort_flag = 1;
    const bool done_ok = mbar_wait(acc_full, 0);
    tc_fence_after();
    float* dvr = dv + ((b * Hkv + hk) * L2 + (live ? key : 0)) * D;
    float* dkr = dk + ((b * Hkv + hk) * L2 + (live ? key : 0)) * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      float x[32], y[32];
      tmem_ld32(lane_base + 256 + c * 32, x);
      tmem_ld32(lane_base + 384 + c * 32, y);
      tmem_wait_ld();
      if (live && ok && done_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const int e = c * 32 + i;
          float4 a = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
          float4 kq = make_float4(y[i] * scale, y[i + 1] * scale, y[i + 2] * scale, y[i + 3] * scale);
          if (e >= hd) {
            a = make_float4(0.f, 0.f, 0.f, 0.f);
            kq = a;
          }
          *reinterpret_cast<float4*>(dvr + e) = a;
          *reinterpret_cast<float4*>(dkr + e) = kq;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

}  // namespace orthrus

namespace orthrus {

// ------------------------------------------------------------------------------------------------
// Forward, two query heads per CTA (ping-pong)
// ------------------------------------------------------------------------------------------------
//
// CTA = 128 query rows of the two query heads 2p, 2p+1 that share one KV head (GQA group size
// even), 320 threads: warp 0 TMA, warp 1 MMA issue, warps 2-5 softmax of head 2p, warps 6-9
// softmax of head 2p+1. Each K / V tile is loaded once for both heads. TMEM: S of head h in
// columns [128h, 128h+128), the O accumulator of head h in [256+128h, ...). While one head's rows
// run their softmax, the tensor core works on the other head's QK^T / PV.
//
// O is accumulated by the MMA itself in TMEM across key tiles. P is computed against a per-row
// reference max m_ref that is only raised when a tile's max exceeds it by more than 2^8 (then the
// row rescales its own O row in TMEM and its running sum); the final O / l uses the same reference,
// so the result is exact while rescales stay rare.

template <int D>
struct Fwd2Smem {
  static constexpr int BOXES = D / 64;
  static constexpr int TILE = BOXES * kAttnTileBytes;  // [128][D]
  static constexpr int OFF_Q = 0;                       // Q of head h at h * TILE
  static constexpr int OFF_RING = 2 * TILE;             // three slots: K(0), V(0), K(1), V(1), ...
  static constexpr int OFF_P = 5 * TILE;                // P of head h at OFF_P + h * 32 KB
  static constexpr int OFF_BAR = OFF_P + 4 * kAttnTileBytes;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
};

constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 256 between rescales

template <int D>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK1,
                        const __grid_constant__ CUtensorMap tmV1, const __grid_constant__ CUtensorMap tmK2,
                        const __grid_constant__ CUtensorMap tmV2, int Hq, int Hkv, int64_t Tq, int hd,
                        float scale_log2, MaskParams mp, bool has2, __nv_bfloat16* __restrict__ o,
                        float* __restrict__ lse) {
  using S = Fwd2Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* slot_full = bars + 1;   // [3] ring slot loaded
  uint64_t* slot_empty = bars + 4;  // [3] ring slot consumed by the MMAs of both heads
  uint64_t* s_full = bars + 7;   // [2] per head
  uint64_t* p_full = bars + 9;   // [2] per head (128 arrivals)
  uint64_t* p_empty = bars + 11; // [2] per head: PV of the head completed
  uint64_t* mma_done = bars + 13;
  uint64_t* s_free = bars + 14;  // [2] per head: the rows loaded S (128 arrivals)
  unsigned long long* red = reinterpret_cast<unsigned long long*>(bars + 16);
  AttnTiles* tiles = reinterpret_cast<AttnTiles*>(bars + 20);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (pair, row, query tile): the query tile varies slowest and runs backwards, so every
  // CTA of the heaviest tiles (most visible keys) is dispatched before any lighter one
  const int64_t q0 = static_cast<int64_t>(gridDim.z - 1 - blockIdx.z) * 128;
  const int pair = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int G = Hq / Hkv;
  const int hk = (2 * pair) / G;
  const int wg = warp >= 2 ? (warp - 2) / 4 : -1;  // softmax warpgroup = head of the pair
  const int row = warp >= 2 ? (warp & 3) * 32 + lane : -1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_empty[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(mma_done, 1);
    red[0] = 0;
    red[1] = ~0ull;
    red[2] = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  // a programmatic dependent launch may start this kernel during the previous one: the tile map,
  // the operands and the outputs belong to the stream order only after griddep_wait()
  griddep_launch_dependents();
  griddep_wait();
  if (warp == 0 && elect_one()) {  // Q does not depend on the tile map: its load overlaps it
    mbar_arrive_expect_tx(q_full, 2 * S::TILE);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int c = 0; c < S::BOXES; ++c)
        tma_load_3d(smem + S::OFF_Q + h * S::TILE + c * kAttnTileBytes, &tmQ, q_full, c * 64,
                    static_cast<int>(q0), static_cast<int>(b * Hq + 2 * pair + h));
  }
  attn_tile_map(mp, b, q0, Tq, has2, wg == 0 ? row : -1, red, tiles);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n1 = tiles->n1, t2a = tiles->t2a;
  const int nt = n1 + tiles->n2;

  if (warp == 0) {
    if (elect_one()) {
      // K and V tiles share a ring of three slots with K one tile ahead of V: K(0), K(1), V(0),
      // K(2), V(1), ..., V(nt - 1). A load may start once the tile three places before it in this
      // order has been consumed, so K(j + 1) is in flight while tile j - 1 is still being read.
      int issued = 0;
      const int z = static_cast<int>(b * Hkv + hk);
      for (int idx = 0; idx < 2 * nt; ++idx) {
        const bool is_v = idx == 2 * nt - 1 || (idx > 0 && (idx & 1) == 0);
        const int j = idx == 2 * nt - 1 ? nt - 1 : is_v ? (idx - 2) / 2 : (idx + 1) / 2;
        const int slot = idx % 3, use = idx / 3;
        const bool src2 = j >= n1;
        const int key0 = (src2 ? t2a + (j - n1) : j) * 128;
        if (*abort_flag || !mbar_wait(&slot_empty[slot], (use & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        const CUtensorMap* map = is_v ? (src2 ? &tmV2 : &tmV1) : (src2 ? &tmK2 : &tmK1);
        uint8_t* dst = smem + S::OFF_RING + slot * S::TILE;
        mbar_arrive_expect_tx(&slot_full[slot], S::TILE);
#pragma unroll
        for (int c = 0; c < S::BOXES; ++c)
          tma_load_3d(dst + c * kAttnTileBytes, map, &slot_full[slot], c * 64, key0, z);
        // the ring holds one tile of lookahead; tile j + 2 goes to L2 now, so its loads do not
        // wait on HBM (the AR keys of the dual view were written long before this kernel)
        if (!is_v && j + 2 < nt) {
          const bool pf2 = j + 2 >= n1;
          const int pkey = (pf2 ? t2a + (j + 2 - n1) : j + 2) * 128;
#pragma unroll
          for (int c = 0; c < S::BOXES; ++c) {
            tma_prefetch_l2_3d(pf2 ? &tmK2 : &tmK1, c * 64, pkey, z);
            tma_prefetch_l2_3d(pf2 ? &tmV2 : &tmV1, c * 64, pkey, z);
          }
        }
        issued = idx + 1;
      }
      if (*abort_flag) {
        mbar_wait_short(q_full, 0);
        for (int idx = max(0, issued - 3); idx < issued; ++idx) mbar_wait_short(&slot_full[idx % 3], (idx / 3) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, false, true);
      // ring positions (slot = position % 3, use = position / 3) in the producer's order
      auto kpos = [&](int j) { return j == 0 ? 0 : 2 * j - 1; };
      auto vpos = [&](int j) { return j == nt - 1 ? 2 * nt - 1 : 2 * j + 2; };
      auto ring = [&](int pos) { return smem_u32(smem + S::OFF_RING + (pos % 3) * S::TILE); };
      auto ring_full = [&](int pos) { return mbar_wait(&slot_full[pos % 3], (pos / 3) & 1); };
      bool ok = mbar_wait(q_full, 0) && (nt == 0 || ring_full(0));
      auto issue_s = [&](int h, int j) {
        const uint32_t q_base = smem_u32(smem + S::OFF_Q + h * S::TILE);
        const uint32_t k_base = ring(kpos(j));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + h * 128, desc_kmajor(q_base, kk), desc_kmajor(k_base, kk), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[h]);
      };
      if (ok && nt > 0) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&slot_empty[0]);
      }
      // per tile j: QK^T of tile j + 1 as soon as the rows of a head have loaded S(j) (it runs
      // under their softmax), then P V of tile j once P(j) is in shared memory
      for (int j = 0; ok && j < nt; ++j) {
        for (int h = 0; ok && h < 2 && j + 1 < nt; ++h) {
          if (*abort_flag || !mbar_wait(&s_free[h], j & 1) || (h == 0 && !ring_full(kpos(j + 1)))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(h, j + 1);
          if (h == 1) umma_commit(&slot_empty[kpos(j + 1) % 3]);
        }
        for (int h = 0; ok && h < 2; ++h) {
          if (*abort_flag || !mbar_wait(&p_full[h], j & 1) || (h == 0 && !ring_full(vpos(j)))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t p_base = smem_u32(smem + S::OFF_P + h * 2 * kAttnTileBytes);
          const uint32_t v_base = ring(vpos(j));
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + 256 + h * 128, desc_kmajor(p_base, kk), desc_mnmajor(v_base, kk), idesc_o,
                     (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&p_empty[h]);
          if (h == 1) umma_commit(&slot_empty[vpos(j) % 3]);
        }
      }
      if (!ok) *abort_flag = 1;
      // drain on its own barrier: no MMA may still run when the CTA frees its TMEM
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else {
    const int h = wg;
    const int64_t t = q0 + row;
    const bool live = t < Tq;
    int64_t e1l = 0, s2l = 0, e2l = 0;
    if (live) query_ranges(mp, b, t, e1l, s2l, e2l);
    // key positions fit 32 bits (sources are < 2^31 rows); narrow them to spare registers for the
    // 128 scores each row holds
    const int s1 = live ? static_cast<int>(source1_start(mp, b, t)) : 0;
    const int e1 = static_cast<int>(e1l), s2 = has2 ? static_cast<int>(s2l) : 0, e2 = has2 ? static_cast<int>(e2l) : 0;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = lane_base + h * 128;
    const uint32_t o_col = lane_base + 256 + h * 128;
    const uint32_t p_base = smem_u32(smem + S::OFF_P + h * 2 * kAttnTileBytes);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (*abort_flag || !mbar_wait(&s_full[h], j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      tmem_ld32(s_col + 0, s);
      tmem_ld32(s_col + 32, s + 32);
      tmem_ld32(s_col + 64, s + 64);
      tmem_ld32(s_col + 96, s + 96);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[h]);  // the MMA warp may overwrite S with the next tile's scores
      const bool src2 = j >= n1;
      const int key0 = (src2 ? t2a + (j - n1) : j) * 128;
      const int lo = (src2 ? s2 : s1) - key0, hi = (src2 ? e2 : e1) - key0;  // visible columns
      const bool full = lo <= 0 && hi >= 128;
      // row max of the raw scores (scale > 0 commutes with max), four independent chains
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full) {
#pragma unroll
        for (int i = 0; i < 128; ++i) mx[i & 3] = fmaxf(mx[i & 3], s[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          s[i] = (i >= lo && i < hi) ? s[i] : -INFINITY;
          mx[i & 3] = fmaxf(mx[i & 3], s[i]);
        }
      }
      const float rmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float tmax = rmax == -INFINITY ? -INFINITY : rmax * scale_log2;
      // raise the reference max only when the tile max exceeds it by more than the threshold
      float alpha = 1.f;
      if (tmax > m_ref + kRescaleThreshold) {
        if (m_ref != -INFINITY) alpha = exp2f(m_ref - tmax);
        m_ref = tmax;
      }
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      // the previous P V of this head must be done before P and O are touched again
      if (j > 0 && !mbar_wait(&p_empty[h], (j - 1) & 1)) {
        ok = false;
        break;
      }
      // P = exp2(s * scale - m_ref) as bf16 pairs, stored 32 columns at a time: no packed copy of
      // the whole row stays live beside the scores (that had spilled registers to local memory)
      float sm[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ex2_approx(fmaf(s[32 * c + i], scale_log2, -mu));
          const float p1 = ex2_approx(fmaf(s[32 * c + i + 1], scale_log2, -mu));
          sm[i & 3] += p0;
          sm[(i + 1) & 3] += p1;
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        store_row32_sw128_packed(p_base, row, c * 32, pk);
      }
      l = fmaf(l, alpha, (sm[0] + sm[1]) + (sm[2] + sm[3]));
      // TMEM loads and stores are warp-collective: the whole warp rescales when any of its rows
      // must (rows that need none multiply by exactly 1)
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          float x[16];
          tmem_ld16(o_col + c * 16, x);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i] *= alpha;
          tmem_st16(o_col + c * 16, x);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&p_full[h]);
    }
    if (!ok) *abort_flag = 1;
    const bool done = ok && nt > 0 && mbar_wait(&p_empty[h], (nt - 1) & 1);
    tc_fence_after();
    float acc[D];
#pragma unroll
    for (int c = 0; c < D / 32; ++c) tmem_ld32(o_col + c * 32, acc + 32 * c);
    tmem_wait_ld();
    if (done && live) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int hh = 2 * pair + h;
      __nv_bfloat16* orow = o + ((b * Tq + t) * Hq + hh) * hd;
      if (hd == D) {
#pragma unroll
        for (int i = 0; i < D; i += 8) {
          uint4 pk = make_uint4(pack_bf16x2(acc[i] * inv, acc[i + 1] * inv), pack_bf16x2(acc[i + 2] * inv, acc[i + 3] * inv),
                                pack_bf16x2(acc[i + 4] * inv, acc[i + 5] * inv), pack_bf16x2(acc[i + 6] * inv, acc[i + 7] * inv));
          *reinterpret_cast<uint4*>(orow + i) = pk;
        }
      } else {
#pragma unroll
        for (int i = 0; i < D; ++i)
          if (i < hd) orow[i] = __float2bfloat16_rn(acc[i] * inv);
      }
      if (lse) lse[(b * Hq + hh) * Tq + t] = (m_ref + log2f(l)) * kLn2;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

}  // namespace orthrus

namespace orthrus {

// ------------------------------------------------------------------------------------------------
// Backward dQ, two query heads per CTA (ping-pong), 64-key tiles
// ------------------------------------------------------------------------------------------------
//
// CTA = 128 query rows of the heads 2p, 2p+1 sharing one KV head; 576 threads (warp 0 TMA, warp 1
// MMA, warps 2-9 / 10-17 the rows of head 2p / 2p+1: each row is shared by two warps, one per
// 32-key half of the tile, so a thread's share of a tile's exponentials is 32). Key tiles of 64
// so that both heads fit in TMEM:
// head h owns S [64h .. +64), dP [128 + 64h .. +64) and its dQ accumulator [256 + 128h .. +128).
// Per tile: S = Q K^T, dP = dO V^T (N = 64), then dS = P (dP - delta), which each row warp writes
// as bf16 pairs over the first 16 of the 32 dP columns it has just read, and dQ += dS K with dS as
// the TMEM operand and K as the MN-major shared-memory operand. A head's next S is issued right
// after its dQ MMA, its next dP only once that dQ MMA has completed (a commit the issuing thread
// waits on: two MMAs with different accumulators are not ordered). Keeping dS out of shared memory
// leaves room for three K/V stages. While one head's rows compute dS, the tensor core runs the
// other head's MMAs.

constexpr int kKeyBox64 = 64 * 64 * 2;  // one [64 rows][64] bf16 box = 8 KB

__device__ __forceinline__ uint64_t desc_kmajor_rows64(uint32_t base, int kk) {  // [64][D] tile
  return umma_desc_sw128(base + (kk >> 2) * kKeyBox64 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor_rows64(uint32_t base, int kk) {  // [64 rows][D]
  return umma_desc_sw128(base + kk * 2048, kKeyBox64, 1024);
}

template <int D>
struct Dq2Smem {
  static constexpr int BOXES = D / 64;
  static constexpr int QT = BOXES * kAttnTileBytes;  // [128][D]
  static constexpr int KT = BOXES * kKeyBox64;       // [64][D]
  static constexpr int OFF_Q = 0;                    // Q of head h at h * QT
  static constexpr int OFF_DO = 2 * QT;              // dO of head h
  static constexpr int STAGES = 3;
  static constexpr int OFF_KV = 4 * QT;              // stage s: K at s * 2KT, V at s * 2KT + KT
  static constexpr int OFF_BAR = OFF_KV + STAGES * 2 * KT;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
};
static_assert(Dq2Smem<128>::SMEM <= 232448, "dQ kernel shared memory");

constexpr int kDq2Threads = 576;

template <int D>
__global__ void __launch_bounds__(kDq2Threads, 1)
    attn_dq_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmK1, const __grid_constant__ CUtensorMap tmV1,
                       const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2, int Hq,
                       int Hkv, int64_t Tq, int hd, float scale, MaskParams mp, bool has2,
                       const float* __restrict__ lse, const float* __restrict__ delta, float* __restrict__ dq) {
  using S = Dq2Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  constexpr int NS = S::STAGES;
  uint64_t* in_full = bars + 0;
  uint64_t* kv_full = bars + 1;            // [NS]
  uint64_t* kv_empty = bars + 1 + NS;      // [NS]
  uint64_t* s_full = bars + 1 + 2 * NS;   // [2] per head: S and dP of the tile in TMEM
  uint64_t* ds_full = s_full + 2;          // [2] per head (8 warp arrivals): dS written to TMEM
  uint64_t* ds_empty = s_full + 4;         // [2] per head: the dQ MMA has consumed dS
  uint64_t* mma_done = s_full + 6;
  static_assert(1 + 2 * NS + 7 <= 16, "dQ kernel barriers");
  unsigned long long* red = reinterpret_cast<unsigned long long*>(bars + 16);
  AttnTiles* tiles = reinterpret_cast<AttnTiles*>(bars + 20);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q0 = static_cast<int64_t>(gridDim.z - 1 - blockIdx.z) * 128;  // heaviest tiles first
  const int pair = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int G = Hq / Hkv;
  const int hk = (2 * pair) / G;
  const int wg = warp >= 2 ? (warp - 2) / 8 : -1;        // head of a row warp
  const int half = warp >= 2 ? ((warp - 2) / 4) & 1 : 0;  // its 32-key half of a tile
  const int row = warp >= 2 ? (warp & 3) * 32 + lane : -1;

  if (threadIdx.x == 0) {
    mbar_init(in_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], 8);
      mbar_init(&ds_empty[i], 1);
    }
    mbar_init(mma_done, 1);
    red[0] = 0;
    red[1] = ~0ull;
    red[2] = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  // a programmatic dependent launch may start this kernel during the previous one: the tile map,
  // the operands and the outputs belong to the stream order only after griddep_wait()
  griddep_launch_dependents();
  griddep_wait();
  if (warp == 0 && elect_one()) {  // Q and dO do not depend on the tile map: their loads overlap it
    mbar_arrive_expect_tx(in_full, 4 * S::QT);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int hh = 2 * pair + h;
#pragma unroll
      for (int c = 0; c < S::BOXES; ++c) {
        tma_load_3d(smem + S::OFF_Q + h * S::QT + c * kAttnTileBytes, &tmQ, in_full, c * 64,
                    static_cast<int>(q0), static_cast<int>(b * Hq + hh));
        tma_load_3d(smem + S::OFF_DO + h * S::QT + c * kAttnTileBytes, &tmDO, in_full, c * 64 + hh * hd,
                    static_cast<int>(q0), static_cast<int>(b));
      }
    }
  }
  attn_tile_map(mp, b, q0, Tq, has2, (wg == 0 && half == 0) ? row : -1, red, tiles);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // 64-key tiles: source 1 covers [0, 64 * n1b), source 2 [64 * t2b, 64 * (t2b + n2b))
  const int n1b = static_cast<int>((red[0] + 63) / 64);
  const int t2b = red[2] > red[1] ? static_cast<int>(red[1] / 64) : 0;
  const int n2b = red[2] > red[1] ? static_cast<int>((red[2] + 63) / 64) - t2b : 0;
  const int nt = n1b + n2b;

  if (warp == 0) {
    if (elect_one()) {
      int issued = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j % NS;
        if (*abort_flag || !mbar_wait(&kv_empty[s], ((j / NS) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        const bool src2 = j >= n1b;
        const int key0 = (src2 ? t2b + (j - n1b) : j) * 64;
        uint8_t* kt = smem + S::OFF_KV + s * 2 * S::KT;
        uint8_t* vt = kt + S::KT;
        mbar_arrive_expect_tx(&kv_full[s], 2 * S::KT);
#pragma unroll
        for (int c = 0; c < S::BOXES; ++c) {
          tma_load_3d(kt + c * kKeyBox64, src2 ? &tmK2 : &tmK1, &kv_full[s], c * 64, key0,
                      static_cast<int>(b * Hkv + hk));
          tma_load_3d(vt + c * kKeyBox64, src2 ? &tmV2 : &tmV1, &kv_full[s], c * 64, key0,
                      static_cast<int>(b * Hkv + hk));
        }
        // three stages of 64 keys: tile j + 4 goes to L2 now (the AR keys come from HBM otherwise)
        if (j + 4 < nt) {
          const bool pf2 = j + 4 >= n1b;
          const int pkey = (pf2 ? t2b + (j + 4 - n1b) : j + 4) * 64;
#pragma unroll
          for (int c = 0; c < S::BOXES; ++c) {
            tma_prefetch_l2_3d(pf2 ? &tmK2 : &tmK1, c * 64, pkey, static_cast<int>(b * Hkv + hk));
            tma_prefetch_l2_3d(pf2 ? &tmV2 : &tmV1, c * 64, pkey, static_cast<int>(b * Hkv + hk));
          }
        }
        issued = j + 1;
      }
      if (*abort_flag) {
        mbar_wait_short(in_full, 0);
        for (int j = max(0, issued - NS); j < issued; ++j) mbar_wait_short(&kv_full[j % NS], (j / NS) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 64, false, false);
      constexpr uint32_t idesc_q = umma_idesc_bf16(128, D, false, true);
      auto issue_s = [&](int h, int j) {  // S = Q K^T
        const uint32_t q_base = smem_u32(smem + S::OFF_Q + h * S::QT);
        const uint32_t k_base = smem_u32(smem + S::OFF_KV + (j % NS) * 2 * S::KT);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + h * 64, desc_kmajor(q_base, kk), desc_kmajor_rows64(k_base, kk), idesc_s,
                   kk > 0 ? 1u : 0u);
      };
      auto issue_dp = [&](int h, int j) {  // dP = dO V^T; then S and dP of the tile are signalled
        const uint32_t do_base = smem_u32(smem + S::OFF_DO + h * S::QT);
        const uint32_t v_base = smem_u32(smem + S::OFF_KV + (j % NS) * 2 * S::KT) + S::KT;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + 128 + h * 64, desc_kmajor(do_base, kk), desc_kmajor_rows64(v_base, kk), idesc_s,
                   kk > 0 ? 1u : 0u);
        umma_commit(&s_full[h]);
      };
      bool ok = mbar_wait(in_full, 0) && (nt == 0 || mbar_wait(&kv_full[0], 0));
      if (ok && nt > 0) {
        tc_fence_after();
        issue_s(0, 0);
        issue_dp(0, 0);
        issue_s(1, 0);
        issue_dp(1, 0);
      }
      for (int j = 0; ok && j < nt; ++j) {
        for (int h = 0; h < 2; ++h) {
          if (*abort_flag || !mbar_wait(&ds_full[h], j & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + S::OFF_KV + (j % NS) * 2 * S::KT);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_tmem_a(tmem + 256 + h * 128, tmem + 128 + h * 64 + (kk >> 1) * 32 + (kk & 1) * 8,
                            desc_mnmajor_rows64(k_base, kk), idesc_q, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&ds_empty[h]);
          if (h == 1) umma_commit(&kv_empty[j % NS]);
          if (j + 1 < nt) {
            if (h == 0 && !mbar_wait(&kv_full[(j + 1) % NS], ((j + 1) / NS) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(h, j + 1);
            // dS lives in this head's dP columns: the next dP waits until the dQ MMA has read it
            if (!mbar_wait(&ds_empty[h], j & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_dp(h, j + 1);
          }
        }
      }
      if (!ok) *abort_flag = 1;
      // drain on its own barrier: no MMA may still run when the CTA frees its TMEM
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else {
    const int h = wg;
    const int hh = 2 * pair + h;
    const int64_t t = q0 + row;
    const bool live = t < Tq;
    int64_t e1 = 0, s2 = 0, e2 = 0;
    if (live) query_ranges(mp, b, t, e1, s2, e2);
    const int64_t s1 = live ? source1_start(mp, b, t) : 0;
    if (!has2) e2 = s2 = 0;
    const int64_t qi = (b * Hq + hh) * Tq + (live ? t : 0);
    const float L2e = live ? lse[qi] * kLog2e : 0.f;
    const float dl = live ? delta[qi] : 0.f;
    const float sl2 = scale * kLog2e;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (*abort_flag || !mbar_wait(&s_full[h], j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool src2 = j >= n1b;
      const int64_t key0 = (src2 ? t2b + (j - n1b) : j) * 64;
      const int64_t lo = (src2 ? s2 : s1) - key0, hi = (src2 ? e2 : e1) - key0;
      const int kind = chunk_kind_warp(lo, hi, 32 * half, 32);  // warp-uniform
      uint32_t pk[16];  // dS of the row's 32 keys of this half as bf16 pairs
      if (kind == 0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = 0u;
      } else {
        float x[32], y[32];
        tmem_ld32(lane_base + h * 64 + 32 * half, x);
        tmem_ld32(lane_base + 128 + h * 64 + 32 * half, y);
        tmem_wait_ld();
        if (kind == 1) {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = ex2_approx(fmaf(x[i], sl2, -L2e)) * (y[i] - dl);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = 32 * half + i;
            const float p = (col >= lo && col < hi) ? ex2_approx(fmaf(x[i], sl2, -L2e)) : 0.f;
            x[i] = p * (y[i] - dl);
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(x[2 * i], x[2 * i + 1]);
      }
      // over the first 16 of the dP columns this warp has just read (the tile's dP MMA is complete)
      tmem_st16_words(lane_base + 128 + h * 64 + 32 * half, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[h]);
    }
    if (!ok) *abort_flag = 1;
    const bool done = ok && nt > 0 && mbar_wait(&ds_empty[h], (nt - 1) & 1);
    tc_fence_after();
    float* out = dq + qi * D;
#pragma unroll 1
    for (int c = 0; c < D / 64; ++c) {  // this warp's half of the head dimension
      const int col0 = half * (D / 2) + 32 * c;
      float v[32];
      tmem_ld32(lane_base + 256 + h * 128 + col0, v);
      tmem_wait_ld();
      if (live && done) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const int e = col0 + i;
          float4 w4 = make_float4(v[i] * scale, v[i + 1] * scale, v[i + 2] * scale, v[i + 3] * scale);
          if (e >= hd) w4 = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(out + e) = w4;
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

}  // namespace orthrus
