// Fused LM head + log-softmax + KL(teacher || student) over the vocabulary, never writing logits.
//
// Reference: FusedLinearForwardKL with _logits / kl_chunk (orthrus/objective.py:303-392).
//
// Three passes over vocabulary tiles (V = 151936 for the 0.6B shape), all on tcgen05 for bf16:
//   1. stats   rows = [student; unique teacher]: logits tile = rows @ W_tile^T in TMEM, online
//              (max, sum exp, first argmax) per row, one partial per (row, vocabulary split);
//              a combine kernel gives lse and argmax per row.
//   2. diff    per student row tile: student and gathered-teacher logits of the same vocabulary
//              tile (two accumulators sharing the W operand), then
//              kl += p_t (log p_t - log p_s) and diff = w (p_s - p_t) in bf16, stored by each
//              row's thread straight to a chunk buffer [chunk_rows, V] (no staging, so four
//              operand stages fit in shared memory);
//   3. grad    grad[chunk] = diff @ W (UMMA with W as the MN-major operand).
// Finalisation (deterministic, fixed summation order): kl_rows, agree, total and the per-offset
// KL / agreement sums of orthrus_loss (orthrus/objective.py:440-452).
// The fp32 path runs the same passes on CUDA cores with exact fp32 arithmetic.
#pragma once

#include "gemm_simt.cuh"
#include "gemm_tc.cuh"

namespace orthrus {

// ------------------------------------------------------------------------------------------------
// Pass 1 (bf16, tcgen05): per-row online max / sum-exp / argmax over a vocabulary range.
// ------------------------------------------------------------------------------------------------

struct StatsTile {
  static constexpr int BM = 128, BN = 256, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;  // 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

__global__ void __launch_bounds__(192, 1)
    lmhead_stats_tc_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW,
                           int R, int V, int D, int tiles_per_split, int rtiles, int units,
                           float* __restrict__ part_m, float* __restrict__ part_s, int* __restrict__ part_i) {
  using T = StatsTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + T::STAGES * T::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + T::STAGES * T::B_BYTES);
  uint64_t* empty = full + T::STAGES;
  uint64_t* acc_full = empty + T::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vtiles = (V + T::BN - 1) / T::BN;
  const int KB = (D + T::BK - 1) / T::BK;
  // persistent CTAs: work unit u = (row tile u % rtiles, vocabulary split u / rtiles), taken
  // round-robin; the stage and accumulator counters run on across units
  auto unit_tiles = [&](int u, int& row0, int& split, int& t0) {
    row0 = (u % rtiles) * T::BM;
    split = u / rtiles;
    t0 = split * tiles_per_split;
    return max(min(vtiles, t0 + tiles_per_split) - t0, 0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmH);
      prefetch_tensormap(&tmW);
      int it = 0, issued = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int row0, split, t0;
        const int ntiles = unit_tiles(u, row0, split, t0);
        for (int t = 0; t < ntiles && !*abort_flag; ++t) {
          const int v0 = (t0 + t) * T::BN;
          for (int kb = 0; kb < KB; ++kb, ++it) {
            const int s = it % T::STAGES;
            const uint32_t ph = (it / T::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
            tma_load_2d(sA + s * T::A_BYTES, &tmH, &full[s], kb * T::BK, row0);
            tma_load_2d(sB + s * T::B_BYTES, &tmW, &full[s], kb * T::BK, v0);
            issued = it + 1;
          }
        }
      }
      if (*abort_flag)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, T::BN, false, false);
      int it = 0, tt = 0;  // stage counter, accumulator tile counter (across units)
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int row0, split, t0;
        const int ntiles = unit_tiles(u, row0, split, t0);
        for (int t = 0; t < ntiles && !*abort_flag; ++t, ++tt) {
          const int b = tt & 1;
          const uint32_t acc = tmem + b * T::BN;
          if (!mbar_wait(&acc_empty[b], ((tt >> 1) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < KB; ++kb, ++it) {
            const int s = it % T::STAGES;
            const uint32_t ph = (it / T::STAGES) & 1;
            if (!mbar_wait(&full[s], ph)) {
              *abort_flag = 1;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(sA + s * T::A_BYTES);
            const uint32_t b_base = smem_u32(sB + s * T::B_BYTES);
#pragma unroll
            for (int k = 0; k < T::BK / 16; ++k)
              umma_f16(acc, umma_desc_sw128(a_base + k * 32, 16, 1024), umma_desc_sw128(b_base + k * 32, 16, 1024),
                       idesc, (kb > 0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          umma_commit(&acc_full[b]);
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    int tt = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
    int row0, split, t0;
    const int ntiles = unit_tiles(u, row0, split, t0);
    const int row = row0 + quarter * 32 + lane;
    float m = -INFINITY, s = 0.f;
    int idx = 0;
    for (int t = 0; t < ntiles; ++t, ++tt) {
      const int b = tt & 1;
      if (*abort_flag || !mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int v0 = (t0 + t) * T::BN;
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * T::BN;
#pragma unroll 1
      for (int c = 0; c < T::BN / 32; ++c) {
        float x[32];
        tmem_ld32(base + c * 32, x);
        tmem_wait_ld();
        const int col0 = v0 + c * 32;
        const int nvalid = min(32, V - col0);
        if (nvalid <= 0) continue;
        // chunk max and its first column: four independent chains (column j in chain j % 4, each
        // keeping its first maximum), then merged preferring the lower column on ties
        float cmv[4];
        int civ[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          cmv[u] = -INFINITY;
          civ[u] = 32;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid && x[j] > cmv[j & 3]) {
            cmv[j & 3] = x[j];
            civ[j & 3] = j;
          }
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (cmv[u + 2] > cmv[u] || (cmv[u + 2] == cmv[u] && civ[u + 2] < civ[u])) {
            cmv[u] = cmv[u + 2];
            civ[u] = civ[u + 2];
          }
        if (cmv[1] > cmv[0] || (cmv[1] == cmv[0] && civ[1] < civ[0])) {
          cmv[0] = cmv[1];
          civ[0] = civ[1];
        }
        const float cm = cmv[0];
        if (cm > m) {
          s *= exp2f((m - cm) * kLog2e);
          m = cm;
          idx = col0 + civ[0];
        }
        const float ml = m * kLog2e;
        float sv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nvalid) sv[j & 3] += ex2_approx(fmaf(x[j], kLog2e, -ml));
        s += (sv[0] + sv[1]) + (sv[2] + sv[3]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (row < R) {
      part_m[static_cast<int64_t>(split) * R + row] = m;
      part_s[static_cast<int64_t>(split) * R + row] = s;
      part_i[static_cast<int64_t>(split) * R + row] = idx;
    }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// Combines the per-split partials of pass 1: lse[r] = M + log(sum_s s_s e^{m_s - M}), argmax[r].
__global__ void lmhead_stats_combine_kernel(const float* __restrict__ part_m, const float* __restrict__ part_s,
                                            const int* __restrict__ part_i, int R, int splits,
                                            float* __restrict__ lse, int* __restrict__ amax) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  float M = -INFINITY;
  int idx = 0;
  for (int s = 0; s < splits; ++s) {
    const float m = part_m[static_cast<int64_t>(s) * R + r];
    if (m > M) {
      M = m;
      idx = part_i[static_cast<int64_t>(s) * R + r];
    }
  }
  float S = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_m[static_cast<int64_t>(s) * R + r];
    if (m > -INFINITY) S += part_s[static_cast<int64_t>(s) * R + r] * expf(m - M);
  }
  lse[r] = M + logf(S);
  amax[r] = idx;
}

// Greedy decoding's argmax of the logits h @ W^T per row from the pass-1 partials: the first
// maximal split in split order, and inside a split the first maximal column (the lowest index on
// ties, as torch.argmax), written as int64. One warp per row: each lane keeps the first maximum of
// its splits (s = lane, lane + 32, ...), then the warp keeps the larger value or, on a tie, the
// lower split, which is the first maximal split.
__global__ void lmhead_argmax_combine_kernel(const float* __restrict__ part_m, const int* __restrict__ part_i, int R,
                                             int splits, int64_t* __restrict__ out) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  float M = -INFINITY;
  int S = INT_MAX;
  for (int s = lane; s < splits; s += 32) {
    const float m = part_m[static_cast<int64_t>(s) * R + r];
    if (m > M) {
      M = m;
      S = s;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, M, off);
    const int os = __shfl_xor_sync(0xffffffffu, S, off);
    if (om > M || (om == M && os < S)) {
      M = om;
      S = os;
    }
  }
  if (lane == 0) out[r] = S == INT_MAX ? 0 : part_i[static_cast<int64_t>(S) * R + r];
}

// ------------------------------------------------------------------------------------------------
// Pass 2 (bf16, tcgen05): KL and the bf16 probability difference of a student row chunk.
// ------------------------------------------------------------------------------------------------

struct DiffTile {
  static constexpr int BM = 128, BN = 128, BK = 64;
  static constexpr int T_BYTES = BM * BK * 2;  // 16 KB per operand tile
  static constexpr int STAGE_BYTES = 3 * T_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

// Rows [c0, c0 + rows) of the student chunk; S rows via tmS (coordinate c0 + ...), gathered
// teacher rows via tmT (same coordinates), W via tmW, output diff [rows, V] (pitch ldd elements).
__global__ void __launch_bounds__(192, 1)
    lmhead_diff_tc_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmT,
                          const __grid_constant__ CUtensorMap tmW, __nv_bfloat16* __restrict__ diff, int64_t ldd,
                          int rows, int c0, int V, int D, int tiles_per_split, int rtiles, int units,
                          const float* __restrict__ lse_s, const float* __restrict__ lse_t_rows,
                          const float* __restrict__ row_weight, float* __restrict__ kl_part) {
  using T = DiffTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + T::STAGES * T::STAGE_BYTES);
  uint64_t* empty = full + T::STAGES;
  uint64_t* acc_full = empty + T::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vtiles = (V + T::BN - 1) / T::BN;
  const int KB = (D + T::BK - 1) / T::BK;
  // persistent CTAs: work unit u = (row tile u % rtiles, vocabulary split u / rtiles), taken
  // round-robin; stage, accumulator and staging-buffer counters run on across units
  auto unit_tiles = [&](int u, int& rt0, int& split, int& t0) {
    rt0 = (u % rtiles) * T::BM;  // row offset inside the chunk
    split = u / rtiles;
    t0 = split * tiles_per_split;
    return max(min(vtiles, t0 + tiles_per_split) - t0, 0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmS);
      prefetch_tensormap(&tmT);
      prefetch_tensormap(&tmW);
      int it = 0, issued = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int rt0, split, t0;
        const int ntiles = unit_tiles(u, rt0, split, t0);
        for (int t = 0; t < ntiles && !*abort_flag; ++t) {
          const int v0 = (t0 + t) * T::BN;
          for (int kb = 0; kb < KB; ++kb, ++it) {
            const int s = it % T::STAGES;
            const uint32_t ph = (it / T::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1)) {
              *abort_flag = 1;
              break;
            }
            uint8_t* st = stages + s * T::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
            tma_load_2d(st, &tmS, &full[s], kb * T::BK, c0 + rt0);
            tma_load_2d(st + T::T_BYTES, &tmT, &full[s], kb * T::BK, c0 + rt0);
            tma_load_2d(st + 2 * T::T_BYTES, &tmW, &full[s], kb * T::BK, v0);
            issued = it + 1;
          }
        }
      }
      if (*abort_flag)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, T::BN, false, false);
      int it = 0, tt = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      int rt0, split, t0;
      const int ntiles = unit_tiles(u, rt0, split, t0);
      for (int t = 0; t < ntiles && !*abort_flag; ++t, ++tt) {
        const int b = tt & 1;
        const uint32_t acc_s = tmem + b * 256, acc_t = acc_s + 128;
        if (!mbar_wait(&acc_empty[b], ((tt >> 1) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % T::STAGES;
          const uint32_t ph = (it / T::STAGES) & 1;
          if (!mbar_wait(&full[s], ph)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(stages + s * T::STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < T::BK / 16; ++k) {
            const uint64_t wdesc = umma_desc_sw128(base + 2 * T::T_BYTES + k * 32, 16, 1024);
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            umma_f16(acc_s, umma_desc_sw128(base + k * 32, 16, 1024), wdesc, idesc, acc);
            umma_f16(acc_t, umma_desc_sw128(base + T::T_BYTES + k * 32, 16, 1024), wdesc, idesc, acc);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int lrow = quarter * 32 + lane;  // row inside the tile (TMEM lane)
    int tt = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
    int rt0, split, t0;
    const int ntiles = unit_tiles(u, rt0, split, t0);
    const int crow = rt0 + lrow;           // row inside the chunk
    const bool live = crow < rows;
    const float ls_off = live ? lse_s[c0 + crow] : 0.f;
    const float lt_off = live ? lse_t_rows[c0 + crow] : 0.f;
    const float w = (live && row_weight != nullptr) ? row_weight[c0 + crow] : 1.f;
    __nv_bfloat16* drow = diff + static_cast<int64_t>(live ? crow : 0) * ldd;
    float kl = 0.f;
    for (int t = 0; t < ntiles; ++t, ++tt) {
      const int b = tt & 1;
      if (*abort_flag || !mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int v0 = (t0 + t) * T::BN;
      const uint32_t base_s = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * 256;
#pragma unroll 1
      for (int c = 0; c < T::BN / 32; ++c) {
        float xs[32], xt[32];
        tmem_ld32(base_s + c * 32, xs);
        tmem_ld32(base_s + 128 + c * 32, xt);
        tmem_wait_ld();
        const int col0 = v0 + c * 32;
        const int nvalid = min(32, V - col0);
        uint32_t packed[16];
        float klv[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains, summed at the end of the chunk
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float d2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float a = xs[j + u] - ls_off;  // log p_s
            const float bb = xt[j + u] - lt_off;  // log p_t
            const float ps = ex2_approx(a * kLog2e), pt = ex2_approx(bb * kLog2e);
            const bool ok = (j + u) < nvalid;
            klv[(j + u) & 3] += ok ? pt * (bb - a) : 0.f;
            d2[u] = ok ? w * (ps - pt) : 0.f;
          }
          packed[j / 2] = pack_bf16x2(d2[0], d2[1]);
        }
        kl += (klv[0] + klv[1]) + (klv[2] + klv[3]);
        // this row's 32 columns: four 16-byte stores (a 64-byte run of the row), or element by
        // element at the end of the vocabulary
        if (live && nvalid == 32) {
          __nv_bfloat16* dst = drow + col0;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + 8 * q) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        } else if (live && nvalid > 0) {
          __nv_bfloat16* dst = drow + col0;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < nvalid) dst[e] = __ushort_as_bfloat16(static_cast<unsigned short>(packed[e >> 1] >> (16 * (e & 1))));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (live) kl_part[static_cast<int64_t>(split) * rows + crow] = kl;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// fp32 path (CUDA cores): same passes with exact fp32 logits.
// ------------------------------------------------------------------------------------------------

// Pass 1 fp32: CTA = 64 rows x a vocabulary range; logits tile in shared memory, 4 threads / row.
template <typename T>
__global__ void __launch_bounds__(256) lmhead_stats_simt_kernel(const T* __restrict__ H, const T* __restrict__ W,
                                                                int R, int V, int D, int tiles_per_split,
                                                                float* __restrict__ part_m,
                                                                float* __restrict__ part_s,
                                                                int* __restrict__ part_i) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  __shared__ float tile[64][64 + 1];
  const int m0 = blockIdx.x * 64, split = blockIdx.y;
  const int vtiles = (V + 63) / 64;
  const int t0 = split * tiles_per_split, t1 = min(vtiles, t0 + tiles_per_split);
  const int tid = threadIdx.x, tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
  const int prow = tid >> 2, pq = tid & 3;  // row and quarter for the online stats
  float m = -INFINITY, s = 0.f;
  int idx = 0;
  for (int t = t0; t < t1; ++t) {
    const int n0 = t * 64;
    float acc[4][4] = {};
    simt_tile_accumulate<T, false>(H, D, W, D, R, V, m0, n0, 0, D, sA, sB, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) tile[tr + i][tc + j] = acc[i][j];
    __syncthreads();
    // thread (prow, pq) scans columns pq*16 .. pq*16+15 of its row
    for (int j = pq * 16; j < pq * 16 + 16; ++j) {
      const int col = n0 + j;
      if (col >= V) break;
      const float x = tile[prow][j];
      if (x > m) {
        s = s * expf(m - x);
        m = x;
        idx = col;
      }
      s += expf(x - m);
    }
    __syncthreads();
  }
  // combine the 4 quarter-threads of a row (lower column ranges first: lowest index wins ties)
  for (int off = 1; off < 4; off <<= 1) {
    const float om = __shfl_down_sync(0xffffffffu, m, off, 4);
    const float os = __shfl_down_sync(0xffffffffu, s, off, 4);
    const int oi = __shfl_down_sync(0xffffffffu, idx, off, 4);
    const float nm = fmaxf(m, om);
    const float ns = (m > -INFINITY ? s * expf(m - nm) : 0.f) + (om > -INFINITY ? os * expf(om - nm) : 0.f);
    if (om > m) idx = oi;
    m = nm;
    s = ns;
  }
  const int row = m0 + prow;
  if (pq == 0 && row < R) {
    part_m[static_cast<int64_t>(split) * R + row] = m;
    part_s[static_cast<int64_t>(split) * R + row] = s;
    part_i[static_cast<int64_t>(split) * R + row] = idx;
  }
}

// Pass 2 fp32: diff chunk [rows, V] fp32 and KL partials.
template <typename T>
__global__ void __launch_bounds__(256) lmhead_diff_simt_kernel(const T* __restrict__ S, const T* __restrict__ Tg,
                                                               const T* __restrict__ W, int rows, int c0,
                                                               int V, int D, int tiles_per_split,
                                                               const float* __restrict__ lse_s,
                                                               const float* __restrict__ lse_t_rows,
                                                               const float* __restrict__ row_weight,
                                                               T* __restrict__ diff, int64_t ldd,
                                                               float* __restrict__ kl_part) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  __shared__ float ts[64][64 + 1];
  __shared__ float tt[64][64 + 1];
  const int m0 = blockIdx.x * 64, split = blockIdx.y;
  const int vtiles = (V + 63) / 64;
  const int t0 = split * tiles_per_split, t1 = min(vtiles, t0 + tiles_per_split);
  const int tid = threadIdx.x, tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
  const int prow = tid >> 2, pq = tid & 3;
  const int crow = m0 + prow;
  const bool live = crow < rows;
  const float ls_off = live ? lse_s[c0 + crow] : 0.f;
  const float lt_off = live ? lse_t_rows[c0 + crow] : 0.f;
  const float w = (live && row_weight) ? row_weight[c0 + crow] : 1.f;
  float kl = 0.f;
  const T* Sc = S + static_cast<int64_t>(c0) * D;
  const T* Tc = Tg + static_cast<int64_t>(c0) * D;
  for (int t = t0; t < t1; ++t) {
    const int n0 = t * 64;
    float acc[4][4] = {};
    simt_tile_accumulate<T, false>(Sc, D, W, D, rows, V, m0, n0, 0, D, sA, sB, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) ts[tr + i][tc + j] = acc[i][j];
    float acc2[4][4] = {};
    simt_tile_accumulate<T, false>(Tc, D, W, D, rows, V, m0, n0, 0, D, sA, sB, acc2);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) tt[tr + i][tc + j] = acc2[i][j];
    __syncthreads();
    for (int j = pq * 16; j < pq * 16 + 16; ++j) {
      const int col = n0 + j;
      if (col >= V || !live) break;
      const float a = ts[prow][j] - ls_off, b = tt[prow][j] - lt_off;
      const float ps = expf(a), pt = expf(b);
      kl += pt * (b - a);
      diff[static_cast<int64_t>(crow) * ldd + col] = from_f32<T>(w * (ps - pt));
    }
    __syncthreads();
  }
  kl += __shfl_down_sync(0xffffffffu, kl, 2, 4);
  kl += __shfl_down_sync(0xffffffffu, kl, 1, 4);
  if (pq == 0 && live) kl_part[static_cast<int64_t>(split) * rows + crow] = kl;
}

// ------------------------------------------------------------------------------------------------
// helpers
// ------------------------------------------------------------------------------------------------

template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ src, const int64_t* __restrict__ index, int64_t n,
                                   int D, T* __restrict__ dst, int64_t src_rows) {
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  int64_t s = index[r];
  if (s < 0 || s >= src_rows) {
    if (threadIdx.x == 0) record_error(ORTHRUS_ERR_BOUNDS);
    s = 0;
  }
  for (int c = threadIdx.x; c < D; c += blockDim.x) dst[r * D + c] = src[s * D + c];
}

// lse_t_rows[r] = lse_t[index[r]] (teacher lse per student row).
__global__ void gather_lse_kernel(const float* __restrict__ lse_t, const int64_t* __restrict__ index, int64_t n,
                                  int64_t m, float* __restrict__ out) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= n) return;
  int64_t s = index[r];
  if (s < 0 || s >= m) s = 0;
  out[r] = lse_t[s];
}

// kl_rows[r] = sum_s kl_part[s][r] (split order); agree[r] = argmax_s[r] == argmax_t[index[r]].
__global__ void lmhead_rows_kernel(const float* __restrict__ kl_part, int splits, int rows, int c0,
                                   const int* __restrict__ amax_s, const int* __restrict__ amax_t,
                                   const int64_t* __restrict__ index, int64_t m, float* __restrict__ kl_rows,
                                   uint8_t* __restrict__ agree) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += kl_part[static_cast<int64_t>(s) * rows + r];
  const int64_t g = c0 + r;
  kl_rows[g] = acc;
  int64_t t = index[g];
  if (t < 0 || t >= m) t = 0;
  agree[g] = amax_s[g] == amax_t[t] ? 1 : 0;
}

// One CTA of 1024 threads: total = sum w_r kl_r (fixed order) and per-offset sums, one warp per
// offset bin scanning every row in order (deterministic, no atomics).
__global__ void __launch_bounds__(1024) lmhead_finalize_kernel(const float* __restrict__ kl_rows,
                                                               const uint8_t* __restrict__ agree,
                                                               const float* __restrict__ row_weight,
                                                               const int64_t* __restrict__ offsets,
                                                               int64_t n, int num_offsets,
                                                               float* __restrict__ total,
                                                               float* __restrict__ kl_by_offset,
                                                               int64_t* __restrict__ agree_by_offset) {
  __shared__ float red[1024];
  float acc = 0.f;
  for (int64_t r = threadIdx.x; r < n; r += 1024) acc += kl_rows[r] * (row_weight ? row_weight[r] : 1.f);
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 512; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = red[0];
  if (offsets == nullptr) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int bin = warp; bin < num_offsets; bin += 32) {
    float k = 0.f;
    long long a = 0;
    for (int64_t r = lane; r < n; r += 32) {
      if (offsets[r] == bin) {
        k += kl_rows[r];
        a += agree[r];
      }
    }
    for (int off = 16; off > 0; off >>= 1) {
      k += __shfl_down_sync(0xffffffffu, k, off);
      a += __shfl_down_sync(0xffffffffu, a, off);
    }
    if (lane == 0) {
      kl_by_offset[bin] = k;
      agree_by_offset[bin] = a;
    }
  }
}

template <typename T>
__global__ void scale_by_scalar_kernel(const T* __restrict__ x, const float* __restrict__ s, T* __restrict__ y,
                                       int64_t count) {
  const float f = *s;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = from_f32<T>(to_f32<T>(x[i]) * to_f32<T>(from_f32<T>(f)));
}

// ------------------------------------------------------------------------------------------------
// host orchestration
// ------------------------------------------------------------------------------------------------

struct LmheadPlan {
  int64_t n, m, V, D, chunk;
  int dtype;
  int stats_splits, diff_splits;
  size_t off_hcat, off_tg, off_pm, off_ps, off_pi, off_lse, off_amax, off_lset, off_klp, off_diff, off_gemm,
      total;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Vocabulary splits for a persistent grid of `sms` CTAs over rtiles x splits work units: the
// smallest split count (at most max_splits) whose units fill the last round of CTAs to within 1 %
// of the best achievable, so no SM idles through a partial last round.
inline int pick_splits(int64_t rtiles, int64_t vtiles, int sms, int max_splits) {
  const int hi = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(vtiles, max_splits)));
  auto eff = [&](int s) {
    const int64_t tps = ceil_div(vtiles, s), actual = ceil_div(vtiles, tps);
    const int64_t units = rtiles * actual;
    return static_cast<double>(units) / static_cast<double>(ceil_div(units, sms) * sms);
  };
  double best = 0.0;
  for (int s = 1; s <= hi; ++s) best = std::max(best, eff(s));
  for (int s = 1; s <= hi; ++s)
    if (eff(s) >= best - 0.01) return s;
  return hi;
}

constexpr int kLmheadMaxSplits = 64;

inline LmheadPlan lmhead_plan(int64_t n, int64_t m, int64_t V, int64_t D, int64_t chunk_rows, int dtype) {
  LmheadPlan p{};
  p.n = n;
  p.m = m;
  p.V = V;
  p.D = D;
  p.dtype = dtype;
  const int64_t tile = dtype == ORTHRUS_BF16 ? 128 : 64;
  int64_t chunk = chunk_rows <= 0 ? 4096 : chunk_rows;
  chunk = std::max<int64_t>(tile, ceil_div(chunk, tile) * tile);
  chunk = std::min<int64_t>(chunk, ceil_div(std::max<int64_t>(n, 1), tile) * tile);
  p.chunk = chunk;
  const int64_t R = n + m;
  const int sms = num_sms();
  if (dtype == ORTHRUS_BF16) {
    p.stats_splits = pick_splits(ceil_div(R, 128), ceil_div(V, 256), sms, kLmheadMaxSplits);
    p.diff_splits = kLmheadMaxSplits;  // workspace bound; each chunk picks its own count
  } else {
    const int64_t rtiles = ceil_div(R, 64), vt = ceil_div(V, 64);
    p.stats_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(vt, ceil_div(4 * sms, rtiles))));
    const int64_t ctiles = ceil_div(chunk, 64);
    p.diff_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(vt, ceil_div(4 * sms, ctiles))));
  }
  const size_t es = dtype == ORTHRUS_BF16 ? 2 : 4;
  const int64_t Vp = ceil_div(V, 8) * 8;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  p.off_hcat = take(static_cast<size_t>(R) * D * es);
  p.off_tg = take(static_cast<size_t>(n) * D * es);
  p.off_pm = take(static_cast<size_t>(p.stats_splits) * R * 4);
  p.off_ps = take(static_cast<size_t>(p.stats_splits) * R * 4);
  p.off_pi = take(static_cast<size_t>(p.stats_splits) * R * 4);
  p.off_lse = take(static_cast<size_t>(R) * 4);
  p.off_amax = take(static_cast<size_t>(R) * 4);
  p.off_lset = take(static_cast<size_t>(n) * 4);
  p.off_klp = take(static_cast<size_t>(p.diff_splits) * chunk * 4);
  p.off_diff = take(static_cast<size_t>(chunk) * Vp * es);
  const size_t gws = dtype == ORTHRUS_BF16 ? gemm_ws_bytes(chunk, D, V) : simt_ws_bytes(chunk, D, V);
  p.off_gemm = take(gws);
  p.total = off;
  return p;
}

// Row argmax of the logits h [R, D] @ W^T [V, D] (bf16, fp32 accumulation) without writing them:
// pass 1 over all SMs (the vocabulary split up to kArgmaxMaxSplits ways for a few rows), then the
// argmax merge. Workspace: three [splits, R] partial arrays.
constexpr int kArgmaxMaxSplits = 296;

inline size_t lmhead_argmax_ws_bytes(int64_t R) {
  return 3 * align_up(static_cast<size_t>(kArgmaxMaxSplits) * R * 4, 256);
}

inline int lmhead_argmax_bf16(const __nv_bfloat16* h, int64_t R, const __nv_bfloat16* W, int64_t V, int64_t D,
                              int64_t* out, void* ws_raw, size_t ws_bytes, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(h && W && out && R >= 1 && V >= 1 && D >= 64 && D % 64 == 0 && R < (1ll << 31) && V < (1ll << 31));
  ORTHRUS_CHECK_ARG(aligned16(h) && aligned16(W));
  if (ws_raw == nullptr || ws_bytes < lmhead_argmax_ws_bytes(R)) return ORTHRUS_EWORKSPACE;
  const size_t part = align_up(static_cast<size_t>(kArgmaxMaxSplits) * R * 4, 256);
  float* pm = reinterpret_cast<float*>(ws_raw);
  float* ps = reinterpret_cast<float*>(static_cast<uint8_t*>(ws_raw) + part);
  int* pi = reinterpret_cast<int*>(static_cast<uint8_t*>(ws_raw) + 2 * part);
  CUtensorMap tmH, tmW;
  if (!make_tmap_2d_bf16(&tmH, h, D, R, D, 64, 128)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tmW, W, D, V, D, 64, 256)) return ORTHRUS_ECUDA;
  const int vt = static_cast<int>(ceil_div(V, 256));
  const int rtiles = static_cast<int>(ceil_div(R, 128));
  const int tps = static_cast<int>(ceil_div(vt, pick_splits(rtiles, vt, num_sms(), kArgmaxMaxSplits)));
  const int splits = static_cast<int>(ceil_div(vt, tps));
  const int units = rtiles * splits;
  ORTHRUS_CHECK_CUDA(ensure_smem(lmhead_stats_tc_kernel, StatsTile::SMEM));
  const unsigned grid = static_cast<unsigned>(std::min(units, num_sms()));
  lmhead_stats_tc_kernel<<<grid, 192, StatsTile::SMEM, stream>>>(tmH, tmW, static_cast<int>(R), static_cast<int>(V),
                                                                 static_cast<int>(D), tps, rtiles, units, pm, ps, pi);
  ORTHRUS_CHECK_LAUNCH();
  lmhead_argmax_combine_kernel<<<static_cast<unsigned>(ceil_div(R, 8)), 256, 0, stream>>>(
      pm, pi, static_cast<int>(R), splits, out);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

template <typename T>
int lmhead_kl_fwd_impl(const T* student, int64_t n, const T* teacher, int64_t m, const int64_t* index,
                       const T* weight, int64_t V, int64_t D, const float* row_weight, const int64_t* offsets,
                       int num_offsets, float* total, float* kl_rows, uint8_t* agree, T* grad,
                       float* kl_by_offset, int64_t* agree_by_offset, int64_t chunk_rows, void* ws_raw,
                       size_t ws_bytes, cudaStream_t stream) {
  constexpr bool kBf16 = sizeof(T) == 2;
  const int dtype = kBf16 ? ORTHRUS_BF16 : ORTHRUS_F32;
  ORTHRUS_CHECK_ARG(n >= 0 && m >= 1 && V >= 1 && D >= 1 && index && weight && total && kl_rows && agree);
  ORTHRUS_CHECK_ARG(n == 0 || (student && teacher));
  ORTHRUS_CHECK_ARG(offsets == nullptr || (kl_by_offset && agree_by_offset && num_offsets > 0));
  ORTHRUS_CHECK_ARG(n + m < (1ll << 31) && V < (1ll << 31));
  if (kBf16) ORTHRUS_CHECK_ARG(D % 64 == 0 && aligned16(student) && aligned16(teacher) && aligned16(weight));
  const LmheadPlan p = lmhead_plan(n, m, V, D, chunk_rows, dtype);
  if (ws_raw == nullptr || ws_bytes < p.total) return ORTHRUS_EWORKSPACE;
  if (n == 0) {
    ORTHRUS_CHECK_CUDA(cudaMemsetAsync(total, 0, sizeof(float), stream));
    if (offsets) {
      ORTHRUS_CHECK_CUDA(cudaMemsetAsync(kl_by_offset, 0, num_offsets * sizeof(float), stream));
      ORTHRUS_CHECK_CUDA(cudaMemsetAsync(agree_by_offset, 0, num_offsets * sizeof(int64_t), stream));
    }
    return ORTHRUS_OK;
  }
  uint8_t* ws = static_cast<uint8_t*>(ws_raw);
  T* hcat = reinterpret_cast<T*>(ws + p.off_hcat);
  T* tg = reinterpret_cast<T*>(ws + p.off_tg);
  float* pm = reinterpret_cast<float*>(ws + p.off_pm);
  float* ps = reinterpret_cast<float*>(ws + p.off_ps);
  int* pi = reinterpret_cast<int*>(ws + p.off_pi);
  float* lse = reinterpret_cast<float*>(ws + p.off_lse);
  int* amax = reinterpret_cast<int*>(ws + p.off_amax);
  float* lset = reinterpret_cast<float*>(ws + p.off_lset);
  float* klp = reinterpret_cast<float*>(ws + p.off_klp);
  T* diff = reinterpret_cast<T*>(ws + p.off_diff);
  void* gws = ws + p.off_gemm;
  const int64_t R = n + m;
  const int64_t Vp = ceil_div(V, 8) * 8;

  // rows = [student; teacher]
  ORTHRUS_CHECK_CUDA(cudaMemcpyAsync(hcat, student, n * D * sizeof(T), cudaMemcpyDeviceToDevice, stream));
  ORTHRUS_CHECK_CUDA(cudaMemcpyAsync(hcat + n * D, teacher, m * D * sizeof(T), cudaMemcpyDeviceToDevice, stream));
  gather_rows_kernel<T><<<static_cast<unsigned>(n), 128, 0, stream>>>(teacher, index, n, static_cast<int>(D), tg, m);
  ORTHRUS_CHECK_LAUNCH();

  // pass 1: lse and argmax of every row
  if constexpr (kBf16) {
    CUtensorMap tmH, tmW;
    if (!make_tmap_2d_bf16(&tmH, hcat, D, R, D, 64, 128)) return ORTHRUS_ECUDA;
    if (!make_tmap_2d_bf16(&tmW, weight, D, V, D, 64, 256)) return ORTHRUS_ECUDA;
    const int vt = static_cast<int>(ceil_div(V, 256));
    const int tps = static_cast<int>(ceil_div(vt, p.stats_splits));
    const int splits = static_cast<int>(ceil_div(vt, tps));
    const int rtiles = static_cast<int>(ceil_div(R, 128));
    const int units = rtiles * splits;
    ORTHRUS_CHECK_CUDA(ensure_smem(lmhead_stats_tc_kernel, StatsTile::SMEM));
    const unsigned grid = static_cast<unsigned>(std::min(units, num_sms()));  // persistent, one CTA per SM
    lmhead_stats_tc_kernel<<<grid, 192, StatsTile::SMEM, stream>>>(tmH, tmW, static_cast<int>(R), static_cast<int>(V),
                                                                   static_cast<int>(D), tps, rtiles, units, pm, ps,
                                                                   pi);
    ORTHRUS_CHECK_LAUNCH();
    lmhead_stats_combine_kernel<<<static_cast<unsigned>(ceil_div(R, 256)), 256, 0, stream>>>(
        pm, ps, pi, static_cast<int>(R), splits, lse, amax);
    ORTHRUS_CHECK_LAUNCH();
  } else {
    const int vt = static_cast<int>(ceil_div(V, 64));
    const int tps = static_cast<int>(ceil_div(vt, p.stats_splits));
    const int splits = static_cast<int>(ceil_div(vt, tps));
    dim3 grid(static_cast<unsigned>(ceil_div(R, 64)), splits);
    lmhead_stats_simt_kernel<T><<<grid, 256, 0, stream>>>(hcat, weight, static_cast<int>(R), static_cast<int>(V),
                                                          static_cast<int>(D), tps, pm, ps, pi);
    ORTHRUS_CHECK_LAUNCH();
    lmhead_stats_combine_kernel<<<static_cast<unsigned>(ceil_div(R, 256)), 256, 0, stream>>>(
        pm, ps, pi, static_cast<int>(R), splits, lse, amax);
    ORTHRUS_CHECK_LAUNCH();
  }
  gather_lse_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, stream>>>(lse + n, index, n, m, lset);
  ORTHRUS_CHECK_LAUNCH();

  // pass 2 + 3 per chunk of student rows
  for (int64_t c0 = 0; c0 < n; c0 += p.chunk) {
    const int rows = static_cast<int>(std::min<int64_t>(p.chunk, n - c0));
    int splits = 1;
    if constexpr (kBf16) {
      CUtensorMap tmS, tmT, tmW;
      if (!make_tmap_2d_bf16(&tmS, student, D, n, D, 64, 128)) return ORTHRUS_ECUDA;
      if (!make_tmap_2d_bf16(&tmT, tg, D, n, D, 64, 128)) return ORTHRUS_ECUDA;
      if (!make_tmap_2d_bf16(&tmW, weight, D, V, D, 64, 128)) return ORTHRUS_ECUDA;
      const int vt = static_cast<int>(ceil_div(V, 128));
      const int rtiles = static_cast<int>(ceil_div(rows, 128));
      const int tps = static_cast<int>(ceil_div(vt, pick_splits(rtiles, vt, num_sms(), p.diff_splits)));
      splits = static_cast<int>(ceil_div(vt, tps));
      const int units = rtiles * splits;
      ORTHRUS_CHECK_CUDA(ensure_smem(lmhead_diff_tc_kernel, DiffTile::SMEM));
      const unsigned grid = static_cast<unsigned>(std::min(units, num_sms()));  // persistent, one CTA per SM
      lmhead_diff_tc_kernel<<<grid, 192, DiffTile::SMEM, stream>>>(tmS, tmT, tmW, diff, Vp, rows, static_cast<int>(c0),
                                                                   static_cast<int>(V), static_cast<int>(D), tps,
                                                                   rtiles, units, lse, lset, row_weight, klp);
      ORTHRUS_CHECK_LAUNCH();
    } else {
      const int vt = static_cast<int>(ceil_div(V, 64));
      const int tps = static_cast<int>(ceil_div(vt, p.diff_splits));
      splits = static_cast<int>(ceil_div(vt, tps));
      dim3 grid(static_cast<unsigned>(ceil_div(rows, 64)), splits);
      lmhead_diff_simt_kernel<T><<<grid, 256, 0, stream>>>(student, tg, weight, rows, static_cast<int>(c0),
                                                           static_cast<int>(V), static_cast<int>(D), tps, lse,
                                                           lset, row_weight, diff, Vp, klp);
      ORTHRUS_CHECK_LAUNCH();
    }
    lmhead_rows_kernel<<<static_cast<unsigned>(ceil_div(rows, 256)), 256, 0, stream>>>(
        klp, splits, rows, static_cast<int>(c0), amax, amax + n, index, m, kl_rows, agree);
    ORTHRUS_CHECK_LAUNCH();
    if (grad != nullptr) {
      int rc;
      if constexpr (kBf16)
        rc = gemm_bf16_impl(diff, Vp, weight, D, grad + c0 * D, D, rows, D, V, /*b_kn=*/1, /*c_f32=*/0, gws,
                            gemm_ws_bytes(p.chunk, D, V), stream, /*batch_invariant=*/false);
      else
        rc = gemm_simt_impl<T, true>(diff, Vp, weight, D, grad + c0 * D, D, rows, D, V, gws,
                                     simt_ws_bytes(p.chunk, D, V), stream);
      if (rc != ORTHRUS_OK) return rc;
    }
  }
  lmhead_finalize_kernel<<<1, 1024, 0, stream>>>(kl_rows, agree, row_weight, offsets, n, num_offsets, total,
                                                 kl_by_offset, agree_by_offset);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // namespace orthrus
