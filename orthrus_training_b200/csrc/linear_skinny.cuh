// Projection GEMMs of the inference passes (prefill, draft, verify): Y = epilogue(X[M, K] @ W^T)
// with many CTAs even when M is a handful of rows.
//
// A decode pass multiplies 32 rows (one block) per sequence by every weight of the model, so a
// projection is a stream of its weights: what bounds it is how many SMs pull weight rows at once.
// Each CTA here owns a 128-row x 64-column output tile (for SwiGLU 32 output columns: 32 gate and
// 32 up rows of W) and the full K, so a [32, 1024] x [1024, 3072] projection runs on 48 CTAs
// instead of the 12 of a 256-column tile. A row's result depends only on its own inputs and the
// fixed k order, never on M: a K-token verification reproduces a one-token greedy pass bit for
// bit, which is what keeps block decoding lossless.
//
// 192 threads: warp 0 TMA producer (8-stage ring of X [128 x 64] and W [64 x 64] k-blocks; for
// at most 32 rows only 32 rows of X are loaded),
// warp 1 TMEM (64 columns) and the single-thread UMMA 128 x 64 x 16 issue, warps 2-5 epilogue
// (tcgen05.ld, residual add or SwiGLU, 16-byte stores of bf16 rows). Every wait is bounded.
#pragma once

#include "linear_tc.cuh"

namespace orthrus {

struct SkinnyTile {
  static constexpr int BM = 128, BN = 64, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;  // 8 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 8;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

// grid (N / 64 output tiles, or F / 32 for SwiGLU; ceil(M / 128)).
template <int EPI>
__global__ void __launch_bounds__(192, 1)
    linear_skinny_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, int M,
                            int N, int K, int f_rows, const __nv_bfloat16* __restrict__ R, int64_t ldr,
                            __nv_bfloat16* __restrict__ Y, int64_t ldy, int a_rows) {
  using T = SkinnyTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + T::STAGES * T::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + T::STAGES * T::B_BYTES);
  uint64_t* empty = full + T::STAGES;
  uint64_t* acc_full = empty + T::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (K + T::BK - 1) / T::BK;
  const int m0 = blockIdx.y * T::BM;
  constexpr bool kSwiGLU = EPI == kLinearSwiGLU;
  const int n0 = blockIdx.x * (kSwiGLU ? T::BN / 2 : T::BN);  // first output column

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmX);
      prefetch_tensormap(&tmW);
      int issued = 0;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % T::STAGES;
        if (!mbar_wait(&empty[s], ((kb / T::STAGES) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        // with at most 32 rows only the first 32 rows of the A tile are loaded: the other lanes of
        // the accumulator are computed from stale shared memory and never stored
        mbar_arrive_expect_tx(&full[s], a_rows * T::BK * 2 + T::B_BYTES);
        tma_load_2d(sA + s * T::A_BYTES, &tmX, &full[s], kb * T::BK, m0);
        if constexpr (kSwiGLU) {  // gate rows [n0, n0 + 32) then up rows [F + n0, F + n0 + 32)
          tma_load_2d(sB + s * T::B_BYTES, &tmW, &full[s], kb * T::BK, n0);
          tma_load_2d(sB + s * T::B_BYTES + T::B_BYTES / 2, &tmW, &full[s], kb * T::BK, f_rows + n0);
        } else {
          tma_load_2d(sB + s * T::B_BYTES, &tmW, &full[s], kb * T::BK, n0);
        }
        issued = kb + 1;
      }
      if (*abort_flag)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, T::BN, false, false);
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % T::STAGES;
        if (*abort_flag || !mbar_wait(&full[s], (kb / T::STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * T::A_BYTES);
        const uint32_t b_base = smem_u32(sB + s * T::B_BYTES);
#pragma unroll
        for (int k = 0; k < T::BK / 16; ++k)
          umma_f16(tmem, umma_desc_sw128(a_base + k * 32, 16, 1024), umma_desc_sw128(b_base + k * 32, 16, 1024),
                   idesc, (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(acc_full);  // also the drain: every MMA issued has completed when it fires
    }
  } else {
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    const bool done = mbar_wait(acc_full, 0) && !*abort_flag;
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float v[64];
    tmem_ld32(base, v);
    tmem_ld32(base + 32, v + 32);
    tmem_wait_ld();
    if (done && row < M) {
      if constexpr (kSwiGLU) {
        // the roundings of silu_mul(x @ [gate; up]^T): g and u rounded, silu rounded, product
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float h[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float gr = round_to_t<__nv_bfloat16>(v[j + e]);
            const float ur = round_to_t<__nv_bfloat16>(v[32 + j + e]);
            h[e] = round_to_t<__nv_bfloat16>(silu_fast(gr)) * ur;
          }
          pk[j / 2] = pack_bf16x2(h[0], h[1]);
        }
        uint4* dst = reinterpret_cast<uint4*>(Y + static_cast<int64_t>(row) * ldy + n0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (n0 + 8 * q < N) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      } else {
        if constexpr (EPI == kLinearResidual) {
          const uint4* src = reinterpret_cast<const uint4*>(R + static_cast<int64_t>(row) * ldr + n0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (n0 + 8 * j >= N) break;
            const uint4 r = src[j];
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[j * 8 + 2 * e] += __uint_as_float(w[e] << 16);
              v[j * 8 + 2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
            }
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(Y + static_cast<int64_t>(row) * ldy + n0);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (n0 + 8 * q < N)
            dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 64);
  }
}

// Y [M, N] (pitch ldy) = X [M, K] @ W^T (+ R), or for SwiGLU Y [M, F] = silu(X gate^T) * (X up^T)
// with W = [gate; up] [2F, K] (N = F). N a multiple of 64 (SwiGLU: 32), K of 8, pitches of 8.
inline int linear_skinny_impl(const void* X, int64_t ldx, const void* W, int64_t ldw, const void* R, void* Y,
                              int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(X && W && Y && M >= 0 && N > 0 && K > 0);
  ORTHRUS_CHECK_ARG(epilogue == kLinearStore || epilogue == kLinearResidual || epilogue == kLinearSwiGLU);
  ORTHRUS_CHECK_ARG(epilogue != kLinearResidual || (R != nullptr && R != Y));
  ORTHRUS_CHECK_ARG(N % (epilogue == kLinearSwiGLU ? 32 : 64) == 0 && K % 8 == 0);
  ORTHRUS_CHECK_ARG(ldx >= K && ldw >= K && ldy >= N && ldx % 8 == 0 && ldw % 8 == 0 && ldy % 8 == 0);
  ORTHRUS_CHECK_ARG(epilogue != kLinearResidual || (R != nullptr && aligned16(R)));
  ORTHRUS_CHECK_ARG(aligned16(X) && aligned16(W) && aligned16(Y));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 30) && K < (1ll << 31));
  if (M == 0) return ORTHRUS_OK;
  using T = SkinnyTile;
  const bool swiglu = epilogue == kLinearSwiGLU;
  CUtensorMap tx, tw;
  const int a_rows = M <= 32 ? 32 : 128;  // rows of X per A box
  if (!make_tmap_2d_bf16(&tx, X, K, M, ldx, 64, a_rows)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tw, W, K, swiglu ? 2 * N : N, ldw, 64, swiglu ? 32 : 64)) return ORTHRUS_ECUDA;
  dim3 grid(static_cast<unsigned>(N / (swiglu ? 32 : 64)), static_cast<unsigned>(ceil_div(M, T::BM)));
  ORTHRUS_CHECK_ARG(grid.y < 65536);
  auto* r = static_cast<const __nv_bfloat16*>(R);
  auto* y = static_cast<__nv_bfloat16*>(Y);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (epilogue == kLinearStore) {
    ORTHRUS_CHECK_CUDA(ensure_smem(linear_skinny_tc_kernel<kLinearStore>, T::SMEM));
    linear_skinny_tc_kernel<kLinearStore><<<grid, 192, T::SMEM, stream>>>(tx, tw, m, n, k, 0, nullptr, 0, y, ldy, a_rows);
  } else if (epilogue == kLinearResidual) {
    ORTHRUS_CHECK_CUDA(ensure_smem(linear_skinny_tc_kernel<kLinearResidual>, T::SMEM));
    linear_skinny_tc_kernel<kLinearResidual><<<grid, 192, T::SMEM, stream>>>(tx, tw, m, n, k, 0, r, ldy, y, ldy, a_rows);
  } else {
    ORTHRUS_CHECK_CUDA(ensure_smem(linear_skinny_tc_kernel<kLinearSwiGLU>, T::SMEM));
    linear_skinny_tc_kernel<kLinearSwiGLU><<<grid, 192, T::SMEM, stream>>>(tx, tw, m, n, k, n, nullptr, 0, y, ldy, a_rows);
  }
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // namespace orthrus
