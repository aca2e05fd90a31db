// Dense bf16 GEMM on the 5th-generation tensor cores: C[M, N] = A[M, K] @ B^T.
//
// One 128 x BN output tile per CTA (BN = 256, or 128 for narrow N), 192 threads:
//   warp 0     TMA producer: A and B k-blocks of 64 (one 128-byte swizzle atom) into a ring of
//              shared-memory stages, completion tracked by full/empty mbarriers;
//   warp 1     TMEM allocation and the single-thread tcgen05.mma issue loop (UMMA 128 x BN x 16),
//              tcgen05.commit frees each stage and finally signals the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of the fp32 accumulator (TMEM lane = output row) and stores.
// B may be K-major ([N, K], e.g. a weight matrix in nn.Linear layout) or MN-major ([K, N], e.g. the
// LM-head weight used as the right operand of diff @ W); both are native UMMA operand layouts.
// Split-K (fixed by N and K only, never by M) writes fp32 partials that a second kernel sums in a
// fixed order, so every output element has the same reduction order whatever M is.
#pragma once

#include "sm100.cuh"

namespace orthrus {

template <int BN, bool B_MN>
struct GemmTile {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Partials layout when splits > 1: ws[split][M][N] fp32.
template <int BN, bool B_MN, bool OUT_F32>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   void* __restrict__ C, int64_t ldc, float* __restrict__ partials, int M, int N,
                   int K, int kb_per_split) {
  using T = GemmTile<BN, B_MN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + T::STAGES * T::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + T::STAGES * T::B_BYTES);
  uint64_t* empty = full + T::STAGES;
  uint64_t* done = empty + T::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * T::BM, n0 = blockIdx.y * BN;
  const int split = blockIdx.z;
  const int KB = (K + T::BK - 1) / T::BK;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(kb0 + kb_per_split, KB);
  const int nk = max(kb1 - kb0, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmA);
      prefetch_tensormap(&tmB);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % T::STAGES;
        const uint32_t ph = (i / T::STAGES) & 1;
        if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1)) {
          *abort_flag = 1;
          break;
        }
        const int kc = (kb0 + i) * T::BK;
        mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
        tma_load_2d(sA + s * T::A_BYTES, &tmA, &full[s], kc, m0);
        if constexpr (!B_MN) {
          tma_load_2d(sB + s * T::B_BYTES, &tmB, &full[s], kc, n0);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            tma_load_2d(sB + s * T::B_BYTES + c * (64 * 64 * 2), &tmB, &full[s], n0 + c * 64, kc);
        }
        issued = i + 1;
      }
      // Drain: every issued stage must have landed before the CTA may exit.
      if (*abort_flag) {
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN, false, B_MN);
      bool issued_any = false;
      for (int i = 0; i < nk; ++i) {
        const int s = i % T::STAGES;
        const uint32_t ph = (i / T::STAGES) & 1;
        if (*abort_flag || !mbar_wait(&full[s], ph)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * T::A_BYTES);
        const uint32_t b_base = smem_u32(sB + s * T::B_BYTES);
#pragma unroll
        for (int k = 0; k < T::BK / 16; ++k) {
          const uint64_t adesc = umma_desc_sw128(a_base + k * 32, 16, 1024);
          const uint64_t bdesc = B_MN ? umma_desc_sw128(b_base + k * 2048, 64 * 64 * 2, 1024)
                                      : umma_desc_sw128(b_base + k * 32, 16, 1024);
          umma_f16(tmem, adesc, bdesc, idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        issued_any = true;
      }
      // `done` fires once all issued MMAs completed (also the drain path after an error).
      umma_commit(done);
      (void)issued_any;
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4).
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    const bool ok = mbar_wait(done, 0);
    if (!ok) *abort_flag = 1;
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      if (nk > 0) {
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      const int col0 = n0 + c * 32;
      if (!ok || row >= M || col0 >= N) continue;
      if (partials != nullptr) {
        float* dst = partials + (static_cast<int64_t>(split) * M + row) * N + col0;
        if (col0 + 32 <= N && (N % 4) == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
          for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = v[j];
        }
      } else if constexpr (OUT_F32) {
        float* dst = reinterpret_cast<float*>(C) + static_cast<int64_t>(row) * ldc + col0;
        if (col0 + 32 <= N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
          for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = v[j];
        }
      } else {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + static_cast<int64_t>(row) * ldc + col0;
        if (col0 + 32 <= N) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                  pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
            *reinterpret_cast<uint4*>(dst + j) = pk;
          }
        } else {
          for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, BN);
  }
}

// Sums split-K partials in split order and converts: C = sum_s ws[s].
template <bool OUT_F32>
__global__ void gemm_splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ C, int64_t ldc,
                                          int M, int N, int splits) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[s * total + i];
    const int64_t r = i / N, c = i % N;
    if constexpr (OUT_F32)
      reinterpret_cast<float*>(C)[r * ldc + c] = acc;
    else
      reinterpret_cast<__nv_bfloat16*>(C)[r * ldc + c] = __float2bfloat16_rn(acc);
  }
}

// Split-K factor: a function of (N, K) only, so results never depend on M.
inline int gemm_splits(int64_t N, int64_t K, int BN) {
  const int64_t ntiles = ceil_div(N, BN);
  const int64_t kb = ceil_div(K, 64);
  int splits = 1;
  const int target = num_sms();
  while (ntiles * splits * 2 <= target && kb / (splits * 2) >= 8) splits *= 2;
  return splits;
}

// Split-K factor chosen with M known, for callers that do not need batch invariance (the LM-head
// gradient GEMM of the training step): the power of two up to gemm_splits that minimises
// (waves of CTAs) x (k-blocks per CTA) plus the fp32 partials' round trip through HBM, both in
// units of one 128 x BN x 64 MMA step (about 0.47 us per SM; partials at about 6 TB/s).
inline int gemm_splits_for_m(int64_t M, int64_t N, int64_t K, int BN) {
  const int cap = gemm_splits(N, K, BN);
  const int64_t tiles = ceil_div(M, 128) * ceil_div(N, BN), kb = ceil_div(K, 64), sms = num_sms();
  int best = 1;
  double best_cost = 0.0;
  for (int s = 1; s <= cap; s *= 2) {
    const double waves = static_cast<double>(ceil_div(tiles * s, sms));
    const double steps = waves * static_cast<double>(ceil_div(kb, s));
    const double partials = s > 1 ? static_cast<double>(s) * M * N * 8.0 / 6.0e12 / 0.47e-6 : 0.0;
    const double cost = steps + partials;
    if (s == 1 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

inline int gemm_bn(int64_t N) { return N >= 256 ? 256 : 128; }

inline size_t gemm_ws_bytes(int64_t M, int64_t N, int64_t K) {
  const int splits = gemm_splits(N, K, gemm_bn(N));
  return splits > 1 ? static_cast<size_t>(splits) * M * N * sizeof(float) : 0;
}

template <int BN, bool B_MN>
int launch_gemm_tc(const CUtensorMap& ta, const CUtensorMap& tb, void* C, int64_t ldc, float* ws, int M, int N,
                   int K, int splits, bool out_f32, cudaStream_t stream) {
  using T = GemmTile<BN, B_MN>;
  const int KB = static_cast<int>(ceil_div(K, 64));
  const int kbps = static_cast<int>(ceil_div(KB, splits));
  dim3 grid(static_cast<unsigned>(ceil_div(M, 128)), static_cast<unsigned>(ceil_div(N, BN)), splits);
  float* part = splits > 1 ? ws : nullptr;
  if (out_f32) {
    auto kern = gemm_tc_kernel<BN, B_MN, true>;
    ORTHRUS_CHECK_CUDA(ensure_smem(kern, T::SMEM));
    kern<<<grid, 192, T::SMEM, stream>>>(ta, tb, C, ldc, part, M, N, K, kbps);
  } else {
    auto kern = gemm_tc_kernel<BN, B_MN, false>;
    ORTHRUS_CHECK_CUDA(ensure_smem(kern, T::SMEM));
    kern<<<grid, 192, T::SMEM, stream>>>(ta, tb, C, ldc, part, M, N, K, kbps);
  }
  ORTHRUS_CHECK_LAUNCH();
  if (splits > 1) {
    const int64_t total = static_cast<int64_t>(M) * N;
    const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), 148 * 16));
    if (out_f32)
      gemm_splitk_reduce_kernel<true><<<blocks, 256, 0, stream>>>(ws, C, ldc, M, N, splits);
    else
      gemm_splitk_reduce_kernel<false><<<blocks, 256, 0, stream>>>(ws, C, ldc, M, N, splits);
    ORTHRUS_CHECK_LAUNCH();
  }
  return ORTHRUS_OK;
}

inline int gemm_bf16_impl(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                          int64_t M, int64_t N, int64_t K, int b_kn, int c_f32, void* ws, size_t ws_bytes,
                          cudaStream_t stream, bool batch_invariant = true) {
  ORTHRUS_CHECK_ARG(A && B && C && M > 0 && N > 0 && K > 0);
  ORTHRUS_CHECK_ARG(lda >= K && ldc >= N && lda % 8 == 0 && ldb % 8 == 0);
  ORTHRUS_CHECK_ARG(b_kn ? ldb >= N : ldb >= K);
  ORTHRUS_CHECK_ARG(aligned16(A) && aligned16(B) && aligned16(C));
  ORTHRUS_CHECK_ARG(c_f32 ? (ldc % 4 == 0) : (ldc % 8 == 0));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31));
  const int bn = gemm_bn(N);
  // at most gemm_splits(N, K): the workspace gemm_ws_bytes reports always suffices
  const int splits = batch_invariant ? gemm_splits(N, K, bn) : gemm_splits_for_m(M, N, K, bn);
  if (splits > 1) {
    if (ws == nullptr || ws_bytes < static_cast<size_t>(splits) * M * N * sizeof(float)) return ORTHRUS_EWORKSPACE;
  }
  CUtensorMap ta, tb;
  if (!make_tmap_2d_bf16(&ta, A, K, M, lda, 64, 128)) return ORTHRUS_ECUDA;
  if (b_kn) {
    if (!make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, 64)) return ORTHRUS_ECUDA;
  } else {
    if (!make_tmap_2d_bf16(&tb, B, K, N, ldb, 64, bn)) return ORTHRUS_ECUDA;
  }
  float* w = static_cast<float*>(ws);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (bn == 256)
    return b_kn ? launch_gemm_tc<256, true>(ta, tb, C, ldc, w, m, n, k, splits, c_f32, stream)
                : launch_gemm_tc<256, false>(ta, tb, C, ldc, w, m, n, k, splits, c_f32, stream);
  return b_kn ? launch_gemm_tc<128, true>(ta, tb, C, ldc, w, m, n, k, splits, c_f32, stream)
              : launch_gemm_tc<128, false>(ta, tb, C, ldc, w, m, n, k, splits, c_f32, stream);
}

}  // namespace orthrus
