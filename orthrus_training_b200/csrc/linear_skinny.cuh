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
// 192 threads: warp 0 TMA producer (ring of X [rows x 64] and W [BN x 64] k-blocks, as many stages
// as about 196 KB holds; for at most 32 rows only 32 rows of X are loaded and stored per stage),
// warp 1 TMEM (max(BN, 32) columns) and the single-thread UMMA 128 x BN x 16 issue, warps 2-5
// epilogue (tcgen05.ld, residual add or SwiGLU, 16-byte stores of bf16 rows). Every wait is
// bounded.
#pragma once

#include "linear_tc.cuh"

namespace orthrus {

template <int BN_, int AROWS_>
struct SkinnyTile {
  static constexpr int BM = 128, BN = BN_, BK = 64, AROWS = AROWS_;
  static constexpr int A_BYTES = AROWS * BK * 2;  // the rows of X a stage holds: 4 KB (32) or 16 KB (128)
  static constexpr int B_BYTES = BN * BK * 2;     // 2 / 4 / 8 KB (a whole number of 1 KB swizzle atoms)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // as many stages as about 196 KB holds (at most 32): what a CTA keeps in flight sets how fast
  // its SM pulls weight rows
  static constexpr int STAGES = (196 * 1024) / STAGE_BYTES < 32 ? (196 * 1024) / STAGE_BYTES : 32;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024;
  // the UMMA reads 128 rows (16 KB) from a stage's A slot: with 32-row slots the rows past 32 come
  // from the slots after it (and, for the last, the B slots), all inside the allocation
  static_assert(AROWS == 128 || STAGES * B_BYTES >= 12 * 1024, "UMMA A reads stay in shared memory");
};

// grid (N / BN output tiles, or F / (BN / 2) for SwiGLU; ceil(M / 128)). Launched as a
// programmatic dependent: the barriers, TMEM and the first STAGES k-blocks of W are set up while
// the previous kernel finishes; X, the residual and Y are touched only after griddep_wait().
template <int EPI, int BN, int AROWS>
__global__ void __launch_bounds__(192, 1)
    linear_skinny_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, int M,
                            int N, int K, int f_rows, const __nv_bfloat16* __restrict__ R, int64_t ldr,
                            __nv_bfloat16* __restrict__ Y, int64_t ldy, int a_rows) {
  using T = SkinnyTile<BN, AROWS>;
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
  constexpr int OUT = kSwiGLU ? BN / 2 : BN;  // output columns of this CTA
  const int n0 = blockIdx.x * OUT;            // first output column

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, T::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  griddep_launch_dependents();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmX);
      prefetch_tensormap(&tmW);
      auto load_w = [&](int kb, int s) {
        if constexpr (kSwiGLU) {  // gate rows [n0, n0 + BN/2) then up rows [F + n0, F + n0 + BN/2)
          tma_load_2d(sB + s * T::B_BYTES, &tmW, &full[s], kb * T::BK, n0);
          tma_load_2d(sB + s * T::B_BYTES + T::B_BYTES / 2, &tmW, &full[s], kb * T::BK, f_rows + n0);
        } else {
          tma_load_2d(sB + s * T::B_BYTES, &tmW, &full[s], kb * T::BK, n0);
        }
      };
      // with at most 32 rows only the first 32 rows of the A tile are loaded: the other lanes of
      // the accumulator are computed from stale shared memory and never stored
      const uint32_t stage_tx = a_rows * T::BK * 2 + T::B_BYTES;
      // the weights do not depend on the previous kernel: the first ring's worth streams in
      // before griddep_wait(), the activations after it
      const int pre = KB < T::STAGES ? KB : T::STAGES;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], stage_tx);
        load_w(kb, kb);
      }
      griddep_wait();
      for (int kb = 0; kb < pre; ++kb) tma_load_2d(sA + kb * T::A_BYTES, &tmX, &full[kb], kb * T::BK, m0);
      int issued = pre;
      for (int kb = pre; kb < KB; ++kb) {
        const int s = kb % T::STAGES;
        if (!mbar_wait(&empty[s], ((kb / T::STAGES) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_2d(sA + s * T::A_BYTES, &tmX, &full[s], kb * T::BK, m0);
        load_w(kb, s);
        issued = kb + 1;
      }
      if (*abort_flag)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN, false, false);
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
    griddep_wait();  // the residual and Y belong to the stream order from here on
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    const bool done = mbar_wait(acc_full, 0) && !*abort_flag;
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float v[BN < 32 ? 32 : BN];  // columns past BN (BN = 16) are allocated but never written
    tmem_ld32(base, v);
    if constexpr (BN == 64) tmem_ld32(base + 32, v + 32);
    tmem_wait_ld();
    if (done && row < M) {
      if constexpr (kSwiGLU) {
        // the roundings of silu_mul(x @ [gate; up]^T): g and u rounded, silu rounded, product
        uint32_t pk[OUT / 2];
#pragma unroll
        for (int j = 0; j < OUT; j += 2) {
          float h[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float gr = round_to_t<__nv_bfloat16>(v[j + e]);
            const float ur = round_to_t<__nv_bfloat16>(v[OUT + j + e]);
            h[e] = round_to_t<__nv_bfloat16>(silu_fast(gr)) * ur;
          }
          pk[j / 2] = pack_bf16x2(h[0], h[1]);
        }
        uint4* dst = reinterpret_cast<uint4*>(Y + static_cast<int64_t>(row) * ldy + n0);
#pragma unroll
        for (int q = 0; q < OUT / 8; ++q)
          if (n0 + 8 * q < N) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      } else {
        if constexpr (EPI == kLinearResidual) {
          const uint4* src = reinterpret_cast<const uint4*>(R + static_cast<int64_t>(row) * ldr + n0);
#pragma unroll
          for (int j = 0; j < OUT / 8; ++j) {
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
        for (int q = 0; q < OUT / 8; ++q)
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
    tmem_free(tmem, T::TMEM_COLS);
  }
}

template <int EPI, int BN, int AROWS>
inline cudaError_t skinny_launch(const CUtensorMap& tx, const CUtensorMap& tw, int M, int N, int K, int f_rows,
                                 const __nv_bfloat16* R, int64_t ldr, __nv_bfloat16* Y, int64_t ldy, int a_rows,
                                 cudaStream_t stream) {
  using T = SkinnyTile<BN, AROWS>;
  auto kernel = linear_skinny_tc_kernel<EPI, BN, AROWS>;
  cudaError_t e = ensure_smem(kernel, T::SMEM);
  if (e != cudaSuccess) return e;
  const int out = EPI == kLinearSwiGLU ? BN / 2 : BN;
  const dim3 grid(static_cast<unsigned>(N / out), static_cast<unsigned>(ceil_div(M, T::BM)));
  return launch_pdl(kernel, grid, dim3(192), T::SMEM, stream, tx, tw, M, N, K, f_rows, R, ldr, Y, ldy, a_rows);
}

// Output columns per CTA: the widest tile (64, 32 or 16 accumulator columns) that still gives at
// least 128 CTAs, else 16. A narrower tile only splits the columns: every output element keeps the
// same k order, so all widths (and the 128 x 256 persistent kernel) give the same bits.
inline int skinny_tile_n(int64_t M, int64_t acc_cols) {
  const int64_t mt = ceil_div(M, 128);
  for (int bn : {64, 32})
    if ((acc_cols / bn) * mt >= 128) return bn;
  return 16;
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
  ORTHRUS_CHECK_ARG(ceil_div(M, 128) < 65536);
  if (M == 0) return ORTHRUS_OK;
  const bool swiglu = epilogue == kLinearSwiGLU;
  const int bn = skinny_tile_n(M, swiglu ? 2 * N : N);
  CUtensorMap tx, tw;
  const int a_rows = M <= 32 ? 32 : 128;  // rows of X per A box
  if (!make_tmap_2d_bf16(&tx, X, K, M, ldx, 64, a_rows)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tw, W, K, swiglu ? 2 * N : N, ldw, 64, swiglu ? bn / 2 : bn)) return ORTHRUS_ECUDA;
  auto* r = static_cast<const __nv_bfloat16*>(R);
  auto* y = static_cast<__nv_bfloat16*>(Y);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  cudaError_t e;
#define ORTHRUS_SKINNY3(EPI_, BN_, AR_)                                                                          \
  e = skinny_launch<EPI_, BN_, AR_>(tx, tw, m, n, k, EPI_ == kLinearSwiGLU ? n : 0,                              \
                                    EPI_ == kLinearResidual ? r : nullptr, ldy, y, ldy, a_rows, stream)
#define ORTHRUS_SKINNY(EPI_, BN_) \
  if (a_rows == 32) ORTHRUS_SKINNY3(EPI_, BN_, 32); else ORTHRUS_SKINNY3(EPI_, BN_, 128)
#define ORTHRUS_SKINNY_BN(EPI_)                      \
  if (bn == 64) {                                    \
    ORTHRUS_SKINNY(EPI_, 64);                        \
  } else if (bn == 32) {                             \
    ORTHRUS_SKINNY(EPI_, 32);                        \
  } else {                                           \
    ORTHRUS_SKINNY(EPI_, 16);                        \
  }
  if (epilogue == kLinearStore) {
    ORTHRUS_SKINNY_BN(kLinearStore);
  } else if (epilogue == kLinearResidual) {
    ORTHRUS_SKINNY_BN(kLinearResidual);
  } else {
    ORTHRUS_SKINNY_BN(kLinearSwiGLU);
  }
#undef ORTHRUS_SKINNY_BN
#undef ORTHRUS_SKINNY
#undef ORTHRUS_SKINNY3
  ORTHRUS_CHECK_CUDA(e);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // namespace orthrus
