// Projection GEMMs of the inference passes (prefill, draft, verify): Y = epilogue(X[M, K] @ W^T)
// with many CTAs even when M is a handful of rows.
//
// A decode pass multiplies 32 rows (one block) per sequence by every weight of the model, so a
// projection is a stream of its weights: what bounds it is how many SMs pull weight rows at once.
// Each CTA here owns a 128-row x BN-column output tile (BN = 64, 32 or 16 accumulator columns; for
// SwiGLU BN/2 gate and BN/2 up rows of W) and the full K, so a [32, 1024] x [1024, 3072]
// projection runs on 96-192 CTAs instead of the 12 of a 256-column tile. A row's result depends
// only on its own inputs and the k order, never on M or BN, and equals what the persistent
// 128 x 256 kernel gives it: a K-token verification reproduces one-token greedy passes bit for
// bit whichever of the two kernels a pass's row count selects, which keeps block decoding
// lossless.
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
  // k-blocks of 64 per stage: a stage is one TMA box of X and one of W spanning KSUB k-blocks (the
  // boxes of a K-blocked tensor map). With 32-row slots four k-blocks per box: a CTA's time is set
  // by how many TMA copies it issues one after another, and this quarters them.
  static constexpr int KSUB = AROWS == 32 ? 4 : 1;
  static constexpr int A_SUB = AROWS * BK * 2;     // one k-block of X: 4 KB (32 rows) or 16 KB (128)
  static constexpr int B_SUB = BN * BK * 2;        // one k-block of W: 2 / 4 / 8 KB (1 KB swizzle atoms)
  static constexpr int A_BYTES = KSUB * A_SUB;
  static constexpr int B_BYTES = KSUB * B_SUB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // as many stages as about 196 KB holds (at most 32)
  static constexpr int STAGES = (196 * 1024) / STAGE_BYTES < 32 ? (196 * 1024) / STAGE_BYTES : 32;
  // One accumulation chain over all k-blocks in order: the k order of the persistent 128 x 256
  // kernel, so the two give a row the same bits. (Four interleaved chains summed at the end were
  // measured: no faster, since a CTA's time here is its TMA and UMMA issue, not UMMA latency.)
  static constexpr int CHAINS = 1;
  static constexpr int TMEM_COLS = CHAINS * BN < 32 ? 32 : CHAINS * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024;
  // the UMMA reads 128 rows (16 KB) from a k-block's A slot: with 32-row slots the rows past 32
  // come from the slots after it (and, for the last, the B slots), all inside the allocation
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
  const int KB = K / T::BK;                        // k-blocks (K is a multiple of 64)
  const int NST = (KB + T::KSUB - 1) / T::KSUB;   // stage loads
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
      // stage st holds k-blocks [st * KSUB, st * KSUB + KSUB): X box (64, rows, KSUB) and W box
      // (64, BN, KSUB), or for SwiGLU (64, BN/2, gate | up, KSUB): per k-block the BN/2 gate rows
      // [n0, n0 + BN/2) and then the BN/2 up rows [F + n0, ...)
      auto load_w = [&](int st, int s) {
        if constexpr (kSwiGLU)
          tma_load_4d(sB + s * T::B_BYTES, &tmW, &full[s], 0, n0, 0, st * T::KSUB);
        else
          tma_load_3d(sB + s * T::B_BYTES, &tmW, &full[s], 0, n0, st * T::KSUB);
      };
      auto load_x = [&](int st, int s) { tma_load_3d(sA + s * T::A_BYTES, &tmX, &full[s], 0, m0, st * T::KSUB); };
      // full boxes are counted even where k-blocks past K are filled with zeros
      const uint32_t stage_tx = T::STAGE_BYTES;
      // the weights do not depend on the previous kernel: the first ring's worth streams in
      // before griddep_wait(), the activations after it
      const int pre = NST < T::STAGES ? NST : T::STAGES;
      for (int st = 0; st < pre; ++st) {
        mbar_arrive_expect_tx(&full[st], stage_tx);
        load_w(st, st);
      }
      griddep_wait();
      for (int st = 0; st < pre; ++st) load_x(st, st);
      int issued = pre;
      for (int st = pre; st < NST; ++st) {
        const int s = st % T::STAGES;
        if (!mbar_wait(&empty[s], ((st / T::STAGES) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], stage_tx);
        load_x(st, s);
        load_w(st, s);
        issued = st + 1;
      }
      if (*abort_flag)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN, false, false);
      bool ok = true;
      for (int st = 0; st < NST; ++st) {
        const int s = st % T::STAGES;
        if (*abort_flag || !mbar_wait(&full[s], (st / T::STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < T::KSUB; ++j) {
          const int kb = st * T::KSUB + j;
          if (kb >= KB) break;
          const uint32_t a_base = smem_u32(sA + s * T::A_BYTES + j * T::A_SUB);
          const uint32_t b_base = smem_u32(sB + s * T::B_BYTES + j * T::B_SUB);
          const uint32_t acc = tmem + (kb % T::CHAINS) * BN;
#pragma unroll
          for (int k = 0; k < T::BK / 16; ++k)
            umma_f16(acc, umma_desc_sw128(a_base + k * 32, 16, 1024), umma_desc_sw128(b_base + k * 32, 16, 1024),
                     idesc, (kb >= T::CHAINS || k > 0) ? 1u : 0u);
        }
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
    // the chains that received k-blocks, summed in chain order (a fixed order for a given K)
    const int nch = KB < T::CHAINS ? KB : T::CHAINS;
    float v[BN];
    auto load_chain = [&](int c, float* dst) {
      if constexpr (BN == 16) {
        tmem_ld16(base + c * BN, dst);
      } else {
        tmem_ld32(base + c * BN, dst);
        if constexpr (BN == 64) tmem_ld32(base + c * BN + 32, dst + 32);
      }
      tmem_wait_ld();
    };
    load_chain(0, v);
#pragma unroll 1
    for (int c = 1; c < nch; ++c) {
      float t[BN];
      load_chain(c, t);
#pragma unroll
      for (int i = 0; i < BN; ++i) v[i] += t[i];
    }
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
// same k order, so all widths, all row counts (and the persistent kernel) give the same bits.
inline int skinny_tile_n(int64_t M, int64_t acc_cols) {
  const int64_t mt = ceil_div(M, 128);
  for (int bn : {64, 32})
    if ((acc_cols / bn) * mt >= 128) return bn;
  return 16;
}

// Y [M, N] (pitch ldy) = X [M, K] @ W^T (+ R), or for SwiGLU Y [M, F] = silu(X gate^T) * (X up^T)
// with W = [gate; up] [2F, K] (N = F). N a multiple of 64 (SwiGLU: 32), K of 64, pitches of 8.
inline int linear_skinny_impl(const void* X, int64_t ldx, const void* W, int64_t ldw, const void* R, void* Y,
                              int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(X && W && Y && M >= 0 && N > 0 && K > 0);
  ORTHRUS_CHECK_ARG(epilogue == kLinearStore || epilogue == kLinearResidual || epilogue == kLinearSwiGLU);
  ORTHRUS_CHECK_ARG(epilogue != kLinearResidual || (R != nullptr && R != Y));
  ORTHRUS_CHECK_ARG(N % (epilogue == kLinearSwiGLU ? 32 : 64) == 0 && K % 64 == 0);
  ORTHRUS_CHECK_ARG(ldx >= K && ldw >= K && ldy >= N && ldx % 8 == 0 && ldw % 8 == 0 && ldy % 8 == 0);
  ORTHRUS_CHECK_ARG(epilogue != kLinearResidual || (R != nullptr && aligned16(R)));
  ORTHRUS_CHECK_ARG(aligned16(X) && aligned16(W) && aligned16(Y));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 30) && K < (1ll << 31));
  ORTHRUS_CHECK_ARG(ceil_div(M, 128) < 65536);
  if (M == 0) return ORTHRUS_OK;
  const bool swiglu = epilogue == kLinearSwiGLU;
  const int bn = skinny_tile_n(M, swiglu ? 2 * N : N);
  CUtensorMap tx, tw;
  const int a_rows = M <= 32 ? 32 : 128;   // rows of X per box
  const int ksub = a_rows == 32 ? 4 : 1;   // k-blocks per box (SkinnyTile::KSUB)
  if (!make_tmap_kblocked_bf16(&tx, X, M, K, ldx, a_rows, ksub)) return ORTHRUS_ECUDA;
  if (!(swiglu ? make_tmap_kblocked_bf16(&tw, W, 2 * N, K, ldw, bn / 2, ksub, 2, N)
               : make_tmap_kblocked_bf16(&tw, W, N, K, ldw, bn, ksub)))
    return ORTHRUS_ECUDA;
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
