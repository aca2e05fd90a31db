// Projection GEMMs on CTA pairs: C[M, N] = epilogue(A @ B^T), bf16 operands, fp32 accumulation in
// the tensor memory of two SMs (tcgen05 cta_group::2, UMMA 256 x 256 x 16).
//
// A cluster of two CTAs owns a 256-row x 256-column tile: each CTA loads its own 128 rows of A and
// its own 128 columns of B (no multicast), the leader CTA (cluster rank 0) issues one UMMA over
// both CTAs' shared memory, and each CTA's TMEM receives its 128 rows of the accumulator. Per
// k-block a CTA loads 32 KB for 128 x 256 x 64 MACs, two thirds of what a one-CTA 128 x 256 tile
// loads, which is what lets the pair keep the tensor pipe fed from L2.
//
// Operand layouts (all three training-step forms of a linear layer y = x W^T):
//   A K-major  [M, K] row-major (activations x, or the output gradient dy)        forward, dX
//   A MN-major [K, M] row-major, i.e. A^T stored (dy for dW = dy^T x)              dW
//   B K-major  [N, K] row-major (the weight W for y = x W^T)                       forward
//   B MN-major [K, N] row-major (W for dX = dy W; x for dW)                        dX, dW
// Epilogues: store (bf16); residual (bf16 R + acc, one rounding: torch.addmm(R, x, W^T)); and the
// SwiGLU backward, where acc = dact = dy @ W_down of the MLP and R = [gate | up] [M, 2N] kept by the
// forward: the epilogue writes C = [dgate | dup] [M, 2N] (the arithmetic and roundings of
// swiglu_bwd_kernel), so dact never goes through HBM.
//
// Persistent: one cluster per SM pair loops over pair tiles (n fastest). 320 threads per CTA:
//   warp 0     TMA producer (both CTAs): this CTA's A and B k-blocks of 64 into a 6-stage ring;
//              completion is signalled on the leader's `full` barrier (the leader posts the byte
//              count of both CTAs);
//   warp 1     TMEM (512 columns, two 256-column accumulators, allocated as a pair) and, in the
//              leader, the single-thread UMMA issue; commits are multicast to both CTAs' barriers;
//   warps 2-9  epilogue (both CTAs): tcgen05.ld of this CTA's rows, the tail, bf16 32 x 64 staging
//              tiles written by TMA stores; the leader's `acc_empty` collects both CTAs' warps.
// Every wait is bounded; on a timeout the CTA records the error, drains its copies and returns.
#pragma once

#include "sm100.cuh"
#include "qkv_prep.cuh"

namespace orthrus {

enum Gemm2Epilogue { kGemm2Store = 0, kGemm2Residual = 1, kGemm2Partial = 2, kGemm2SwiGLUBwd = 3 };

struct Gemm2Base {
  static constexpr int BM = 128;                  // rows per CTA (256 per pair)
  static constexpr int BN = 256;                  // accumulator columns per tile
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;     // 16 KB
  static constexpr int B_BYTES = 128 * BK * 2;    // 16 KB: this CTA's 128 columns of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGING = 32 * 64 * 2;     // per epilogue warp: 32 rows x 64 bf16
  static constexpr int BOX_MN = 64 * 64 * 2;      // one [64 k][64 mn] box of an MN-major operand
};

// The SwiGLU-backward epilogue also reads [gate | up]: per epilogue warp a 4 KB buffer that TMA
// fills with the next 32 x 32 gate and up boxes, paid for with one stage of the ring (its K is
// short: the MLP's hidden size).
template <int EPI>
struct Gemm2Tile : Gemm2Base {
  static constexpr int STAGES = EPI == 3 ? 5 : 6;
  static constexpr int IN_STAGING = EPI == 3 ? 2 * 32 * 32 * 2 : 0;
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_WARPS * (STAGING + IN_STAGING) + 1024 + 256;
};

struct Gemm2Geometry {
  int M, N, K;
  int npairs;    // pair tiles along N
  int tiles;     // pair tiles x k-splits: the work units
  int splits;    // k-splits per tile (kGemm2Partial: fp32 partials, reduced by gemm2_reduce_kernel)
  int kb_split;  // k-blocks of 64 per split
  int m_pad;     // rows of one split's partial slab (M rounded up to 256)
};

// K-major operand tile of 128 rows: rows of 64 elements (128 B), 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t g2_desc_k(uint32_t base, int kk) {
  return umma_desc_sw128(base + kk * 32, 16, 1024);
}
// MN-major operand tile [64 k][128 mn] stored as two [64 k][64 mn] boxes: k-step kk = 16 rows.
__device__ __forceinline__ uint64_t g2_desc_mn(uint32_t base, int kk) {
  return umma_desc_sw128(base + kk * 2048, Gemm2Base::BOX_MN, 1024);
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(Gemm2Base::THREADS, 1)
    gemm2_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                    const Gemm2Geometry g, const __nv_bfloat16* __restrict__ R, int64_t ldr) {
  using T = Gemm2Tile<EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + T::STAGES * T::A_BYTES;
  uint8_t* staging = sB + T::STAGES * T::B_BYTES;
  uint8_t* in_staging = staging + T::EPI_WARPS * T::STAGING;  // kGemm2SwiGLUBwd only
  uint64_t* full = reinterpret_cast<uint64_t*>(in_staging + T::EPI_WARPS * T::IN_STAGING);
  uint64_t* empty = full + T::STAGES;
  uint64_t* acc_full = empty + T::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2], leader only: both CTAs' epilogue warps arrive
  uint64_t* mma_drain = acc_empty + 2;
  uint64_t* in_full = mma_drain + 1;       // [EPI_WARPS], kGemm2SwiGLUBwd: [gate | up] boxes landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(in_full + T::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int KB = (g.K + T::BK - 1) / T::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * T::EPI_WARPS);
    }
    mbar_init(mma_drain, 1);
    for (int w = 0; w < T::EPI_WARPS; ++w) mbar_init(&in_full[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before anyone signals them
  // launched as a programmatic dependent: the set-up above overlaps the previous kernel's tail;
  // operands, the residual and C belong to the stream order from here on
  griddep_launch_dependents();
  griddep_wait();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // unit u = (pair tile u / splits, k-split u % splits)
  auto tile_coords = [&](int u, int& m0, int& n0, int& kb0, int& nkb) {
    const int t = u / g.splits, sp = u % g.splits;
    m0 = (t / g.npairs) * 256 + static_cast<int>(rank) * 128;  // this CTA's rows
    n0 = (t % g.npairs) * 256;                                   // the pair's columns
    kb0 = sp * g.kb_split;
    nkb = max(0, min(KB, kb0 + g.kb_split) - kb0);
  };

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmA);
      prefetch_tensormap(&tmB);
      int it = 0, issued = 0;
      for (int t = cluster; t < g.tiles && !*abort_flag; t += nclusters) {
        int m0, n0, kb0, nkb;
        tile_coords(t, m0, n0, kb0, nkb);
        const int nb = n0 + static_cast<int>(rank) * 128;  // this CTA's columns of B
        for (int kb = kb0; kb < kb0 + nkb; ++kb, ++it) {
          const int s = it % T::STAGES;
          if (!mbar_wait(&empty[s], ((it / T::STAGES) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * T::STAGE_BYTES);
          uint8_t* a = sA + s * T::A_BYTES;
          uint8_t* b = sB + s * T::B_BYTES;
          if constexpr (A_MN) {
            tma_load_2d_pair(a, &tmA, bar, m0, kb * T::BK);
            tma_load_2d_pair(a + T::BOX_MN, &tmA, bar, m0 + 64, kb * T::BK);
          } else {
            tma_load_2d_pair(a, &tmA, bar, kb * T::BK, m0);
          }
          if constexpr (B_MN) {
            tma_load_2d_pair(b, &tmB, bar, nb, kb * T::BK);
            tma_load_2d_pair(b + T::BOX_MN, &tmB, bar, nb + 64, kb * T::BK);
          } else {
            tma_load_2d_pair(b, &tmB, bar, kb * T::BK, nb);
          }
          issued = it + 1;
        }
      }
      // after an abort, the copies still in flight complete before the CTA leaves (the leader
      // sees them on its own barriers; the peer's land on the leader's, which the leader drains)
      if (*abort_flag && leader)
        for (int i = max(0, issued - T::STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % T::STAGES], (i / T::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(256, T::BN, A_MN, B_MN);
      int it = 0, tt = 0;
      for (int t = cluster; t < g.tiles && !*abort_flag; t += nclusters, ++tt) {
        const int b = tt & 1;
        const uint32_t acc = tmem + b * T::BN;
        if (!mbar_wait_cluster(&acc_empty[b], ((tt >> 1) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        int m0, n0, kb0, nkb;
        tile_coords(t, m0, n0, kb0, nkb);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % T::STAGES;
          if (!mbar_wait(&full[s], (it / T::STAGES) & 1)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * T::A_BYTES);
          const uint32_t b_base = smem_u32(sB + s * T::B_BYTES);
#pragma unroll
          for (int k = 0; k < T::BK / 16; ++k) {
            const uint64_t ad = A_MN ? g2_desc_mn(a_base, k) : g2_desc_k(a_base, k);
            const uint64_t bd = B_MN ? g2_desc_mn(b_base, k) : g2_desc_k(b_base, k);
            umma_f16_pair(acc, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[s], 3);
        }
        umma_commit_pair(&acc_full[b], 3);
      }
      // every MMA issued has completed (in both CTAs' TMEM) before either frees its columns
      umma_commit_pair(mma_drain, 3);
      mbar_wait(mma_drain, 0);
    } else if (!leader && elect_one()) {
      mbar_wait(mma_drain, 0);  // the leader's last MMAs also wrote this CTA's TMEM
    }
  } else {
    const int quarter = warp & 3;      // TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;  // which half of the tile's columns it takes
    const uint32_t stage = smem_u32(staging + (warp - 2) * T::STAGING);
    int tt = 0;
    auto flush = [&](int col0, int row0) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < g.M && col0 < g.N) {
        tma_store_2d(&tmC, staging + (warp - 2) * T::STAGING, col0, row0);
        tma_store_commit();
      }
    };
    auto reuse = [&]() {  // the previous store has finished reading the staging tile
      if (lane == 0) tma_store_wait_read_all();
      __syncwarp();
    };
    // kGemm2SwiGLUBwd: this warp's [gate | up] buffer, one 32 x 32 box of each, one load in flight
    uint8_t* inb = in_staging + (warp - 2) * T::IN_STAGING;
    uint64_t* ib = &in_full[warp - 2];
    uint32_t in_issued = 0, in_used = 0;
    auto in_issue = [&](int col0, int r0) {
      if (lane == 0) {
        fence_proxy_async_smem();  // the lanes' reads of the previous chunk precede the overwrite
        mbar_arrive_expect_tx(ib, T::IN_STAGING);
        tma_load_2d(inb, &tmR, ib, col0, r0);
        tma_load_2d(inb + T::IN_STAGING / 2, &tmR, ib, g.N + col0, r0);
      }
      ++in_issued;
    };
    auto in_issue_tile = [&](int u, int j) {  // chunk j of this warp's rows in work unit u
      int um0, un0, ukb0, unkb;
      tile_coords(u, um0, un0, ukb0, unkb);
      in_issue(un0 + (4 * half + j) * 32, um0 + quarter * 32);
    };
    auto in_wait = [&]() -> bool {  // the oldest chunk issued has landed
      const bool ok = mbar_wait(ib, in_used & 1);
      ++in_used;
      if (!ok) *abort_flag = 1;
      return ok;
    };
    if constexpr (EPI == kGemm2SwiGLUBwd)
      if (cluster < g.tiles) in_issue_tile(cluster, 0);
    for (int t = cluster; t < g.tiles && !*abort_flag; t += nclusters, ++tt) {
      const int b = tt & 1;
      if (!mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int m0, n0, kb0, nkb;
      tile_coords(t, m0, n0, kb0, nkb);
      const int row0 = m0 + quarter * 32;
      const int row = row0 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * T::BN;
      if constexpr (EPI == kGemm2Partial) {
        // fp32 partial of this k-split into rows [split * m_pad + row] of the partial slabs, in
        // 32 x 32 boxes (128-byte rows); rows past M stay inside this split's padded slab
        const int prow0 = (t % g.splits) * g.m_pad + row0;
#pragma unroll 1
        for (int c = 4 * half; c < 4 * half + 4; ++c) {
          reuse();
          float v[32];
          tmem_ld32(base + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            st_shared_v4(stage + sw128_offset(lane, q), __float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                         __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < g.M && n0 + c * 32 < g.N) {
            tma_store_2d(&tmC, staging + (warp - 2) * T::STAGING, n0 + c * 32, prow0);
            tma_store_commit();
          }
        }
      } else if constexpr (EPI == kGemm2SwiGLUBwd) {
        // [gate | up] of this warp's 32 rows arrives 32 columns at a time by TMA into its own
        // buffer, one chunk ahead of the one being computed (across tiles too). dgate leaves
        // through the staging tile 64 columns at a time, then dup (kept packed meanwhile).
#pragma unroll 1
        for (int pair = 0; pair < 2; ++pair) {
          reuse();
          uint32_t dup[2][16];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int j = 2 * pair + cc;  // chunk of this warp's four
            uint4 gq[4], uq[4];
            const bool have = in_wait();
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // 64-byte swizzle: 16-byte unit q of row `lane`
              const uint32_t off = lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4);
              gq[q] = ld_shared_v4(smem_u32(inb) + off);
              uq[q] = ld_shared_v4(smem_u32(inb) + 2048 + off);
            }
            __syncwarp();
            if (j < 3)
              in_issue(n0 + (4 * half + j + 1) * 32, row0);
            else if (t + nclusters < g.tiles)
              in_issue_tile(t + nclusters, 0);
            float v[32];
            tmem_ld32(base + (4 * half + j) * 32, v);
            tmem_wait_ld();
            float dg[32];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t gw[4] = {gq[q].x, gq[q].y, gq[q].z, gq[q].w};
              const uint32_t uw[4] = {uq[q].x, uq[q].y, uq[q].z, uq[q].w};
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int i = 8 * q + e;
                const float gv = have ? __uint_as_float((e & 1) ? (gw[e / 2] & 0xffff0000u) : (gw[e / 2] << 16)) : 0.f;
                const float uv = have ? __uint_as_float((e & 1) ? (uw[e / 2] & 0xffff0000u) : (uw[e / 2] << 16)) : 0.f;
                const float d = bf16_round(v[i]);  // dact as the GEMM output
                const float sg = sigmoid_fast(gv);
                const float sl = bf16_round(gv * sg);
                const float ds = bf16_round(d * uv);
                dg[i] = ds * sg * (1.f + gv * (1.f - sg));
                v[i] = d * sl;  // dup
              }
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) dup[cc][q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_shared_v4(stage + sw128_offset(lane, cc * 4 + q), pack_bf16x2(dg[8 * q], dg[8 * q + 1]),
                           pack_bf16x2(dg[8 * q + 2], dg[8 * q + 3]), pack_bf16x2(dg[8 * q + 4], dg[8 * q + 5]),
                           pack_bf16x2(dg[8 * q + 6], dg[8 * q + 7]));
          }
          const int col0 = n0 + (4 * half + 2 * pair) * 32;
          flush(col0, row0);
          reuse();
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_shared_v4(stage + sw128_offset(lane, cc * 4 + q), dup[cc][4 * q], dup[cc][4 * q + 1],
                           dup[cc][4 * q + 2], dup[cc][4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < g.M && col0 < g.N) {
            tma_store_2d(&tmC, staging + (warp - 2) * T::STAGING, g.N + col0, row0);
            tma_store_commit();
          }
        }
      } else {
#pragma unroll 1
      for (int pair = 0; pair < 2; ++pair) {
        reuse();
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 4 * half + 2 * pair + cc;
          const int col0 = n0 + c * 32;
          uint4 rv[4];
          if constexpr (EPI == kGemm2Residual) {
            if (row < g.M && col0 < g.N) {
              const uint4* src = reinterpret_cast<const uint4*>(R + static_cast<int64_t>(row) * ldr + col0);
#pragma unroll
              for (int j = 0; j < 4; ++j) rv[j] = src[j];
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) rv[j] = make_uint4(0u, 0u, 0u, 0u);
            }
          }
          float v[32];
          tmem_ld32(base + c * 32, v);
          tmem_wait_ld();
          if constexpr (EPI == kGemm2Residual) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t w[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                v[j * 8 + 2 * e] += __uint_as_float(w[e] << 16);
                v[j * 8 + 2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_shared_v4(stage + sw128_offset(lane, cc * 4 + q), pack_bf16x2(v[8 * q], v[8 * q + 1]),
                         pack_bf16x2(v[8 * q + 2], v[8 * q + 3]), pack_bf16x2(v[8 * q + 4], v[8 * q + 5]),
                         pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        }
        flush(n0 + (4 * half + 2 * pair) * 32, row0);
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[b]), 0));
    }
    if constexpr (EPI == kGemm2SwiGLUBwd)
      for (; in_used < in_issued; ++in_used) mbar_wait_short(ib, in_used & 1);  // no copy outlives the CTA
    if (lane == 0) tma_store_wait_all();
  }
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or leaves while the other may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_free_pair(tmem, 512);
  }
}

// C = bf16(sum over splits of the fp32 partials, in split order (+ R)): deterministic, one rounding.
__global__ void gemm2_reduce_kernel(const float* __restrict__ part, int splits, int64_t m_pad, int M, int N,
                                    const __nv_bfloat16* __restrict__ R, int64_t ldr, __nv_bfloat16* __restrict__ C,
                                    int64_t ldc) {
  const int64_t groups = static_cast<int64_t>(M) * (N / 4);
  griddep_launch_dependents();  // launched as a programmatic dependent
  griddep_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / (N / 4);
    const int n = static_cast<int>(i % (N / 4)) * 4;
    float4 acc = *reinterpret_cast<const float4*>(part + m * N + n);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 p = *reinterpret_cast<const float4*>(part + (sp * m_pad + m) * N + n);
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    if (R != nullptr) {
      const __nv_bfloat16* r = R + m * ldr + n;
      acc.x += __bfloat162float(r[0]);
      acc.y += __bfloat162float(r[1]);
      acc.z += __bfloat162float(r[2]);
      acc.w += __bfloat162float(r[3]);
    }
    __nv_bfloat16* c = C + m * ldc + n;
    *reinterpret_cast<__nv_bfloat162*>(c) = __floats2bfloat162_rn(acc.x, acc.y);
    *reinterpret_cast<__nv_bfloat162*>(c + 2) = __floats2bfloat162_rn(acc.z, acc.w);
  }
}

// Largest number of co-resident 2-CTA clusters of a gemm2 kernel (cached per kernel).
template <int EPI, typename Kern>
inline int gemm2_max_clusters(Kern kernel) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(Gemm2Base::THREADS);
  cfg.dynamicSmemBytes = Gemm2Tile<EPI>::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) n = num_sms() / 2;
  cache[key] = n;
  return n;
}

template <int EPI, bool A_MN, bool B_MN>
inline int gemm2_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tr,
                        const Gemm2Geometry& g, const __nv_bfloat16* R, int64_t ldr, cudaStream_t stream) {
  auto kernel = gemm2_tc_kernel<EPI, A_MN, B_MN>;
  ORTHRUS_CHECK_CUDA(ensure_smem(kernel, Gemm2Tile<EPI>::SMEM));
  const int clusters = std::min(g.tiles, gemm2_max_clusters<EPI>(kernel));  // g.tiles: work units
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
  cfg.blockDim = dim3(Gemm2Base::THREADS);
  cfg.dynamicSmemBytes = Gemm2Tile<EPI>::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  ORTHRUS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, tr, g, R, ldr));
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

// k-splits of a (M, N, K) problem: only when the pair tiles fill less than one wave of clusters.
// Modelled time of a split count: the MMA work at an assumed 1.2 PF/s over the fraction of the
// cluster waves the units fill, plus the fp32 partials written and read back at 5 TB/s; the split
// count with the least modelled time, each split at least 16 k-blocks.
inline int gemm2_splits(int64_t M, int64_t N, int64_t K, int clusters) {
  const int64_t tiles = ceil_div(M, 256) * ceil_div(N, 256), kb = ceil_div(K, 64);
  if (tiles >= clusters) return 1;
  const double mma_s = 2.0 * M * N * K / 1.2e15;
  auto modelled = [&](int64_t s) {
    const int64_t units = tiles * s;
    const double fill = static_cast<double>(units) / static_cast<double>(ceil_div(units, clusters) * clusters);
    const double partial_s = s > 1 ? (8.0 * s * M * N + 2.0 * M * N) / 5e12 : 0.0;
    return mma_s / fill + partial_s;
  };
  int best = 1;
  for (int s = 2; s <= 8 && kb / s >= 16; ++s)
    if (modelled(s) < modelled(best)) best = s;
  return best;
}

inline size_t gemm2_ws_bytes(int64_t M, int64_t N, int64_t K) {
  const int s = gemm2_splits(M, N, K, num_sms() / 2);
  return s > 1 ? static_cast<size_t>(s) * ceil_div(M, 256) * 256 * N * 4 : 0;
}

// C[M, N] (pitch ldc) = A @ B^T (+ R), with A [M, K] (a_mn = 0; pitch lda) or A^T stored as
// [K, M] (a_mn = 1), B [N, K] (b_mn = 0) or B^T stored as [K, N] (b_mn = 1). All bf16; pitches
// multiples of 8 elements; pointers 16-byte aligned; R has the pitch ldr and may not alias C.
// Problems whose pair tiles fill less than one wave are split over k into fp32 partials in the
// workspace (gemm2_ws_bytes) and reduced in a fixed order.
inline int gemm2_bf16_impl(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C,
                           int64_t ldc, const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue,
                           void* ws, size_t ws_bytes, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(A && B && C && M >= 0 && N > 0 && K > 0);
  // ABI epilogue 2 is the SwiGLU backward: R = [gate | up] and C = [dgate | dup], both [M, 2N]
  const bool swiglu_bwd = epilogue == 2;
  ORTHRUS_CHECK_ARG(epilogue == kGemm2Store || ((epilogue == kGemm2Residual || swiglu_bwd) && R != nullptr && R != C));
  ORTHRUS_CHECK_ARG(!swiglu_bwd || (!a_mn && N % 64 == 0 && ldr >= 2 * N && ldc >= 2 * N));
  ORTHRUS_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0 && (R == nullptr || ldr % 8 == 0));
  ORTHRUS_CHECK_ARG(lda >= (a_mn ? M : K) && ldb >= (b_mn ? N : K) && ldc >= N && (R == nullptr || ldr >= N));
  ORTHRUS_CHECK_ARG(N % 32 == 0 && K % 8 == 0 && (!a_mn || M % 8 == 0));
  ORTHRUS_CHECK_ARG(aligned16(A) && aligned16(B) && aligned16(C) && (R == nullptr || aligned16(R)));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 30) && K < (1ll << 31));
  if (M == 0) return ORTHRUS_OK;
  if (!swiglu_bwd && (ws_bytes < gemm2_ws_bytes(M, N, K) || (gemm2_ws_bytes(M, N, K) > 0 && ws == nullptr)))
    return ORTHRUS_EWORKSPACE;
  CUtensorMap ta, tb, tc, tr{};
  const bool ok_a = a_mn ? make_tmap_2d_bf16(&ta, A, M, K, lda, 64, 64) : make_tmap_2d_bf16(&ta, A, K, M, lda, 64, 128);
  const bool ok_b = b_mn ? make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, 64) : make_tmap_2d_bf16(&tb, B, K, N, ldb, 64, 128);
  if (!ok_a || !ok_b) return ORTHRUS_ECUDA;
  Gemm2Geometry g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.npairs = static_cast<int>(ceil_div(N, 256));
  g.splits = swiglu_bwd ? 1 : gemm2_splits(M, N, K, num_sms() / 2);
  g.kb_split = static_cast<int>(ceil_div(ceil_div(K, 64), g.splits));
  g.m_pad = static_cast<int>(ceil_div(M, 256) * 256);
  const int64_t tiles = ceil_div(M, 256) * g.npairs * g.splits;
  ORTHRUS_CHECK_ARG(tiles < (1ll << 31));
  g.tiles = static_cast<int>(tiles);
  auto* r = static_cast<const __nv_bfloat16*>(R);
  if (g.splits > 1) {
    float* part = static_cast<float*>(ws);
    if (!make_tmap_2d_f32(&tc, part, N, static_cast<uint64_t>(g.splits) * g.m_pad, N, 32, 32)) return ORTHRUS_ECUDA;
    const int key = (a_mn ? 2 : 0) | (b_mn ? 1 : 0);
    int rc = key == 0   ? gemm2_launch<kGemm2Partial, false, false>(ta, tb, tc, tr, g, nullptr, 0, stream)
             : key == 1 ? gemm2_launch<kGemm2Partial, false, true>(ta, tb, tc, tr, g, nullptr, 0, stream)
             : key == 2 ? gemm2_launch<kGemm2Partial, true, false>(ta, tb, tc, tr, g, nullptr, 0, stream)
                        : gemm2_launch<kGemm2Partial, true, true>(ta, tb, tc, tr, g, nullptr, 0, stream);
    if (rc != ORTHRUS_OK) return rc;
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(M * (N / 4), 256), num_sms() * 8));
    ORTHRUS_CHECK_CUDA(launch_pdl(gemm2_reduce_kernel, dim3(blocks), dim3(256), 0, stream,
                                  static_cast<const float*>(part), g.splits, static_cast<int64_t>(g.m_pad), g.M,
                                  g.N, r, ldr, static_cast<__nv_bfloat16*>(C), ldc));
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  if (!make_tmap_2d_bf16(&tc, C, swiglu_bwd ? 2 * N : N, M, ldc, 64, 32)) return ORTHRUS_ECUDA;
  // [gate | up] boxes of 32 rows x 32 columns (64 bytes, 64-byte swizzle) for the SwiGLU backward
  if (swiglu_bwd && !make_tmap_2d_bf16(&tr, R, 2 * N, M, ldr, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return ORTHRUS_ECUDA;
  if (swiglu_bwd)
    return b_mn ? gemm2_launch<kGemm2SwiGLUBwd, false, true>(ta, tb, tc, tr, g, r, ldr, stream)
                : gemm2_launch<kGemm2SwiGLUBwd, false, false>(ta, tb, tc, tr, g, r, ldr, stream);
  const int key = (epilogue == kGemm2Residual ? 4 : 0) | (a_mn ? 2 : 0) | (b_mn ? 1 : 0);
  switch (key) {
    case 0: return gemm2_launch<kGemm2Store, false, false>(ta, tb, tc, tr, g, r, ldr, stream);
    case 1: return gemm2_launch<kGemm2Store, false, true>(ta, tb, tc, tr, g, r, ldr, stream);
    case 2: return gemm2_launch<kGemm2Store, true, false>(ta, tb, tc, tr, g, r, ldr, stream);
    case 3: return gemm2_launch<kGemm2Store, true, true>(ta, tb, tc, tr, g, r, ldr, stream);
    case 4: return gemm2_launch<kGemm2Residual, false, false>(ta, tb, tc, tr, g, r, ldr, stream);
    case 5: return gemm2_launch<kGemm2Residual, false, true>(ta, tb, tc, tr, g, r, ldr, stream);
    default: return ORTHRUS_EINVAL;  // a residual needs A in its row-major form
  }
}

}  // namespace orthrus
