// Projection GEMMs of the Qwen3 layers with their elementwise tails fused into the epilogue:
// Y = epilogue(X[M, K] @ W^T), bf16 operands, fp32 accumulation in tensor memory.
//
//   kLinearStore     Y[M, N] = acc                                   (F.linear)
//   kLinearResidual  Y[M, N] = R[M, N] + acc, one rounding            (torch.addmm(R, X, W^T))
//   kLinearSwiGLU    W = [gate; up] of shape [2F, K]; Y[M, F] = silu(g) * u with g and u rounded
//                    to bf16 first and silu rounded before the product (F.linear followed by
//                    F.silu(gate) * up, orthrus/objective.py:146-149), so [gate | up] is never
//                    written to or read back from HBM.
//   kLinearSwiGLUKeep  the SwiGLU form that also writes [gate | up] (bf16, the F.linear output),
//                    which the backward of the activation needs (the trainable view's MLP).
//   kLinearQkvRope   W = [q; k; v] heads of 128: the q and k heads get the per-head RMSNorm and
//                    RoPE of the attention prologue (orthrus/objective.py:136-143, the arithmetic
//                    and roundings of qkv_prep_fwd_row_kernel) and every head is written head-major
//                    ([B, H, L, 128]) for the attention kernels. The frozen view writes nothing
//                    else; the trainable view also keeps the q / k columns of the token-major
//                    projection and rstd, which the prologue's backward reads.
//
// One CTA per SM loops over 128-row x 256-accumulator-column tiles in m-major order (the CTAs in
// flight share one weight panel in L2 and read each activation panel from HBM once), 320 threads:
//   warp 0     TMA producer: X and W k-blocks of 64 (one 128-byte swizzle atom) into a 4-stage ring;
//              W arrives as two 128-row boxes (the two halves of the tile, or gate and up rows);
//   warp 1     TMEM allocation and the single-thread tcgen05.mma issue loop (UMMA 128 x 256 x 16)
//              into one of two 256-column accumulators, so the epilogue of tile t overlaps the
//              mainloop of tile t + 1;
//   warps 2-9  epilogue, two warps per TMEM lane quarter splitting the columns: tcgen05.ld
//              (TMEM lane = output row), the fused tail, bf16 rows into a per-warp 32 x 64 staging
//              tile (128-byte swizzle) that one TMA store writes out (clipped at M and N).
// Every wait is bounded; on a timeout the CTA records the error, drains its copies and returns.
#pragma once

#include "sm100.cuh"
#include "qkv_prep.cuh"
#include "rowwise.cuh"

namespace orthrus {

enum LinearEpilogue {
  kLinearStore = 0,
  kLinearResidual = 1,
  kLinearSwiGLU = 2,
  kLinearQkvRope = 3,
  kLinearSwiGLUKeep = 4
};

// Operands of the q|k|v epilogue: rows are tokens t of L per sequence (M = B * L, L a multiple of
// 128, RoPE position = t); cos / sin [L][64] hold cos(t * inv_freq[i]) rounded to bf16.
struct QkvRopeParams {
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  const int64_t* positions;  // RoPE position per row, or null for t
  float* rstd_out;           // [rows, Hq + Hkv] rsqrt(mean(x^2) + eps) per q / k head, or null
  bool keep;                 // also write the q / k columns of the projection token-major (tmP)
  int L, Hq, Hkv;
  int64_t table_rows;        // rows of rope_cos / rope_sin
  float eps;
};

struct LinearTile {
  static constexpr int BM = 128, BN = 256, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;    // 16 KB
  static constexpr int B_HALF = 128 * BK * 2;    // 16 KB: one 128-row W box
  static constexpr int B_BYTES = 2 * B_HALF;     // 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGING = 32 * 64 * 2;  // per epilogue warp: 32 rows x 64 bf16
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_WARPS * STAGING + 1024 + 256;
};

// silu(g) = g / (1 + exp(-g)) with exp(-g) = 2^(-g log2 e) on ex2.approx and an approximate
// reciprocal: within a few fp32 ulps of the IEEE form, far below the bf16 rounding that follows.
__device__ __forceinline__ float silu_fast(float g) {
  return __fdividef(g, 1.f + ex2_approx(-g * kLog2e));
}

// Tile t -> (m tile, n tile) and the first W row of each 128-row half of the accumulator.
struct LinearGeometry {
  int M, N, K, ntiles, tiles, f_rows;  // f_rows: F (up rows start there) for SwiGLU, else 0
  // pair: tiles of 256 rows over a CTA pair, this CTA's 128 rows at rank * 128
  __device__ __forceinline__ void tile(int t, int epi, int& m0, int& n0, int& w0, int& w1, bool pair = false,
                                       int rank = 0) const {
    const int mt = t / ntiles, nt = t % ntiles;
    m0 = pair ? mt * 2 * LinearTile::BM + rank * LinearTile::BM : mt * LinearTile::BM;
    if (epi == kLinearSwiGLU || epi == kLinearSwiGLUKeep) {
      n0 = nt * 128;
      w0 = n0;
      w1 = f_rows + n0;
    } else {
      n0 = nt * LinearTile::BN;
      w0 = n0;
      // N is a multiple of 128: the upper half is either wholly inside W or wholly past its end,
      // in which case the lower rows are loaded again and their columns never stored
      w1 = n0 + 128 < N ? n0 + 128 : n0;
    }
  }
};

// PAIR: the same kernel on CTA pairs (tcgen05 cta_group::2, UMMA 256 x 256 x 16): each CTA of the
// pair loads its own 128 rows of X and one of the two 128-row W boxes (no multicast), the leader
// issues the MMA over both CTAs' shared memory, and each CTA's TMEM holds the accumulator of its
// rows with exactly the one-CTA column layout, so every epilogue is unchanged. Per k-block a CTA
// loads 32 KB instead of 48 KB for the same MACs.
template <int EPI, bool PAIR = false>
__global__ void __launch_bounds__(LinearTile::THREADS, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmP,
                     const LinearGeometry g, int64_t ldr, const __nv_bfloat16* __restrict__ R,
                     const QkvRopeParams qp) {
  using T = LinearTile;
  // one-CTA ring: 4 stages of X (16 KB) + both W boxes (32 KB); pair ring: 6 stages of X + one box
  constexpr int STAGES = PAIR ? 6 : T::STAGES;
  constexpr int B_STAGE = PAIR ? T::B_HALF : T::B_BYTES;
  constexpr int STAGE_BYTES = T::A_BYTES + B_STAGE;
  static_assert(STAGES * STAGE_BYTES == T::STAGES * T::STAGE_BYTES, "both rings fill the same space");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * T::A_BYTES;
  uint8_t* staging = sB + STAGES * B_STAGE;  // 1024-aligned: the ring is a multiple of 1 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + T::EPI_WARPS * T::STAGING);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* mma_drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (g.K + T::BK - 1) / T::BK;
  const int rank = PAIR ? static_cast<int>(cluster_ctarank()) : 0;
  const bool leader = rank == 0;
  const int first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int stride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], (PAIR ? 2 : 1) * T::EPI_WARPS);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, 512);
    else
      tmem_alloc(tmem_slot, 512);
  }
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // the peer's barriers exist before anyone signals them
  // launched as a programmatic dependent: the set-up above overlaps the previous kernel's tail;
  // operands and outputs belong to the stream order from here on
  griddep_launch_dependents();
  griddep_wait();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tensormap(&tmX);
      prefetch_tensormap(&tmW);
      int it = 0, issued = 0;
      for (int t = first; t < g.tiles && !*abort_flag; t += stride) {
        int m0, n0, w0, w1;
        g.tile(t, EPI, m0, n0, w0, w1, PAIR, rank);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          if constexpr (PAIR) {
            // this CTA's rows and its W box (rank 0: the first 128 accumulator columns); the leader
            // posts the bytes of both CTAs on its own barrier, which both CTAs' copies complete
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
            tma_load_2d_pair(sA + s * T::A_BYTES, &tmX, bar, kb * T::BK, m0);
            tma_load_2d_pair(sB + s * B_STAGE, &tmW, bar, kb * T::BK, rank == 0 ? w0 : w1);
          } else {
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(sA + s * T::A_BYTES, &tmX, &full[s], kb * T::BK, m0);
            tma_load_2d(sB + s * B_STAGE, &tmW, &full[s], kb * T::BK, w0);
            tma_load_2d(sB + s * B_STAGE + T::B_HALF, &tmW, &full[s], kb * T::BK, w1);
          }
          issued = it + 1;
        }
      }
      if (*abort_flag && leader)
        for (int i = max(0, issued - STAGES); i < issued; ++i)
          mbar_wait_short(&full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(PAIR ? 256 : 128, T::BN, false, false);
      int it = 0, tt = 0;
      for (int t = first; t < g.tiles && !*abort_flag; t += stride, ++tt) {
        const int b = tt & 1;
        const uint32_t acc = tmem + b * T::BN;
        const bool free_acc = PAIR ? mbar_wait_cluster(&acc_empty[b], ((tt >> 1) & 1) ^ 1)
                                   : mbar_wait(&acc_empty[b], ((tt >> 1) & 1) ^ 1);
        if (!free_acc) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * T::A_BYTES);
          const uint32_t b_base = smem_u32(sB + s * B_STAGE);
#pragma unroll
          for (int k = 0; k < T::BK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(b_base + k * 32, 16, 1024);
            if constexpr (PAIR)
              umma_f16_pair(acc, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else
              umma_f16(acc, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            umma_commit_pair(&empty[s], 3);
          else
            umma_commit(&empty[s]);
        }
        if constexpr (PAIR)
          umma_commit_pair(&acc_full[b], 3);
        else
          umma_commit(&acc_full[b]);
      }
      // every MMA this thread issued has completed before the accumulators are freed
      if constexpr (PAIR)
        umma_commit_pair(mma_drain, 3);
      else
        umma_commit(mma_drain);
      mbar_wait_short(mma_drain, 0);
    } else if (PAIR && !leader && elect_one()) {
      mbar_wait(mma_drain, 0);  // the leader's MMAs also write this CTA's TMEM
    }
  } else {
    const int quarter = warp & 3;          // TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;      // which half of the tile's columns it takes
    const uint32_t stage = smem_u32(staging + (warp - 2) * T::STAGING);
    int tt = 0;
    // 64 output columns [col0, col0 + 64) of this warp's 32 rows from the staging tile; a box
    // that starts past the last row or column is not stored at all (the rest is clipped by TMA)
    auto flush = [&](int col0, int row0) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < g.M && col0 < g.N) {
        tma_store_2d(&tmY, staging + (warp - 2) * T::STAGING, col0, row0);
        tma_store_commit();
      }
    };
    auto reuse = [&]() {  // the previous store has finished reading the staging tile
      if (lane == 0) tma_store_wait_read_all();
      __syncwarp();
    };
    for (int t = first; t < g.tiles && !*abort_flag; t += stride, ++tt) {
      const int b = tt & 1;
      if (!mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int m0, n0, w0, w1;
      g.tile(t, EPI, m0, n0, w0, w1, PAIR, rank);
      const int row0 = m0 + quarter * 32;
      const int row = row0 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * T::BN;
      if constexpr (EPI == kLinearQkvRope) {
        // this warp: head n0 / 128 + half, 32 tokens t0 .. t0 + 31 of sequence bq
        const int head = n0 / 128 + half;
        const int kind = head < qp.Hq ? 0 : head < qp.Hq + qp.Hkv ? 1 : 2;
        const int bq = m0 / qp.L, t0 = m0 % qp.L + quarter * 32;
        int64_t tok = qp.positions != nullptr ? qp.positions[row] : static_cast<int64_t>(t0 + lane);
        if (tok < 0 || tok >= qp.table_rows) {  // a position past the table: clamp and report
          record_error(ORTHRUS_ERR_BOUNDS);
          tok = tok < 0 ? 0 : qp.table_rows - 1;
        }
        const int hk = kind == 0 ? head : kind == 1 ? head - qp.Hq : head - qp.Hq - qp.Hkv;
        const int out_row0 = (bq * (kind == 0 ? qp.Hq : qp.Hkv) + hk) * qp.L + t0;
        const CUtensorMap* omap = kind == 0 ? &tmY : kind == 1 ? &tmK : &tmV;
        const uint32_t hbase = base + half * 128;
        float rstd = 1.f;
        if (kind < 2) {
          // the prologue's sum of squares: lane l of its warp held elements 4l..4l+3, then an xor
          // butterfly over the 32 lanes; replayed in the same order on this thread's row
          float part[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(hbase + c * 32, v);
            tmem_wait_ld();
            round_all<__nv_bfloat16, 32>(v);
#pragma unroll
            for (int l = 0; l < 8; ++l) {
              float ss = 0.f;
#pragma unroll
              for (int k = 0; k < 4; ++k) ss = fmaf(v[4 * l + k], v[4 * l + k], ss);
              part[c * 8 + l] = ss;
            }
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int l = 0; l < off; ++l) part[l] += part[l + off];
          rstd = rsqrtf(part[0] / 128.f + qp.eps);
          if (qp.rstd_out != nullptr) qp.rstd_out[static_cast<int64_t>(row) * (qp.Hq + qp.Hkv) + head] = rstd;
        }
        const __nv_bfloat16* wn = kind == 0 ? qp.q_norm_w : qp.k_norm_w;
#pragma unroll 1
        for (int cp = 0; cp < 2; ++cp) {  // elements i = cp*32 + j and their RoPE partners i + 64
          reuse();
          float lo[32], hi[32];
          tmem_ld32(hbase + cp * 32, lo);
          tmem_ld32(hbase + (cp + 2) * 32, hi);
          tmem_wait_ld();
          round_all<__nv_bfloat16, 32>(lo);
          round_all<__nv_bfloat16, 32>(hi);
          if (qp.keep && kind < 2) {  // the projection itself, token-major, for the backward
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              st_shared_v4(stage + sw64_offset(lane, q), pack_bf16x2(lo[8 * q], lo[8 * q + 1]),
                           pack_bf16x2(lo[8 * q + 2], lo[8 * q + 3]), pack_bf16x2(lo[8 * q + 4], lo[8 * q + 5]),
                           pack_bf16x2(lo[8 * q + 6], lo[8 * q + 7]));
              st_shared_v4(stage + 2048 + sw64_offset(lane, q), pack_bf16x2(hi[8 * q], hi[8 * q + 1]),
                           pack_bf16x2(hi[8 * q + 2], hi[8 * q + 3]), pack_bf16x2(hi[8 * q + 4], hi[8 * q + 5]),
                           pack_bf16x2(hi[8 * q + 6], hi[8 * q + 7]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              uint8_t* sbuf = staging + (warp - 2) * T::STAGING;
              tma_store_2d(&tmP, sbuf, head * 128 + cp * 32, row0);
              tma_store_2d(&tmP, sbuf + 2048, head * 128 + 64 + cp * 32, row0);
              tma_store_commit();
            }
            reuse();
          }
          if (kind < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              lo[j] *= rstd;
              hi[j] *= rstd;
            }
            round_all<__nv_bfloat16, 32>(lo);
            round_all<__nv_bfloat16, 32>(hi);
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {
              float wl[8], wh[8], cs[8], sn[8];
              load_elems<__nv_bfloat16, 8>(wn + cp * 32 + g8 * 8, wl);
              load_elems<__nv_bfloat16, 8>(wn + 64 + cp * 32 + g8 * 8, wh);
              load_elems<__nv_bfloat16, 8>(qp.rope_cos + static_cast<int64_t>(tok) * 64 + cp * 32 + g8 * 8, cs);
              load_elems<__nv_bfloat16, 8>(qp.rope_sin + static_cast<int64_t>(tok) * 64 + cp * 32 + g8 * 8, sn);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                lo[g8 * 8 + e] *= wl[e];
                hi[g8 * 8 + e] *= wh[e];
              }
              round_all<__nv_bfloat16, 8>(lo + g8 * 8);
              round_all<__nv_bfloat16, 8>(hi + g8 * 8);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float a = lo[g8 * 8 + e], bb = hi[g8 * 8 + e];
                const float ra = -bb, rb = a;  // rotate_half: the lower half takes -upper
                lo[g8 * 8 + e] = a * cs[e] + ra * sn[e];
                hi[g8 * 8 + e] = bb * cs[e] + rb * sn[e];
              }
            }
          }
          // two 32 x 32 staging boxes (64-byte rows): columns cp*32.. and 64 + cp*32..
          const uint32_t box_lo = stage, box_hi = stage + 2048;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            st_shared_v4(box_lo + sw64_offset(lane, q), pack_bf16x2(lo[8 * q], lo[8 * q + 1]),
                         pack_bf16x2(lo[8 * q + 2], lo[8 * q + 3]), pack_bf16x2(lo[8 * q + 4], lo[8 * q + 5]),
                         pack_bf16x2(lo[8 * q + 6], lo[8 * q + 7]));
            st_shared_v4(box_hi + sw64_offset(lane, q), pack_bf16x2(hi[8 * q], hi[8 * q + 1]),
                         pack_bf16x2(hi[8 * q + 2], hi[8 * q + 3]), pack_bf16x2(hi[8 * q + 4], hi[8 * q + 5]),
                         pack_bf16x2(hi[8 * q + 6], hi[8 * q + 7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            uint8_t* sbuf = staging + (warp - 2) * T::STAGING;
            tma_store_2d(omap, sbuf, cp * 32, out_row0);
            tma_store_2d(omap, sbuf + 2048, 64 + cp * 32, out_row0);
            tma_store_commit();
          }
        }
      } else if constexpr (EPI == kLinearSwiGLUKeep) {
        // per 32-column chunk: silu(g) * u to Y and g to [gate | up], then u, through two 32 x 32
        // staging boxes (64-byte rows)
        uint8_t* sbuf = staging + (warp - 2) * T::STAGING;
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          float gv[32], uv[32];
          tmem_ld32(base + c * 32, gv);
          tmem_ld32(base + 128 + c * 32, uv);
          tmem_wait_ld();
          round_all<__nv_bfloat16, 32>(gv);
          round_all<__nv_bfloat16, 32>(uv);
          reuse();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float hq[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) hq[e] = round_to_t<__nv_bfloat16>(silu_fast(gv[8 * q + e])) * uv[8 * q + e];
            st_shared_v4(stage + sw64_offset(lane, q), pack_bf16x2(hq[0], hq[1]), pack_bf16x2(hq[2], hq[3]),
                         pack_bf16x2(hq[4], hq[5]), pack_bf16x2(hq[6], hq[7]));
            st_shared_v4(stage + 2048 + sw64_offset(lane, q), pack_bf16x2(gv[8 * q], gv[8 * q + 1]),
                         pack_bf16x2(gv[8 * q + 2], gv[8 * q + 3]), pack_bf16x2(gv[8 * q + 4], gv[8 * q + 5]),
                         pack_bf16x2(gv[8 * q + 6], gv[8 * q + 7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < g.M) {
            tma_store_2d(&tmY, sbuf, n0 + c * 32, row0);
            tma_store_2d(&tmK, sbuf + 2048, n0 + c * 32, row0);
            tma_store_commit();
          }
          reuse();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_shared_v4(stage + sw64_offset(lane, q), pack_bf16x2(uv[8 * q], uv[8 * q + 1]),
                         pack_bf16x2(uv[8 * q + 2], uv[8 * q + 3]), pack_bf16x2(uv[8 * q + 4], uv[8 * q + 5]),
                         pack_bf16x2(uv[8 * q + 6], uv[8 * q + 7]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < g.M) {
            tma_store_2d(&tmK, sbuf, g.f_rows + n0 + c * 32, row0);
            tma_store_commit();
          }
        }
      } else if constexpr (EPI == kLinearSwiGLU) {
        reuse();
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          float gv[32], uv[32];
          tmem_ld32(base + c * 32, gv);
          tmem_ld32(base + 128 + c * 32, uv);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float h[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float gr = round_to_t<__nv_bfloat16>(gv[j + e]);
              const float ur = round_to_t<__nv_bfloat16>(uv[j + e]);
              h[e] = round_to_t<__nv_bfloat16>(silu_fast(gr)) * ur;
            }
            pk[j / 2] = pack_bf16x2(h[0], h[1]);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_shared_v4(stage + sw128_offset(lane, (c & 1) * 4 + q), pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                         pk[4 * q + 3]);
        }
        flush(n0 + half * 64, row0);
      } else {
#pragma unroll 1
        for (int pair = 0; pair < 2; ++pair) {
          reuse();
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 4 * half + 2 * pair + cc;
            const int col0 = n0 + c * 32;
            uint4 rv[4];
            if constexpr (EPI == kLinearResidual) {
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
            if constexpr (EPI == kLinearResidual) {
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
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[b]), 0));
        else
          mbar_arrive(&acc_empty[b]);
      }
    }
    if (lane == 0) tma_store_wait_all();
  }
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // neither CTA frees TMEM or leaves while the other may signal it
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_free_pair(tmem, 512);
    else
      tmem_free(tmem, 512);
  }
}

// Largest number of co-resident clusters of two of a pair-mode linear kernel (cached per kernel).
template <typename Kern>
inline int linear_pair_max_clusters(Kern kernel) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(LinearTile::THREADS);
  cfg.dynamicSmemBytes = LinearTile::SMEM;
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

// Launches linear_tc_kernel<EPI> on g.tiles tiles of 128 rows, or, with pair, linear_tc_kernel<EPI,
// true> on clusters of two over tiles of 256 rows (g.tiles recomputed for them).
template <int EPI>
inline int linear_launch(bool pair, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ty,
                         const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tp, LinearGeometry g,
                         int64_t ldr, const __nv_bfloat16* R, const QkvRopeParams& qp, cudaStream_t stream) {
  using T = LinearTile;
  if (!pair) {
    ORTHRUS_CHECK_CUDA(ensure_smem(linear_tc_kernel<EPI>, T::SMEM));
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(g.tiles, num_sms()));
    ORTHRUS_CHECK_CUDA(launch_pdl(linear_tc_kernel<EPI>, dim3(grid), dim3(T::THREADS), T::SMEM, stream, tx, tw, ty, tk,
                                  tv, tp, g, ldr, R, qp));
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  auto kernel = linear_tc_kernel<EPI, true>;
  ORTHRUS_CHECK_CUDA(ensure_smem(kernel, T::SMEM));
  g.tiles = static_cast<int>(ceil_div(g.M, 2 * T::BM) * g.ntiles);
  const int clusters = std::min(g.tiles, linear_pair_max_clusters(kernel));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
  cfg.blockDim = dim3(T::THREADS);
  cfg.dynamicSmemBytes = T::SMEM;
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
  ORTHRUS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kernel, tx, tw, ty, tk, tv, tp, g, ldr, R, qp));
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

// cos / sin [P][half] of the RoPE angle p * inv_freq[i], rounded to bf16, by sincosf as the
// attention prologue computes them.
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int64_t P, int half,
                                  __nv_bfloat16* __restrict__ cos_out, __nv_bfloat16* __restrict__ sin_out) {
  const int64_t n = P * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float sv, cv;
    sincosf(static_cast<float>(i / half) * inv_freq[i % half], &sv, &cv);
    cos_out[i] = __float2bfloat16_rn(cv);
    sin_out[i] = __float2bfloat16_rn(sv);
  }
}

inline int rope_table_impl(const float* inv_freq, int64_t P, int half, void* cos_out, void* sin_out,
                           cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(inv_freq && cos_out && sin_out && P > 0 && half > 0 && P * half < (1ll << 40));
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(P * half, 256), 148 * 8));
  rope_table_kernel<<<blocks, 256, 0, stream>>>(inv_freq, P, half, static_cast<__nv_bfloat16*>(cos_out),
                                                static_cast<__nv_bfloat16*>(sin_out));
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

// Host side. N is the number of output columns (F for SwiGLU, whose W has 2F rows); N must be a
// multiple of 128, K a multiple of 8, leading dimensions multiples of 8 elements. R (residual) has
// the leading dimension of Y and is a separate buffer.
// epilogue | kLinearPairFlag runs the kernel on CTA pairs (the training step's sizes; inference
// keeps the one-CTA kernel, so its per-row results never depend on the launch form).
constexpr int kLinearPairFlag = 0x100;

inline int linear_bf16_impl(const void* X, int64_t ldx, const void* W, int64_t ldw, const void* R, void* Y,
                            int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue, cudaStream_t stream) {
  const bool pair = (epilogue & kLinearPairFlag) != 0;
  epilogue &= ~kLinearPairFlag;
  ORTHRUS_CHECK_ARG(X && W && Y && M >= 0 && N > 0 && K > 0);
  ORTHRUS_CHECK_ARG(epilogue == kLinearStore || epilogue == kLinearResidual || epilogue == kLinearSwiGLU);  // q|k|v: linear_qkv_rope_impl
  ORTHRUS_CHECK_ARG(epilogue != kLinearResidual || (R != nullptr && R != Y));
  ORTHRUS_CHECK_ARG(N % 128 == 0 && K % 8 == 0 && ldx >= K && ldw >= K && ldy >= N);
  ORTHRUS_CHECK_ARG(ldx % 8 == 0 && ldw % 8 == 0 && ldy % 8 == 0);
  ORTHRUS_CHECK_ARG(aligned16(X) && aligned16(W) && aligned16(Y) && (R == nullptr || aligned16(R)));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && N < (1ll << 30) && K < (1ll << 31));
  if (M == 0) return ORTHRUS_OK;
  using T = LinearTile;
  const int64_t w_rows = epilogue == kLinearSwiGLU ? 2 * N : N;
  CUtensorMap tx, tw, ty;
  if (!make_tmap_2d_bf16(&tx, X, K, M, ldx, 64, 128)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tw, W, K, w_rows, ldw, 64, 128)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&ty, Y, N, M, ldy, 64, 32)) return ORTHRUS_ECUDA;
  LinearGeometry g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.ntiles = static_cast<int>(epilogue == kLinearSwiGLU ? N / 128 : ceil_div(N, T::BN));
  const int64_t tiles = ceil_div(M, T::BM) * g.ntiles;
  ORTHRUS_CHECK_ARG(tiles < (1ll << 31));
  g.tiles = static_cast<int>(tiles);
  g.f_rows = epilogue == kLinearSwiGLU ? static_cast<int>(N) : 0;
  auto* r = static_cast<const __nv_bfloat16*>(R);
  const QkvRopeParams none{};
  if (epilogue == kLinearStore)
    return linear_launch<kLinearStore>(pair, tx, tw, ty, ty, ty, ty, g, ldy, nullptr, none, stream);
  if (epilogue == kLinearResidual)
    return linear_launch<kLinearResidual>(pair, tx, tw, ty, ty, ty, ty, g, ldy, r, none, stream);
  return linear_launch<kLinearSwiGLU>(pair, tx, tw, ty, ty, ty, ty, g, ldy, nullptr, none, stream);
}

// silu(x gate^T) * (x up^T) into y [M, F] and the projection [gate | up] into gate_up [M, 2F].
inline int linear_swiglu_keep_impl(const void* X, const void* W, int64_t M, int64_t F, int64_t K, void* Y,
                                   void* GU, cudaStream_t stream) {
  ORTHRUS_CHECK_ARG(X && W && Y && GU && M >= 0 && F > 0 && F % 128 == 0 && K > 0 && K % 8 == 0);
  ORTHRUS_CHECK_ARG(aligned16(X) && aligned16(W) && aligned16(Y) && aligned16(GU));
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && F < (1ll << 29) && K < (1ll << 31));
  if (M == 0) return ORTHRUS_OK;
  using T = LinearTile;
  CUtensorMap tx, tw, ty, tgu;
  if (!make_tmap_2d_bf16(&tx, X, K, M, K, 64, 128)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tw, W, K, 2 * F, K, 64, 128)) return ORTHRUS_ECUDA;
  // 32 x 32 boxes of 64-byte rows, 64-byte swizzle (bank-conflict-free staging stores)
  if (!make_tmap_2d_bf16(&ty, Y, F, M, F, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tgu, GU, 2 * F, M, 2 * F, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return ORTHRUS_ECUDA;
  LinearGeometry g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(F);
  g.K = static_cast<int>(K);
  g.ntiles = static_cast<int>(F / 128);
  const int64_t tiles = ceil_div(M, T::BM) * g.ntiles;
  ORTHRUS_CHECK_ARG(tiles < (1ll << 31));
  g.tiles = static_cast<int>(tiles);
  g.f_rows = static_cast<int>(F);
  const QkvRopeParams none{};
  // the trainable view's MLP (thousands of rows): CTA pairs
  return linear_launch<kLinearSwiGLUKeep>(M >= 2048, tx, tw, ty, tgu, tgu, tgu, g, 0, nullptr, none, stream);
}

// q|k|v projection of x [B*L, K] by w [(Hq + 2 Hkv) * 128, K] with the attention prologue in the
// epilogue; q_out [B, Hq, L, 128], k_out / v_out [B, Hkv, L, 128] (head dim 128, positions 0..L-1).
inline int linear_qkv_rope_impl(const void* X, const void* W, const void* q_norm_w, const void* k_norm_w,
                                const void* rope_cos, const void* rope_sin, int64_t B, int64_t L, int64_t K,
                                int Hq, int Hkv, float eps, void* q_out, void* k_out, void* v_out,
                                cudaStream_t stream, int64_t table_rows, const int64_t* positions = nullptr,
                                void* qkv_keep = nullptr, float* rstd_out = nullptr) {
  ORTHRUS_CHECK_ARG(X && W && q_norm_w && k_norm_w && rope_cos && rope_sin && q_out && k_out && v_out);
  ORTHRUS_CHECK_ARG(B > 0 && L > 0 && L % 128 == 0 && K > 0 && K % 8 == 0 && Hq > 0 && Hkv > 0);
  ORTHRUS_CHECK_ARG((Hq + 2 * Hkv) % 2 == 0);  // two whole heads per 256-column tile
  ORTHRUS_CHECK_ARG(table_rows >= (positions == nullptr ? L : 1));
  ORTHRUS_CHECK_ARG(aligned16(X) && aligned16(W) && aligned16(q_norm_w) && aligned16(k_norm_w) &&
                    aligned16(rope_cos) && aligned16(rope_sin) && aligned16(q_out) && aligned16(k_out) &&
                    aligned16(v_out));
  const int64_t M = B * L, N = static_cast<int64_t>(Hq + 2 * Hkv) * 128;
  ORTHRUS_CHECK_ARG(M < (1ll << 31) && B * Hq * L < (1ll << 31) && N < (1ll << 30) && K < (1ll << 31));
  using T = LinearTile;
  CUtensorMap tx, tw, tq, tk, tv;
  if (!make_tmap_2d_bf16(&tx, X, K, M, K, 64, 128)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tw, W, K, N, K, 64, 128)) return ORTHRUS_ECUDA;
  // 32 x 32 boxes of 64-byte rows with 64-byte swizzle: the epilogue's staging stores (one row
  // per lane) then fall on distinct shared-memory banks
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
  if (!make_tmap_2d_bf16(&tq, q_out, 128, B * Hq * L, 128, 32, 32, sw)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tk, k_out, 128, B * Hkv * L, 128, 32, 32, sw)) return ORTHRUS_ECUDA;
  if (!make_tmap_2d_bf16(&tv, v_out, 128, B * Hkv * L, 128, 32, 32, sw)) return ORTHRUS_ECUDA;
  CUtensorMap tp = tv;
  ORTHRUS_CHECK_ARG(qkv_keep == nullptr || aligned16(qkv_keep));
  if (qkv_keep != nullptr && !make_tmap_2d_bf16(&tp, qkv_keep, N, M, N, 32, 32, sw)) return ORTHRUS_ECUDA;
  LinearGeometry g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.ntiles = static_cast<int>(N / T::BN);  // two heads per tile
  g.tiles = static_cast<int>(ceil_div(M, T::BM) * g.ntiles);
  g.f_rows = 0;
  QkvRopeParams qp;
  qp.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  qp.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  qp.rope_cos = static_cast<const __nv_bfloat16*>(rope_cos);
  qp.rope_sin = static_cast<const __nv_bfloat16*>(rope_sin);
  qp.positions = positions;
  qp.table_rows = table_rows;
  qp.rstd_out = rstd_out;
  qp.keep = qkv_keep != nullptr;
  qp.L = static_cast<int>(L);
  qp.Hq = Hq;
  qp.Hkv = Hkv;
  qp.eps = eps;
  // the training step's q|k|v projections (thousands of rows): CTA pairs
  return linear_launch<kLinearQkvRope>(M >= 2048, tx, tw, tq, tk, tv, tp, g, 0, nullptr, qp, stream);
}

}  // namespace orthrus
