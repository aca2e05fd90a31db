// dK / dV of the dual view's own-block keys when a block is 32 keys and the head dim is 128.
//
// The diffusion view's source-2 keys are seen only by the queries of their own block, so their
// gradients are 32 x 32 problems per (block, query head): S^T = K Q^T and dP^T = V dO^T over the
// head dim, P^T = exp(S^T scale - lse), dS^T = P^T (dP^T - delta), then dV = sum_h P^T dO and
// dK = scale * sum_h dS^T Q over the query heads h of the KV head (orthrus/objective.py:160-165 and
// the backward of its block mask, orthrus/modeling_orthrus.py:58-85). Work per block is 2 MFLOP
// against 176 KB of operands and results, so the kernel is bound by HBM, not by tensor throughput:
// it is written for occupancy (3 CTAs of 4 warps per SM, every operand fetched with cp.async at
// once) with warp-level bf16 MMAs (mma.sync m16n8k16, fp32 accumulation) on 32 x 32 tiles that a
// 128-row tcgen05 tile would pad four times over.
//
// One CTA per (32-key block, KV head, batch row), 128 threads:
//   load   K, V [32 x 128] and Q_h, dO_h [32 x 128] of the G query heads into padded shared rows
//          (272 bytes: conflict-free ldmatrix), lse * log2 e and delta per query;
//   phase1 warp g < G: S^T_g and dP^T_g as 2 x 4 m16n8 tiles over 8 k-steps, then P^T_g and
//          dS^T_g rounded to bf16 into shared memory;
//   phase2 warp w: columns [32 w, 32 w + 32) of dV and dK, summed over g (k = the 32 queries),
//          stored as fp32 [B, Hkv, L2, 128].
// P^T and dS^T are rounded to bf16 before they are multiplied, as in the tcgen05 kernels; the
// k order differs from them, so results agree to fp32 accumulation, not bit for bit.
#pragma once

#include "sm100.cuh"

namespace orthrus {

struct BlockKvSmem {
  static constexpr int ROW = 272;               // 128 bf16 + 16 bytes of padding
  static constexpr int TILE = 32 * ROW;         // one [32][128] operand
  static constexpr int PROW = 80;               // 32 bf16 + 16 bytes of padding
  static constexpr int PTILE = 32 * PROW;       // one [32 keys][32 queries] bf16 tile
  template <int G>
  static constexpr int bytes() {
    return (2 + 2 * G) * TILE + 2 * G * PTILE + 2 * G * 32 * 4;
  }
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D (16 x 8, fp32) += A (16 x 16, bf16, row) * B (16 x 8, bf16, col)
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// grid (Tq / 32, Hkv, B); L2 >= Tq source-2 keys, key j of a row seen by queries of its own block.
template <int G>
__global__ void __launch_bounds__(128, 3)
    attn_dkdv_block32_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k2,
                             const __nv_bfloat16* __restrict__ v2, int64_t s2h, int64_t s2b,
                             const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
                             const float* __restrict__ delta, int Hq, int Hkv, int64_t Tq, int64_t L2, float scale,
                             float* __restrict__ dk, float* __restrict__ dv) {
  using S = BlockKvSmem;
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  const uint32_t sK = base, sV = base + S::TILE;
  auto sQ = [&](int g) { return base + (2 + g) * S::TILE; };
  auto sDO = [&](int g) { return base + (2 + G + g) * S::TILE; };
  const uint32_t sP0 = base + (2 + 2 * G) * S::TILE;  // P^T_g at sP0 + g * PTILE, dS^T_g after them
  auto sP = [&](int g) { return sP0 + g * S::PTILE; };
  auto sDS = [&](int g) { return sP0 + (G + g) * S::PTILE; };
  float* stat = reinterpret_cast<float*>(smem + (2 + 2 * G) * S::TILE + 2 * G * S::PTILE);  // [G][lse2 | delta]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;  // keys = queries of this block
  const int hk = blockIdx.y;
  const int64_t b = blockIdx.z;

  // every operand at once: 16-byte pieces, 512 per [32][128] tile, 4 per thread
  const __nv_bfloat16* kr = k2 + b * s2b + hk * s2h + k0 * 128;
  const __nv_bfloat16* vr = v2 + b * s2b + hk * s2h + k0 * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int piece = tid + 128 * i, r = piece >> 4, c = piece & 15;
    const uint32_t off = r * S::ROW + c * 16;
    cp_async16(sK + off, kr + r * 128 + c * 8);
    cp_async16(sV + off, vr + r * 128 + c * 8);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int h = hk * G + g;
      cp_async16(sQ(g) + off, q + ((b * Hq + h) * Tq + k0 + r) * 128 + c * 8);
      cp_async16(sDO(g) + off, dout + ((b * Tq + k0 + r) * Hq + h) * 128 + c * 8);
    }
  }
  if (tid < 32 * G) {
    const int g = tid >> 5, h = hk * G + g;
    stat[g * 64 + lane] = lse[(b * Hq + h) * Tq + k0 + lane] * kLog2e;
    stat[g * 64 + 32 + lane] = delta[(b * Hq + h) * Tq + k0 + lane];
  }
  cp_async_wait_all();
  __syncthreads();

  const int lr = lane & 15, lk = (lane >> 4) * 8;  // ldmatrix: row and k offset of this lane's address
  const float sl2 = scale * kLog2e;
  for (int g = warp; g < G; g += 4) {
    // S^T = K Q_g^T and dP^T = V dO_g^T: rows = keys (2 m-tiles), columns = queries (4 n-tiles)
    float acc_s[2][4][4], acc_p[2][4][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc_s[m][n][e] = acc_p[m][n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t ak[2][4], av[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const uint32_t off = (m * 16 + lr) * S::ROW + (ks * 16 + lk) * 2;
        ldsm_x4(sK + off, ak[m][0], ak[m][1], ak[m][2], ak[m][3]);
        ldsm_x4(sV + off, av[m][0], av[m][1], av[m][2], av[m][3]);
      }
      // B from rows of Q_g / dO_g (k contiguous): one x4 gives two n-tiles (lanes 16-31: n + 8)
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int nrow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kof = ks * 16 + ((lane >> 3) & 1) * 8;
        const uint32_t off = nrow * S::ROW + kof * 2;
        uint32_t bq[4], bd[4];
        ldsm_x4(sQ(g) + off, bq[0], bq[1], bq[2], bq[3]);
        ldsm_x4(sDO(g) + off, bd[0], bd[1], bd[2], bd[3]);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          mma_bf16_16816(acc_s[m][2 * np], ak[m], bq[0], bq[1]);
          mma_bf16_16816(acc_s[m][2 * np + 1], ak[m], bq[2], bq[3]);
          mma_bf16_16816(acc_p[m][2 * np], av[m], bd[0], bd[1]);
          mma_bf16_16816(acc_p[m][2 * np + 1], av[m], bd[2], bd[3]);
        }
      }
    }
    // P^T and dS^T of this head, bf16, rows = keys, columns = queries
    const float* lse2 = stat + g * 64;
    const float* dl = lse2 + 32;
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
          const int key = m * 16 + (lane >> 2) + 8 * hrow;
          const int qc = n * 8 + (lane & 3) * 2;
          const float p0 = ex2_approx(fmaf(acc_s[m][n][2 * hrow], sl2, -lse2[qc]));
          const float p1 = ex2_approx(fmaf(acc_s[m][n][2 * hrow + 1], sl2, -lse2[qc + 1]));
          const float d0 = p0 * (acc_p[m][n][2 * hrow] - dl[qc]);
          const float d1 = p1 * (acc_p[m][n][2 * hrow + 1] - dl[qc + 1]);
          const uint32_t off = key * S::PROW + qc * 2;
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(sP(g) + off), "r"(pack_bf16x2(p0, p1)) : "memory");
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(sDS(g) + off), "r"(pack_bf16x2(d0, d1)) : "memory");
        }
  }
  __syncthreads();

  // dV[:, cols] = sum_g P^T_g dO_g[:, cols]; dK[:, cols] = scale sum_g dS^T_g Q_g[:, cols]
  const int c0 = warp * 32;
  float acc_v[2][4][4], acc_k[2][4][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc_v[m][n][e] = acc_k[m][n][e] = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {  // k = queries 16 ks .. 16 ks + 15
      uint32_t ap[2][4], ad[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const uint32_t off = (m * 16 + lr) * S::PROW + (ks * 16 + lk) * 2;
        ldsm_x4(sP(g) + off, ap[m][0], ap[m][1], ap[m][2], ap[m][3]);
        ldsm_x4(sDS(g) + off, ad[m][0], ad[m][1], ad[m][2], ad[m][3]);
      }
      // B = dO_g / Q_g rows [k = query][n = column]: transposed loads, two n-tiles per x4
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int krow = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ncol = c0 + np * 16 + (lane >> 4) * 8;
        const uint32_t off = krow * S::ROW + ncol * 2;
        uint32_t bo[4], bq[4];
        ldsm_x4_t(sDO(g) + off, bo[0], bo[1], bo[2], bo[3]);
        ldsm_x4_t(sQ(g) + off, bq[0], bq[1], bq[2], bq[3]);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          mma_bf16_16816(acc_v[m][2 * np], ap[m], bo[0], bo[1]);
          mma_bf16_16816(acc_v[m][2 * np + 1], ap[m], bo[2], bo[3]);
          mma_bf16_16816(acc_k[m][2 * np], ad[m], bq[0], bq[1]);
          mma_bf16_16816(acc_k[m][2 * np + 1], ad[m], bq[2], bq[3]);
        }
      }
    }
  }
  float* dvb = dv + ((b * Hkv + hk) * L2 + k0) * 128;
  float* dkb = dk + ((b * Hkv + hk) * L2 + k0) * 128;
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int key = m * 16 + (lane >> 2) + 8 * hrow;
        const int col = c0 + n * 8 + (lane & 3) * 2;
        *reinterpret_cast<float2*>(dvb + key * 128 + col) =
            make_float2(acc_v[m][n][2 * hrow], acc_v[m][n][2 * hrow + 1]);
        *reinterpret_cast<float2*>(dkb + key * 128 + col) =
            make_float2(acc_k[m][n][2 * hrow] * scale, acc_k[m][n][2 * hrow + 1] * scale);
      }
}

}  // namespace orthrus
