// The C ABI of liborthrus_b200.so (declared in include/orthrus_b200.h). The whole library is one
// translation unit, so device symbols (the error word) need no relocatable device code.
#include <algorithm>
#include <cstdlib>

#include "host_common.h"
#include "sm100.cuh"

#include "attention_simt.cuh"
#include "attention_tc.cuh"
#include "attention_blockkv.cuh"
#include "attention_decode.cuh"
#include "decode.cuh"
#include "sampling.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "gemm2_tc.cuh"
#include "linear_tc.cuh"
#include "linear_skinny.cuh"
#include "lmhead_kl.cuh"
#include "qkv_prep.cuh"
#include "rowwise.cuh"
#include "selftest.cuh"

using namespace orthrus;

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int orthrus_version(void) { return 100; }

unsigned long long orthrus_launch_count(void) { return launch_counter().load(std::memory_order_relaxed); }

int orthrus_device_error(int device, unsigned int* word, int clear) {
  ORTHRUS_CHECK_ARG(word != nullptr);
  int prev = 0;
  ORTHRUS_CHECK_CUDA(cudaGetDevice(&prev));
  ORTHRUS_CHECK_CUDA(cudaSetDevice(device));
  ORTHRUS_CHECK_CUDA(cudaDeviceSynchronize());
  unsigned int w = 0;
  ORTHRUS_CHECK_CUDA(cudaMemcpyFromSymbol(&w, g_device_error, sizeof(w)));
  if (clear && w) {
    const unsigned int zero = 0;
    ORTHRUS_CHECK_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
  }
  ORTHRUS_CHECK_CUDA(cudaSetDevice(prev));
  *word = w;
  return w ? ORTHRUS_EDEVICE : ORTHRUS_OK;
}

int orthrus_selftest_bounded_wait(const void* tile64x64, uint64_t limit_ns, unsigned int* status, void* stream) {
  ORTHRUS_CHECK_ARG(tile64x64 && status && aligned16(tile64x64) && limit_ns > 0 && limit_ns <= 100000000ull);
  CUtensorMap tm;
  if (!make_tmap_2d_bf16(&tm, tile64x64, 64, 64, 64, 64, 64)) return ORTHRUS_ECUDA;
  bounded_wait_selftest_kernel<<<1, 64, 0, as_stream(stream)>>>(tm, limit_ns, status);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

size_t orthrus_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) { return gemm_ws_bytes(M, N, K); }

int orthrus_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                      int64_t N, int64_t K, int b_kn, int c_f32, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return gemm_bf16_impl(A, lda, B, ldb, C, ldc, M, N, K, b_kn, c_f32, workspace, workspace_bytes,
                        as_stream(stream));
}

size_t orthrus_gemm2_workspace_bytes(int64_t M, int64_t N, int64_t K) { return gemm2_ws_bytes(M, N, K); }

int orthrus_gemm2_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C,
                       int64_t ldc, const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue,
                       void* workspace, size_t workspace_bytes, void* stream) {
  return gemm2_bf16_impl(A, lda, a_mn, B, ldb, b_mn, C, ldc, R, ldr, M, N, K, epilogue, workspace,
                         workspace_bytes, as_stream(stream));
}

int orthrus_linear_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* residual, void* y,
                        int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue, void* stream) {
  return linear_bf16_impl(x, ldx, w, ldw, residual, y, ldy, M, N, K, epilogue, as_stream(stream));
}

int orthrus_linear_skinny_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* residual, void* y,
                               int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue, void* stream) {
  return linear_skinny_impl(x, ldx, w, ldw, residual, y, ldy, M, N, K, epilogue, as_stream(stream));
}

int orthrus_linear_swiglu_keep_bf16(const void* x, const void* w_gate_up, int64_t M, int64_t F, int64_t K, void* y,
                                    void* gate_up, void* stream) {
  return linear_swiglu_keep_impl(x, w_gate_up, M, F, K, y, gate_up, as_stream(stream));
}

int orthrus_linear_qkv_rope_keep_bf16(const void* x, const void* w_qkv, const void* q_norm_w, const void* k_norm_w,
                                      const void* rope_cos, const void* rope_sin, int64_t table_rows,
                                      const int64_t* positions, int64_t B,
                                      int64_t L, int64_t K, int Hq, int Hkv, float eps, void* q_out, void* k_out,
                                      void* v_out, void* qkv_out, float* rstd_out, void* stream) {
  ORTHRUS_CHECK_ARG(positions && qkv_out && rstd_out);
  return linear_qkv_rope_impl(x, w_qkv, q_norm_w, k_norm_w, rope_cos, rope_sin, B, L, K, Hq, Hkv, eps, q_out,
                              k_out, v_out, as_stream(stream), table_rows, positions, qkv_out, rstd_out);
}

int orthrus_rope_table_bf16(const float* inv_freq, int64_t positions, int half, void* cos_out, void* sin_out,
                            void* stream) {
  return rope_table_impl(inv_freq, positions, half, cos_out, sin_out, as_stream(stream));
}

int orthrus_linear_qkv_rope_bf16(const void* x, const void* w_qkv, const void* q_norm_w, const void* k_norm_w,
                                 const void* rope_cos, const void* rope_sin, int64_t B, int64_t L, int64_t K, int Hq,
                                 int Hkv, float eps, void* q_out, void* k_out, void* v_out, void* stream) {
  return linear_qkv_rope_impl(x, w_qkv, q_norm_w, k_norm_w, rope_cos, rope_sin, B, L, K, Hq, Hkv, eps, q_out,
                              k_out, v_out, as_stream(stream), L);
}

size_t orthrus_gemm_simt_workspace_bytes(int64_t M, int64_t N, int64_t K) { return simt_ws_bytes(M, N, K); }

int orthrus_gemm_simt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                      int64_t N, int64_t K, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype == ORTHRUS_F32)
    return gemm_simt_impl<float, false>(static_cast<const float*>(A), lda, static_cast<const float*>(B), ldb,
                                        static_cast<float*>(C), ldc, M, N, K, workspace, workspace_bytes,
                                        as_stream(stream));
  if (dtype == ORTHRUS_BF16)
    return gemm_simt_impl<__nv_bfloat16, false>(
        static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(B), ldb,
        static_cast<__nv_bfloat16*>(C), ldc, M, N, K, workspace, workspace_bytes, as_stream(stream));
  return ORTHRUS_EINVAL;
}

size_t orthrus_lmhead_argmax_workspace_bytes(int64_t R) { return R > 0 ? lmhead_argmax_ws_bytes(R) : 0; }

int orthrus_lmhead_argmax_bf16(const void* h, int64_t R, const void* weight, int64_t V, int64_t d, int64_t* out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  return lmhead_argmax_bf16(static_cast<const __nv_bfloat16*>(h), R, static_cast<const __nv_bfloat16*>(weight), V, d,
                            out, workspace, workspace_bytes, as_stream(stream));
}

int orthrus_decode_draft_ids(const int64_t* ids, int64_t B, int K, const int64_t* anchor, const uint8_t* done,
                             int64_t* verify_ids, void* stream) {
  ORTHRUS_CHECK_ARG(ids && anchor && verify_ids && B > 0 && K >= 1);
  decode_draft_ids_kernel<<<static_cast<unsigned>(ceil_div(B * K, 256)), 256, 0, as_stream(stream)>>>(
      ids, B, K, anchor, done, verify_ids);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_decode_accept_ids(const int64_t* ar_tokens, int64_t B, int K, const int64_t* verify_ids,
                              const int64_t* eos, int n_eos, const int32_t* max_len, int32_t* start, int64_t* anchor,
                              uint8_t* done, int64_t* out_tokens, int32_t* out_len, int64_t out_cap,
                              int32_t* accepted_log, int32_t* cycle, int64_t log_cap, void* stream) {
  ORTHRUS_CHECK_ARG(ar_tokens && verify_ids && max_len && start && anchor && done && out_tokens && out_len &&
                    accepted_log && cycle && B > 0 && K >= 1);
  ORTHRUS_CHECK_ARG(n_eos == 0 || eos != nullptr);
  decode_accept_kernel<<<static_cast<unsigned>(ceil_div(B, 128)), 128, 0, as_stream(stream)>>>(
      B, K, verify_ids, ar_tokens, eos, n_eos, max_len, start, anchor, done, out_tokens, out_len, out_cap,
      accepted_log, cycle, log_cap);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

size_t orthrus_lmhead_kl_workspace_bytes(int64_t n, int64_t m, int64_t V, int64_t d, int64_t chunk_rows,
                                         int dtype) {
  return lmhead_plan(n, m, V, d, chunk_rows, dtype).total;
}

int orthrus_lmhead_kl_fwd(const void* student, int64_t n, const void* teacher, int64_t m, const int64_t* index,
                          const void* weight, int64_t V, int64_t d, const float* row_weight,
                          const int64_t* offsets, int num_offsets, float* total, float* kl_rows, uint8_t* agree,
                          void* grad, float* kl_by_offset, int64_t* agree_by_offset, int64_t chunk_rows,
                          void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  if (dtype == ORTHRUS_BF16)
    return lmhead_kl_fwd_impl<__nv_bfloat16>(
        static_cast<const __nv_bfloat16*>(student), n, static_cast<const __nv_bfloat16*>(teacher), m, index,
        static_cast<const __nv_bfloat16*>(weight), V, d, row_weight, offsets, num_offsets, total, kl_rows,
        agree, static_cast<__nv_bfloat16*>(grad), kl_by_offset, agree_by_offset, chunk_rows, workspace,
        workspace_bytes, as_stream(stream));
  if (dtype == ORTHRUS_F32)
    return lmhead_kl_fwd_impl<float>(static_cast<const float*>(student), n, static_cast<const float*>(teacher), m,
                                     index, static_cast<const float*>(weight), V, d, row_weight, offsets,
                                     num_offsets, total, kl_rows, agree, static_cast<float*>(grad), kl_by_offset,
                                     agree_by_offset, chunk_rows, workspace, workspace_bytes, as_stream(stream));
  return ORTHRUS_EINVAL;
}

int orthrus_lmhead_kl_bwd(const void* grad, const float* grad_total, void* grad_student, int64_t count,
                          int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(grad && grad_total && grad_student && count >= 0);
  if (count == 0) return ORTHRUS_OK;
  const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(count, 256), 148 * 8));
  if (dtype == ORTHRUS_BF16)
    scale_by_scalar_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(grad), grad_total, static_cast<__nv_bfloat16*>(grad_student), count);
  else if (dtype == ORTHRUS_F32)
    scale_by_scalar_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const float*>(grad), grad_total, static_cast<float*>(grad_student), count);
  else
    return ORTHRUS_EINVAL;
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// q/k prep, attention, decoding
// ------------------------------------------------------------------------------------------------

namespace {

__global__ void attn_tilemap_kernel(const int64_t* __restrict__ anchors, int64_t B, int64_t A, int block,
                                    int64_t L1, int32_t* __restrict__ out) {
  const int64_t Tq = A * block;
  const int64_t ntiles = (Tq + 127) / 128;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= B * ntiles) return;
  const int64_t b = i / ntiles, tile = i % ntiles;
  const int64_t q0 = tile * 128, q1 = min(Tq, q0 + 128);
  int64_t e1 = 0, s2 = INT64_MAX, e2 = 0;
  for (int64_t blk = q0 / block; blk <= (q1 - 1) / block; ++blk) {
    e1 = max(e1, min(L1, anchors[b * A + blk]));
    s2 = min(s2, blk * block);
    e2 = max(e2, (blk + 1) * block);
  }
  out[i * 4 + 0] = static_cast<int32_t>((e1 + 127) / 128);
  out[i * 4 + 1] = static_cast<int32_t>(e1);
  out[i * 4 + 2] = static_cast<int32_t>(s2);
  out[i * 4 + 3] = static_cast<int32_t>(e2);
}

// bf16 rows of 64 or 128 take the tensor-core kernels for every mask. A row's result there does
// not depend on the other rows of its tile (key tiles that a row cannot see contribute exact
// zeros), so a K-token verification reproduces the one-token pass bit for bit. Keys past a
// sequence's cached length must be finite (the caches start zeroed).
bool use_tensor_cores(int dtype, int hd, int D, int mask, const int32_t*) {
  return dtype == ORTHRUS_BF16 && hd == D && (D == 64 || D == 128) && mask >= ORTHRUS_MASK_CAUSAL &&
         mask <= ORTHRUS_MASK_TREE;
}

template <typename Kern>
int set_smem(Kern k, int bytes) {
  ORTHRUS_CHECK_CUDA(ensure_smem(k, bytes));
  return ORTHRUS_OK;
}

struct AttnMaps {
  CUtensorMap q, k1, v1, k2, v2, dout;
};

bool make_attn_maps(AttnMaps& m, const void* q, const void* k1, const void* v1, int64_t s1h, int64_t L1,
                    const void* k2, const void* v2, int64_t s2h, int64_t L2, int64_t B, int Hq, int Hkv,
                    int64_t Tq, int hd, int D, const void* dout, uint32_t key_box = 128) {
  bool ok = make_tmap_3d_bf16(&m.q, q, D, Tq, B * Hq, D, Tq * D, 64, 128) &&
            make_tmap_3d_bf16(&m.k1, k1, D, L1, B * Hkv, D, s1h, 64, key_box) &&
            make_tmap_3d_bf16(&m.v1, v1, D, L1, B * Hkv, D, s1h, 64, key_box);
  if (k2 != nullptr)
    ok = ok && make_tmap_3d_bf16(&m.k2, k2, D, L2, B * Hkv, D, s2h, 64, key_box) &&
         make_tmap_3d_bf16(&m.v2, v2, D, L2, B * Hkv, D, s2h, 64, key_box);
  else {
    m.k2 = m.k1;
    m.v2 = m.v1;
  }
  if (dout != nullptr)
    ok = ok && make_tmap_3d_bf16(&m.dout, dout, static_cast<uint64_t>(Hq) * hd, Tq, B, static_cast<uint64_t>(Hq) * hd,
                                 Tq * Hq * hd, 64, 128);
  return ok;
}

}  // namespace

extern "C" {

int orthrus_qkv_prep_fwd(const void* qkv, const int64_t* positions, const float* inv_freq, const void* q_norm_w,
                         const void* k_norm_w, int64_t B, int64_t T, int Hq, int Hkv, int hd, int D, float eps,
                         void* q_out, void* k_out, void* v_out, int64_t cap, const int32_t* offset, float* rstd,
                         int dtype, void* stream) {
  if (dtype == ORTHRUS_BF16)
    return qkv_prep_fwd_impl<__nv_bfloat16>(
        static_cast<const __nv_bfloat16*>(qkv), positions, inv_freq, static_cast<const __nv_bfloat16*>(q_norm_w),
        static_cast<const __nv_bfloat16*>(k_norm_w), B, T, Hq, Hkv, hd, D, eps, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(v_out), cap, offset, rstd, as_stream(stream));
  if (dtype == ORTHRUS_F32)
    return qkv_prep_fwd_impl<float>(static_cast<const float*>(qkv), positions, inv_freq,
                                    static_cast<const float*>(q_norm_w), static_cast<const float*>(k_norm_w), B, T,
                                    Hq, Hkv, hd, D, eps, static_cast<float*>(q_out), static_cast<float*>(k_out),
                                    static_cast<float*>(v_out), cap, offset, rstd, as_stream(stream));
  return ORTHRUS_EINVAL;
}

size_t orthrus_qkv_prep_bwd_workspace_bytes(int64_t, int64_t, int hd) { return qkv_prep_bwd_ws(hd); }

int orthrus_qkv_prep_bwd(const void* qkv, const int64_t* positions, const float* inv_freq, const void* q_norm_w,
                         const void* k_norm_w, const float* rstd, const float* dq, const float* dk, const float* dv,
                         int64_t B, int64_t T, int Hq, int Hkv, int hd, int D, void* dqkv, float* dq_norm_w,
                         float* dk_norm_w, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  if (dtype == ORTHRUS_BF16)
    return qkv_prep_bwd_impl<__nv_bfloat16>(
        static_cast<const __nv_bfloat16*>(qkv), positions, inv_freq, static_cast<const __nv_bfloat16*>(q_norm_w),
        static_cast<const __nv_bfloat16*>(k_norm_w), rstd, dq, dk, dv, B, T, Hq, Hkv, hd, D,
        static_cast<__nv_bfloat16*>(dqkv), dq_norm_w, dk_norm_w, workspace, workspace_bytes, as_stream(stream));
  if (dtype == ORTHRUS_F32)
    return qkv_prep_bwd_impl<float>(static_cast<const float*>(qkv), positions, inv_freq,
                                    static_cast<const float*>(q_norm_w), static_cast<const float*>(k_norm_w), rstd, dq,
                                    dk, dv, B, T, Hq, Hkv, hd, D, static_cast<float*>(dqkv), dq_norm_w, dk_norm_w,
                                    workspace, workspace_bytes, as_stream(stream));
  return ORTHRUS_EINVAL;
}

int orthrus_attn_tilemap(const int64_t* anchors, int64_t B, int64_t A, int block, int64_t L1, int32_t* tilemap,
                         void* stream) {
  ORTHRUS_CHECK_ARG(anchors && tilemap && B > 0 && A > 0 && block > 0 && L1 >= 0);
  const int64_t n = B * ceil_div(A * block, 128);
  attn_tilemap_kernel<<<static_cast<unsigned>(ceil_div(n, 128)), 128, 0, as_stream(stream)>>>(anchors, B, A, block,
                                                                                            L1, tilemap);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

static int attn_fwd_impl(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                         const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq,
                         int Hkv, int64_t Tq, int hd, int D, float scale, int mask, const int64_t* anchors, int64_t A,
                         int block, const int32_t* offset, const int32_t* limit2, const int32_t* doc_start, void* o,
                         float* lse, int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(q && k1 && v1 && o && B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Tq > 0 && L1 >= 0);
  ORTHRUS_CHECK_ARG(hd > 0 && hd <= D && D <= 128 && mask >= 0 && mask <= ORTHRUS_MASK_TREE);
  ORTHRUS_CHECK_ARG(mask != ORTHRUS_MASK_DUAL || (anchors && A > 0 && block > 0 && k2 && v2));
  ORTHRUS_CHECK_ARG(mask != ORTHRUS_MASK_DRAFT || k2 != nullptr);
  ORTHRUS_CHECK_ARG(mask != ORTHRUS_MASK_TREE || (k2 && v2 && offset && limit2));
  ORTHRUS_CHECK_ARG(B < 65536 && Hq < 65536);
  const bool has2 = k2 != nullptr && mask != ORTHRUS_MASK_CAUSAL;
  MaskParams mp{mask, anchors, A, block, offset, limit2, L1, has2 ? L2 : 0};
  mp.doc_start = doc_start;
  cudaStream_t st = as_stream(stream);
  if (use_tensor_cores(dtype, hd, D, mask, offset)) {
    ORTHRUS_CHECK_ARG(s1b == Hkv * s1h && (!has2 || s2b == Hkv * s2h));
    ORTHRUS_CHECK_ARG(aligned16(q) && aligned16(k1) && aligned16(v1) && aligned16(o));
    AttnMaps m;
    if (!make_attn_maps(m, q, k1, v1, s1h, L1, has2 ? k2 : nullptr, has2 ? v2 : nullptr, s2h, L2, B, Hq, Hkv, Tq,
                        hd, D, nullptr))
      return ORTHRUS_ECUDA;
    const float sl2 = scale * kLog2e;
    if ((Hq / Hkv) % 2 == 0) {  // two query heads of one KV head per CTA
      ORTHRUS_CHECK_ARG(ceil_div(Tq, 128) < 65536);
      dim3 grid2(Hq / 2, static_cast<unsigned>(B), static_cast<unsigned>(ceil_div(Tq, 128)));
      if (D == 128) {
        if (set_smem(attn_fwd_tc2_kernel<128>, Fwd2Smem<128>::SMEM)) return ORTHRUS_ECUDA;
        ORTHRUS_CHECK_CUDA(launch_pdl(attn_fwd_tc2_kernel<128>, grid2, dim3(320), Fwd2Smem<128>::SMEM, st, m.q,
                                      m.k1, m.v1, m.k2, m.v2, Hq, Hkv, Tq, hd, sl2, mp, has2,
                                      static_cast<__nv_bfloat16*>(o), lse));
      } else {
        if (set_smem(attn_fwd_tc2_kernel<64>, Fwd2Smem<64>::SMEM)) return ORTHRUS_ECUDA;
        ORTHRUS_CHECK_CUDA(launch_pdl(attn_fwd_tc2_kernel<64>, grid2, dim3(320), Fwd2Smem<64>::SMEM, st, m.q, m.k1,
                                      m.v1, m.k2, m.v2, Hq, Hkv, Tq, hd, sl2, mp, has2,
                                      static_cast<__nv_bfloat16*>(o), lse));
      }
      ORTHRUS_CHECK_LAUNCH();
      return ORTHRUS_OK;
    }
    dim3 grid(static_cast<unsigned>(ceil_div(Tq, 128)), Hq, static_cast<unsigned>(B));
    if (D == 128) {
      if (set_smem(attn_fwd_tc_kernel<128>, FwdSmem<128>::SMEM)) return ORTHRUS_ECUDA;
      ORTHRUS_CHECK_CUDA(launch_pdl(attn_fwd_tc_kernel<128>, grid, dim3(192), FwdSmem<128>::SMEM, st, m.q, m.k1,
                                    m.v1, m.k2, m.v2, Hq, Hkv, Tq, hd, sl2, mp, has2,
                                    static_cast<__nv_bfloat16*>(o), lse));
    } else {
      if (set_smem(attn_fwd_tc_kernel<64>, FwdSmem<64>::SMEM)) return ORTHRUS_ECUDA;
      ORTHRUS_CHECK_CUDA(launch_pdl(attn_fwd_tc_kernel<64>, grid, dim3(192), FwdSmem<64>::SMEM, st, m.q, m.k1,
                                    m.v1, m.k2, m.v2, Hq, Hkv, Tq, hd, sl2, mp, has2,
                                    static_cast<__nv_bfloat16*>(o), lse));
    }
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  dim3 grid(static_cast<unsigned>(ceil_div(Tq, kSimtQ)), Hq, static_cast<unsigned>(B));
  if (dtype == ORTHRUS_BF16) {
    using T = __nv_bfloat16;
    attn_fwd_simt_kernel<T><<<grid, 32 * kSimtQ, 0, st>>>(
        static_cast<const T*>(q), static_cast<const T*>(k1), static_cast<const T*>(v1), s1h, s1b,
        static_cast<const T*>(k2), static_cast<const T*>(v2), s2h, s2b, Hq, Hkv, Tq, hd, D, scale, mp,
        static_cast<T*>(o), lse);
  } else if (dtype == ORTHRUS_F32) {
    attn_fwd_simt_kernel<float><<<grid, 32 * kSimtQ, 0, st>>>(
        static_cast<const float*>(q), static_cast<const float*>(k1), static_cast<const float*>(v1), s1h, s1b,
        static_cast<const float*>(k2), static_cast<const float*>(v2), s2h, s2b, Hq, Hkv, Tq, hd, D, scale, mp,
        static_cast<float*>(o), lse);
  } else {
    return ORTHRUS_EINVAL;
  }
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

size_t orthrus_attn_decode_workspace_bytes(int64_t B, int Hq, int64_t Tq, int64_t L1) {
  if (B <= 0 || Hq <= 0 || Tq <= 0 || L1 < 0) return 0;
  const size_t rows = static_cast<size_t>(decode_splits1(L1) + 1) * B * Hq * Tq;
  return rows * 128 * sizeof(float) + rows * 2 * sizeof(float);
}

int orthrus_attn_decode_fwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                            const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq,
                            int Hkv, int64_t Tq, float scale, int mask, const int32_t* offset, const int32_t* limit2,
                            void* o, void* workspace, size_t workspace_bytes, void* stream) {
  ORTHRUS_CHECK_ARG(q && k1 && v1 && o && workspace && B > 0 && B < 65536 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0);
  ORTHRUS_CHECK_ARG(Tq > 0 && Tq <= kDecSub && (Hq / Hkv) * Tq <= kDecMaxRows && L1 > 0 && Hkv < 65536);
  ORTHRUS_CHECK_ARG(mask == ORTHRUS_MASK_CAUSAL || (mask == ORTHRUS_MASK_DRAFT && k2 && v2 && L2 > 0 && L2 <= kDecSub));
  ORTHRUS_CHECK_ARG(workspace_bytes >= orthrus_attn_decode_workspace_bytes(B, Hq, Tq, L1));
  ORTHRUS_CHECK_ARG(aligned16(q) && aligned16(k1) && aligned16(v1) && aligned16(o) && aligned16(workspace));
  ORTHRUS_CHECK_ARG(s1h % 8 == 0 && s1b % 8 == 0 && (mask == ORTHRUS_MASK_CAUSAL || (s2h % 8 == 0 && s2b % 8 == 0)));
  const bool has2 = mask == ORTHRUS_MASK_DRAFT;
  MaskParams mp{mask, nullptr, 0, 0, offset, limit2, L1, has2 ? L2 : 0};
  const int ns1 = static_cast<int>(decode_splits1(L1));
  const size_t rows = static_cast<size_t>(ns1 + 1) * B * Hq * Tq;
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + rows * 128;
  cudaStream_t st = as_stream(stream);
  const int qrows = static_cast<int>(ceil_div((Hq / Hkv) * Tq, 16)) * 16;
  const int smem = decode_smem_bytes(qrows);
  if (set_smem(attn_decode_split_kernel, smem)) return ORTHRUS_ECUDA;
  const dim3 grid(static_cast<unsigned>(ns1 + (has2 ? 1 : 0)), static_cast<unsigned>(Hkv), static_cast<unsigned>(B));
  const auto* K2 = static_cast<const __nv_bfloat16*>(has2 ? k2 : k1);
  const auto* V2 = static_cast<const __nv_bfloat16*>(has2 ? v2 : v1);
  ORTHRUS_CHECK_CUDA(launch_pdl(attn_decode_split_kernel, grid, dim3(2 * qrows), smem, st,
                                static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k1),
                                static_cast<const __nv_bfloat16*>(v1), s1h, s1b, K2, V2, has2 ? s2h : s1h,
                                has2 ? s2b : s1b, Hq, Hkv, static_cast<int>(Tq), scale * kLog2e, mp, ns1, part_o,
                                part_ml));
  ORTHRUS_CHECK_LAUNCH();
  const int64_t items = B * Hq * Tq;
  ORTHRUS_CHECK_CUDA(launch_pdl(attn_decode_combine_kernel, dim3(static_cast<unsigned>(ceil_div(items, 8))), dim3(256),
                                0, st, static_cast<const float*>(part_o), static_cast<const float*>(part_ml), B, Hq,
                                static_cast<int>(Tq), ns1, mp, static_cast<__nv_bfloat16*>(o)));
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

size_t orthrus_attn_bwd_workspace_bytes(int64_t B, int Hq, int64_t Tq) {
  return static_cast<size_t>(B) * Hq * Tq * sizeof(float);
}

namespace {

// A second stream per device, with a fork and a join event, so that the dK/dV kernel of the
// backward runs beside the dQ kernel and fills the SMs its last partial wave leaves idle. Created
// on the first backward on each device; the join makes the caller's stream wait for the side
// stream, so the caller sees one ordered call (stream capture records it as a fork and a join).
// The events are shared by every caller on the device, so `use` is held from the fork record to
// the join wait: another host thread cannot re-record the fork between one call's record and its
// side-stream wait (which would make that call's dK/dV wait on the other caller's stream instead).
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex use;
};

SideStream* side_stream_on_current_device() {
  static std::mutex mu;
  static SideStream side[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  SideStream& s = side[dev];
  if (s.stream == nullptr) {
    if (cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
  }
  return &s;
}

}  // namespace

static int attn_bwd_impl(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                         const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq,
                         int Hkv, int64_t Tq, int hd, int D, float scale, const int64_t* anchors, int64_t A, int block,
                         const int32_t* doc_start, const void* o, const float* lse, const void* do_, float* dq,
                         float* dk2, float* dv2, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(q && k1 && v1 && k2 && v2 && anchors && o && lse && do_ && dq && dk2 && dv2);
  ORTHRUS_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Tq > 0 && hd > 0 && hd <= D && D <= 128);
  ORTHRUS_CHECK_ARG(A > 0 && block > 0 && L2 >= Tq && B < 65536 && Hq < 65536);
  if (workspace == nullptr || workspace_bytes < orthrus_attn_bwd_workspace_bytes(B, Hq, Tq)) return ORTHRUS_EWORKSPACE;
  float* delta = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  MaskParams mp{ORTHRUS_MASK_DUAL, anchors, A, block, nullptr, nullptr, L1, L2};
  mp.doc_start = doc_start;
  const int64_t items = B * Tq * Hq;
  const bool tc = use_tensor_cores(dtype, hd, D, ORTHRUS_MASK_DUAL, nullptr) && (128 % block == 0) &&
                  (Hq / Hkv) <= DkvSmem<128>::MAX_GROUP;
  if (dtype == ORTHRUS_BF16 && hd == 128 && aligned16(o) && aligned16(do_)) {
    ORTHRUS_CHECK_CUDA(launch_pdl(attn_delta128_bf16_kernel, dim3(static_cast<unsigned>(ceil_div(items, 16))),
                                  dim3(256), 0, st, static_cast<const __nv_bfloat16*>(o),
                                  static_cast<const __nv_bfloat16*>(do_), B, Hq, Tq, delta));
  } else if (dtype == ORTHRUS_BF16) {
    using T = __nv_bfloat16;
    attn_delta_kernel<T><<<static_cast<unsigned>(ceil_div(items, 8)), 256, 0, st>>>(
        static_cast<const T*>(o), static_cast<const T*>(do_), B, Hq, Tq, hd, delta);
  } else if (dtype == ORTHRUS_F32) {
    attn_delta_kernel<float><<<static_cast<unsigned>(ceil_div(items, 8)), 256, 0, st>>>(
        static_cast<const float*>(o), static_cast<const float*>(do_), B, Hq, Tq, hd, delta);
  } else {
    return ORTHRUS_EINVAL;
  }
  ORTHRUS_CHECK_LAUNCH();
  if (tc) {
    ORTHRUS_CHECK_ARG(s1b == Hkv * s1h && s2b == Hkv * s2h);
    ORTHRUS_CHECK_ARG(aligned16(q) && aligned16(k1) && aligned16(v1) && aligned16(k2) && aligned16(v2) &&
                      aligned16(do_) && aligned16(dq) && aligned16(dk2) && aligned16(dv2));
    AttnMaps m;
    if (!make_attn_maps(m, q, k1, v1, s1h, L1, k2, v2, s2h, L2, B, Hq, Hkv, Tq, hd, D, do_)) return ORTHRUS_ECUDA;
    dim3 grid(static_cast<unsigned>(ceil_div(Tq, 128)), Hq, static_cast<unsigned>(B));
    dim3 grid_kv(static_cast<unsigned>(ceil_div(L2, 128)), Hkv, static_cast<unsigned>(B));
    if ((Hq / Hkv) % 2 == 0) {  // dQ with two query heads per CTA and 64-key tiles
      AttnMaps m64;
      if (!make_attn_maps(m64, q, k1, v1, s1h, L1, k2, v2, s2h, L2, B, Hq, Hkv, Tq, hd, D, do_, 64))
        return ORTHRUS_ECUDA;
      ORTHRUS_CHECK_ARG(ceil_div(Tq, 128) < 65536);
      dim3 grid2(Hq / 2, static_cast<unsigned>(B), static_cast<unsigned>(ceil_div(Tq, 128)));
      // dQ on the caller's stream, dK/dV on the side stream (both only read delta and the inputs)
      SideStream* side = side_stream_on_current_device();
      if (side == nullptr) return ORTHRUS_ECUDA;
      std::lock_guard<std::mutex> in_use(side->use);  // fork record .. join wait (launches only)
      ORTHRUS_CHECK_CUDA(cudaEventRecord(side->fork, st));
      if (D == 128) {
        if (set_smem(attn_dq_tc2_kernel<128>, Dq2Smem<128>::SMEM)) return ORTHRUS_ECUDA;
        if (set_smem(attn_dkdv_tc_kernel<128>, DkvSmem<128>::SMEM)) return ORTHRUS_ECUDA;
        ORTHRUS_CHECK_CUDA(launch_pdl(attn_dq_tc2_kernel<128>, grid2, dim3(kDq2Threads), Dq2Smem<128>::SMEM, st, m64.q,
                                      m64.dout, m64.k1, m64.v1, m64.k2, m64.v2, Hq, Hkv, Tq, hd, scale, mp, true,
                                      lse, static_cast<const float*>(delta), dq));
        ORTHRUS_CHECK_LAUNCH();
        ORTHRUS_CHECK_CUDA(cudaStreamWaitEvent(side->stream, side->fork, 0));
        const int G = Hq / Hkv;
        if (block == 32 && hd == 128 && Tq % 32 == 0 && (G == 2 || G == 4) && s2h % 8 == 0 && s2b % 8 == 0 &&
            Tq / 32 < (1ll << 31)) {
          // 32-key blocks: the HBM-bound own-block kernel (32 x 32 problems, no 128-row padding)
          const dim3 grid_b(static_cast<unsigned>(Tq / 32), Hkv, static_cast<unsigned>(B));
          auto* qb = static_cast<const __nv_bfloat16*>(q);
          auto* k2b = static_cast<const __nv_bfloat16*>(k2);
          auto* v2b = static_cast<const __nv_bfloat16*>(v2);
          auto* dob = static_cast<const __nv_bfloat16*>(do_);
          if (G == 2) {
            if (set_smem(attn_dkdv_block32_kernel<2>, BlockKvSmem::bytes<2>())) return ORTHRUS_ECUDA;
            attn_dkdv_block32_kernel<2><<<grid_b, 128, BlockKvSmem::bytes<2>(), side->stream>>>(
                qb, k2b, v2b, s2h, s2b, dob, lse, delta, Hq, Hkv, Tq, L2, scale, dk2, dv2);
          } else {
            if (set_smem(attn_dkdv_block32_kernel<4>, BlockKvSmem::bytes<4>())) return ORTHRUS_ECUDA;
            attn_dkdv_block32_kernel<4><<<grid_b, 128, BlockKvSmem::bytes<4>(), side->stream>>>(
                qb, k2b, v2b, s2h, s2b, dob, lse, delta, Hq, Hkv, Tq, L2, scale, dk2, dv2);
          }
        } else {
          attn_dkdv_tc_kernel<128><<<grid_kv, 192, DkvSmem<128>::SMEM, side->stream>>>(
              m.q, m.dout, m.k2, m.v2, Hq, Hkv, Tq, L2, hd, block, scale, lse, delta, dk2, dv2);
        }
      } else {
        if (set_smem(attn_dq_tc2_kernel<64>, Dq2Smem<64>::SMEM)) return ORTHRUS_ECUDA;
        if (set_smem(attn_dkdv_tc_kernel<64>, DkvSmem<64>::SMEM)) return ORTHRUS_ECUDA;
        attn_dq_tc2_kernel<64><<<grid2, kDq2Threads, Dq2Smem<64>::SMEM, st>>>(
            m64.q, m64.dout, m64.k1, m64.v1, m64.k2, m64.v2, Hq, Hkv, Tq, hd, scale, mp, true, lse, delta, dq);
        ORTHRUS_CHECK_LAUNCH();
        ORTHRUS_CHECK_CUDA(cudaStreamWaitEvent(side->stream, side->fork, 0));
        attn_dkdv_tc_kernel<64><<<grid_kv, 192, DkvSmem<64>::SMEM, side->stream>>>(
            m.q, m.dout, m.k2, m.v2, Hq, Hkv, Tq, L2, hd, block, scale, lse, delta, dk2, dv2);
      }
      ORTHRUS_CHECK_LAUNCH();
      ORTHRUS_CHECK_CUDA(cudaEventRecord(side->join, side->stream));
      ORTHRUS_CHECK_CUDA(cudaStreamWaitEvent(st, side->join, 0));
      return ORTHRUS_OK;
    }
    if (D == 128) {
      if (set_smem(attn_dq_tc_kernel<128>, DqSmem<128>::SMEM)) return ORTHRUS_ECUDA;
      attn_dq_tc_kernel<128><<<grid, 192, DqSmem<128>::SMEM, st>>>(m.q, m.dout, m.k1, m.v1, m.k2, m.v2, Hq, Hkv, Tq,
                                                                     hd, scale, mp, true, lse, delta, dq);
      ORTHRUS_CHECK_LAUNCH();
      if (set_smem(attn_dkdv_tc_kernel<128>, DkvSmem<128>::SMEM)) return ORTHRUS_ECUDA;
      attn_dkdv_tc_kernel<128><<<grid_kv, 192, DkvSmem<128>::SMEM, st>>>(m.q, m.dout, m.k2, m.v2, Hq, Hkv, Tq, L2,
                                                                           hd, block, scale, lse, delta, dk2, dv2);
    } else {
      if (set_smem(attn_dq_tc_kernel<64>, DqSmem<64>::SMEM)) return ORTHRUS_ECUDA;
      attn_dq_tc_kernel<64><<<grid, 192, DqSmem<64>::SMEM, st>>>(m.q, m.dout, m.k1, m.v1, m.k2, m.v2, Hq, Hkv, Tq, hd,
                                                                   scale, mp, true, lse, delta, dq);
      ORTHRUS_CHECK_LAUNCH();
      if (set_smem(attn_dkdv_tc_kernel<64>, DkvSmem<64>::SMEM)) return ORTHRUS_ECUDA;
      attn_dkdv_tc_kernel<64><<<grid_kv, 192, DkvSmem<64>::SMEM, st>>>(m.q, m.dout, m.k2, m.v2, Hq, Hkv, Tq, L2, hd,
                                                                         block, scale, lse, delta, dk2, dv2);
    }
    ORTHRUS_CHECK_LAUNCH();
    return ORTHRUS_OK;
  }
  dim3 grid(static_cast<unsigned>(ceil_div(Tq, kSimtQ)), Hq, static_cast<unsigned>(B));
  dim3 grid_kv(static_cast<unsigned>(ceil_div(L2, 8)), Hkv, static_cast<unsigned>(B));
  if (dtype == ORTHRUS_BF16) {
    using T = __nv_bfloat16;
    attn_dq_simt_kernel<T><<<grid, 32 * kSimtQ, 0, st>>>(
        static_cast<const T*>(q), static_cast<const T*>(k1), static_cast<const T*>(v1), s1h, s1b,
        static_cast<const T*>(k2), static_cast<const T*>(v2), s2h, s2b, Hq, Hkv, Tq, hd, D, scale, mp, lse, delta,
        static_cast<const T*>(do_), dq);
    ORTHRUS_CHECK_LAUNCH();
    attn_dkdv_block_simt_kernel<T><<<grid_kv, 256, 0, st>>>(static_cast<const T*>(q), static_cast<const T*>(k2),
                                                            static_cast<const T*>(v2), s2h, s2b, Hq, Hkv, Tq, hd, D,
                                                            scale, block, L2, lse, delta, static_cast<const T*>(do_),
                                                            dk2, dv2);
  } else {
    attn_dq_simt_kernel<float><<<grid, 32 * kSimtQ, 0, st>>>(
        static_cast<const float*>(q), static_cast<const float*>(k1), static_cast<const float*>(v1), s1h, s1b,
        static_cast<const float*>(k2), static_cast<const float*>(v2), s2h, s2b, Hq, Hkv, Tq, hd, D, scale, mp, lse,
        delta, static_cast<const float*>(do_), dq);
    ORTHRUS_CHECK_LAUNCH();
    attn_dkdv_block_simt_kernel<float><<<grid_kv, 256, 0, st>>>(
        static_cast<const float*>(q), static_cast<const float*>(k2), static_cast<const float*>(v2), s2h, s2b, Hq, Hkv,
        Tq, hd, D, scale, block, L2, lse, delta, static_cast<const float*>(do_), dk2, dv2);
  }
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_argmax_rows(const float* logits, int64_t ldl, int64_t R, int64_t V, int64_t* out, void* stream) {
  ORTHRUS_CHECK_ARG(logits && out && R >= 0 && V > 0 && ldl >= V);
  if (R == 0) return ORTHRUS_OK;
  argmax_rows_kernel<<<static_cast<unsigned>(R), 512, 0, as_stream(stream)>>>(logits, ldl, V, out);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_decode_draft(const float* logits, int64_t B, int K, int64_t V, const int64_t* anchor, const uint8_t* done,
                         int64_t* verify_ids, void* stream) {
  ORTHRUS_CHECK_ARG(logits && anchor && verify_ids && B > 0 && K >= 1 && V > 0 && B < 65536);
  if (K == 1) return ORTHRUS_OK;
  dim3 grid(K - 1, static_cast<unsigned>(B));
  decode_draft_kernel<<<grid, 512, 0, as_stream(stream)>>>(logits, K, V, anchor, done, verify_ids);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_decode_verify_accept(const float* logits, int64_t B, int K, int64_t V, const int64_t* verify_ids,
                                 int64_t* ar_tokens, const int64_t* eos, int n_eos, const int32_t* max_len,
                                 int32_t* start, int64_t* anchor, uint8_t* done, int64_t* out_tokens,
                                 int32_t* out_len, int64_t out_cap, int32_t* accepted_log, int32_t* cycle,
                                 int64_t log_cap, void* stream) {
  ORTHRUS_CHECK_ARG(logits && verify_ids && ar_tokens && max_len && start && anchor && done && out_tokens &&
                    out_len && accepted_log && cycle && B > 0 && K >= 1 && V > 0);
  ORTHRUS_CHECK_ARG(n_eos == 0 || eos != nullptr);
  cudaStream_t st = as_stream(stream);
  argmax_rows_kernel<<<static_cast<unsigned>(B * K), 512, 0, st>>>(logits, V, V, ar_tokens);
  ORTHRUS_CHECK_LAUNCH();
  decode_accept_kernel<<<static_cast<unsigned>(ceil_div(B, 128)), 128, 0, st>>>(
      B, K, verify_ids, ar_tokens, eos, n_eos, max_len, start, anchor, done, out_tokens, out_len, out_cap,
      accepted_log, cycle, log_cap);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

static bool sample_args_ok(int C, float temperature, int top_k, float top_p) {
  return C >= 1 && C <= kSampleMaxCand && temperature > 0.f && top_k >= 1 && top_k <= C && top_p > 0.f;
}

int orthrus_sample_probs(const float* cand_vals, int64_t R, int C, float temperature, int top_k, float top_p,
                         float* probs, void* stream) {
  ORTHRUS_CHECK_ARG(cand_vals && probs && R >= 0 && sample_args_ok(C, temperature, top_k, top_p));
  if (R == 0) return ORTHRUS_OK;
  sample_probs_kernel<<<static_cast<unsigned>(ceil_div(R, 128)), 128, 0, as_stream(stream)>>>(
      cand_vals, R, C, temperature, top_k, top_p, probs);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_sample_rows(const float* cand_vals, const int64_t* cand_ids, int64_t R, int C, float temperature,
                        int top_k, float top_p, uint64_t seed, const int32_t* cycle, int64_t* tokens, void* stream) {
  ORTHRUS_CHECK_ARG(cand_vals && cand_ids && tokens && R >= 0 && sample_args_ok(C, temperature, top_k, top_p));
  if (R == 0) return ORTHRUS_OK;
  sample_rows_kernel<<<static_cast<unsigned>(ceil_div(R, 128)), 128, 0, as_stream(stream)>>>(
      cand_vals, cand_ids, R, C, temperature, top_k, top_p, seed, cycle, tokens);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_decode_sample_draft(const float* cand_vals, const int64_t* cand_ids, int64_t B, int K, int C,
                                float temperature, int top_k, float top_p, uint64_t seed, const int32_t* cycle,
                                const int64_t* anchor, const uint8_t* done, int64_t* verify_ids, float* draft_probs,
                                void* stream) {
  ORTHRUS_CHECK_ARG(cand_vals && cand_ids && cycle && anchor && done && verify_ids && draft_probs && B > 0 &&
                    B < (1 << 30) && K >= 2 && K <= kSampleMaxBlock && sample_args_ok(C, temperature, top_k, top_p));
  decode_sample_draft_kernel<<<static_cast<unsigned>(B), kSampleMaxBlock, 0, as_stream(stream)>>>(
      cand_vals, cand_ids, K, C, temperature, top_k, top_p, seed, cycle, anchor, done, verify_ids, draft_probs);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_decode_sample_accept(const float* cand_vals, const int64_t* cand_ids, const float* draft_probs,
                                 const int64_t* draft_ids, int64_t B, int K, int C, float temperature, int top_k,
                                 float top_p, uint64_t seed, const int64_t* verify_ids, const int64_t* eos, int n_eos,
                                 const int32_t* max_len, int32_t* start, int64_t* anchor, uint8_t* done,
                                 int64_t* out_tokens, int32_t* out_len, int64_t out_cap, int32_t* accepted_log,
                                 int32_t* cycle, int64_t log_cap, void* stream) {
  ORTHRUS_CHECK_ARG(cand_vals && cand_ids && draft_probs && draft_ids && verify_ids && max_len && start && anchor &&
                    done && out_tokens && out_len && accepted_log && cycle && B > 0 && B < (1 << 30) && K >= 2 &&
                    K <= kSampleMaxBlock && sample_args_ok(C, temperature, top_k, top_p));
  ORTHRUS_CHECK_ARG(n_eos == 0 || eos != nullptr);
  decode_sample_accept_kernel<<<static_cast<unsigned>(B), kSampleMaxBlock, 0, as_stream(stream)>>>(
      cand_vals, cand_ids, draft_probs, draft_ids, K, C, temperature, top_k, top_p, seed, verify_ids, eos, n_eos,
      max_len, start, anchor, done, out_tokens, out_len, out_cap, accepted_log, cycle, log_cap);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_philox4x32_10(const uint32_t* counter_key, int64_t n, uint32_t* out, void* stream) {
  ORTHRUS_CHECK_ARG(counter_key && out && n >= 0);
  if (n == 0) return ORTHRUS_OK;
  philox_kernel<<<static_cast<unsigned>(ceil_div(n, 128)), 128, 0, as_stream(stream)>>>(counter_key, n, out);
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

int orthrus_attn_fwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                     const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq, int Hkv,
                     int64_t Tq, int hd, int D, float scale, int mask, const int64_t* anchors, int64_t A, int block,
                     const int32_t* offset, const int32_t* limit2, void* o, float* lse, int dtype, void* stream) {
  return attn_fwd_impl(q, k1, v1, s1h, s1b, L1, k2, v2, s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, scale, mask, anchors, A,
                       block, offset, limit2, nullptr, o, lse, dtype, stream);
}

int orthrus_attn_fwd_doc(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                         const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq,
                         int Hkv, int64_t Tq, int hd, int D, float scale, int mask, const int64_t* anchors, int64_t A,
                         int block, const int32_t* offset, const int32_t* limit2, const int32_t* doc_start, void* o,
                         float* lse, int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(doc_start != nullptr && L1 > 0);
  return attn_fwd_impl(q, k1, v1, s1h, s1b, L1, k2, v2, s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, scale, mask, anchors, A,
                       block, offset, limit2, doc_start, o, lse, dtype, stream);
}

int orthrus_attn_bwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                     const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq, int Hkv,
                     int64_t Tq, int hd, int D, float scale, const int64_t* anchors, int64_t A, int block,
                     const void* o, const float* lse, const void* do_, float* dq, float* dk2, float* dv2,
                     void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  return attn_bwd_impl(q, k1, v1, s1h, s1b, L1, k2, v2, s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, scale, anchors, A, block,
                       nullptr, o, lse, do_, dq, dk2, dv2, workspace, workspace_bytes, dtype, stream);
}

int orthrus_attn_bwd_doc(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b, int64_t L1,
                         const void* k2, const void* v2, int64_t s2h, int64_t s2b, int64_t L2, int64_t B, int Hq,
                         int Hkv, int64_t Tq, int hd, int D, float scale, const int64_t* anchors, int64_t A,
                         int block, const int32_t* doc_start, const void* o, const float* lse, const void* do_,
                         float* dq, float* dk2, float* dv2, void* workspace, size_t workspace_bytes, int dtype,
                         void* stream) {
  ORTHRUS_CHECK_ARG(doc_start != nullptr && L1 > 0);
  return attn_bwd_impl(q, k1, v1, s1h, s1b, L1, k2, v2, s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, scale, anchors, A, block,
                       doc_start, o, lse, do_, dq, dk2, dv2, workspace, workspace_bytes, dtype, stream);
}

}  // extern "C"

namespace {

// The register-resident RMSNorm kernels take bf16 rows of 256, 512, 1024 or 2048 elements (one to
// eight 16-byte vectors per lane); other widths keep the strided kernels.
int rmsnorm_reg_chunks(int d) { return (d == 256 || d == 512 || d == 1024 || d == 2048) ? d / 256 : 0; }

cudaError_t rmsnorm_fwd_reg(int chunks, unsigned blocks, cudaStream_t st, const __nv_bfloat16* x,
                            const __nv_bfloat16* w, int64_t rows, float eps, __nv_bfloat16* y, float* rstd) {
  using T = __nv_bfloat16;
  switch (chunks) {
    case 1: return launch_pdl(rmsnorm_fwd_reg_kernel<T, 1>, dim3(blocks), dim3(256), 0, st, x, w, rows, eps, y, rstd);
    case 2: return launch_pdl(rmsnorm_fwd_reg_kernel<T, 2>, dim3(blocks), dim3(256), 0, st, x, w, rows, eps, y, rstd);
    case 4: return launch_pdl(rmsnorm_fwd_reg_kernel<T, 4>, dim3(blocks), dim3(256), 0, st, x, w, rows, eps, y, rstd);
    default: return launch_pdl(rmsnorm_fwd_reg_kernel<T, 8>, dim3(blocks), dim3(256), 0, st, x, w, rows, eps, y, rstd);
  }
}

template <bool ADD>
cudaError_t rmsnorm_bwd_reg(int chunks, unsigned blocks, cudaStream_t st, const __nv_bfloat16* x,
                            const __nv_bfloat16* w, const float* rstd, const __nv_bfloat16* dy, int64_t rows,
                            __nv_bfloat16* dx, const __nv_bfloat16* dres) {
  using T = __nv_bfloat16;
  switch (chunks) {
    case 1: return launch_pdl(rmsnorm_bwd_reg_kernel<T, 1, ADD>, dim3(blocks), dim3(256), 0, st, x, w, rstd, dy, rows, dx, dres);
    case 2: return launch_pdl(rmsnorm_bwd_reg_kernel<T, 2, ADD>, dim3(blocks), dim3(256), 0, st, x, w, rstd, dy, rows, dx, dres);
    case 4: return launch_pdl(rmsnorm_bwd_reg_kernel<T, 4, ADD>, dim3(blocks), dim3(256), 0, st, x, w, rstd, dy, rows, dx, dres);
    default: return launch_pdl(rmsnorm_bwd_reg_kernel<T, 8, ADD>, dim3(blocks), dim3(256), 0, st, x, w, rstd, dy, rows, dx, dres);
  }
}

}  // namespace

extern "C" int orthrus_rmsnorm(const void* x, const void* w, int64_t rows, int d, float eps, void* y, float* rstd,
                               int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(x && w && y && rows >= 0 && d > 0);
  if (rows == 0) return ORTHRUS_OK;
  const unsigned blocks = static_cast<unsigned>(ceil_div(rows, 8));
  const bool vec = aligned16(x) && aligned16(w) && aligned16(y) && d % (dtype == ORTHRUS_BF16 ? 256 : 128) == 0;
  if (dtype == ORTHRUS_BF16) {
    using T = __nv_bfloat16;
    if (vec && rmsnorm_reg_chunks(d) > 0)
      ORTHRUS_CHECK_CUDA(rmsnorm_fwd_reg(rmsnorm_reg_chunks(d), blocks, as_stream(stream), static_cast<const T*>(x),
                                         static_cast<const T*>(w), rows, eps, static_cast<T*>(y), rstd));
    else if (vec)
      ORTHRUS_CHECK_CUDA(launch_pdl(rmsnorm_fwd_vec_kernel<T>, dim3(blocks), dim3(256), 0, as_stream(stream),
                                    static_cast<const T*>(x), static_cast<const T*>(w), rows, d, eps,
                                    static_cast<T*>(y), rstd));
    else
      rmsnorm_kernel<T><<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const T*>(x), static_cast<const T*>(w), rows,
                                                              d, eps, static_cast<T*>(y), rstd);
  } else if (dtype == ORTHRUS_F32) {
    if (vec)
      rmsnorm_fwd_vec_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
          static_cast<const float*>(x), static_cast<const float*>(w), rows, d, eps, static_cast<float*>(y), rstd);
    else
      rmsnorm_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const float*>(x),
                                                                 static_cast<const float*>(w), rows, d, eps,
                                                                 static_cast<float*>(y), rstd);
  } else {
    return ORTHRUS_EINVAL;
  }
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

extern "C" int orthrus_rmsnorm_bwd_add(const void* x, const void* w, const float* rstd, const void* dy,
                                       const void* dres, int64_t rows, int d, void* dx, void* stream) {
  ORTHRUS_CHECK_ARG(x && w && rstd && dy && dres && dx && rows >= 0 && d > 0 && d % 256 == 0);
  ORTHRUS_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(dy) && aligned16(dres) && aligned16(dx));
  if (rows == 0) return ORTHRUS_OK;
  using T = __nv_bfloat16;
  if (rmsnorm_reg_chunks(d) > 0)
    ORTHRUS_CHECK_CUDA(rmsnorm_bwd_reg<true>(rmsnorm_reg_chunks(d), static_cast<unsigned>(ceil_div(rows, 8)),
                                             as_stream(stream), static_cast<const T*>(x), static_cast<const T*>(w),
                                             rstd, static_cast<const T*>(dy), rows, static_cast<T*>(dx),
                                             static_cast<const T*>(dres)));
  else
    ORTHRUS_CHECK_CUDA(launch_pdl(rmsnorm_bwd_vec_kernel<T>, dim3(static_cast<unsigned>(ceil_div(rows, 8))),
                                  dim3(256), 0, as_stream(stream), static_cast<const T*>(x),
                                  static_cast<const T*>(w), rstd, static_cast<const T*>(dy), rows, d,
                                  static_cast<T*>(dx), static_cast<const T*>(dres)));
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

extern "C" int orthrus_rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, int64_t rows,
                                   int d, void* dx, int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(x && w && rstd && dy && dx && rows >= 0 && d > 0);
  if (rows == 0) return ORTHRUS_OK;
  const unsigned blocks = static_cast<unsigned>(ceil_div(rows, 8));
  const bool vec = aligned16(x) && aligned16(w) && aligned16(dy) && aligned16(dx) &&
                   d % (dtype == ORTHRUS_BF16 ? 256 : 128) == 0;
  if (dtype == ORTHRUS_BF16) {
    using T = __nv_bfloat16;
    if (vec && rmsnorm_reg_chunks(d) > 0)
      ORTHRUS_CHECK_CUDA(rmsnorm_bwd_reg<false>(rmsnorm_reg_chunks(d), blocks, as_stream(stream), static_cast<const T*>(x),
                                                static_cast<const T*>(w), rstd, static_cast<const T*>(dy), rows,
                                                static_cast<T*>(dx), static_cast<const T*>(nullptr)));
    else if (vec)
      ORTHRUS_CHECK_CUDA(launch_pdl(rmsnorm_bwd_vec_kernel<T>, dim3(blocks), dim3(256), 0, as_stream(stream),
                                    static_cast<const T*>(x), static_cast<const T*>(w), rstd,
                                    static_cast<const T*>(dy), rows, d, static_cast<T*>(dx),
                                    static_cast<const T*>(nullptr)));
    else
      rmsnorm_bwd_kernel<T><<<blocks, 256, 0, as_stream(stream)>>>(
          static_cast<const T*>(x), static_cast<const T*>(w), rstd, static_cast<const T*>(dy), rows, d,
          static_cast<T*>(dx));
  } else if (dtype == ORTHRUS_F32) {
    if (vec)
      rmsnorm_bwd_vec_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
          static_cast<const float*>(x), static_cast<const float*>(w), rstd, static_cast<const float*>(dy), rows, d,
          static_cast<float*>(dx));
    else
      rmsnorm_bwd_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
          static_cast<const float*>(x), static_cast<const float*>(w), rstd, static_cast<const float*>(dy), rows, d,
          static_cast<float*>(dx));
  } else {
    return ORTHRUS_EINVAL;
  }
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

extern "C" int orthrus_swiglu_fwd(const void* gate_up, int64_t rows, int inter, void* out, int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(gate_up && out && rows >= 0 && inter > 0 && aligned16(gate_up) && aligned16(out));
  ORTHRUS_CHECK_ARG(inter % (dtype == ORTHRUS_BF16 ? 8 : 4) == 0);
  if (rows == 0) return ORTHRUS_OK;
  const int64_t items = rows * inter / (dtype == ORTHRUS_BF16 ? 8 : 4);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(items, 256), 148 * 16));
  if (dtype == ORTHRUS_BF16)
    swiglu_fwd_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(gate_up), rows, inter, static_cast<__nv_bfloat16*>(out));
  else if (dtype == ORTHRUS_F32)
    swiglu_fwd_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const float*>(gate_up), rows, inter,
                                                                     static_cast<float*>(out));
  else
    return ORTHRUS_EINVAL;
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

extern "C" int orthrus_swiglu_bwd(const void* gate_up, const void* dout, int64_t rows, int inter, void* dgate_up,
                                  int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(gate_up && dout && dgate_up && rows >= 0 && inter > 0);
  ORTHRUS_CHECK_ARG(aligned16(gate_up) && aligned16(dout) && aligned16(dgate_up));
  ORTHRUS_CHECK_ARG(inter % (dtype == ORTHRUS_BF16 ? 8 : 4) == 0);
  if (rows == 0) return ORTHRUS_OK;
  const int64_t items = rows * inter / (dtype == ORTHRUS_BF16 ? 8 : 4);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(items, 256), 148 * 16));
  if (dtype == ORTHRUS_BF16)
    swiglu_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(gate_up), static_cast<const __nv_bfloat16*>(dout), rows, inter,
        static_cast<__nv_bfloat16*>(dgate_up));
  else if (dtype == ORTHRUS_F32)
    swiglu_bwd_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>(
        static_cast<const float*>(gate_up), static_cast<const float*>(dout), rows, inter, static_cast<float*>(dgate_up));
  else
    return ORTHRUS_EINVAL;
  ORTHRUS_CHECK_LAUNCH();
  return ORTHRUS_OK;
}

// ------------------------------------------------------------------------------------------------
// Attention backward without any allocation
// ------------------------------------------------------------------------------------------------
//
// For callers that cannot allocate device memory (see orthrus_attn_bwd_noalloc in the header):
// the per-query scratch of the backward (delta = rowsum(dO * O), one fp32 per query row per head)
// lives in a fixed array of this translation unit instead of a caller workspace.

namespace {

static __device__ __align__(256) float g_attn_bwd_noalloc_scratch[ORTHRUS_ATTN_BWD_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;

// Device address of the scratch array on the current device. Host code only sees a host-side
// stand-in under the array's name, so the address is looked up once per device (with that device
// current) through cudaGetSymbolAddress and cached.
void* noalloc_scratch_on_current_device() {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_bwd_noalloc_scratch) != cudaSuccess) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace

extern "C" int orthrus_attn_bwd_noalloc(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                                        int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                                        int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, int hd, int D,
                                        float scale, const int64_t* anchors, int64_t A, int block, const void* o,
                                        const float* lse, const void* do_, float* dq, float* dk2, float* dv2,
                                        int dtype, void* stream) {
  ORTHRUS_CHECK_ARG(B > 0 && Hq > 0 && Tq > 0);
  if (B * static_cast<int64_t>(Hq) * Tq > ORTHRUS_ATTN_BWD_NOALLOC_MAX_ROWS) {
    if (getenv("ORTHRUS_DEBUG"))
      fprintf(stderr, "orthrus_attn_bwd_noalloc: B*Hq*Tq = %lld exceeds the %d rows of fixed scratch\n",
              static_cast<long long>(B * static_cast<int64_t>(Hq) * Tq), ORTHRUS_ATTN_BWD_NOALLOC_MAX_ROWS);
    return ORTHRUS_EINVAL;
  }
  void* scratch = noalloc_scratch_on_current_device();
  if (scratch == nullptr) return ORTHRUS_ECUDA;
  // every row of delta the kernels read is written first by the delta kernel: nothing to clear
  return orthrus_attn_bwd(q, k1, v1, s1h, s1b, L1, k2, v2, s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, scale, anchors, A,
                          block, o, lse, do_, dq, dk2, dv2, scratch, sizeof(g_attn_bwd_noalloc_scratch), dtype,
                          stream);
}
