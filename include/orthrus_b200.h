/*
 * orthrus_b200.h — C ABI of the Blackwell (sm_100a) kernels behind the Orthrus dual-view path.
 *
 * The Python drop-in modules (orthrus_training_b200.modeling_orthrus / objective / decoding) call
 * these entry points through ctypes; any other host (C++, a cgo or JNI binding) can call them the
 * same way. Conventions shared by every entry point:
 *   - plain device pointers and sizes, no framework types; every buffer is allocated by the caller
 *     (outputs and, where a *_workspace_bytes query exists, scratch memory);
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); work is enqueued asynchronously;
 *   - the return value is a status: ORTHRUS_OK, or a negative ORTHRUS_E* code for bad arguments or a
 *     failed launch. Kernels never trap: a device-side wait that runs out of time (2 s) records a
 *     bit in the device error word, read with orthrus_device_error();
 *   - dtype codes: ORTHRUS_BF16 (tensor-core path) or ORTHRUS_F32 (exact fp32 path on CUDA cores);
 *   - no global mutable state besides the device error word and a host-side launch counter.
 *
 * Each entry point names the reference interface it replaces (paths inside the reference project
 * ekonst41/orthrus-training).
 */
#ifndef ORTHRUS_B200_H
#define ORTHRUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------ */
#define ORTHRUS_OK 0
#define ORTHRUS_EINVAL (-1)       /* bad argument: shape, pointer alignment, unsupported size   */
#define ORTHRUS_ECUDA (-2)        /* a CUDA runtime call or kernel launch failed                */
#define ORTHRUS_EWORKSPACE (-3)   /* caller workspace smaller than *_workspace_bytes reported    */
#define ORTHRUS_EDEVICE (-4)      /* orthrus_device_error found the device error word non-zero   */

/* ---- device error word bits ------------------------------------------------------------- */
#define ORTHRUS_ERR_TIMEOUT 1u    /* a bounded wait (mbarrier / flag) ran out of time            */
#define ORTHRUS_ERR_BOUNDS 2u     /* a device-side index check failed; the access was skipped    */

/* ---- dtypes ----------------------------------------------------------------------------- */
#define ORTHRUS_BF16 0
#define ORTHRUS_F32 1

/* ---- attention mask modes (orthrus_attn_fwd / orthrus_attn_bwd) ------------------------- */
/* Query t of batch b sees source-1 keys [0, e1) and source-2 keys [s2, e2):                   */
#define ORTHRUS_MASK_CAUSAL 0  /* e1 = t + 1 + offset[b] (offset NULL = 0); no source 2         */
#define ORTHRUS_MASK_DUAL 1    /* blk = t / block: e1 = min(anchors[b, blk], L1),               */
                               /* [s2, e2) = [blk*block, blk*block + block)                     */
#define ORTHRUS_MASK_DRAFT 2   /* e1 = offset[b]; [s2, e2) = [0, min(L2, limit2[b]))             */
#define ORTHRUS_MASK_TREE 3    /* tree verification over a cache holding the new tokens at rows   */
                               /* offset[b] + t, passed as both sources: e1 = offset[b] + 1 (the  */
                               /* prefix and the root t = 0), [s2, e2) = [offset[b] + limit2[t],  */
                               /* offset[b] + t + 1) (the query's own branch up to itself; limit2 */
                               /* is per query here, >= 1). Forward only.                         */

/* Library version (major*10000 + minor*100 + patch). */
int orthrus_version(void);

/* Number of kernels this process has launched through the library so far (diagnostics). */
unsigned long long orthrus_launch_count(void);

/* Reads the device error word of `device` (synchronizes that device) into *word; clears it when
 * `clear` is non-zero. Returns ORTHRUS_OK, or ORTHRUS_EDEVICE when the word was non-zero. */
int orthrus_device_error(int device, unsigned int* word, int clear);

/* ---- dense GEMM building block (tcgen05) ------------------------------------------------- */
/* C[M, N] = A[M, K] @ B^T, bf16 inputs, fp32 accumulation in tensor memory.
 *   b_kn = 0: B is [N, K] row-major (ldb >= K); b_kn = 1: B is [K, N] row-major (ldb >= N).
 *   c_f32 = 1 writes fp32 C, else bf16. Leading dimensions are in elements and multiples of 8.
 *   The per-element reduction order depends on (N, K) only, never on M: results for a row are
 *   bit-identical whatever M is (used for lossless decoding).
 * Replaces the cuBLAS GEMM of F.linear / torch.mm (orthrus/objective.py:139-149,303-313,384). */
size_t orthrus_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
int orthrus_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                      int64_t M, int64_t N, int64_t K, int b_kn, int c_f32, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Projection GEMM on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles over two SMs):
 * C[M, N] (pitch ldc) = A @ B^T, or R + A @ B^T with epilogue ORTHRUS_GEMM2_RESIDUAL (one
 * rounding, R [M, N] pitch ldr, not aliasing C). A is [M, K] row-major (a_mn = 0) or stored
 * transposed as [K, M] (a_mn = 1); B is [N, K] (b_mn = 0) or stored transposed as [K, N]
 * (b_mn = 1). All bf16 with fp32 accumulation; pitches multiples of 8 elements, N a multiple of
 * 32, pointers 16-byte aligned; the residual form takes a row-major A.
 * Replaces the F.linear projections of the training step and their autograd backward
 * (orthrus/objective.py:136-149,160-165): y = x W^T (+ residual), dX = dY W (b_mn = 1),
 * dW = dY^T X (a_mn = b_mn = 1). A problem whose tiles fill less than one wave of SM pairs is
 * split over K into fp32 partials in the workspace (orthrus_gemm2_workspace_bytes, 0 when not
 * split) and reduced in a fixed order, so results do not depend on timing. */
#define ORTHRUS_GEMM2_STORE 0
#define ORTHRUS_GEMM2_RESIDUAL 1
#define ORTHRUS_GEMM2_SWIGLU_BWD 2  /* R = [gate | up] [M, 2N] of the MLP forward (pitch ldr); C = [dgate | dup]
                                      [M, 2N] (pitch ldc), from the accumulator dact = dY @ W_down, with the
                                      arithmetic of orthrus_swiglu_bwd */
size_t orthrus_gemm2_workspace_bytes(int64_t M, int64_t N, int64_t K);
int orthrus_gemm2_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                       void* C, int64_t ldc, const void* R, int64_t ldr, int64_t M, int64_t N,
                       int64_t K, int epilogue, void* workspace, size_t workspace_bytes, void* stream);

/* Projection GEMM with the layer's elementwise tail in the epilogue, bf16 in and out:
 *   ORTHRUS_LINEAR_STORE     y[M, N] = x[M, K] @ w[N, K]^T                      (F.linear)
 *   ORTHRUS_LINEAR_RESIDUAL  y = residual + x @ w^T, fp32 sum rounded once      (torch.addmm)
 *   ORTHRUS_LINEAR_SWIGLU    w = [gate; up] [2N, K]: y[M, N] = silu(g) * u, g and u rounded to bf16
 *                            and silu rounded before the product (F.linear then F.silu(gate) * up)
 * N a multiple of 128, K a multiple of 8, leading dimensions multiples of 8 elements, pointers
 * 16-byte aligned; residual has leading dimension ldy and does not alias y. Persistent tcgen05
 * kernel, one CTA per SM. Replaces the projections and activations of _attention_inputs and
 * _mlp_residual (orthrus/objective.py:136-149) on the frozen teacher pass. */
#define ORTHRUS_LINEAR_STORE 0
#define ORTHRUS_LINEAR_RESIDUAL 1
#define ORTHRUS_LINEAR_SWIGLU 2
#define ORTHRUS_LINEAR_PAIR 0x100  /* flag: the same kernel on CTA pairs (tcgen05 cta_group::2, 256-row tiles) */
int orthrus_linear_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* residual,
                        void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int epilogue,
                        void* stream);

/* The same three epilogues (STORE, RESIDUAL, SWIGLU) on 128-row x 64-column tiles (32 output
 * columns for SWIGLU), one tile per CTA with the full K: many CTAs stream weights when M is a
 * few rows (the decode passes). N a multiple of 64 (SWIGLU: 32). Per-row results depend only on
 * the row's inputs and the fixed k order, as for orthrus_linear_bf16.
 * Replaces the F.linear projections of the generation passes (orthrus/modeling_orthrus.py:469-497
 * through Qwen3Attention / Qwen3MLP). */
int orthrus_linear_skinny_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw,
                               const void* residual, void* y, int64_t ldy, int64_t M, int64_t N,
                               int64_t K, int epilogue, void* stream);

/* The same for the trainable view, whose prologue has a backward: RoPE at positions [B*L] (int64,
 * below table_rows, the rows of rope_cos / rope_sin; a position outside is clamped and reported
 * through ORTHRUS_ERR_BOUNDS) instead of t, and the q / k columns of the token-major projection
 * qkv_out [B*L, (Hq + 2 Hkv) * 128] (bf16, the F.linear output; v columns untouched) and rstd_out
 * [B*L, Hq + Hkv] fp32 are kept for orthrus_qkv_prep_bwd. Replaces F.linear + the prologue of
 * the diffusion layer (orthrus/objective.py:136-143,160-165). */
int orthrus_linear_qkv_rope_keep_bf16(const void* x, const void* w_qkv, const void* q_norm_w,
                                      const void* k_norm_w, const void* rope_cos,
                                      const void* rope_sin, int64_t table_rows,
                                      const int64_t* positions, int64_t B,
                                      int64_t L, int64_t K, int Hq, int Hkv, float eps, void* q_out,
                                      void* k_out, void* v_out, void* qkv_out, float* rstd_out,
                                      void* stream);

/* SwiGLU projection that also keeps the projection for the backward of the activation:
 * y [M, F] = silu(g) * u as ORTHRUS_LINEAR_SWIGLU, and gate_up [M, 2F] = x @ w_gate_up^T rounded
 * to bf16 (the F.linear output). F a multiple of 128, K of 8, contiguous rows. Replaces F.linear +
 * the activation of _mlp_residual in the trainable view (orthrus/objective.py:146-149,160-165). */
int orthrus_linear_swiglu_keep_bf16(const void* x, const void* w_gate_up, int64_t M, int64_t F,
                                    int64_t K, void* y, void* gate_up, void* stream);

/* RoPE table: cos_out / sin_out [positions][half] bf16 = cos / sin(p * inv_freq[i]) by sincosf,
 * rounded to bf16 (the rotary table of the attention prologue, orthrus/objective.py:136-143). */
int orthrus_rope_table_bf16(const float* inv_freq, int64_t positions, int half, void* cos_out,
                            void* sin_out, void* stream);

/* q|k|v projection with the attention prologue in the epilogue, bf16, head dim 128:
 * x [B*L, K] @ w_qkv[(Hq + 2 Hkv) * 128, K]^T, then per q / k head the RMSNorm (q_norm_w /
 * k_norm_w [128], eps) and RoPE at position t (rope_cos / rope_sin [L][64] from
 * orthrus_rope_table_bf16), written head-major: q_out [B, Hq, L, 128], k_out and v_out
 * [B, Hkv, L, 128]. The same arithmetic and roundings as orthrus_gemm_bf16 followed by
 * orthrus_qkv_prep_fwd, without the token-major projection in HBM. L a multiple of 128, K of 8,
 * Hq + 2 Hkv even. Replaces _attention_inputs of the frozen AR pass (orthrus/objective.py:136-143,
 * 152-157). */
int orthrus_linear_qkv_rope_bf16(const void* x, const void* w_qkv, const void* q_norm_w,
                                 const void* k_norm_w, const void* rope_cos, const void* rope_sin,
                                 int64_t B, int64_t L, int64_t K, int Hq, int Hkv, float eps,
                                 void* q_out, void* k_out, void* v_out, void* stream);

/* Same contract for fp32 (or bf16-in, fp32-accumulate) operands on CUDA cores, B as [N, K]:
 * exact fp32 arithmetic with a fixed reduction order that does not depend on M. */
size_t orthrus_gemm_simt_workspace_bytes(int64_t M, int64_t N, int64_t K);
int orthrus_gemm_simt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                      int64_t M, int64_t N, int64_t K, int dtype, void* workspace,
                      size_t workspace_bytes, void* stream);

/* RMSNorm of `rows` rows of length d: y = w * (x * rsqrt(mean(x^2) + eps)), the normalised value
 * rounded to dtype before the weight multiply (transformers Qwen3RMSNorm, orthrus/objective.py:128-133).
 * One warp per row, fixed reduction order. rstd [rows] fp32 receives rsqrt(mean(x^2) + eps) when
 * not NULL (for the backward). */
int orthrus_rmsnorm(const void* x, const void* w, int64_t rows, int d, float eps, void* y,
                    float* rstd, int dtype, void* stream);

/* Backward of orthrus_rmsnorm with respect to x (the norm weights of the model are frozen):
 * dx = rstd * (w dy - xhat * mean(w dy xhat)), xhat = x * rstd, from the rstd [rows] fp32 the
 * forward wrote.
 * Replaces the autograd backward of _rms_norm (orthrus/objective.py:128-133). */
int orthrus_rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy,
                        int64_t rows, int d, void* dx, int dtype, void* stream);
/* The same backward (bf16, d a multiple of 256) plus the gradient dres [rows, d] that reaches x
 * through a residual connection, summed before the single rounding: dx = dres + dnorm. Replaces
 * the sum autograd forms for x used both by the pre-norm and by the residual add of a Qwen3 layer
 * (orthrus/objective.py:146-149,160-165). */
int orthrus_rmsnorm_bwd_add(const void* x, const void* w, const float* rstd, const void* dy,
                            const void* dres, int64_t rows, int d, void* dx, void* stream);

/* SwiGLU activation of the fused [gate | up] projection gate_up [rows, 2 * inter]:
 * out [rows, inter] = silu(gate) * up (silu rounded to dtype first, as F.silu(gate) * up), and its
 * backward dgate_up [rows, 2 * inter] from dout [rows, inter]. inter must be a multiple of 8 (bf16)
 * / 4 (fp32). Replaces the activation of _mlp_residual (orthrus/objective.py:146-149). */
int orthrus_swiglu_fwd(const void* gate_up, int64_t rows, int inter, void* out, int dtype,
                       void* stream);
int orthrus_swiglu_bwd(const void* gate_up, const void* dout, int64_t rows, int inter,
                       void* dgate_up, int dtype, void* stream);

/* ---- q/k RMSNorm + RoPE + head-major layout (fused prologue of the attention) ------------- */
/* qkv: [rows = B*T, (Hq + 2*Hkv) * hd] token-major projection output (q | k | v columns).
 * positions: [B, T] int64 RoPE positions; inv_freq: [hd/2] fp32 RoPE inverse frequencies
 * (1 / theta^(2i/hd), computed by the caller exactly as the rotary embedding does). Writes
 *   q_out [B, Hq, T, D]            (norm + RoPE), D = padded head dim (>= hd, zero padding)
 *   k_out [B, Hkv, cap, D] at row offset[b] + t (norm + RoPE), v_out likewise (copy);
 *   rstd [rows, Hq + Hkv] fp32 (saved for the backward; may be NULL).
 * offset may be NULL (0). cap >= offset[b] + T. dtype applies to qkv and all outputs.
 * Replaces _attention_inputs (orthrus/objective.py:136-143) and the q/k norm + apply_rotary_pos_emb
 * of OrthrusAttention.forward (orthrus/modeling_orthrus.py:153-159) plus DynamicCache.update. */
int orthrus_qkv_prep_fwd(const void* qkv, const int64_t* positions, const float* inv_freq,
                         const void* q_norm_w, const void* k_norm_w, int64_t B, int64_t T, int Hq,
                         int Hkv, int hd, int D, float eps, void* q_out, void* k_out, void* v_out,
                         int64_t cap, const int32_t* offset, float* rstd, int dtype, void* stream);

/* Backward of orthrus_qkv_prep_fwd for training (offset 0, cap = T):
 *   dq [B, Hq, T, D] fp32, dk [B, Hkv, T, D] fp32, dv [B, Hkv, T, D] fp32 (any may be NULL = 0)
 *   -> dqkv [rows, (Hq + 2 Hkv) hd] (dtype), dq_norm_w / dk_norm_w [hd] fp32 (overwritten).
 * workspace: orthrus_qkv_prep_bwd_workspace_bytes(). */
size_t orthrus_qkv_prep_bwd_workspace_bytes(int64_t B, int64_t T, int hd);
int orthrus_qkv_prep_bwd(const void* qkv, const int64_t* positions, const float* inv_freq,
                         const void* q_norm_w, const void* k_norm_w, const float* rstd,
                         const float* dq, const float* dk, const float* dv, int64_t B, int64_t T,
                         int Hq, int Hkv, int hd, int D, void* dqkv, float* dq_norm_w,
                         float* dk_norm_w, void* workspace, size_t workspace_bytes, int dtype,
                         void* stream);

/* ---- failure detection ------------------------------------------------------------------- */
/* Self-test of the bounded-wait protocol of the tcgen05 / TMA kernels (no reference counterpart:
 * the reference has no device code). One CTA issues a TMA load of the 64 x 64 bf16 tile at
 * tile64x64 (16-byte aligned, row pitch 64), then waits limit_ns (at most 0.1 s) on an mbarrier
 * that nothing arrives on; the wait runs out and sets ORTHRUS_ERR_TIMEOUT in the device error word,
 * the kernel drains its copy, frees its TMEM and returns. *status (device, zeroed by the caller)
 * receives bit 1 = timed out, 2 = copy drained, 4 = TMEM freed. The context stays usable. */
int orthrus_selftest_bounded_wait(const void* tile64x64, uint64_t limit_ns, unsigned int* status,
                                  void* stream);

/* ---- dual-view attention --------------------------------------------------------------- */
/* Per-anchor tile map of the dual-view mask (K3): for every 128-query tile of each row,
 * tilemap[b, tile] = {source-1 key tiles to visit, source-1 keys visible to the tile (largest
 * anchor, clipped to L1), first and one-past-last source-2 key}.
 * anchors [B, A] int64 sorted per row, block = K. Output int32 [B, ceil(A*K/128), 4].
 * Replaces build_block_mask / create_block_mask (orthrus/modeling_orthrus.py:58-74) and
 * skip_ar_key_grads (orthrus/objective.py:168-198): the backward never visits source-1 keys
 * for dK/dV. */
int orthrus_attn_tilemap(const int64_t* anchors, int64_t B, int64_t A, int block, int64_t L1,
                         int32_t* tilemap, void* stream);

/* Forward. q [B, Hq, Tq, D]; source 1: k1/v1 with row pitch D, head stride s1h, batch stride s1b
 * (elements), L1 rows; source 2: k2/v2 (stride s2h, s2b, L2 rows; NULL when unused).
 * o: token-major [B, Tq, Hq, hd] (the o_proj input), lse [B, Hq, Tq] fp32 (may be NULL).
 * mask: ORTHRUS_MASK_* with anchors [B, A] int64 (DUAL), offset [B] int32 (CAUSAL/DRAFT) and
 * limit2 [B] int32 (DRAFT, may be NULL). scale = 1/sqrt(hd).
 * bf16 runs the tcgen05 tile kernel (D = 128 or 64); fp32 runs the exact CUDA-core kernel.
 * Replaces F.scaled_dot_product_attention (orthrus/objective.py:155), flex_attention with the
 * dual-pass BlockMask (orthrus/objective.py:163; orthrus/modeling_orthrus.py:77-85) and the
 * generation-time attention of OrthrusAttention (orthrus/modeling_orthrus.py:167-188). */
int orthrus_attn_fwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                     int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                     int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, int hd, int D, float scale,
                     int mask, const int64_t* anchors, int64_t A, int block, const int32_t* offset,
                     const int32_t* limit2, void* o, float* lse, int dtype, void* stream);

/* The attention of the decode passes, bf16 with hd = D = 128: a block of Tq <= 64 query rows per
 * sequence ((Hq / Hkv) * Tq <= 128) over its KV cache, with the CAUSAL mask (verification and
 * one-token greedy passes: row t of sequence b sees cache rows [0, offset[b] + t]) or the DRAFT
 * mask (the cache rows [0, offset[b]) plus the block's own keys k2 / v2 [0, limit2[b]), L2 <= 64).
 * Same arguments and output as orthrus_attn_fwd (no lse). The keys are split into 128-key ranges
 * from key 0, one CTA per (range, KV head, sequence), merged per row in range order: a row's
 * result depends on its visible keys only, so a Tq-row pass equals Tq one-row passes bit for bit.
 * workspace: orthrus_attn_decode_workspace_bytes(B, Hq, Tq, L1) (per-range partial states).
 * Replaces the generation-time attention of OrthrusAttention (orthrus/modeling_orthrus.py:167-188)
 * in diffusion_generate's draft and verify passes (:469-497). */
size_t orthrus_attn_decode_workspace_bytes(int64_t B, int Hq, int64_t Tq, int64_t L1);
int orthrus_attn_decode_fwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                            int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                            int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, float scale, int mask,
                            const int32_t* offset, const int32_t* limit2, void* o, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Backward of the DUAL mask (training): from do_ [B, Tq, Hq, hd] (token-major), o, lse, q and the
 * two sources, writes dq [B, Hq, Tq, D] fp32 and dk2 / dv2 [B, Hkv, L2, D] fp32 (source-2 keys
 * only: source-1 keys are the frozen teacher's and get no gradient).
 * workspace: orthrus_attn_bwd_workspace_bytes().
 * bf16 with an even GQA group runs dK/dV on a library-owned side stream of the device, forked
 * from and joined back into `stream` inside the call; the fork/join events are shared per device
 * and guarded by a mutex, so host threads may call this concurrently with their own workspaces. */
size_t orthrus_attn_bwd_workspace_bytes(int64_t B, int Hq, int64_t Tq);
int orthrus_attn_bwd(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                     int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                     int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, int hd, int D, float scale,
                     const int64_t* anchors, int64_t A, int block, const void* o, const float* lse,
                     const void* do_, float* dq, float* dk2, float* dv2, void* workspace,
                     size_t workspace_bytes, int dtype, void* stream);

/* Opt-in document mask for packed rows of several documents (the reference runs without one:
 * SDPA is_causal over the whole row, orthrus/objective.py:155, and the block mask's AR prefix
 * kv < anchor, orthrus/modeling_orthrus.py:58-74). doc_start is int32 [B, L1]: the first position
 * of each position's document. With it a causal query t sees source-1 keys [doc_start[t], t] and
 * a dual-view query of the block anchored at a sees [doc_start[a], a) plus its own block; the
 * other masks are unchanged. Otherwise as orthrus_attn_fwd / orthrus_attn_bwd. */
int orthrus_attn_fwd_doc(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                         int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                         int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, int hd, int D,
                         float scale, int mask, const int64_t* anchors, int64_t A, int block,
                         const int32_t* offset, const int32_t* limit2, const int32_t* doc_start,
                         void* o, float* lse, int dtype, void* stream);
int orthrus_attn_bwd_doc(const void* q, const void* k1, const void* v1, int64_t s1h, int64_t s1b,
                         int64_t L1, const void* k2, const void* v2, int64_t s2h, int64_t s2b,
                         int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq, int hd, int D,
                         float scale, const int64_t* anchors, int64_t A, int block,
                         const int32_t* doc_start, const void* o, const float* lse, const void* do_,
                         float* dq, float* dk2, float* dv2, void* workspace, size_t workspace_bytes,
                         int dtype, void* stream);

/* The same backward for callers that must not allocate device memory at all: no workspace
 * argument, and no cudaMalloc, cudaFree or allocating library call inside. It exists for hosts
 * that cannot hand this library a workspace: a runtime that owns every device byte in its own pool
 * (an embedding service behind cgo / JNI), or a hot loop where cudaMalloc's implicit device
 * synchronisation is not acceptable. This entry point has no counterpart in the reference.
 * Its scratch (one fp32 per query row per head) is a fixed array compiled into the library, held
 * by every GPU that loads it until the process exits, so B * Hq * Tq must not exceed
 * ORTHRUS_ATTN_BWD_NOALLOC_MAX_ROWS (262144 rows = 1 MiB); larger sizes return ORTHRUS_EINVAL.
 * The first call on a device looks up the array's device address with that device current; make
 * that first call before any stream capture. Every call reuses the same array and fully rewrites
 * the part it reads, so nothing needs clearing, but calls that overlap on the GPU (two streams,
 * two threads) race on it. Like orthrus_attn_bwd, a bf16 call with an even GQA group runs its
 * dK/dV kernel on the library's per-device side stream, which every backward on that device
 * shares: "overlapping calls" includes any other backward whose dK/dV is still in flight there.
 * Arguments and outputs as orthrus_attn_bwd. */
#define ORTHRUS_ATTN_BWD_NOALLOC_MAX_ROWS 262144
int orthrus_attn_bwd_noalloc(const void* q, const void* k1, const void* v1, int64_t s1h,
                             int64_t s1b, int64_t L1, const void* k2, const void* v2, int64_t s2h,
                             int64_t s2b, int64_t L2, int64_t B, int Hq, int Hkv, int64_t Tq,
                             int hd, int D, float scale, const int64_t* anchors, int64_t A,
                             int block, const void* o, const float* lse, const void* do_,
                             float* dq, float* dk2, float* dv2, int dtype, void* stream);

/* ---- fused LM head + log-softmax + KL(teacher || student) ------------------------------- */
/* total = sum_r w_r KL(softmax(W t[index[r]]) || softmax(W s[r])), kl_rows[r], agree[r] (top-1
 * match, lowest index wins ties), and, when grad != NULL, grad[r] = w_r (p_s - p_t)[r] @ W
 * (the d(total)/d(student) that the reference saves for backward).
 * student [n, d], teacher [m, d] (unique target rows), index [n] non-decreasing in [0, m),
 * weight [V, d], row_weight [n] fp32 or NULL (w = 1), offsets [n] int64 (block offset of each row)
 * or NULL; per-offset outputs kl_by_offset [num_offsets] fp32 and agree_by_offset
 * [num_offsets] int64 when offsets != NULL. Logits are never written to memory; the bf16
 * probability difference of chunk_rows rows at a time lives in the workspace.
 * Replaces FusedLinearForwardKL (orthrus/objective.py:338-392) with _logits / kl_chunk
 * (:303-332) and the stats of orthrus_loss (:440-452). */
size_t orthrus_lmhead_kl_workspace_bytes(int64_t n, int64_t m, int64_t V, int64_t d,
                                         int64_t chunk_rows, int dtype);
int orthrus_lmhead_kl_fwd(const void* student, int64_t n, const void* teacher, int64_t m,
                          const int64_t* index, const void* weight, int64_t V, int64_t d,
                          const float* row_weight, const int64_t* offsets, int num_offsets,
                          float* total, float* kl_rows, uint8_t* agree, void* grad,
                          float* kl_by_offset, int64_t* agree_by_offset, int64_t chunk_rows,
                          void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* grad_student[i] = grad[i] * grad_total[0], count elements (FusedLinearForwardKL.backward,
 * orthrus/objective.py:389-392). */
int orthrus_lmhead_kl_bwd(const void* grad, const float* grad_total, void* grad_student,
                          int64_t count, int dtype, void* stream);

/* ---- parallel block decoding ----------------------------------------------------------- */
/* Row-wise argmax of fp32 logits [R, V] (lowest index on ties, as torch.argmax), R rows at
 * row pitch ldl: out[r] int64. */
int orthrus_argmax_rows(const float* logits, int64_t ldl, int64_t R, int64_t V, int64_t* out,
                        void* stream);

/* Draft step (K7) for B sequences: logits [B, K, V] fp32 of the diffusion pass over
 * [anchor, mask x K-1]; writes verify_ids [B, K] = [anchor, argmax of positions 0..K-2].
 * Sequences with done[b] != 0 are left untouched.
 * Replaces the draft half of OrthrusLM.diffusion_generate (orthrus/modeling_orthrus.py:469-487)
 * and ModelBackend.draft (orthrus/decoding.py:178-206). */
int orthrus_decode_draft(const float* logits, int64_t B, int K, int64_t V, const int64_t* anchor,
                         const uint8_t* done, int64_t* verify_ids, void* stream);

/* Verify + greedy accept + rollback (K8) for B sequences, entirely on device:
 *   ar_tokens [B, K] = argmax(verify logits [B, K, V]) (written, int64);
 *   accepted = longest prefix with drafts == ar_tokens, limited to
 *   block_len - 1 = min(K, max_len[b] - start[b]) - 1 and ending after an accepted EOS;
 *   appends the kept tokens and the bonus token to out_tokens [B, out_cap] at out_len[b];
 *   start[b] += accepted + 1 (the KV-cache length rollback: positions past it are dead);
 *   anchor[b] = bonus; accepted_log[b, cycle[b]] = accepted; done[b] on EOS or max length.
 * eos: int64 [n_eos] (n_eos may be 0).
 * Replaces the verify / accept / truncate_cache half of OrthrusLM.diffusion_generate
 * (orthrus/modeling_orthrus.py:489-533), decoding._verify / _advance / ModelBackend.commit
 * (orthrus/decoding.py:248-264,336-369). */
int orthrus_decode_verify_accept(const float* logits, int64_t B, int K, int64_t V,
                                 const int64_t* verify_ids, int64_t* ar_tokens,
                                 const int64_t* eos, int n_eos,
                                 const int32_t* max_len, int32_t* start, int64_t* anchor,
                                 uint8_t* done, int64_t* out_tokens, int32_t* out_len,
                                 int64_t out_cap, int32_t* accepted_log, int32_t* cycle,
                                 int64_t log_cap, void* stream);

/* The LM head's argmax without logits, for greedy decoding: out int64 [R] = argmax over the V
 * columns of h [R, d] @ weight [V, d]^T (bf16, fp32 accumulation, d % 64 == 0), the lowest index
 * on ties (torch.argmax). The logits tiles are computed as orthrus_gemm_bf16 computes them and
 * reduced on chip; nothing of size [R, V] is written. workspace:
 * orthrus_lmhead_argmax_workspace_bytes(R). Replaces lm_head + argmax of diffusion_generate's
 * greedy pick (orthrus/modeling_orthrus.py:437-439). */
size_t orthrus_lmhead_argmax_workspace_bytes(int64_t R);
int orthrus_lmhead_argmax_bf16(const void* h, int64_t R, const void* weight, int64_t V, int64_t d,
                               int64_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* orthrus_decode_draft and orthrus_decode_verify_accept with the rows' argmax ids [B * K] (from
 * orthrus_lmhead_argmax_bf16) in place of their logits. */
int orthrus_decode_draft_ids(const int64_t* ids, int64_t B, int K, const int64_t* anchor,
                             const uint8_t* done, int64_t* verify_ids, void* stream);
int orthrus_decode_accept_ids(const int64_t* ar_tokens, int64_t B, int K, const int64_t* verify_ids,
                              const int64_t* eos, int n_eos, const int32_t* max_len, int32_t* start,
                              int64_t* anchor, uint8_t* done, int64_t* out_tokens, int32_t* out_len,
                              int64_t out_cap, int32_t* accepted_log, int32_t* cycle, int64_t log_cap,
                              void* stream);

/* ---- sampled decoding (temperature > 0) ----
 * A row's sampling distribution lives on its C top candidates: cand_vals fp32 [R, C] sorted
 * descending and cand_ids int64 [R, C] (the logits' top C, e.g. torch.topk), with
 * 1 <= top_k <= C <= 128 and C - top_k spare candidates to keep ties at the top_k-th value.
 * The filter is the reference's `pick` (orthrus/modeling_orthrus.py:437-449): divide by the
 * temperature, drop values below the top_k-th, keep the smallest descending prefix whose mass
 * exceeds top_p (the first always), softmax. Random draws are Philox4x32-10 keyed by `seed` and
 * counted by (sequence, cycle[b], position, purpose), so a decode is reproducible from its seed
 * and a cycle replays as a CUDA graph. */

/* probs fp32 [R, C]: the filtered distribution of each candidate row (0 for dropped ones). */
int orthrus_sample_probs(const float* cand_vals, int64_t R, int C, float temperature, int top_k,
                         float top_p, float* probs, void* stream);

/* tokens int64 [R]: one draw per row from its filtered distribution, counter (r, cycle[r] or 0 if
 * cycle is null, 0, first): the prefill's first token (modeling_orthrus.py:460-462). */
int orthrus_sample_rows(const float* cand_vals, const int64_t* cand_ids, int64_t R, int C,
                        float temperature, int top_k, float top_p, uint64_t seed,
                        const int32_t* cycle, int64_t* tokens, void* stream);

/* Draft step of a sampled cycle (modeling_orthrus.py:472-483 with pick): candidate rows
 * [B, K-1, C] of the diffusion pass; verify_ids[b] = [anchor[b], d_0 .. d_{K-2}] with d_i drawn
 * from q_i, kept in draft_probs fp32 [B, K-1, C]. Sequences with done[b] are left alone.
 * 2 <= K <= 64. */
int orthrus_decode_sample_draft(const float* cand_vals, const int64_t* cand_ids, int64_t B, int K,
                                int C, float temperature, int top_k, float top_p, uint64_t seed,
                                const int32_t* cycle, const int64_t* anchor, const uint8_t* done,
                                int64_t* verify_ids, float* draft_probs, void* stream);

/* Verify / accept step of a sampled cycle: exact rejection sampling
 * (modeling_orthrus.py:498-511). cand_vals / cand_ids [B, K, C] are the verify pass's rows,
 * draft_probs / draft_ids [B, K-1, C] the draft step's. Draft i is kept while
 * u_i < min(1, p_i(d_i) / max(q_i(d_i), 1e-8)) (and stops after an accepted EOS); the bonus token
 * comes from the normalised max(p - q, 0) at the first rejection (p if its mass is <= 1e-5), or
 * from p after a full accept. The commit is orthrus_decode_verify_accept's. */
int orthrus_decode_sample_accept(const float* cand_vals, const int64_t* cand_ids,
                                 const float* draft_probs, const int64_t* draft_ids, int64_t B,
                                 int K, int C, float temperature, int top_k, float top_p,
                                 uint64_t seed, const int64_t* verify_ids, const int64_t* eos,
                                 int n_eos, const int32_t* max_len, int32_t* start,
                                 int64_t* anchor, uint8_t* done, int64_t* out_tokens,
                                 int32_t* out_len, int64_t out_cap, int32_t* accepted_log,
                                 int32_t* cycle, int64_t log_cap, void* stream);

/* out uint32 [n, 4] = Philox4x32-10(counter_key[r, 0:4], key counter_key[r, 4:6]): the known-answer
 * check of the decode's generator. */
int orthrus_philox4x32_10(const uint32_t* counter_key, int64_t n, uint32_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ORTHRUS_B200_H */
