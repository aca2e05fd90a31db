"""Thin torch-facing wrappers over the C ABI: allocate outputs and workspaces with torch, pass raw
pointers and the current stream, check the status. No computation happens in Python."""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass

import torch

from orthrus_training_b200 import _lib as L


class KernelTimer:
    """CUDA-event timing of individual entry points on the stream they launch on, with the
    algorithmic work (FLOPs) of each launch. Enabled by assigning an instance to ``ops.TIMER``."""

    def __init__(self):
        self.records = defaultdict(list)

    def begin(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def end(self, name, e0, work):
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.records[name].append((e0, e1, work))

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for name, recs in self.records.items():
            ms = sum(a.elapsed_time(b) for a, b, _ in recs)
            work = sum(float(w) for _, _, w in recs)
            out[name] = {"launches": len(recs), "ms": ms, "flops": work}
        return out


TIMER: KernelTimer | None = None


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("orthrus_training_b200 ops run on CUDA tensors only (no CPU fallback)")


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def gemm(a: torch.Tensor, b: torch.Tensor, *, b_kn: bool = False, out_dtype=None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """a [M, K] @ (b [N, K])^T (or a @ b for b [K, N] with b_kn). bf16 inputs run on tcgen05 tensor
    cores, fp32 inputs on the exact CUDA-core kernel; fp32 accumulation either way."""
    _require_cuda(a, b)
    if a.dim() != 2 or b.dim() != 2 or a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("gemm takes row-major 2-D operands")
    M, K = a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    if (b.shape[0] if b_kn else b.shape[1]) != K:
        raise ValueError(f"gemm shape mismatch {tuple(a.shape)} x {tuple(b.shape)}")
    lib = L.lib()
    stream = L.stream_of(a.device)
    if a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        out_dtype = out_dtype or torch.bfloat16
        c = out if out is not None else torch.empty(M, N, dtype=out_dtype, device=a.device)
        ws = _workspace(lib.orthrus_gemm_workspace_bytes(M, N, K), a.device)
        L.check(lib.orthrus_gemm_bf16(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                      c.data_ptr(), c.stride(0), M, N, K, int(b_kn),
                                      int(c.dtype == torch.float32), L.ptr(ws),
                                      0 if ws is None else ws.numel(), stream), "gemm_bf16")
        return c
    if b_kn:
        raise ValueError("the CUDA-core gemm takes b as [N, K]")
    code = L.dtype_code(a.dtype)
    c = out if out is not None else torch.empty(M, N, dtype=a.dtype, device=a.device)
    ws = _workspace(lib.orthrus_gemm_simt_workspace_bytes(M, N, K), a.device)
    L.check(lib.orthrus_gemm_simt(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                  c.data_ptr(), c.stride(0), M, N, K, code, L.ptr(ws),
                                  0 if ws is None else ws.numel(), stream), "gemm_simt")
    return c


def gemm2(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = False,
          residual: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 GEMM on CTA pairs (orthrus_gemm2_bf16): C = A @ B^T (+ residual), where A is `a`
    [M, K], or `a`^T when a_t (a stored as [K, M]), and B is `b` [N, K], or `b`^T when b_t (b
    stored as [K, N]). So y = x W^T is gemm2(x, W), dX = dY W is gemm2(dY, W, b_t=True) and
    dW = dY^T X is gemm2(dY, X, a_t=True, b_t=True)."""
    _require_cuda(a, b, residual)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.dim() != 2 or b.dim() != 2:
        raise ValueError("gemm2 takes 2-D bf16 operands")
    a, b = a.contiguous(), b.contiguous()
    M, K = (a.shape[1], a.shape[0]) if a_t else a.shape
    N, Kb = (b.shape[1], b.shape[0]) if b_t else b.shape
    if Kb != K:
        raise ValueError(f"gemm2 shape mismatch: A {tuple(a.shape)} (t={a_t}), B {tuple(b.shape)} (t={b_t})")
    c = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    epi = 0
    if residual is not None:
        residual = residual.contiguous()
        if residual.shape != (M, N) or residual.dtype != torch.bfloat16:
            raise ValueError("residual must be bf16 [M, N]")
        epi = 1
    lib = L.lib()
    ws = _workspace(lib.orthrus_gemm2_workspace_bytes(M, N, K), a.device)
    L.check(lib.orthrus_gemm2_bf16(a.data_ptr(), a.stride(0), int(a_t), b.data_ptr(), b.stride(0), int(b_t),
                                   c.data_ptr(), N, L.ptr(residual), N if residual is not None else 0,
                                   M, N, K, epi, L.ptr(ws), 0 if ws is None else ws.numel(),
                                   L.stream_of(a.device)), "gemm2_bf16")
    return c


def gemm2_swiglu_backward(dy: torch.Tensor, w_down: torch.Tensor, gate_up: torch.Tensor) -> torch.Tensor:
    """[dgate | dup] [M, 2F] of the MLP from the gradient dy [M, d] of its output: the CTA-pair
    GEMM dact = dy @ w_down (w_down [d, F]) with the SwiGLU backward of gate_up [M, 2F] in its
    epilogue (silu_mul_backward(gate_up, dy @ w_down) without writing dact)."""
    _require_cuda(dy, w_down, gate_up)
    dy, w_down, gate_up = dy.contiguous(), w_down.contiguous(), gate_up.contiguous()
    M, d = dy.shape
    F = w_down.shape[1]
    if w_down.shape[0] != d or gate_up.shape != (M, 2 * F) or F % 64 or dy.dtype != torch.bfloat16:
        raise ValueError("gemm2_swiglu_backward takes bf16 dy [M, d], w_down [d, F], gate_up [M, 2F]")
    dgu = torch.empty(M, 2 * F, dtype=torch.bfloat16, device=dy.device)
    L.check(L.lib().orthrus_gemm2_bf16(dy.data_ptr(), d, 0, w_down.data_ptr(), F, 1, dgu.data_ptr(), 2 * F,
                                       gate_up.data_ptr(), 2 * F, M, F, d, 2, None, 0, L.stream_of(dy.device)),
            "gemm2_swiglu_bwd")
    return dgu


LINEAR_STORE, LINEAR_RESIDUAL, LINEAR_SWIGLU = 0, 1, 2


def fused_linear_supported(x: torch.Tensor, w: torch.Tensor, n_out: int) -> bool:
    """Shapes and dtypes orthrus_linear_bf16 takes (bf16, N a multiple of 128, K of 8)."""
    return (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and n_out % 128 == 0 and x.shape[1] % 8 == 0)


LINEAR_PAIR = 0x100  # epilogue flag of orthrus_linear_bf16: run on CTA pairs


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
           skinny: bool = False, pair: bool = False) -> torch.Tensor:
    """x [M, K] @ w [N, K]^T, plus residual [M, N] in the epilogue when given (torch.addmm with
    beta = 1), on the persistent tcgen05 projection kernel, or with skinny on the inference
    passes' kernel (128-row tiles of 16-64 columns, many CTAs for a few rows; K a multiple of 64;
    a row's result independent of the row count)."""
    _require_cuda(x, w, residual)
    x = x.contiguous()
    w = w.contiguous()
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K or not fused_linear_supported(x, w, N):
        raise ValueError(f"linear takes bf16 x [M, K] and w [N, K] with N % 128 == 0, K % 8 == 0; "
                         f"got {tuple(x.shape)} {x.dtype} x {tuple(w.shape)} {w.dtype}")
    y = torch.empty(M, N, dtype=x.dtype, device=x.device)
    epi = LINEAR_STORE
    if residual is not None:
        residual = residual.contiguous()
        if residual.shape != (M, N) or residual.dtype != x.dtype:
            raise ValueError("residual must be [M, N] in the dtype of x")
        epi = LINEAR_RESIDUAL
    fn = L.lib().orthrus_linear_skinny_bf16 if skinny else L.lib().orthrus_linear_bf16
    L.check(fn(x.data_ptr(), K, w.data_ptr(), K, L.ptr(residual), y.data_ptr(), N, M, N, K,
               epi | (LINEAR_PAIR if pair and not skinny else 0), L.stream_of(x.device)), "linear_bf16")
    return y


def linear_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, keep_gate_up: bool = False,
                  skinny: bool = False, pair: bool = False):
    """silu(x @ gate^T) * (x @ up^T) for w_gate_up = [gate; up] [2F, K], without writing the
    [gate | up] projection (same roundings as silu_mul(x @ w_gate_up^T)). With keep_gate_up the
    projection [M, 2F] is written as well and (y, gate_up) is returned."""
    _require_cuda(x, w_gate_up)
    x = x.contiguous()
    w_gate_up = w_gate_up.contiguous()
    M, K = x.shape
    F = w_gate_up.shape[0] // 2
    if w_gate_up.shape != (2 * F, K) or not fused_linear_supported(x, w_gate_up, F):
        raise ValueError(f"linear_swiglu takes bf16 x [M, K] and w [2F, K] with F % 128 == 0; got "
                         f"{tuple(x.shape)} x {tuple(w_gate_up.shape)}")
    y = torch.empty(M, F, dtype=x.dtype, device=x.device)
    if keep_gate_up:
        gu = torch.empty(M, 2 * F, dtype=x.dtype, device=x.device)
        L.check(L.lib().orthrus_linear_swiglu_keep_bf16(x.data_ptr(), w_gate_up.data_ptr(), M, F, K,
                                                        y.data_ptr(), gu.data_ptr(), L.stream_of(x.device)),
                "linear_swiglu_keep")
        return y, gu
    fn = L.lib().orthrus_linear_skinny_bf16 if skinny else L.lib().orthrus_linear_bf16
    L.check(fn(x.data_ptr(), K, w_gate_up.data_ptr(), K, None, y.data_ptr(), F, M, F, K,
               LINEAR_SWIGLU | (LINEAR_PAIR if pair and not skinny else 0), L.stream_of(x.device)),
            "linear_swiglu")
    return y


def rope_table(inv_freq: torch.Tensor, positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 (cos, sin) [positions, hd/2] of p * inv_freq[i] (sincosf, rounded to bf16)."""
    _require_cuda(inv_freq)
    inv_freq = inv_freq.float().contiguous()
    half = inv_freq.numel()
    cos = torch.empty(positions, half, dtype=torch.bfloat16, device=inv_freq.device)
    sin = torch.empty_like(cos)
    L.check(L.lib().orthrus_rope_table_bf16(inv_freq.data_ptr(), positions, half, cos.data_ptr(),
                                            sin.data_ptr(), L.stream_of(inv_freq.device)), "rope_table")
    return cos, sin


def fused_qkv_rope_supported(x: torch.Tensor, hd: int, D: int, L_: int, Hq: int, Hkv: int) -> bool:
    """Shapes the q|k|v projection with the prologue epilogue takes."""
    return (x.dtype == torch.bfloat16 and hd == 128 and D == 128 and L_ % 128 == 0
            and x.shape[1] % 8 == 0 and (Hq + 2 * Hkv) % 2 == 0)


def linear_qkv_rope(x, w_qkv, q_norm_w, k_norm_w, rope, B: int, L_: int, Hq: int, Hkv: int, eps: float,
                    positions: torch.Tensor | None = None, keep: bool = False):
    """q|k|v projection with q/k RMSNorm + RoPE in the GEMM epilogue (positions 0..L-1 per
    sequence, or the int64 [B, L] positions given). Returns head-major q [B, Hq, L, 128], k, v
    [B, Hkv, L, 128] (same values as qkv_prep(x @ w_qkv^T, ...) up to the GEMM's accumulation
    order); with keep also the token-major projection [B*L, (Hq + 2 Hkv) * 128] (q / k columns
    written, for the prologue's backward) and rstd [B*L, Hq + Hkv]."""
    _require_cuda(x, w_qkv, q_norm_w, k_norm_w, positions)
    x, w_qkv = x.contiguous(), w_qkv.contiguous()
    cos, sin = rope
    if positions is None and cos.shape[0] < L_:
        # rows take positions 0..L-1; with explicit positions (the trainable view's block rows,
        # whose count A*K may exceed the sequence) the kernel bounds-checks each position instead
        raise ValueError("the RoPE table is shorter than the sequence")
    dev, dt = x.device, x.dtype
    q = torch.empty(B, Hq, L_, 128, dtype=dt, device=dev)
    k = torch.empty(B, Hkv, L_, 128, dtype=dt, device=dev)
    v = torch.empty(B, Hkv, L_, 128, dtype=dt, device=dev)
    if keep:
        if positions is None:
            raise ValueError("keep needs the positions of the rows")
        positions = positions.to(torch.int64).contiguous()
        if positions.numel() != B * L_:
            raise ValueError("positions must hold one int64 per row")
        qkv = torch.empty(B * L_, w_qkv.shape[0], dtype=dt, device=dev)
        rstd = torch.empty(B * L_, Hq + Hkv, dtype=torch.float32, device=dev)
        L.check(L.lib().orthrus_linear_qkv_rope_keep_bf16(
            x.data_ptr(), w_qkv.data_ptr(), q_norm_w.contiguous().data_ptr(), k_norm_w.contiguous().data_ptr(),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], positions.data_ptr(), B, L_, x.shape[1], Hq, Hkv,
            float(eps),
            q.data_ptr(), k.data_ptr(), v.data_ptr(), qkv.data_ptr(), rstd.data_ptr(), L.stream_of(dev)),
            "linear_qkv_rope_keep")
        return q, k, v, qkv, rstd
    if positions is not None:
        raise ValueError("positions other than 0..L-1 are taken with keep=True only")
    L.check(L.lib().orthrus_linear_qkv_rope_bf16(
        x.data_ptr(), w_qkv.data_ptr(), q_norm_w.contiguous().data_ptr(), k_norm_w.contiguous().data_ptr(),
        cos.data_ptr(), sin.data_ptr(), B, L_, x.shape[1], Hq, Hkv, float(eps), q.data_ptr(), k.data_ptr(),
        v.data_ptr(), L.stream_of(dev)), "linear_qkv_rope")
    return q, k, v


def lmhead_kl(student, teacher, index, weight, row_weight=None, offsets=None, num_offsets=0,
              need_grad=True, chunk_rows=4096):
    """Fused LM head + log-softmax + KL(teacher || student) (FusedLinearForwardKL.forward math).
    Returns (total fp32 [], kl_rows fp32 [n], agree bool [n], grad [n, d] or None,
    kl_by_offset fp32 [num_offsets] or None, agree_by_offset int64 [num_offsets] or None)."""
    _require_cuda(student, teacher, index, weight, row_weight, offsets)
    dt = student.dtype
    code = L.dtype_code(dt)
    if teacher.dtype != dt or weight.dtype != dt:
        raise ValueError("student, teacher and weight must share a dtype")
    student, teacher, weight = student.contiguous(), teacher.contiguous(), weight.contiguous()
    index = index.to(torch.int64).contiguous()
    n, d = student.shape
    m = teacher.shape[0]
    V = weight.shape[0]
    dev = student.device
    pad = (-d) % 64 if dt == torch.bfloat16 else 0
    if pad:  # the tensor-core path consumes the hidden dimension in 64-wide k-blocks
        student = torch.nn.functional.pad(student, (0, pad))
        teacher = torch.nn.functional.pad(teacher, (0, pad))
        weight = torch.nn.functional.pad(weight, (0, pad))
    dp = d + pad
    lib = L.lib()
    total = torch.empty((), dtype=torch.float32, device=dev)
    kl_rows = torch.empty(n, dtype=torch.float32, device=dev)
    agree = torch.empty(n, dtype=torch.uint8, device=dev)
    grad = torch.empty(n, dp, dtype=dt, device=dev) if need_grad else None
    kbo = abo = None
    if offsets is not None:
        offsets = offsets.to(torch.int64).contiguous()
        kbo = torch.empty(num_offsets, dtype=torch.float32, device=dev)
        abo = torch.empty(num_offsets, dtype=torch.int64, device=dev)
    if row_weight is not None:
        row_weight = row_weight.to(torch.float32).contiguous()
    nbytes = lib.orthrus_lmhead_kl_workspace_bytes(n, m, V, dp, chunk_rows, code)
    ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
    t0 = TIMER.begin() if TIMER is not None else None
    L.check(lib.orthrus_lmhead_kl_fwd(
        L.ptr(student), n, L.ptr(teacher), m, L.ptr(index), L.ptr(weight), V, dp, L.ptr(row_weight),
        L.ptr(offsets), int(num_offsets), L.ptr(total), L.ptr(kl_rows), L.ptr(agree), L.ptr(grad),
        L.ptr(kbo), L.ptr(abo), chunk_rows, L.ptr(ws), ws.numel(), code, L.stream_of(dev)),
        "lmhead_kl_fwd")
    if t0 is not None:  # student logits + unique teacher logits + grad GEMM
        TIMER.end("lmhead_kl", t0, 2.0 * d * V * ((2 if need_grad else 1) * n + m))
    if grad is not None and pad:
        grad = grad[:, :d]
    return total, kl_rows, agree.bool(), grad, kbo, abo


def lmhead_kl_backward(grad: torch.Tensor, grad_total: torch.Tensor) -> torch.Tensor:
    """grad * grad_total, as FusedLinearForwardKL.backward."""
    _require_cuda(grad, grad_total)
    grad = grad.contiguous()
    out = torch.empty_like(grad)
    gt = grad_total.to(torch.float32).reshape(1).contiguous()
    L.check(L.lib().orthrus_lmhead_kl_bwd(grad.data_ptr(), gt.data_ptr(), out.data_ptr(),
                                          grad.numel(), L.dtype_code(grad.dtype),
                                          L.stream_of(grad.device)), "lmhead_kl_bwd")
    return out


# --- q/k norm + RoPE ---------------------------------------------------------------------------


def rope_inv_freq(head_dim: int, theta: float, device) -> torch.Tensor:
    """1 / theta^(2i/hd) in fp32, computed with the same torch ops as the rotary embedding of the
    reference model (transformers Qwen3RotaryEmbedding, default rope)."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim
    return (1.0 / (theta ** exponent)).to(device)


def qkv_prep(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, q_norm_w, k_norm_w,
             B: int, T: int, Hq: int, Hkv: int, hd: int, D: int, eps: float, *, k_cache=None,
             v_cache=None, offset=None, want_rstd=False):
    """q/k RMSNorm + RoPE of the fused projection output qkv [B*T, (Hq+2Hkv)*hd].
    Returns (q [B, Hq, T, D], k, v, rstd); k / v are [B, Hkv, T, D] unless caches
    [B, Hkv, cap, D] are given, in which case rows offset[b] + t of the caches are written."""
    _require_cuda(qkv, positions)
    dt = qkv.dtype
    dev = qkv.device
    qkv = qkv.contiguous()
    q = torch.empty(B, Hq, T, D, dtype=dt, device=dev)
    if k_cache is None:
        k_cache = torch.empty(B, Hkv, T, D, dtype=dt, device=dev)
        v_cache = torch.empty(B, Hkv, T, D, dtype=dt, device=dev)
    cap = k_cache.shape[2]
    rstd = torch.empty(B * T, Hq + Hkv, dtype=torch.float32, device=dev) if want_rstd else None
    L.check(L.lib().orthrus_qkv_prep_fwd(
        qkv.data_ptr(), positions.contiguous().data_ptr(), inv_freq.data_ptr(),
        q_norm_w.contiguous().data_ptr(), k_norm_w.contiguous().data_ptr(), B, T, Hq, Hkv, hd, D,
        float(eps), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), cap, L.ptr(offset),
        L.ptr(rstd), L.dtype_code(dt), L.stream_of(dev)), "qkv_prep_fwd")
    return q, k_cache, v_cache, rstd


def qkv_prep_backward(qkv, positions, inv_freq, q_norm_w, k_norm_w, rstd, dq, dk, dv, B, T, Hq, Hkv,
                      hd, D):
    """Gradients of qkv_prep (training layout): dq/dk/dv fp32 head-major -> (dqkv, dq_norm_w,
    dk_norm_w)."""
    dt = qkv.dtype
    dev = qkv.device
    dqkv = torch.empty_like(qkv)
    dqw = torch.empty(hd, dtype=torch.float32, device=dev)
    dkw = torch.empty(hd, dtype=torch.float32, device=dev)
    lib = L.lib()
    ws = torch.empty(int(lib.orthrus_qkv_prep_bwd_workspace_bytes(B, T, hd)), dtype=torch.uint8,
                     device=dev)
    L.check(lib.orthrus_qkv_prep_bwd(
        qkv.data_ptr(), positions.contiguous().data_ptr(), inv_freq.data_ptr(),
        q_norm_w.contiguous().data_ptr(), k_norm_w.contiguous().data_ptr(), rstd.data_ptr(),
        L.ptr(dq), L.ptr(dk), L.ptr(dv), B, T, Hq, Hkv, hd, D, dqkv.data_ptr(), dqw.data_ptr(),
        dkw.data_ptr(), ws.data_ptr(), ws.numel(), L.dtype_code(dt), L.stream_of(dev)),
        "qkv_prep_bwd")
    return dqkv, dqw, dkw


# --- attention ---------------------------------------------------------------------------------


def _src(t):
    if t is None:
        return 0, 0, 0
    if t.stride(3) != 1 or t.stride(2) != t.shape[3]:
        raise ValueError("attention sources must have contiguous rows of D elements")
    return t.stride(1), t.stride(0), t.shape[2]


def attention_fwd(q, k1, v1, k2=None, v2=None, *, mask: int, hd: int, scale: float,
                  anchors=None, block: int = 0, offset=None, limit2=None, L1: int | None = None,
                  want_lse: bool = True, doc_start=None):
    """Dual-view / causal / draft / tree attention. q [B, Hq, Tq, D]; sources [B, Hkv, rows, D].
    For the tree mask (3) k2/v2 are the cache k1/v1 holding the new tokens at rows offset[b] + t
    and limit2 is int32 [Tq]: the first new-token index of each query's branch (>= 1).
    doc_start (opt-in document mask, int32 [B, L1], see objective.document_starts) keeps the
    source-1 keys of a query to its own document (causal) or to its anchor's document (dual).
    Returns (o [B, Tq, Hq, hd] token-major, lse [B, Hq, Tq] fp32 or None)."""
    _require_cuda(q, k1, v1, k2, v2, anchors, offset, limit2, doc_start)
    B, Hq, Tq, D = q.shape
    if mask == 3 and (offset is None or limit2 is None or limit2.dtype != torch.int32
                      or limit2.numel() != Tq or not limit2.is_contiguous()):
        raise ValueError("the tree mask takes offset int32 [B] and limit2 int32 [Tq] (branch starts)")
    Hkv = k1.shape[1]
    s1h, s1b, rows1 = _src(k1)
    if v1.stride() != k1.stride():
        raise ValueError("k1 and v1 must share strides")
    s2h, s2b, L2 = _src(k2)
    L1 = rows1 if L1 is None else L1
    q = q.contiguous()
    o = torch.empty(B, Tq, Hq, hd, dtype=q.dtype, device=q.device)
    lse = torch.empty(B, Hq, Tq, dtype=torch.float32, device=q.device) if want_lse else None
    A = anchors.shape[1] if anchors is not None else 0
    if anchors is not None:
        anchors = anchors.to(torch.int64).contiguous()
    t0 = TIMER.begin() if TIMER is not None else None
    if (not want_lse and doc_start is None and anchors is None and offset is not None
            and _decode_attention_ok(q, mask, hd, D, Tq, Hq, Hkv, k2, L2)):
        ws = torch.empty(int(L.lib().orthrus_attn_decode_workspace_bytes(B, Hq, Tq, L1)), dtype=torch.uint8,
                         device=q.device)
        L.check(L.lib().orthrus_attn_decode_fwd(
            q.data_ptr(), k1.data_ptr(), v1.data_ptr(), s1h, s1b, L1, L.ptr(k2), L.ptr(v2), s2h, s2b, L2, B, Hq,
            Hkv, Tq, float(scale), mask, offset.data_ptr(), L.ptr(limit2), o.data_ptr(), ws.data_ptr(), ws.numel(),
            L.stream_of(q.device)), "attn_decode_fwd")
    elif doc_start is None:
        L.check(L.lib().orthrus_attn_fwd(
            q.data_ptr(), k1.data_ptr(), v1.data_ptr(), s1h, s1b, L1, L.ptr(k2), L.ptr(v2), s2h, s2b,
            L2, B, Hq, Hkv, Tq, hd, D, float(scale), mask, L.ptr(anchors), A, block, L.ptr(offset),
            L.ptr(limit2), o.data_ptr(), L.ptr(lse), L.dtype_code(q.dtype), L.stream_of(q.device)),
            "attn_fwd")
    else:
        doc_start = _doc_start_arg(doc_start, B, L1)
        L.check(L.lib().orthrus_attn_fwd_doc(
            q.data_ptr(), k1.data_ptr(), v1.data_ptr(), s1h, s1b, L1, L.ptr(k2), L.ptr(v2), s2h, s2b,
            L2, B, Hq, Hkv, Tq, hd, D, float(scale), mask, L.ptr(anchors), A, block, L.ptr(offset),
            L.ptr(limit2), doc_start.data_ptr(), o.data_ptr(), L.ptr(lse), L.dtype_code(q.dtype),
            L.stream_of(q.device)), "attn_fwd_doc")
    if t0 is not None:
        TIMER.end(f"attn_fwd_{('causal', 'dual', 'draft', 'tree')[mask]}", t0,
                  attention_flops(mask, B, Hq, Tq, hd, anchors, block, L1))
    return o, lse


def _decode_attention_ok(q, mask, hd, D, Tq, Hq, Hkv, k2, L2) -> bool:
    """The decode passes' split-key kernel takes bf16 blocks of at most 64 rows per sequence with
    hd = 128, causal over a cache (with offsets) or the draft mask."""
    return (q.dtype == torch.bfloat16 and hd == 128 and D == 128 and Tq <= 64 and (Hq // Hkv) * Tq <= 128
            and (mask == 0 or (mask == 2 and k2 is not None and 0 < L2 <= 64)))


def attention_flops(mask, B, Hq, Tq, hd, anchors=None, block=0, L1=0):
    """Algorithmic forward FLOPs: 4 hd per (query, visible key) per head (2 for QK^T, 2 for PV);
    a device scalar for the dual mask (anchors stay on the device)."""
    if mask == 0:
        return 4.0 * hd * Hq * B * Tq * (Tq + 1) / 2
    if mask == 1:
        vis = anchors.clamp(max=L1).sum() * block + anchors.numel() * block * block
        return 4.0 * hd * Hq * vis
    return 0.0


def _doc_start_arg(doc_start, B: int, L1: int) -> torch.Tensor:
    """int32 [B, L1] document starts of the source-1 positions (a longer row is cut to L1)."""
    if doc_start.dtype != torch.int32 or doc_start.dim() != 2 or doc_start.shape[0] != B \
            or doc_start.shape[1] < L1:
        raise ValueError(f"doc_start must be int32 [B, >= L1] = [{B}, >= {L1}], got "
                         f"{doc_start.dtype} {tuple(doc_start.shape)}")
    return doc_start[:, :L1].contiguous()


def attention_bwd(q, k1, v1, k2, v2, anchors, block, o, lse, dout, *, hd: int, scale: float,
                  doc_start=None):
    """Backward of the dual mask: (dq [B, Hq, Tq, D], dk2, dv2 [B, Hkv, L2, D]) fp32. doc_start as
    in attention_fwd (the same mask as the forward's)."""
    B, Hq, Tq, D = q.shape
    Hkv = k1.shape[1]
    s1h, s1b, L1 = _src(k1)
    s2h, s2b, L2 = _src(k2)
    dev = q.device
    dq = torch.empty(B, Hq, Tq, D, dtype=torch.float32, device=dev)
    dk2 = torch.empty(B, Hkv, L2, D, dtype=torch.float32, device=dev)
    dv2 = torch.empty(B, Hkv, L2, D, dtype=torch.float32, device=dev)
    lib = L.lib()
    ws = torch.empty(int(lib.orthrus_attn_bwd_workspace_bytes(B, Hq, Tq)), dtype=torch.uint8,
                     device=dev)
    anchors = anchors.to(torch.int64).contiguous()
    dout = dout.contiguous()
    t0 = TIMER.begin() if TIMER is not None else None
    if doc_start is None:
        L.check(lib.orthrus_attn_bwd(
            q.data_ptr(), k1.data_ptr(), v1.data_ptr(), s1h, s1b, L1, k2.data_ptr(), v2.data_ptr(),
            s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, float(scale), anchors.data_ptr(), anchors.shape[1],
            block, o.data_ptr(), lse.data_ptr(), dout.data_ptr(), dq.data_ptr(), dk2.data_ptr(),
            dv2.data_ptr(), ws.data_ptr(), ws.numel(), L.dtype_code(q.dtype), L.stream_of(dev)),
            "attn_bwd")
    else:
        doc_start = _doc_start_arg(doc_start, B, L1)
        L.check(lib.orthrus_attn_bwd_doc(
            q.data_ptr(), k1.data_ptr(), v1.data_ptr(), s1h, s1b, L1, k2.data_ptr(), v2.data_ptr(),
            s2h, s2b, L2, B, Hq, Hkv, Tq, hd, D, float(scale), anchors.data_ptr(), anchors.shape[1],
            block, doc_start.data_ptr(), o.data_ptr(), lse.data_ptr(), dout.data_ptr(), dq.data_ptr(),
            dk2.data_ptr(), dv2.data_ptr(), ws.data_ptr(), ws.numel(), L.dtype_code(q.dtype),
            L.stream_of(dev)), "attn_bwd_doc")
    if t0 is not None:  # QK^T recompute, dP and dQ: 1.5x the forward FLOPs
        TIMER.end("attn_bwd_dual", t0, 1.5 * attention_flops(1, B, Hq, Tq, hd, anchors, block, L1))
    return dq, dk2, dv2


def attention_tilemap(anchors: torch.Tensor, block: int, L1: int) -> torch.Tensor:
    """Per 128-query tile: (source-1 tiles, visible source-1 keys, source-2 key range) int32."""
    _require_cuda(anchors)
    anchors = anchors.to(torch.int64).contiguous()
    B, A = anchors.shape
    ntiles = (A * block + 127) // 128
    out = torch.empty(B, ntiles, 4, dtype=torch.int32, device=anchors.device)
    L.check(L.lib().orthrus_attn_tilemap(anchors.data_ptr(), B, A, block, L1, out.data_ptr(),
                                         L.stream_of(anchors.device)), "attn_tilemap")
    return out


# --- decoding ----------------------------------------------------------------------------------


def argmax_rows(logits: torch.Tensor) -> torch.Tensor:
    """Row-wise argmax of fp32 logits [R, V] (lowest index on ties)."""
    _require_cuda(logits)
    if logits.dtype != torch.float32 or logits.stride(-1) != 1:
        raise ValueError("argmax_rows takes row-major fp32 logits")
    R, V = logits.shape
    out = torch.empty(R, dtype=torch.int64, device=logits.device)
    L.check(L.lib().orthrus_argmax_rows(logits.data_ptr(), logits.stride(0), R, V, out.data_ptr(),
                                        L.stream_of(logits.device)), "argmax_rows")
    return out


def decode_draft(logits, anchor, done, verify_ids):
    B, K, V = logits.shape
    L.check(L.lib().orthrus_decode_draft(logits.data_ptr(), B, K, V, anchor.data_ptr(),
                                         L.ptr(done), verify_ids.data_ptr(),
                                         L.stream_of(logits.device)), "decode_draft")


def decode_verify_accept(logits, verify_ids, ar_tokens, eos, max_len, start, anchor, done,
                         out_tokens, out_len, accepted_log, cycle):
    B, K, V = logits.shape
    L.check(L.lib().orthrus_decode_verify_accept(
        logits.data_ptr(), B, K, V, verify_ids.data_ptr(), ar_tokens.data_ptr(), L.ptr(eos),
        0 if eos is None else eos.numel(), max_len.data_ptr(), start.data_ptr(), anchor.data_ptr(),
        done.data_ptr(), out_tokens.data_ptr(), out_len.data_ptr(), out_tokens.shape[1],
        accepted_log.data_ptr(), cycle.data_ptr(), accepted_log.shape[1],
        L.stream_of(logits.device)), "decode_verify_accept")


def lmhead_argmax(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """argmax over the vocabulary of hidden [R, d] @ weight [V, d]^T (bf16) without writing the
    logits; int64 [R], the lowest index on ties (the argmax of gemm(..., out_dtype=fp32))."""
    _require_cuda(hidden, weight)
    h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    R, d = h.shape
    out = torch.empty(R, dtype=torch.int64, device=h.device)
    lib = L.lib()
    ws = torch.empty(int(lib.orthrus_lmhead_argmax_workspace_bytes(R)), dtype=torch.uint8, device=h.device)
    L.check(lib.orthrus_lmhead_argmax_bf16(h.data_ptr(), R, weight.data_ptr(), weight.shape[0], d, out.data_ptr(),
                                           ws.data_ptr(), ws.numel(), L.stream_of(h.device)), "lmhead_argmax")
    return out


def decode_draft_ids(ids, anchor, done, verify_ids):
    B, K = verify_ids.shape
    L.check(L.lib().orthrus_decode_draft_ids(ids.data_ptr(), B, K, anchor.data_ptr(), L.ptr(done),
                                             verify_ids.data_ptr(), L.stream_of(ids.device)), "decode_draft_ids")


def decode_accept_ids(ar_tokens, verify_ids, eos, max_len, start, anchor, done, out_tokens, out_len,
                      accepted_log, cycle):
    B, K = verify_ids.shape
    L.check(L.lib().orthrus_decode_accept_ids(
        ar_tokens.data_ptr(), B, K, verify_ids.data_ptr(), L.ptr(eos), 0 if eos is None else eos.numel(),
        max_len.data_ptr(), start.data_ptr(), anchor.data_ptr(), done.data_ptr(), out_tokens.data_ptr(),
        out_len.data_ptr(), out_tokens.shape[1], accepted_log.data_ptr(), cycle.data_ptr(), accepted_log.shape[1],
        L.stream_of(ar_tokens.device)), "decode_accept_ids")


# --- sampled decoding ---------------------------------------------------------------------------

SAMPLE_MAX_TOP_K = 112  # top_k of the device sampler (candidates: top_k + 16 spares, at most 128)


@dataclass(frozen=True)
class SamplingParams:
    """The sampling knobs of diffusion_generate (orthrus/modeling_orthrus.py:405-449) and the seed
    of the decode's Philox draws."""

    temperature: float
    top_k: int = 20
    top_p: float = 0.8
    seed: int = 0

    def candidates(self, vocab: int) -> int:
        """C: the top-k candidates kept per row, plus spares for ties at the k-th value."""
        if not self.temperature > 0:
            raise ValueError("sampling needs a temperature > 0")
        if not 1 <= self.top_k <= SAMPLE_MAX_TOP_K:
            raise ValueError(f"the device sampler takes 1 <= top_k <= {SAMPLE_MAX_TOP_K} (got {self.top_k})")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        k = min(self.top_k, vocab)
        return min(k + 16, vocab, 128)



def sample_candidates(logits: torch.Tensor, params: SamplingParams):
    """(values fp32 [..., C] descending, ids int64 [..., C]): each row's top C logits."""
    _require_cuda(logits)
    C = params.candidates(logits.shape[-1])
    vals, ids = torch.topk(logits.float(), C, dim=-1, sorted=True)
    return vals.contiguous(), ids.contiguous()


def sample_probs(vals: torch.Tensor, params: SamplingParams) -> torch.Tensor:
    """The filtered distribution [..., C] of candidate rows (the reference's `pick` filter)."""
    _require_cuda(vals)
    C = vals.shape[-1]
    v = vals.reshape(-1, C).contiguous()
    out = torch.empty_like(v)
    L.check(L.lib().orthrus_sample_probs(v.data_ptr(), v.shape[0], C, float(params.temperature),
                                         min(params.top_k, C), float(params.top_p),
                                         out.data_ptr(), L.stream_of(v.device)), "sample_probs")
    return out.view_as(vals)


def sample_rows(vals: torch.Tensor, ids: torch.Tensor, params: SamplingParams, cycle=None) -> torch.Tensor:
    """One token per candidate row [R, C] (draw (r, cycle[r] or 0, 0, first))."""
    _require_cuda(vals, ids, cycle)
    R, C = vals.shape
    out = torch.empty(R, dtype=torch.int64, device=vals.device)
    L.check(L.lib().orthrus_sample_rows(vals.data_ptr(), ids.data_ptr(), R, C, float(params.temperature),
                                        min(params.top_k, C), float(params.top_p), params.seed & (2 ** 64 - 1),
                                        L.ptr(cycle), out.data_ptr(), L.stream_of(vals.device)), "sample_rows")
    return out


def decode_sample_draft(vals, ids, params: SamplingParams, cycle, anchor, done, verify_ids, draft_probs):
    """Drafts of a sampled cycle from the diffusion pass's candidate rows [B, K-1, C]."""
    B, K1, C = vals.shape
    L.check(L.lib().orthrus_decode_sample_draft(
        vals.data_ptr(), ids.data_ptr(), B, K1 + 1, C, float(params.temperature), min(params.top_k, C),
        float(params.top_p), params.seed & (2 ** 64 - 1), cycle.data_ptr(), anchor.data_ptr(), done.data_ptr(),
        verify_ids.data_ptr(), draft_probs.data_ptr(), L.stream_of(vals.device)), "decode_sample_draft")


def decode_sample_accept(vals, ids, draft_probs, draft_ids, params: SamplingParams, verify_ids, eos, max_len,
                         start, anchor, done, out_tokens, out_len, accepted_log, cycle):
    """Rejection-sampling accept of a sampled cycle from the verify pass's candidate rows [B, K, C]."""
    B, K, C = vals.shape
    L.check(L.lib().orthrus_decode_sample_accept(
        vals.data_ptr(), ids.data_ptr(), draft_probs.data_ptr(), draft_ids.data_ptr(), B, K, C,
        float(params.temperature), min(params.top_k, C), float(params.top_p), params.seed & (2 ** 64 - 1),
        verify_ids.data_ptr(), L.ptr(eos), 0 if eos is None else eos.numel(), max_len.data_ptr(),
        start.data_ptr(), anchor.data_ptr(), done.data_ptr(), out_tokens.data_ptr(), out_len.data_ptr(),
        out_tokens.shape[1], accepted_log.data_ptr(), cycle.data_ptr(), accepted_log.shape[1],
        L.stream_of(vals.device)), "decode_sample_accept")


def philox4x32_10(counter_key: torch.Tensor) -> torch.Tensor:
    """Philox4x32-10 of int32 [n, 6] (counter words 0-3, key words 0-1, as 32-bit patterns) ->
    int32 [n, 4] bit patterns, on the device of the input."""
    _require_cuda(counter_key)
    ck = counter_key.to(torch.int32).contiguous()
    out = torch.empty(ck.shape[0], 4, dtype=torch.int32, device=ck.device)
    L.check(L.lib().orthrus_philox4x32_10(ck.data_ptr(), ck.shape[0], out.data_ptr(), L.stream_of(ck.device)),
            "philox4x32_10")
    return out


# --- row-local elementwise pieces ---------------------------------------------------------------


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, want_rstd: bool = False):
    """Qwen3RMSNorm over the last dim with a fixed per-row reduction order (no autograd).
    Returns y, or (y, rstd fp32 [rows]) with want_rstd."""
    _require_cuda(x, weight)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    y = torch.empty_like(x2)
    w = weight.to(x.dtype).contiguous()
    rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device) if want_rstd else None
    L.check(L.lib().orthrus_rmsnorm(x2.data_ptr(), w.data_ptr(), x2.shape[0], x2.shape[1],
                                    float(eps), y.data_ptr(), L.ptr(rstd), L.dtype_code(x.dtype),
                                    L.stream_of(x.device)), "rmsnorm")
    return (y.view(shape), rstd) if want_rstd else y.view(shape)


def rms_norm_backward(x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor,
                      dy: torch.Tensor, dres: torch.Tensor | None = None) -> torch.Tensor:
    """dx of rms_norm (the weight is frozen); with dres, dres + dx in one rounding (the gradient
    of a tensor that also feeds a residual add)."""
    shape = x.shape
    if dres is not None:
        x2 = x.reshape(-1, shape[-1]).contiguous()
        if x.dtype != torch.bfloat16 or shape[-1] % 256:
            return rms_norm_backward(x, weight, rstd, dy) + dres
        dy2 = dy.reshape(-1, shape[-1]).contiguous().to(x.dtype)
        r2 = dres.reshape(-1, shape[-1]).contiguous().to(x.dtype)
        w = weight.to(x.dtype).contiguous()
        dx = torch.empty_like(x2)
        L.check(L.lib().orthrus_rmsnorm_bwd_add(x2.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy2.data_ptr(),
                                                r2.data_ptr(), x2.shape[0], x2.shape[1], dx.data_ptr(),
                                                L.stream_of(x.device)), "rmsnorm_bwd_add")
        return dx.view(shape)
    x2 = x.reshape(-1, shape[-1]).contiguous()
    dy2 = dy.reshape(-1, shape[-1]).contiguous().to(x.dtype)
    w = weight.to(x.dtype).contiguous()
    dx = torch.empty_like(x2)
    L.check(L.lib().orthrus_rmsnorm_bwd(x2.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy2.data_ptr(),
                                        x2.shape[0], x2.shape[1], dx.data_ptr(),
                                        L.dtype_code(x.dtype), L.stream_of(x.device)), "rmsnorm_bwd")
    return dx.view(shape)


def add(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Residual add (elementwise, order-free)."""
    return x + y


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """SwiGLU activation of the fused [gate | up] projection output (orthrus_swiglu_fwd)."""
    _require_cuda(gate_up)
    shape = gate_up.shape
    g2 = gate_up.reshape(-1, shape[-1]).contiguous()
    inter = shape[-1] // 2
    out = torch.empty(g2.shape[0], inter, dtype=gate_up.dtype, device=gate_up.device)
    L.check(L.lib().orthrus_swiglu_fwd(g2.data_ptr(), g2.shape[0], inter, out.data_ptr(),
                                       L.dtype_code(gate_up.dtype), L.stream_of(gate_up.device)),
            "swiglu_fwd")
    return out.view(*shape[:-1], inter)


def silu_mul_backward(gate_up: torch.Tensor, dout: torch.Tensor) -> torch.Tensor:
    shape = gate_up.shape
    g2 = gate_up.reshape(-1, shape[-1]).contiguous()
    inter = shape[-1] // 2
    d2 = dout.reshape(-1, inter).contiguous().to(gate_up.dtype)
    dgu = torch.empty_like(g2)
    L.check(L.lib().orthrus_swiglu_bwd(g2.data_ptr(), d2.data_ptr(), g2.shape[0], inter,
                                       dgu.data_ptr(), L.dtype_code(gate_up.dtype),
                                       L.stream_of(gate_up.device)), "swiglu_bwd")
    return dgu.view(shape)


# --- per-entry-point timing (the breakdown pass of bench.py) -------------------------------------
# Every public op below records CUDA events on its launching stream around the call when ops.TIMER
# is set (attention and the LM head record their own, with their FLOP counts). Projections carry
# their GEMM FLOPs and the "proj_" prefix; the row kernels report time only. Nested timed calls
# are not counted twice.

_timing_depth = 0


def _timed(fn, label, work):
    import functools

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        global _timing_depth
        if TIMER is None or _timing_depth:
            return fn(*args, **kwargs)
        _timing_depth += 1
        try:
            t0 = TIMER.begin()
            out = fn(*args, **kwargs)
            TIMER.end(label, t0, work(*args, **kwargs) if work is not None else 0.0)
        finally:
            _timing_depth -= 1
        return out

    return wrapper


def _gemm2_work(a, b, *, a_t=False, b_t=False, residual=None):
    M, K = (a.shape[1], a.shape[0]) if a_t else a.shape
    return 2.0 * M * (b.shape[1] if b_t else b.shape[0]) * K


def _rows_cols_work(x, w, *args, **kwargs):  # x [M, K] @ w [N, K]^T
    return 2.0 * x.shape[0] * w.shape[0] * x.shape[1]


def _gemm_work(a, b, *, b_kn=False, **kwargs):
    return 2.0 * a.shape[0] * (b.shape[1] if b_kn else b.shape[0]) * a.shape[1]


for _name, _label, _work in (
        ("gemm2", "proj_gemm2", _gemm2_work),
        ("gemm2_swiglu_backward", "proj_gemm2_swiglu_bwd",
         lambda dy, w, gu: 2.0 * dy.shape[0] * w.shape[1] * dy.shape[1]),
        ("linear", "proj_linear", _rows_cols_work),
        ("linear_swiglu", "proj_linear_swiglu", _rows_cols_work),
        ("linear_qkv_rope", "proj_linear_qkv_rope", _rows_cols_work),
        ("gemm", "proj_gemm", _gemm_work),
        ("qkv_prep", "qkv_prep", None),
        ("qkv_prep_backward", "qkv_prep_bwd", None),
        ("rms_norm", "rms_norm", None),
        ("rms_norm_backward", "rms_norm_bwd", None),
        ("silu_mul", "swiglu", None),
        ("silu_mul_backward", "swiglu_bwd", None),
        ("lmhead_kl_backward", "lmhead_kl_bwd_scale", None),
        ("add", "add", None),
        ("rope_table", "rope_table", None)):
    globals()[_name] = _timed(globals()[_name], _label, _work)
