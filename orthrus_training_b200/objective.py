"""Orthrus training objective on the Blackwell kernels: drop-in for orthrus/objective.py.

Same functions, signatures and return values as the reference module. Both views run through
``liborthrus_b200.so``:

- teacher (frozen, no grad): per layer RMSNorm -> fused q|k|v projection -> q/k norm + RoPE
  prologue -> causal tcgen05 attention -> o projection -> SwiGLU MLP; its K/V become the AR cache
  (orthrus/objective.py:152-157,248-255);
- student (diffusion view, autograd): twin q|k|v projection -> ``DualViewAttention`` (prologue +
  dual-view tcgen05 attention with the per-anchor tile map; backward = dQ over every visible key
  tile plus dK/dV of the own-block keys only, the reference's skip_ar_key_grads) -> twin o
  projection -> frozen MLP (orthrus/objective.py:160-165,257-272);
- KL: ``FusedLinearForwardKL`` over the fused LM-head + log-softmax + KL kernels, which also emit the
  per-offset KL / agreement sums (orthrus/objective.py:298-392,440-452).

Every projection GEMM of the bf16 training step (forward, dX and dW) runs on this package's tcgen05
kernels: the persistent one-CTA kernel where an epilogue fuses the q/k prologue or SwiGLU, the
CTA-pair kernel (orthrus_gemm2_bf16) for the rest; every attention, norm + RoPE, LM-head and KL
computation is a kernel of this package as well. The fp32 path keeps torch matmuls for its
projections (exact fp32 parity runs). There is no CPU path.
"""

from __future__ import annotations

import logging

import torch
import torch.nn.functional as F

from orthrus_training_b200 import ops
from orthrus_training_b200._lib import MASK_CAUSAL, MASK_DUAL
from orthrus_training_b200.modeling_orthrus import (
    OrthrusLM,
    build_block_mask,
    diffusion_attention,  # noqa: F401  (re-exported like the reference module)
    padded_head_dim,
)

log = logging.getLogger(__name__)

SKIP_AR_KEY_GRADS = True  # always: the AR keys are the frozen teacher's and never get dK/dV


def sample_anchors(assistant_mask: torch.Tensor, block_size: int, num_anchors: int,
                   generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
    """Sorted anchors drawn without replacement from assistant positions in [1, L-K]; spare slots
    repeat the last anchor and are invalid (orthrus/objective.py:37-63). The same torch RNG calls
    as the reference (one randperm per row over its candidate count), so one generator state
    yields the reference's anchors. The candidate counts of all rows come to the host in one read;
    each row's candidates are its assistant positions in ascending order, taken on the device
    from a stable sort instead of a boolean gather (which would read back a size per row)."""
    batch, seq_len = assistant_mask.shape
    slots = min(num_anchors, seq_len - block_size)
    span = seq_len - block_size  # candidate positions 1 .. span
    device = assistant_mask.device
    positions = torch.arange(1, span + 1, device=device)
    eligible = assistant_mask[:, 1: span + 1].bool()
    counts = eligible.sum(1).tolist()
    # per row: the eligible positions first, ascending (stable sort on "not eligible")
    ranked = torch.sort((~eligible).to(torch.uint8), dim=1, stable=True).indices + 1
    anchors = torch.zeros((batch, slots), dtype=torch.long, device=device)
    valid = torch.zeros((batch, slots), dtype=torch.bool, device=device)
    for row in range(batch):
        has_targets = counts[row] > 0
        n = counts[row] if has_targets else span
        candidates = ranked[row] if has_targets else positions
        order = torch.randperm(n, generator=generator, device=device)
        taken = min(slots, n)
        picked = candidates[order[:slots]].sort().values
        anchors[row, :taken] = picked
        anchors[row, taken:] = picked[-1]
        valid[row, :taken] = has_targets
    return anchors, valid


def supervision_mask(assistant_mask, anchors, valid, block_size):
    """keep[b, a, i]: target anchor+i+1 is an assistant token and the slot is valid
    (orthrus/objective.py:66-73). Shape [batch, slots, K-1]."""
    targets = anchors[:, :, None] + torch.arange(1, block_size, device=anchors.device)
    keep = assistant_mask.gather(1, targets.flatten(1)).view_as(targets)
    return keep & valid[:, :, None]


def position_weights(block_size: int, gamma: float, device=None) -> torch.Tensor | None:
    """exp(-i/gamma), i = 0..K-2, or None for gamma <= 0 (orthrus/objective.py:76-81)."""
    if gamma <= 0:
        return None
    return torch.exp(-torch.arange(block_size - 1, device=device, dtype=torch.float32) / gamma)


class _RMSNorm(torch.autograd.Function):
    """Qwen3RMSNorm (orthrus/objective.py:128-133) on the row kernels: forward saves rstd, backward
    returns dx only (the norm weights of the model are frozen)."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = ops.rms_norm(x, weight, eps, want_rstd=True)
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        return ops.rms_norm_backward(x, weight, rstd, dy), None, None


class _NormWithSkip(torch.autograd.Function):
    """RMSNorm of a block input that also feeds the block's residual add: returns (n(x), x). Its
    backward receives both gradients of x and sums them inside the RMSNorm backward kernel (one
    rounding), instead of autograd adding the residual gradient in a separate pass."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = ops.rms_norm(x, weight, eps, want_rstd=True)
        ctx.save_for_backward(x, weight, rstd)
        return y, x.view_as(x)

    @staticmethod
    def backward(ctx, dy, dskip):
        x, weight, rstd = ctx.saved_tensors
        return ops.rms_norm_backward(x, weight, rstd, dy, dres=dskip), None, None


class _SwiGLU(torch.autograd.Function):
    """silu(gate) * up of the fused [gate | up] projection (orthrus/objective.py:146-149)."""

    @staticmethod
    def forward(ctx, gate_up):
        ctx.save_for_backward(gate_up)
        return ops.silu_mul(gate_up)

    @staticmethod
    def backward(ctx, dout):
        (gate_up,) = ctx.saved_tensors
        return ops.silu_mul_backward(gate_up, dout)


class _GateUpSwiGLU(torch.autograd.Function):
    """F.linear(h, [gate; up]) followed by the SwiGLU activation in one persistent kernel that also
    keeps [gate | up] for the backward (orthrus/objective.py:146-149). The MLP weights are frozen,
    so the backward returns dh = dgate_up @ W only."""

    @staticmethod
    def forward(ctx, h, w_gate_up):
        if w_gate_up.requires_grad:
            raise ValueError("the MLP weights of the dual-view model are frozen")
        act, gate_up = ops.linear_swiglu(h, w_gate_up, keep_gate_up=True)
        ctx.save_for_backward(gate_up, w_gate_up)
        return act

    @staticmethod
    def backward(ctx, dact):
        gate_up, w = ctx.saved_tensors
        dgu = ops.silu_mul_backward(gate_up, dact.contiguous())
        return _dx(dgu, w), None


def _rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3RMSNorm with autograd for the student path (frozen weight)."""
    if weight.requires_grad:
        raise ValueError("the RMSNorm weights of the dual-view model are frozen")
    return _RMSNorm.apply(x, weight, eps)


def _pair_gemm_ok(*tensors) -> bool:
    """Whether the CTA-pair GEMM takes these operands (bf16, sizes multiples of 32)."""
    return all(t.dtype == torch.bfloat16 and t.shape[-1] % 32 == 0 for t in tensors)


def _add_projection(x: torch.Tensor, a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x + a @ w^T (torch.addmm(x, a, w.t())) without autograd, on the CTA-pair GEMM with the
    residual in its epilogue for bf16."""
    if _pair_gemm_ok(x, a, w):
        return ops.gemm2(a, w, residual=x)
    return torch.addmm(x, a, w.t())


class _ProjectionResidual(torch.autograd.Function):
    """x + a @ w^T (orthrus/objective.py:160-165 o projection, :146-149 down projection) on the
    CTA-pair GEMM: the forward carries the residual in its epilogue; the backward is dx = dy,
    da = dy @ w and, for a trainable w, dw = dy^T @ a (the two GEMMs autograd runs for
    torch.addmm), on the same kernel."""

    @staticmethod
    def forward(ctx, x, a, w):
        ctx.save_for_backward(a, w)
        return ops.gemm2(a, w, residual=x)

    @staticmethod
    def backward(ctx, dy):
        a, w = ctx.saved_tensors
        dy = dy.contiguous()
        da = ops.gemm2(dy, w, b_t=True) if ctx.needs_input_grad[1] else None
        dw = ops.gemm2(dy, a, a_t=True, b_t=True) if ctx.needs_input_grad[2] else None
        return dy, da, dw


def _projection_residual(x: torch.Tensor, a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if _pair_gemm_ok(x, a, w):
        return _ProjectionResidual.apply(x, a, w)
    return torch.addmm(x, a, w.t())


def _dx(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """dy @ w: the input gradient of a projection with weight w [N, K]."""
    dy = dy.contiguous()
    return ops.gemm2(dy, w, b_t=True) if _pair_gemm_ok(dy, w) else dy @ w


def _dw(dy: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    """dy^T @ a: the weight gradient of a projection of the rows a."""
    dy = dy.contiguous()
    return ops.gemm2(dy, a, a_t=True, b_t=True) if _pair_gemm_ok(dy, a) and dy.shape[1] % 8 == 0 \
        else dy.t() @ a


class _MLPBlock(torch.autograd.Function):
    """The MLP half of a trainable-view layer, x + down(silu(gate(n(x))) * up(n(x))) with n the
    post-attention RMSNorm (orthrus/objective.py:146-149), as one Function so that its backward
    fuses what autograd would run as separate passes: the SwiGLU backward rides in the epilogue of
    the dact = dy @ W_down GEMM (dact never reaches HBM), and the residual gradient dy is added in
    the RMSNorm backward kernel. The MLP and norm weights are frozen: only dx is returned."""

    @staticmethod
    def forward(ctx, x, norm_w, w_gate_up, w_down, eps):
        h, rstd = ops.rms_norm(x, norm_w, eps, want_rstd=True)
        act, gate_up = ops.linear_swiglu(h, w_gate_up, keep_gate_up=True)
        ctx.save_for_backward(x, norm_w, rstd, gate_up, w_gate_up, w_down)
        return ops.gemm2(act, w_down, residual=x)

    @staticmethod
    def backward(ctx, dy):
        x, norm_w, rstd, gate_up, w_gate_up, w_down = ctx.saved_tensors
        dy = dy.contiguous()
        dgu = ops.gemm2_swiglu_backward(dy, w_down, gate_up)
        dh = _dx(dgu, w_gate_up)
        return ops.rms_norm_backward(x, norm_w, rstd, dh, dres=dy), None, None, None, None


def _mlp_block_ok(x, w_gu, w_down) -> bool:
    F = w_gu.shape[0] // 2
    return (_pair_gemm_ok(x, w_down) and ops.fused_linear_supported(x, w_gu, F) and F % 64 == 0
            and x.shape[-1] % 256 == 0 and not w_gu.requires_grad and not w_down.requires_grad)


class DualViewAttention(torch.autograd.Function):
    """Diffusion-view attention of one layer from the twin projection output.

    forward: q/k RMSNorm + RoPE prologue (orthrus_qkv_prep_fwd) of qkv [B*Q, (Hq+2Hkv) hd], then
    the dual-view attention (orthrus_attn_fwd, mask DUAL) over source 1 = the teacher's K/V and
    source 2 = the block's own K/V. Returns o [B*Q, Hq*hd] (the o_proj input).
    backward: orthrus_attn_bwd (dQ for every visible key, dK/dV of the own-block keys only), then
    orthrus_qkv_prep_bwd back to dqkv and the q/k norm weight gradients.
    """

    @staticmethod
    def forward(ctx, qkv, q_norm_w, k_norm_w, ar_k, ar_v, positions, anchors, inv_freq, meta,
                doc_start=None):
        B, Q, Hq, Hkv, hd, D, K, eps = meta
        q, k2, v2, rstd = ops.qkv_prep(qkv, positions, inv_freq, q_norm_w, k_norm_w, B, Q, Hq, Hkv,
                                       hd, D, eps, want_rstd=True)
        o, lse = ops.attention_fwd(q, ar_k, ar_v, k2, v2, mask=MASK_DUAL, hd=hd, scale=hd ** -0.5,
                                   anchors=anchors, block=K, doc_start=doc_start)
        ctx.doc_start = doc_start
        ctx.save_for_backward(qkv, q_norm_w, k_norm_w, ar_k, ar_v, positions, anchors, inv_freq, q,
                              k2, v2, o, lse, rstd)
        ctx.meta = meta
        return o.view(B * Q, Hq * hd)

    @staticmethod
    def backward(ctx, grad_o):
        qkv, qn, kn, ar_k, ar_v, positions, anchors, inv, q, k2, v2, o, lse, rstd = ctx.saved_tensors
        B, Q, Hq, Hkv, hd, D, K, eps = ctx.meta
        dout = grad_o.contiguous().view(B, Q, Hq, hd).to(q.dtype)
        dq, dk2, dv2 = ops.attention_bwd(q, ar_k, ar_v, k2, v2, anchors, K, o, lse, dout, hd=hd,
                                         scale=hd ** -0.5, doc_start=ctx.doc_start)
        dqkv, dqw, dkw = ops.qkv_prep_backward(qkv, positions, inv, qn, kn, rstd, dq, dk2, dv2, B,
                                               Q, Hq, Hkv, hd, D)
        return dqkv, dqw.to(qn.dtype), dkw.to(kn.dtype), None, None, None, None, None, None, None


class DualViewAttentionFused(torch.autograd.Function):
    """DualViewAttention with the twin q|k|v projection folded in (orthrus/objective.py:136-143,
    160-165): forward = the projection GEMM with the q/k RMSNorm + RoPE prologue in its epilogue
    (orthrus_linear_qkv_rope_keep_bf16, which also keeps the q / k columns of the projection and
    rstd), then the dual-view attention; backward = the attention backward, the prologue backward,
    then dh = dqkv W and dW = dqkv^T h. One Function, so the fp32 dq / dk / dv of the attention
    backward reach the prologue backward without a cast."""

    @staticmethod
    def forward(ctx, h, w_qkv, q_norm_w, k_norm_w, ar_k, ar_v, positions, anchors, inv_freq, rope_cos,
                rope_sin, meta, doc_start=None):
        B, Q, Hq, Hkv, hd, D, K, eps = meta
        q, k2, v2, qkv, rstd = ops.linear_qkv_rope(h, w_qkv, q_norm_w, k_norm_w, (rope_cos, rope_sin), B, Q,
                                                   Hq, Hkv, eps, positions=positions, keep=True)
        o, lse = ops.attention_fwd(q, ar_k, ar_v, k2, v2, mask=MASK_DUAL, hd=hd, scale=hd ** -0.5,
                                   anchors=anchors, block=K, doc_start=doc_start)
        ctx.doc_start = doc_start
        ctx.save_for_backward(h, w_qkv, qkv, q_norm_w, k_norm_w, ar_k, ar_v, positions, anchors, inv_freq,
                              q, k2, v2, o, lse, rstd)
        ctx.meta = meta
        return o.view(B * Q, Hq * hd)

    @staticmethod
    def backward(ctx, grad_o):
        h, w, qkv, qn, kn, ar_k, ar_v, positions, anchors, inv, q, k2, v2, o, lse, rstd = ctx.saved_tensors
        B, Q, Hq, Hkv, hd, D, K, eps = ctx.meta
        dout = grad_o.contiguous().view(B, Q, Hq, hd).to(q.dtype)
        dq, dk2, dv2 = ops.attention_bwd(q, ar_k, ar_v, k2, v2, anchors, K, o, lse, dout, hd=hd,
                                         scale=hd ** -0.5, doc_start=ctx.doc_start)
        dqkv, dqw, dkw = ops.qkv_prep_backward(qkv, positions, inv, qn, kn, rstd, dq, dk2, dv2, B,
                                               Q, Hq, Hkv, hd, D)
        dh = _dx(dqkv, w)
        dw = _dw(dqkv, h)
        return (dh, dw, dqw.to(qn.dtype), dkw.to(kn.dtype), None, None, None, None, None, None, None,
                None, None)


def _teacher_layer(backbone, i, x, pos, B, L, inv, rope=None, doc_start=None):
    cfg = backbone.config
    layer = backbone.layers[i]
    attn = layer.self_attn
    Hq, Hkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    D = padded_head_dim(hd)
    eps = cfg.rms_norm_eps
    h = ops.rms_norm(x, layer.input_layernorm.weight, eps)
    if rope is not None:
        # q|k|v GEMM with the q/k norm + RoPE prologue in its epilogue, written head-major
        q, k, v = ops.linear_qkv_rope(h, attn.packed_qkv(False), attn.q_norm.weight,
                                      attn.k_norm.weight, rope, B, L, Hq, Hkv, eps)
    else:
        qkv = h @ attn.packed_qkv(False).t()
        q, k, v, _ = ops.qkv_prep(qkv, pos, inv, attn.q_norm.weight, attn.k_norm.weight, B, L, Hq,
                                  Hkv, hd, D, eps)
    o, _ = ops.attention_fwd(q, k, v, mask=MASK_CAUSAL, hd=hd, scale=hd ** -0.5, want_lse=False,
                             doc_start=doc_start)
    # residual adds ride in the GEMM epilogue
    x = _add_projection(x, o.view(B * L, Hq * hd), attn.o_proj.weight)
    h = ops.rms_norm(x, layer.post_attention_layernorm.weight, eps)
    w_gu = layer.mlp.packed_gate_up()
    if ops.fused_linear_supported(h, w_gu, w_gu.shape[0] // 2):
        # gate/up GEMM with SwiGLU in its epilogue: [gate | up] never goes through HBM
        act = ops.linear_swiglu(h, w_gu, pair=h.shape[0] >= 2048)
    else:
        act = ops.silu_mul(h @ w_gu.t())
    x = _add_projection(x, act, layer.mlp.down_proj.weight)
    return x, k, v


def _diffusion_layer(backbone, i, x, ar_k, ar_v, positions, anchors, inv, B, Q, rope=None, doc_start=None):
    cfg = backbone.config
    layer = backbone.layers[i]
    attn = layer.self_attn
    Hq, Hkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    eps = cfg.rms_norm_eps
    meta = (B, Q, Hq, Hkv, hd, padded_head_dim(hd), cfg.block_size, eps)
    if torch.is_grad_enabled() and not layer.input_layernorm.weight.requires_grad:
        h, x = _NormWithSkip.apply(x, layer.input_layernorm.weight, eps)
    else:
        h = _rms_norm(x, layer.input_layernorm.weight, eps)
    w_qkv = torch.cat([attn.q_proj_diff.weight, attn.k_proj_diff.weight, attn.v_proj_diff.weight], 0)
    if rope is not None and ops.fused_qkv_rope_supported(h, hd, padded_head_dim(hd), Q, Hq, Hkv):
        o = DualViewAttentionFused.apply(h, w_qkv, attn.q_norm_diff.weight, attn.k_norm_diff.weight, ar_k,
                                         ar_v, positions, anchors, inv, rope[0], rope[1], meta, doc_start)
    else:
        qkv = F.linear(h, w_qkv)
        o = DualViewAttention.apply(qkv, attn.q_norm_diff.weight, attn.k_norm_diff.weight, ar_k, ar_v,
                                    positions, anchors, inv, meta, doc_start)
    x = _projection_residual(x, o, attn.o_proj_diff.weight)
    w_gu, w_down = layer.mlp.packed_gate_up(), layer.mlp.down_proj.weight
    if _mlp_block_ok(x, w_gu, w_down) and not layer.post_attention_layernorm.weight.requires_grad:
        return _MLPBlock.apply(x, layer.post_attention_layernorm.weight, w_gu, w_down, eps)
    h = _rms_norm(x, layer.post_attention_layernorm.weight, eps)
    if ops.fused_linear_supported(h, w_gu, w_gu.shape[0] // 2):
        act = _GateUpSwiGLU.apply(h, w_gu)
    else:
        act = _SwiGLU.apply(F.linear(h, w_gu))
    return _projection_residual(x, act, w_down)


def _backbone(model):
    """The decoder stack of an OrthrusLM, or the stack itself."""
    return model.model if isinstance(model, OrthrusLM) else model


def _student_stack(backbone, x, cache, anchors, positions, rope, inv, doc_start=None):
    """The differentiable diffusion view: every layer over x [B*Q, d] (the block embeddings) with
    the teacher's keys / values cache[i] = (k, v) [B, Hkv, >= L, D], then the final norm."""
    B, Q = positions.shape
    checkpoint = backbone.gradient_checkpointing and torch.is_grad_enabled()
    for i, (k, v) in enumerate(cache):
        args = (backbone, i, x, k, v, positions, anchors, inv, B, Q, rope, doc_start)
        if checkpoint:
            x = torch.utils.checkpoint.checkpoint(_diffusion_layer, *args, use_reentrant=False)
        else:
            x = _diffusion_layer(*args)
    return _rms_norm(x, backbone.norm.weight, backbone.config.rms_norm_eps)


def _rope_for(x, backbone, rows: int, Q: int):
    cfg = backbone.config
    hd = cfg.head_dim
    if ops.fused_qkv_rope_supported(x, hd, padded_head_dim(hd), Q, cfg.num_attention_heads,
                                    cfg.num_key_value_heads):
        return ops.rope_table(backbone.inv_freq(x.device), rows)
    return None


def diffusion_states(backbone, x: torch.Tensor, cache, positions: torch.Tensor,
                     block_mask) -> torch.Tensor:
    """The diffusion view of OrthrusModel.forward with the training mask and gradients enabled:
    block embeddings x [B*Q, d] at positions [B, Q] over the AR cache (a KVCache holding the
    teacher's keys and values of block_mask.ar_len positions), differentiable w.r.t. the twins
    (orthrus/modeling_orthrus.py:129-189 through flex attention). Returns [B*Q, d]."""
    ar_len = block_mask.ar_len
    if block_mask.block_size != backbone.config.block_size:
        raise ValueError("the mask's block size differs from the model's")
    B, Q = positions.shape
    anchors = block_mask.anchors.to(torch.int64).contiguous()
    layers = [(k[:, :, :ar_len], v[:, :, :ar_len]) for k, v in cache.buffers()]
    rope = _rope_for(x, backbone, ar_len, Q)
    return _student_stack(backbone, x, layers, anchors, positions.contiguous(), rope,
                          backbone.inv_freq(x.device))


def document_starts(assistant_mask: torch.Tensor) -> torch.Tensor:
    """First position of each position's document in packed rows, int32 [B, L]. Rows concatenate
    conversations as prompt then response (orthrus/data.py:43-69), so a new document begins at
    position 0 and wherever an unsupervised token follows a supervised one. A conversation whose
    response is empty shows no boundary and stays joined to its neighbour."""
    m = assistant_mask.to(torch.bool)
    B, L = m.shape
    boundary = torch.zeros_like(m)
    boundary[:, 0] = True
    boundary[:, 1:] = m[:, :-1] & ~m[:, 1:]
    pos = torch.arange(L, device=m.device, dtype=torch.int32).expand(B, L)
    starts = torch.where(boundary, pos, torch.zeros_like(pos))
    return starts.cummax(dim=1).values.to(torch.int32).contiguous()


class TeacherPass:
    """The frozen AR view over the clean rows: final hidden states [B, L, d] and every layer's
    keys / values, plus the rotary tables the diffusion view reuses and the document starts
    (document_starts) both views were masked with, or None."""

    def __init__(self, states, cache, rope, inv, input_ids, doc_start=None):
        self.states, self.cache, self.rope, self.inv = states, cache, rope, inv
        self.input_ids, self.doc_start = input_ids, doc_start


@torch.no_grad()
def teacher_pass(model: OrthrusLM, input_ids: torch.Tensor,
                 doc_start: torch.Tensor | None = None) -> TeacherPass:
    """The AR half of model_states (orthrus/objective.py:247-254, the frozen teacher over the clean
    rows). It depends on the input ids only, so a caller may queue it before the anchors are
    drawn and let the host-side anchor work overlap it. `doc_start` (document_starts, int32
    [B, L]) keeps each query inside its own document; the reference has no such mask (None)."""
    backbone = _backbone(model)
    cfg = backbone.config
    if any(t != "full_attention" for t in getattr(cfg, "layer_types", ["full_attention"])
           [: cfg.num_hidden_layers]):
        raise ValueError("model_states supports full attention layers only (no sliding window)")
    if not input_ids.is_cuda:
        raise ValueError("model_states runs on CUDA tensors only (no CPU fallback)")
    B, L = input_ids.shape
    d = cfg.hidden_size
    inv = backbone.inv_freq(input_ids.device)
    x = F.embedding(input_ids, backbone.embed_tokens.weight).reshape(B * L, d)
    pos = torch.arange(L, device=x.device)[None].expand(B, L).contiguous()
    rope = _rope_for(x, backbone, L, L)
    cache = []
    for i in range(cfg.num_hidden_layers):
        x, k, v = _teacher_layer(backbone, i, x, pos, B, L, inv, rope, doc_start)
        cache.append((k, v))
    states = ops.rms_norm(x, backbone.norm.weight, cfg.rms_norm_eps).view(B, L, d)
    return TeacherPass(states, cache, rope, inv, input_ids, doc_start)


def model_states(model: OrthrusLM, input_ids: torch.Tensor, anchors: torch.Tensor,
                 compiled: bool = False, kernel_options: dict | None = None, *,
                 teacher: TeacherPass | None = None, doc_start: torch.Tensor | None = None):
    """Final hidden states of the diffusion view over all anchor blocks [B, A*K, d] and of the
    frozen AR view over the clean rows [B, L, d] (orthrus/objective.py:228-272). `compiled` and
    `kernel_options` are accepted for signature compatibility; the kernels are fixed. `teacher`
    is the result of teacher_pass(model, input_ids) when the caller queued it already; otherwise
    `doc_start` (document_starts) opts both views into the document mask."""
    backbone = _backbone(model)
    cfg = backbone.config
    if teacher is None:
        teacher = teacher_pass(model, input_ids, doc_start)
    elif teacher.input_ids is not input_ids:
        raise ValueError("the teacher pass was run on other input ids")
    elif doc_start is not None and teacher.doc_start is not doc_start:
        raise ValueError("the teacher pass was run with other document starts")
    K = cfg.block_size
    B, L = input_ids.shape
    d = cfg.hidden_size
    anchors = anchors.to(torch.int64).contiguous()
    positions = (anchors[:, :, None] + torch.arange(K, device=anchors.device)).flatten(1).contiguous()
    block_ids = torch.full((B, anchors.shape[1], K), cfg.mask_token_id, dtype=torch.long,
                           device=anchors.device)
    block_ids[:, :, 0] = input_ids.gather(1, anchors)
    Q = anchors.shape[1] * K
    x = F.embedding(block_ids.flatten(1), backbone.embed_tokens.weight).reshape(B * Q, d)
    student = _student_stack(backbone, x, teacher.cache, anchors, positions, teacher.rope, teacher.inv,
                             teacher.doc_start)
    return student.view(B, Q, d), teacher.states


@torch.no_grad()
def reference_states(model: OrthrusLM, input_ids: torch.Tensor, anchors: torch.Tensor):
    """model_states through the module forward (OrthrusLM.forward with the dual-view mask), as the
    reference's reference_states (orthrus/objective.py:275-295)."""
    K, mask_token_id = model.config.block_size, model.config.mask_token_id
    B, L = input_ids.shape
    teacher = model(input_ids=input_ids, use_cache=True, logits_to_keep=1)
    positions = anchors[:, :, None] + torch.arange(K, device=anchors.device)
    block_ids = torch.full_like(positions, mask_token_id)
    block_ids[:, :, 0] = input_ids.gather(1, anchors)
    student = model(input_ids=block_ids.flatten(1), position_ids=positions.flatten(1),
                    past_key_values=teacher.past_key_values, use_cache=False, is_diffusion_pass=True,
                    ar_seq_len=L, flex_block_mask=build_block_mask(anchors, L, K), logits_to_keep=1)
    return student.last_hidden_state, teacher.last_hidden_state


class _FusedKL(torch.autograd.Function):
    """LM head + KL with the kernel's per-offset statistics; gradient computed in the forward."""

    @staticmethod
    def forward(ctx, student, teacher, index, weight, chunk_size, row_weight, offsets, num_offsets):
        total, kl_rows, agree, grad, kbo, abo = ops.lmhead_kl(
            student, teacher, index, weight, row_weight, offsets, num_offsets,
            need_grad=ctx.needs_input_grad[0], chunk_rows=max(int(chunk_size), 128))
        ctx.save_for_backward(grad)
        outs = [kl_rows, agree] + ([kbo, abo] if offsets is not None else [])
        ctx.mark_non_differentiable(*outs)
        if offsets is None:
            return total, kl_rows, agree
        return total, kl_rows, agree, kbo, abo

    @staticmethod
    def backward(ctx, grad_total, *unused):
        (grad,) = ctx.saved_tensors
        if grad is None:
            return (None,) * 8
        return ops.lmhead_kl_backward(grad, grad_total), None, None, None, None, None, None, None


class FusedLinearForwardKL:
    """sum_r w_r KL(softmax(W teacher[index[r]]) || softmax(W student[r])), per-row KL and top-1
    agreement (orthrus/objective.py:338-392). Same apply() signature and outputs (total,
    kl_rows, agree), differentiable w.r.t. the student rows; `compiled` is ignored."""

    @staticmethod
    def apply(student, teacher, index, weight, chunk_size, compiled=False, row_weight=None):
        return _FusedKL.apply(student, teacher, index, weight, chunk_size, row_weight, None, 0)


class SupervisedLayout:
    """The supervised block positions of a batch, settled before the forward: kept (row, anchor,
    offset) indices ordered by their unique target position, the gather indices of the student
    and teacher rows, per-offset counts and weights (orthrus/objective.py:418-429,448)."""

    def __init__(self, assistant_mask, anchors, valid, K, gamma):
        batch, seq_len = assistant_mask.shape
        self.keep = supervision_mask(assistant_mask, anchors, valid, K)
        targets = anchors[:, :, None] + torch.arange(K - 1, device=anchors.device)
        targets = targets + seq_len * torch.arange(batch, device=anchors.device)[:, None, None]
        kept = torch.nonzero(self.keep.flatten()).squeeze(1)  # flat (row, anchor, offset) indices
        self.positions, index = torch.unique(targets.flatten()[kept], return_inverse=True)
        order = torch.argsort(index, stable=True)
        kept = kept[order]
        self.index = index[order]
        self.offsets = kept % (K - 1)
        self.student_rows = (kept // (K - 1)) * K + self.offsets  # row in [B * A * K]
        self.tokens_by_offset = torch.bincount(self.offsets, minlength=K - 1)
        weights = position_weights(K, gamma, self.keep.device)
        self.row_weight = weights[self.offsets] if weights is not None else None
        self.count = self.keep.sum()

    def tensors(self) -> list[torch.Tensor]:
        return [t for t in (self.keep, self.positions, self.index, self.offsets, self.student_rows,
                            self.tokens_by_offset, self.row_weight, self.count) if t is not None]


def orthrus_loss(model: OrthrusLM, input_ids: torch.Tensor, assistant_mask: torch.Tensor,
                 anchors: torch.Tensor, valid: torch.Tensor, kl_chunk_size: int,
                 compiled: bool = False, kernel_options: dict | None = None, gamma: float = 0.0, *,
                 teacher: TeacherPass | None = None, layout: SupervisedLayout | None = None,
                 document_mask: bool = False):
    """Mean (or position-weighted mean) forward KL over supervised block positions and its
    statistics (orthrus/objective.py:395-453). `teacher` (teacher_pass) and `layout`
    (SupervisedLayout) may be prepared by the caller: the training step queues the teacher first
    and settles the layout's host reads on a side stream meanwhile. `document_mask` (off, as in
    the reference) keeps attention inside each packed conversation (document_starts); a prepared
    teacher carries its own choice."""
    K = model.config.block_size
    # The supervised rows depend on the inputs only. Their layout is settled before the forward is
    # queued, so its host reads (the kept-row and unique-target counts, bincount's size) happen
    # while the device is idle rather than between the forward and the LM head.
    if layout is None:
        layout = SupervisedLayout(assistant_mask, anchors, valid, K, gamma)
    doc_start = None
    if document_mask and teacher is None:
        doc_start = document_starts(assistant_mask)
    student, teacher = model_states(model, input_ids, anchors, compiled, kernel_options,
                                    teacher=teacher, doc_start=doc_start)
    hidden = student.shape[-1]
    row_weight = layout.row_weight
    total, kl_rows, agree, kl_by_offset, agree_by_offset = _FusedKL.apply(
        student.reshape(-1, hidden).index_select(0, layout.student_rows),
        teacher.flatten(0, 1)[layout.positions].to(student.dtype),
        layout.index,
        model.lm_head.weight,
        kl_chunk_size,
        row_weight,
        layout.offsets,
        K - 1,
    )
    count = layout.count
    norm = row_weight.sum() if row_weight is not None else count.float()
    stats = {
        "tokens": count.detach(),
        "kl_sum": kl_rows.sum(),
        "weighted_kl_sum": total.detach(),
        "weight_sum": norm.detach(),
        "agree": agree.sum(),
        "kl_by_offset": kl_by_offset,
        "agree_by_offset": agree_by_offset,
        "tokens_by_offset": layout.tokens_by_offset,
        "valid_anchors": valid.float().mean(),
    }
    return total / norm.clamp_min(1e-6), stats
