"""fp32 CPU restatement of the Orthrus dual-view hot path (test infrastructure only).

Every function states the reference behaviour it restates as ``file:line`` inside the reference
project (ekonst41/orthrus-training); ``tf:`` marks the third-party Qwen3 module math in
``transformers/models/qwen3/modeling_qwen3.py`` that the reference calls.

The model is a plain ``dict`` of tensors keyed by the reference's own parameter names
(``model.layers.{i}.self_attn.q_proj_diff.weight`` ...), so a state dict of the reference's
``OrthrusLM`` or of ``orthrus_training_b200.modeling_orthrus.OrthrusLM`` can be passed directly.
All arithmetic runs in the dtype of the tensors given (fp32 for parity checks).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

__all__ = [
    "OracleConfig",
    "rms_norm",
    "rope_cos_sin",
    "apply_rope",
    "dense_block_mask",
    "masked_attention",
    "attention_inputs",
    "ar_layer",
    "diffusion_layer",
    "model_states",
    "sample_anchors",
    "supervision_mask",
    "position_weights",
    "fused_linear_forward_kl",
    "orthrus_loss",
    "OracleCache",
    "forward_logits",
    "ar_generate",
    "diffusion_generate",
    "decode_base",
    "lr_scale",
    "sampling_probs",
    "rejection_accept",
]


@dataclass(frozen=True)
class OracleConfig:
    """Shape of a Qwen3-architecture Orthrus model (reference: Qwen3Config + block_size and
    mask_token_id, orthrus/modeling_orthrus.py:12-14,44)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 32
    mask_token_id: int = 0

    @staticmethod
    def from_hf(config) -> "OracleConfig":
        theta = getattr(config, "rope_theta", None)
        if theta is None:
            theta = config.rope_parameters["rope_theta"]
        return OracleConfig(
            vocab_size=config.vocab_size,
            hidden_size=config.hidden_size,
            intermediate_size=config.intermediate_size,
            num_layers=config.num_hidden_layers,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            head_dim=config.head_dim,
            rms_norm_eps=config.rms_norm_eps,
            rope_theta=float(theta),
            block_size=config.block_size,
            mask_token_id=config.mask_token_id,
        )


def _p(params: dict, layer: int, name: str) -> torch.Tensor:
    return params[f"model.layers.{layer}.{name}"]


# --- Qwen3 layer math -------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3RMSNorm (tf:50-64; reference orthrus/objective.py:128-133): normalise in fp32, cast
    back to the input dtype, then scale by the weight."""
    dtype = x.dtype
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return weight * xf.to(dtype)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, dtype=torch.float32):
    """Default RoPE tables (tf Qwen3RotaryEmbedding: inv_freq = 1/theta^(2i/hd), freqs =
    pos * inv_freq, emb = cat(freqs, freqs)); positions [B, T] -> cos, sin [B, T, hd]."""
    inv_freq = 1.0 / (
        theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim)
    )
    freqs = positions.float()[..., None] * inv_freq.to(positions.device)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """tf apply_rotary_pos_emb on [B, H, T, hd] with cos/sin [B, T, hd]:
    x*cos + rotate_half(x)*sin, rotate_half(x) = cat(-x2, x1)."""
    cos, sin = cos[:, None], sin[:, None]
    half = x.shape[-1] // 2
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rotated * sin


def attention_inputs(h, params, layer, suffix, cos, sin, cfg: OracleConfig):
    """q, k, v [B, heads, T, hd] after q/k RMSNorm and RoPE (orthrus/objective.py:136-143)."""
    hd = cfg.head_dim
    shape = (*h.shape[:-1], -1, hd)
    attn = f"self_attn.{{}}{suffix}.weight"
    q = F.linear(h, _p(params, layer, attn.format("q_proj"))).view(shape)
    k = F.linear(h, _p(params, layer, attn.format("k_proj"))).view(shape)
    v = F.linear(h, _p(params, layer, attn.format("v_proj"))).view(shape)
    q = rms_norm(q, _p(params, layer, attn.format("q_norm")), cfg.rms_norm_eps).transpose(1, 2)
    k = rms_norm(k, _p(params, layer, attn.format("k_norm")), cfg.rms_norm_eps).transpose(1, 2)
    v = v.transpose(1, 2)
    return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v


def mlp_residual(x, params, layer, cfg: OracleConfig):
    """x + down(silu(gate(n(x))) * up(n(x))) (orthrus/objective.py:146-149; tf Qwen3MLP)."""
    h = rms_norm(x, _p(params, layer, "post_attention_layernorm.weight"), cfg.rms_norm_eps)
    gate = F.linear(h, _p(params, layer, "mlp.gate_proj.weight"))
    up = F.linear(h, _p(params, layer, "mlp.up_proj.weight"))
    return x + F.linear(F.silu(gate) * up, _p(params, layer, "mlp.down_proj.weight"))


def masked_attention(q, k, v, mask: torch.Tensor | None, causal: bool = False):
    """softmax(q k^T / sqrt(hd) + mask) v with GQA (keys repeated per query group): the dense SDPA
    path the reference runs on CPU (orthrus/modeling_orthrus.py:84-85; tf:184-219).
    mask: bool [B or 1, Q, Kv] (True = visible) or None."""
    groups = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(groups, dim=1)
    v = v.repeat_interleave(groups, dim=1)
    scores = (q @ k.transpose(-1, -2)) / (q.shape[-1] ** 0.5)
    if causal:
        ql, kl = q.shape[2], k.shape[2]
        mask_c = torch.ones(ql, kl, dtype=torch.bool, device=q.device).tril(kl - ql)
        scores = scores.masked_fill(~mask_c, float("-inf"))
    if mask is not None:
        scores = scores.masked_fill(~mask[:, None], float("-inf"))
    return torch.softmax(scores.float(), dim=-1).to(q.dtype) @ v


def dense_block_mask(anchors: torch.Tensor, ar_len: int, block_size: int) -> torch.Tensor:
    """Dual-pass training mask materialised densely, [B, A*K, ar_len + A*K] bool
    (orthrus/modeling_orthrus.py:58-74): query of block b sees AR keys strictly before
    anchors[:, b] and every key of its own block, never another block."""
    batch, blocks = anchors.shape
    q_len = blocks * block_size
    q = torch.arange(q_len, device=anchors.device)[:, None]
    kv = torch.arange(ar_len + q_len, device=anchors.device)[None, :]
    block = q // block_size
    ar_visible = (kv < ar_len) & (kv < anchors[:, block])
    same = (kv >= ar_len) & ((kv - ar_len) // block_size == block)
    return ar_visible | same


def ar_layer(x, cos, sin, params, layer, cfg: OracleConfig):
    """Frozen causal layer over the whole packed row, returns (x, k, v)
    (orthrus/objective.py:152-157)."""
    h = rms_norm(x, _p(params, layer, "input_layernorm.weight"), cfg.rms_norm_eps)
    q, k, v = attention_inputs(h, params, layer, "", cos, sin, cfg)
    out = masked_attention(q, k, v, None, causal=True)
    x = x + F.linear(out.transpose(1, 2).flatten(2), _p(params, layer, "self_attn.o_proj.weight"))
    return mlp_residual(x, params, layer, cfg), k, v


def diffusion_layer(x, cos, sin, ar_k, ar_v, mask, params, layer, cfg: OracleConfig):
    """Twin attention over cat([AR cache, block keys]) with the dual-pass mask, shared MLP
    (orthrus/objective.py:160-165)."""
    h = rms_norm(x, _p(params, layer, "input_layernorm.weight"), cfg.rms_norm_eps)
    q, k, v = attention_inputs(h, params, layer, "_diff", cos, sin, cfg)
    out = masked_attention(q, torch.cat([ar_k, k], 2), torch.cat([ar_v, v], 2), mask)
    o = _p(params, layer, "self_attn.o_proj_diff.weight")
    x = x + F.linear(out.transpose(1, 2).flatten(2), o)
    return mlp_residual(x, params, layer, cfg)


def model_states(params, cfg: OracleConfig, input_ids, anchors):
    """(student [B, A*K, d], teacher [B, L, d]) final hidden states (orthrus/objective.py:228-272):
    teacher = causal pass over the clean rows without grad; block ids = [anchor token, mask x K-1]
    at positions anchor..anchor+K-1; student = diffusion layers with the dual-pass mask."""
    K = cfg.block_size
    batch, seq_len = input_ids.shape
    embed = params["model.embed_tokens.weight"]
    with torch.no_grad():
        x = F.embedding(input_ids, embed)
        pos = torch.arange(seq_len, device=x.device)[None].expand(batch, -1)
        cos, sin = rope_cos_sin(pos, cfg.head_dim, cfg.rope_theta, x.dtype)
        cache = []
        for layer in range(cfg.num_layers):
            x, k, v = ar_layer(x, cos, sin, params, layer, cfg)
            cache.append((k, v))
        teacher = rms_norm(x, params["model.norm.weight"], cfg.rms_norm_eps)
    positions = anchors[:, :, None] + torch.arange(K, device=anchors.device)
    block_ids = torch.full_like(positions, cfg.mask_token_id)
    block_ids[:, :, 0] = input_ids.gather(1, anchors)
    x = F.embedding(block_ids.flatten(1), embed)
    cos, sin = rope_cos_sin(positions.flatten(1), cfg.head_dim, cfg.rope_theta, x.dtype)
    mask = dense_block_mask(anchors, seq_len, K)
    for layer, (k, v) in enumerate(cache):
        x = diffusion_layer(x, cos, sin, k, v, mask, params, layer, cfg)
    return rms_norm(x, params["model.norm.weight"], cfg.rms_norm_eps), teacher


# --- anchors, supervision and the KL objective --------------------------------------------------


def sample_anchors(assistant_mask, block_size, num_anchors, generator):
    """Sorted anchors drawn without replacement from assistant positions in [1, L-K]; spare slots
    repeat the last anchor and are invalid (orthrus/objective.py:37-63). Uses the same torch RNG
    calls, so one generator state gives the reference's anchors."""
    batch, seq_len = assistant_mask.shape
    slots = min(num_anchors, seq_len - block_size)
    device = assistant_mask.device
    positions = torch.arange(1, seq_len - block_size + 1, device=device)
    anchors = torch.zeros((batch, slots), dtype=torch.long, device=device)
    valid = torch.zeros((batch, slots), dtype=torch.bool, device=device)
    for row in range(batch):
        candidates = positions[assistant_mask[row, positions]]
        has_targets = candidates.numel() > 0
        if not has_targets:
            candidates = positions
        order = torch.randperm(candidates.numel(), generator=generator, device=device)
        picked = candidates[order[:slots]].sort().values
        anchors[row, : len(picked)] = picked
        anchors[row, len(picked):] = picked[-1]
        valid[row, : len(picked)] = has_targets
    return anchors, valid


def supervision_mask(assistant_mask, anchors, valid, block_size):
    """keep[b, a, i] = mask[anchor+i+1] & valid[b, a], i = 0..K-2 (orthrus/objective.py:66-73)."""
    targets = anchors[:, :, None] + torch.arange(1, block_size, device=anchors.device)
    keep = assistant_mask.gather(1, targets.flatten(1)).view_as(targets)
    return keep & valid[:, :, None]


def position_weights(block_size, gamma, device=None):
    """exp(-i/gamma) for i = 0..K-2, None for gamma <= 0 (orthrus/objective.py:76-81)."""
    if gamma <= 0:
        return None
    return torch.exp(-torch.arange(block_size - 1, device=device, dtype=torch.float32) / gamma)


def fused_linear_forward_kl(student, teacher, index, weight, row_weight=None):
    """sum_r w_r KL(softmax(W t[index[r]]) || softmax(W s[r])), per-row KL, top-1 agreement and
    d(total)/d(student) = w_r (p_s - p_t) W (orthrus/objective.py:303-392), unchunked, logits in
    fp32. Returns (total, kl_rows, agree, grad)."""
    ls = student.float() @ weight.float().t()
    lt = teacher.float() @ weight.float().t()
    log_pt = lt.log_softmax(-1)[index]
    log_ps = ls.log_softmax(-1)
    p_t = log_pt.exp()
    kl = (p_t * (log_pt - log_ps)).sum(-1)
    agree = ls.argmax(-1) == lt.argmax(-1)[index]
    diff = log_ps.exp() - p_t
    if row_weight is not None:
        diff = diff * row_weight[:, None]
    grad = diff @ weight.float()
    total = (kl * row_weight).sum() if row_weight is not None else kl.sum()
    return total, kl, agree, grad


def orthrus_loss(params, cfg: OracleConfig, input_ids, assistant_mask, anchors, valid, gamma=0.0):
    """Mean (or position-weighted mean) forward KL over supervised block positions and its stats
    (orthrus/objective.py:395-453). Differentiable w.r.t. the twin parameters through autograd:
    the gradient of the KL sum w.r.t. the student logits is w (p_s - p_t), as in the reference's
    fused backward."""
    K = cfg.block_size
    batch, seq_len = input_ids.shape
    student, teacher = model_states(params, cfg, input_ids, anchors)
    hidden = student.shape[-1]
    student = student.view(batch, -1, K, hidden)[:, :, :-1]
    keep = supervision_mask(assistant_mask, anchors, valid, K)
    targets = anchors[:, :, None] + torch.arange(K - 1, device=anchors.device)
    targets = targets + seq_len * torch.arange(batch, device=anchors.device)[:, None, None]
    positions, index = torch.unique(targets[keep], return_inverse=True)
    order = torch.argsort(index, stable=True)
    offsets = torch.arange(K - 1, device=keep.device).expand_as(keep)[keep][order]
    weights = position_weights(K, gamma, keep.device)
    row_weight = weights[offsets] if weights is not None else None
    weight = params["lm_head.weight"] if "lm_head.weight" in params else params[
        "model.embed_tokens.weight"]
    s_rows = student[keep][order]
    t_rows = teacher.flatten(0, 1)[positions].to(student.dtype)
    idx = index[order]
    ls = s_rows.float() @ weight.float().t()
    lt = t_rows.float() @ weight.float().t()
    log_pt = lt.log_softmax(-1)[idx]
    log_ps = ls.log_softmax(-1)
    kl_rows = (log_pt.exp() * (log_pt - log_ps)).sum(-1)
    agree = ls.argmax(-1) == lt.argmax(-1)[idx]
    total = (kl_rows * row_weight).sum() if row_weight is not None else kl_rows.sum()
    count = keep.sum()
    norm = row_weight.sum() if row_weight is not None else count.float()
    kl_d = kl_rows.detach()
    stats = {
        "tokens": count,
        "kl_sum": kl_d.sum(),
        "weighted_kl_sum": total.detach(),
        "weight_sum": norm.detach(),
        "agree": agree.sum(),
        "kl_by_offset": torch.zeros(K - 1).index_add_(0, offsets, kl_d),
        "agree_by_offset": torch.bincount(offsets[agree], minlength=K - 1),
        "tokens_by_offset": torch.bincount(offsets, minlength=K - 1),
        "valid_anchors": valid.float().mean(),
    }
    return total / norm.clamp_min(1e-6), stats


def lr_scale(step: int, warmup: int, total: int, min_ratio: float) -> float:
    """Linear warmup then cosine decay to min_ratio (orthrus/train.py:71-76)."""
    import math

    if warmup > 0 and step < warmup:
        return (step + 1) / warmup
    progress = min(1.0, max(0.0, (step - warmup) / max(1, total - warmup)))
    return min_ratio + (1.0 - min_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress))


# --- decoding ----------------------------------------------------------------------------------


class OracleCache:
    """Per-layer (keys, values) [B, Hkv, len, hd] with crop, the DynamicCache operations the
    reference uses (update = append along the sequence, crop = keep a prefix)."""

    def __init__(self, num_layers: int):
        self.layers = [None] * num_layers

    def length(self) -> int:
        return 0 if self.layers[0] is None else self.layers[0][0].shape[2]

    def append(self, layer, k, v):
        if self.layers[layer] is None:
            self.layers[layer] = (k, v)
        else:
            pk, pv = self.layers[layer]
            self.layers[layer] = (torch.cat([pk, k], 2), torch.cat([pv, v], 2))
        return self.layers[layer]

    def crop(self, length: int) -> None:
        """truncate_cache (orthrus/modeling_orthrus.py:107-111)."""
        self.layers = [
            None if kv is None else (kv[0][:, :, :length], kv[1][:, :, :length])
            for kv in self.layers
        ]


def forward_logits(params, cfg: OracleConfig, ids, positions, cache: OracleCache, diffusion=False):
    """OrthrusLM.forward over ids at positions with a cache (orthrus/modeling_orthrus.py:238-362):
    AR view = causal over cache + new tokens, appended to the cache (HF Qwen3Attention with
    DynamicCache.update); diffusion view = twin q/k/v over cat([cache, block]) with no mask and no
    cache update (orthrus/modeling_orthrus.py:153-189). Returns fp32 logits [B, T, V]."""
    x = F.embedding(ids, params["model.embed_tokens.weight"])
    cos, sin = rope_cos_sin(positions, cfg.head_dim, cfg.rope_theta, x.dtype)
    for layer in range(cfg.num_layers):
        h = rms_norm(x, _p(params, layer, "input_layernorm.weight"), cfg.rms_norm_eps)
        if diffusion:
            q, k, v = attention_inputs(h, params, layer, "_diff", cos, sin, cfg)
            ck, cv = cache.layers[layer]
            out = masked_attention(q, torch.cat([ck, k], 2), torch.cat([cv, v], 2), None)
            o = _p(params, layer, "self_attn.o_proj_diff.weight")
        else:
            q, k, v = attention_inputs(h, params, layer, "", cos, sin, cfg)
            ck, cv = cache.append(layer, k, v)
            out = masked_attention(q, ck, cv, None, causal=True)
            o = _p(params, layer, "self_attn.o_proj.weight")
        x = x + F.linear(out.transpose(1, 2).flatten(2), o)
        x = mlp_residual(x, params, layer, cfg)
    x = rms_norm(x, params["model.norm.weight"], cfg.rms_norm_eps)
    weight = params.get("lm_head.weight", params["model.embed_tokens.weight"])
    return (x @ weight.t()).float()


@torch.no_grad()
def ar_generate(params, cfg: OracleConfig, prompt: torch.Tensor, max_new_tokens: int, eos=(),
                gaps: list | None = None):
    """Plain greedy decoding with the frozen AR view (orthrus/evaluate.py:59-76): prompt [1, P] ->
    list of new tokens (stops after an EOS token or max_new_tokens). When `gaps` is a list, the
    top-1 minus top-2 logit gap of every token is appended to it (the reference returns the same
    gaps to tell rounding ties from bugs)."""
    cache = OracleCache(cfg.num_layers)
    pos = torch.arange(prompt.shape[1])[None]
    logits = forward_logits(params, cfg, prompt, pos, cache)
    tokens = []
    while True:
        token = int(logits[0, -1].argmax())
        tokens.append(token)
        if gaps is not None:
            top2 = logits[0, -1].topk(2).values
            gaps.append(float(top2[0] - top2[1]))
        if token in eos or len(tokens) == max_new_tokens:
            return tokens
        pos = torch.tensor([[cache.length()]])
        logits = forward_logits(params, cfg, torch.tensor([[token]]), pos, cache)


@torch.no_grad()
def diffusion_generate(params, cfg: OracleConfig, prompt, max_new_tokens, eos=(), drafts=None):
    """Greedy Orthrus decoding (orthrus/modeling_orthrus.py:404-534, temperature 0): draft K-1
    tokens with the diffusion view over [anchor, mask x K-1], verify [anchor, drafts] causally,
    accept the longest agreeing prefix plus the AR bonus token, crop the cache.

    drafts: optional callable (start, block_len) -> list of block_len-1 draft tokens that replaces
    the diffusion pass (the scripted-draft mode of tests/test_decoding.py:127-155).
    Returns (tokens [1, n], accepted per cycle)."""
    K, mask_id = cfg.block_size, cfg.mask_token_id
    prompt_len = prompt.shape[1]
    max_length = prompt_len + max_new_tokens
    cache = OracleCache(cfg.num_layers)
    output = torch.full((1, max_length + K), mask_id, dtype=torch.long)
    output[:, :prompt_len] = prompt
    accepted_log = []
    logits = forward_logits(params, cfg, prompt, torch.arange(prompt_len)[None], cache)
    start = prompt_len
    nxt = int(logits[0, -1].argmax())
    output[0, start] = nxt
    if nxt in eos:
        return output[:, : start + 1], accepted_log
    while start < max_length - 1:
        block_len = min(K, max_length - start)
        positions = torch.arange(start, start + block_len)[None]
        if drafts is not None:
            draft_tokens = torch.tensor([list(drafts(start, block_len))], dtype=torch.long)
        else:
            block = torch.full((1, block_len), mask_id, dtype=torch.long)
            block[0, 0] = output[0, start]
            dl = forward_logits(params, cfg, block, positions, cache, diffusion=True)
            draft_tokens = dl[:, :-1].argmax(-1)
        proposed = torch.cat([output[:, start:start + 1], draft_tokens], 1)
        vl = forward_logits(params, cfg, proposed, positions, cache)
        ar_tokens = vl.argmax(-1)
        matches = draft_tokens == ar_tokens[:, :-1]
        accepted = int(matches.cumprod(1).sum())
        nxt = int(ar_tokens[0, accepted])
        accepted_log.append(accepted)
        kept = proposed[0, : accepted + 1].tolist()
        hits = [i for i, t in enumerate(kept) if t in eos]
        if hits:
            end = start + hits[0] + 1
            output[0, start:end] = torch.tensor(kept[: hits[0] + 1])
            return output[:, :end], accepted_log
        output[0, start:start + accepted + 1] = torch.tensor(kept)
        start += accepted + 1
        cache.crop(start)
        if start < max_length:
            output[0, start] = nxt
            if nxt in eos:
                return output[:, : start + 1], accepted_log
    return output[:, :max_length], accepted_log


def decode_base(params, cfg, prompt_ids: list, max_new_tokens: int, eos=(), drafts=None):
    """decoding.decode with the base strategy (orthrus/decoding.py:391-429): prefill, then per
    cycle draft -> verify -> accept, where acceptance stops after an accepted EOS (_verify,
    orthrus/decoding.py:336-351) and _advance (:354-369) appends the kept drafts and the AR bonus.
    drafts: optional callable (start, block_len) -> block_len-1 scripted draft tokens.
    Returns (new tokens, accepted per cycle, forward passes)."""
    K, mask_id = cfg.block_size, cfg.mask_token_id
    eos = set(eos)
    prompt_len = len(prompt_ids)
    max_length = prompt_len + max_new_tokens
    cache = OracleCache(cfg.num_layers)
    logits = forward_logits(params, cfg, torch.tensor([prompt_ids]),
                            torch.arange(prompt_len)[None], cache)
    tokens = [int(logits[0, -1].argmax())]
    passes = 1
    accepted_log = []
    done = tokens[-1] in eos
    start = prompt_len
    while not done and start < max_length - 1:
        block_len = min(K, max_length - start)
        root = tokens[-1]
        positions = torch.arange(start, start + block_len)[None]
        if drafts is not None:
            draft_tokens = list(drafts(start, block_len))
        else:
            block = torch.full((1, block_len), mask_id, dtype=torch.long)
            block[0, 0] = root
            dl = forward_logits(params, cfg, block, positions, cache, diffusion=True)
            draft_tokens = dl[0, :-1].argmax(-1).tolist()
        passes += 1
        proposed = torch.tensor([[root] + draft_tokens])
        preds = forward_logits(params, cfg, proposed, positions, cache)[0].argmax(-1).tolist()
        passes += 1
        accepted = 0
        while accepted < len(draft_tokens) and draft_tokens[accepted] == preds[accepted]:
            accepted += 1
            if draft_tokens[accepted - 1] in eos:
                break
        cache.crop(start + 1 + accepted)
        accepted_log.append(accepted)
        kept, bonus = draft_tokens[:accepted], preds[accepted]
        hit = next((i for i, t in enumerate(kept) if t in eos), None)
        if hit is not None:
            tokens.extend(kept[: hit + 1])
            break
        tokens.extend(kept)
        start += len(kept) + 1
        if start < max_length:
            tokens.append(bonus)
            if bonus in eos:
                break
        done = start >= max_length - 1
    return tokens, accepted_log, passes


def sampling_probs(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """The sampling distribution of diffusion_generate's `pick` (orthrus/modeling_orthrus.py:
    437-449): logits / temperature; keep the values >= the top_k-th largest (ties kept); then keep
    the smallest descending prefix whose softmax mass exceeds top_p (the first token always kept);
    softmax over what is left. logits [..., V] -> probs [..., V] fp32."""
    x = logits.float() / temperature
    if top_k > 0:
        kth = torch.topk(x, min(top_k, x.shape[-1])).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    if top_p < 1.0:
        sx, order = torch.sort(x, descending=True)
        cum = torch.cumsum(torch.softmax(sx, dim=-1), dim=-1)
        drop = torch.zeros_like(cum, dtype=torch.bool)
        drop[..., 1:] = cum[..., :-1] > top_p
        x = x.masked_fill(torch.zeros_like(drop).scatter(-1, order, drop), float("-inf"))
    return torch.softmax(x, dim=-1)


def rejection_accept(draft_tokens, draft_probs, ar_probs, uniforms):
    """Exact rejection sampling of one verify cycle (orthrus/modeling_orthrus.py:498-511): draft i
    is kept while u_i < min(1, p_i(d_i) / max(q_i(d_i), 1e-8)); at the first rejection the next
    token comes from the normalised residual max(p - q, 0) (p itself if the residual's mass is
    <= 1e-5); after a full accept from p of the next position. draft_tokens [n], draft_probs
    [n, V], ar_probs [n + 1, V], uniforms [n] -> (accepted, next-token distribution [V])."""
    accepted = 0
    for i in range(draft_tokens.shape[0]):
        t = int(draft_tokens[i])
        ratio = ar_probs[i, t] / draft_probs[i, t].clamp_min(1e-8)
        if float(uniforms[i]) < float(ratio.clamp(max=1.0)):
            accepted += 1
        else:
            break
    target = ar_probs[accepted]
    if accepted < draft_tokens.shape[0]:
        residual = (target - draft_probs[accepted]).clamp_min(0.0)
        target = residual / residual.sum() if residual.sum() > 1e-5 else target
    return accepted, target
