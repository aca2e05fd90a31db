"""Orthrus dual-view model on the Blackwell kernels: drop-in for orthrus/modeling_orthrus.py.

Same class names, parameter names (so reference checkpoints and state dicts load unchanged), config
fields (a Qwen3 config plus ``block_size`` and ``mask_token_id``) and call signatures as the
reference module. The arithmetic behind them runs in ``liborthrus_b200.so``:

- q/k RMSNorm + RoPE + cache write: ``ops.qkv_prep`` (orthrus/modeling_orthrus.py:153-159),
- attention: ``ops.attention_fwd`` with the causal, dual-view or draft mask
  (orthrus/modeling_orthrus.py:58-85,167-188),
- projections: ``ops.linear`` / ``ops.linear_swiglu`` for bf16 (the persistent tcgen05 kernel, no
  split-K, the residual add and SwiGLU in its epilogue) and ``ops.gemm`` otherwise; the LM head:
  ``ops.gemm`` (fp32 logits). Every one gives per-row results that do not depend on the number of
  rows, so a K-token verification reproduces a one-token greedy pass bit for bit,
- RMSNorm and the SwiGLU activation: row-local kernels of fixed reduction order.

There is no CPU path: every forward requires CUDA tensors and the built library.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

from orthrus_training_b200 import ops
from orthrus_training_b200._lib import MASK_CAUSAL, MASK_DRAFT, MASK_DUAL, MASK_TREE
from orthrus_training_b200.kv_cache import KVCache

try:  # the reference configures the model with a plain Qwen3Config plus two fields
    from transformers import Qwen3Config as OrthrusConfig
except ImportError:  # pragma: no cover - transformers is part of the image
    OrthrusConfig = None

DIFF_MODULES = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")
DynamicCache = KVCache  # the cache class the reference passes around (transformers DynamicCache)


def _theta(config) -> float:
    theta = getattr(config, "rope_theta", None)
    if theta is None:
        theta = config.rope_parameters["rope_theta"]
    return float(theta)


def padded_head_dim(head_dim: int) -> int:
    """Head dim as stored for the attention kernels: 64 or 128 (zero padded), or the head dim itself
    when it is larger than 128 is not supported."""
    if head_dim > 128:
        raise ValueError("head_dim > 128 is not supported by the attention kernels")
    return 64 if head_dim <= 64 else 128


class RMSNorm(nn.Module):
    """Qwen3RMSNorm parameters (transformers Qwen3RMSNorm); forward runs the row kernel."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.variance_epsilon)


def _positions_of(position_ids, B: int, T: int, start: int, device) -> torch.Tensor:
    """int64 [B, T] positions: the given ids broadcast over the batch, else start .. start + T."""
    if position_ids is None:
        position_ids = torch.arange(start, start + T, device=device)[None]
    return position_ids.to(device=device, dtype=torch.int64).expand(B, T).contiguous()


def _cached_weight(owner: nn.Module, key, tensors: list[torch.Tensor]) -> torch.Tensor:
    """torch.cat(tensors) cached on the module (inference only), rebuilt when one of them changes
    (its version counter or storage)."""
    stamp = tuple((t._version, t.data_ptr()) for t in tensors)
    cache = owner.__dict__.setdefault("_packed_weights", {})
    hit = cache.get(key)
    if hit is None or hit[0] != stamp:
        with torch.no_grad():
            hit = (stamp, torch.cat(list(tensors), 0).contiguous())
        cache[key] = hit
    return hit[1]


def _few_row_kernel(rows: int, cols: int, K: int) -> bool:
    """Whether a projection of `rows` rows, `cols` output (accumulator) columns and depth K runs on
    the few-row kernel: when 128 x 256 tiles would leave most SMs idle and K is a multiple of 64.
    The two kernels give every row the same bits, so the choice never changes a result."""
    return K % 64 == 0 and -(-rows // 128) * -(-cols // 256) < 74


def _project(a: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """a @ w^T (+ residual). Every kernel here is batch-invariant: a row's result does not depend
    on how many rows the call has."""
    if a.dtype == torch.bfloat16 and ops.fused_linear_supported(a, w, w.shape[0]):
        return ops.linear(a, w, residual=residual, skinny=_few_row_kernel(a.shape[0], w.shape[0], a.shape[1]))
    y = ops.gemm(a, w)
    return y if residual is None else ops.add(residual, y)


class OrthrusMLP(nn.Module):
    """Qwen3MLP (down(silu(gate(x)) * up(x))) on the fused gate/up + SwiGLU kernel."""

    def __init__(self, config):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)

    def packed_gate_up(self) -> torch.Tensor:
        """[gate; up] as one [2F, d] weight (cached)."""
        return _cached_weight(self, "gate_up", [self.gate_proj.weight, self.up_proj.weight])

    def activation(self, h: torch.Tensor) -> torch.Tensor:
        """silu(h @ gate^T) * (h @ up^T) for h [rows, d]."""
        w = self.packed_gate_up()
        if h.dtype == torch.bfloat16 and ops.fused_linear_supported(h, w, w.shape[0] // 2):
            return ops.linear_swiglu(h, w, skinny=_few_row_kernel(h.shape[0], w.shape[0], h.shape[1]))
        return ops.silu_mul(ops.gemm(h, w))

    @torch.no_grad()
    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        h = x.reshape(-1, shape[-1]).contiguous()
        r = None if residual is None else residual.reshape(-1, shape[-1]).contiguous()
        return _project(self.activation(h), self.down_proj.weight, r).view(shape)


class OrthrusAttention(nn.Module):
    """Frozen autoregressive attention and its trainable diffusion twin (*_diff), with the
    parameter layout and forward signature of orthrus/modeling_orthrus.py:114-189.

    forward() runs one layer's attention for inference on this package's kernels:
    - AR pass (is_diffusion_pass False): q|k|v projection, q/k RMSNorm + RoPE, the new keys and
      values appended to past_key_values at this layer's committed length, causal attention over
      the cache and the new tokens (a 4-D tree-verification mask is accepted and converted);
    - diffusion pass: the twin projections, keys = cat[cache[:ar_seq_len], block], with the
      dual-view training mask (flex_block_mask, or the equivalent dense 4-D attention_mask of
      orthrus/decoding.py:463-481) or, with no mask, full attention of the block over the cache
      and itself (generation).
    RoPE positions come from the position_ids / cache_position the decoder passes down (the kernels
    compute cos / sin from them, the values position_embeddings holds for the default RoPE), else
    they continue the cache. Returns (output [B, T, d], None)."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = config.head_dim
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        q_dim, kv_dim = self.num_heads * self.head_dim, self.num_kv_heads * self.head_dim
        bias = bool(getattr(config, "attention_bias", False))
        if bias:
            raise ValueError("attention_bias is not supported (Qwen3 has no projection biases)")
        for suffix in ("", "_diff"):
            setattr(self, f"q_proj{suffix}", nn.Linear(config.hidden_size, q_dim, bias=False))
            setattr(self, f"k_proj{suffix}", nn.Linear(config.hidden_size, kv_dim, bias=False))
            setattr(self, f"v_proj{suffix}", nn.Linear(config.hidden_size, kv_dim, bias=False))
            setattr(self, f"o_proj{suffix}", nn.Linear(q_dim, config.hidden_size, bias=False))
            setattr(self, f"q_norm{suffix}", RMSNorm(self.head_dim, config.rms_norm_eps))
            setattr(self, f"k_norm{suffix}", RMSNorm(self.head_dim, config.rms_norm_eps))

    def view_weights(self, diffusion: bool):
        s = "_diff" if diffusion else ""
        g = lambda n: getattr(self, f"{n}{s}")  # noqa: E731
        return g("q_proj").weight, g("k_proj").weight, g("v_proj").weight, g("o_proj").weight, \
            g("q_norm").weight, g("k_norm").weight

    def packed_qkv(self, diffusion: bool) -> torch.Tensor:
        """[q; k; v] weights of one view as a single [(Hq + 2 Hkv) hd, d] matrix (cached)."""
        wq, wk, wv, *_ = self.view_weights(diffusion)
        return _cached_weight(self, ("qkv", diffusion), [wq, wk, wv])

    def attend(self, h, positions, mode: str, *, kv=None, offsets=None, ar_len=None, limit2=None,
               block_mask=None, tree_lo=None, inv_freq=None) -> torch.Tensor:
        """Attention output [B*T, Hq*hd] (the o projection's input) of h [B*T, d] at positions
        [B, T]; the modes of OrthrusModel.run_layers, kv = this layer's (key, value) buffers."""
        cfg = self.config
        B, T = positions.shape
        Hq, Hkv, hd = self.num_heads, self.num_kv_heads, self.head_dim
        D = padded_head_dim(hd)
        eps = cfg.rms_norm_eps
        diffusion = mode not in ("ar", "tree")
        _, _, _, _, qn, kn = self.view_weights(diffusion)
        inv = inv_freq if inv_freq is not None else ops.rope_inv_freq(hd, _theta(cfg), h.device)
        qkv = _project(h, self.packed_qkv(diffusion))
        if mode in ("ar", "tree") and kv is not None:
            kb, vb = kv
            q, _, _, _ = ops.qkv_prep(qkv, positions, inv, qn, kn, B, T, Hq, Hkv, hd, D, eps,
                                      k_cache=kb, v_cache=vb, offset=offsets)
            if mode == "tree":
                o, _ = ops.attention_fwd(q, kb, vb, kb, vb, mask=MASK_TREE, hd=hd, scale=self.scaling,
                                         offset=offsets, limit2=tree_lo, want_lse=False)
            else:
                o, _ = ops.attention_fwd(q, kb, vb, mask=MASK_CAUSAL, hd=hd, scale=self.scaling,
                                         offset=offsets, want_lse=False)
        elif mode == "ar":
            q, k, v, _ = ops.qkv_prep(qkv, positions, inv, qn, kn, B, T, Hq, Hkv, hd, D, eps)
            o, _ = ops.attention_fwd(q, k, v, mask=MASK_CAUSAL, hd=hd, scale=self.scaling, want_lse=False)
        else:
            q, k2, v2, _ = ops.qkv_prep(qkv, positions, inv, qn, kn, B, T, Hq, Hkv, hd, D, eps)
            kb, vb = kv
            if mode == "dual":
                o, _ = ops.attention_fwd(q, kb, vb, k2, v2, mask=MASK_DUAL, hd=hd, scale=self.scaling,
                                         anchors=block_mask.anchors, block=block_mask.block_size,
                                         L1=ar_len, want_lse=False)
            else:
                o, _ = ops.attention_fwd(q, kb, vb, k2, v2, mask=MASK_DRAFT, hd=hd, scale=self.scaling,
                                         offset=offsets, limit2=limit2, want_lse=False)
        return o.reshape(B * T, Hq * hd)

    @torch.no_grad()
    def forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                past_key_values: KVCache | None = None, is_diffusion_pass: bool = False,
                ar_seq_len: int | None = None, flex_block_mask: "DualViewMask | None" = None,
                **kwargs):
        B, T, d = hidden_states.shape
        cache = past_key_values
        if cache is not None and not isinstance(cache, KVCache):
            raise ValueError("past_key_values must be this package's KVCache (exported as DynamicCache)")
        seen = cache.get_seq_length(self.layer_idx) if cache is not None else 0
        position_ids = kwargs.get("position_ids")
        if position_ids is None:
            position_ids = kwargs.get("cache_position")
        positions = _positions_of(position_ids, B, T, seen, hidden_states.device)
        h = hidden_states.reshape(B * T, d).contiguous()
        common = dict(inv_freq=None)
        if not is_diffusion_pass:
            tree_lo = None
            if attention_mask is not None and attention_mask.dim() == 4:
                tree_lo = tree_mask_to_lo(attention_mask, seen, T).to(h.device)
            if cache is None:
                if tree_lo is not None:
                    raise ValueError("tree verification runs over a cache")
                o = self.attend(h, positions, "ar", **common)
            else:
                cache.allocate(B, h.dtype, h.device)
                cache.reserve(seen + T)
                kv = (cache.k[self.layer_idx], cache.v[self.layer_idx])
                o = self.attend(h, positions, "tree" if tree_lo is not None else "ar", kv=kv,
                                offsets=cache.offsets(B, self.layer_idx), tree_lo=tree_lo, **common)
                cache.lengths[self.layer_idx] = seen + T
        else:
            if cache is None or ar_seq_len is None:
                raise ValueError("the diffusion pass needs the AR cache (past_key_values) and ar_seq_len")
            if seen != ar_seq_len:
                raise ValueError(f"AR cache holds {seen} positions, expected {ar_seq_len}")
            kv = (cache.k[self.layer_idx][:, :, :ar_seq_len], cache.v[self.layer_idx][:, :, :ar_seq_len])
            if flex_block_mask is None and attention_mask is not None:
                flex_block_mask = dense_mask_to_dual(attention_mask, ar_seq_len, T)
            if flex_block_mask is not None:
                o = self.attend(h, positions, "dual", kv=kv, ar_len=ar_seq_len, block_mask=flex_block_mask,
                                **common)
            else:
                offsets = cache.offsets(B, self.layer_idx)
                limit2 = torch.full((B,), T, dtype=torch.int32, device=h.device)
                o = self.attend(h, positions, "draft", kv=kv, offsets=offsets, limit2=limit2, **common)
        wo = self.view_weights(is_diffusion_pass)[3]
        return _project(o, wo).view(B, T, d), None


class OrthrusDecoderLayer(nn.Module):
    """Pre-norm Qwen3 decoder layer (orthrus/modeling_orthrus.py:192-221): x + attn(norm(x)), then
    + mlp(norm(x)); the residual adds ride in the projection epilogues."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.self_attn = OrthrusAttention(config, layer_idx)
        self.mlp = OrthrusMLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)

    @torch.no_grad()
    def forward(self, hidden_states: torch.Tensor, attention_mask=None, position_embeddings=None,
                past_key_values: KVCache | None = None, **kwargs) -> torch.Tensor:
        attn, _ = self.self_attn(hidden_states=self.input_layernorm(hidden_states),
                                 attention_mask=attention_mask, position_embeddings=position_embeddings,
                                 past_key_values=past_key_values, **kwargs)
        x = hidden_states + attn
        return self.mlp(self.post_attention_layernorm(x), residual=x)


class OrthrusModel(nn.Module):
    """The decoder stack (orthrus/modeling_orthrus.py:224-296). forward() has the reference's
    signature and returns last_hidden_state (final norm applied) and the cache. The AR pass and
    generation-time diffusion passes run the fused no-grad layer loop (run_layers); a diffusion
    pass with the training mask and gradients enabled runs the differentiable dual-view layers of
    objective.model_states, so its output backpropagates into the twins."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.padding_idx = getattr(config, "pad_token_id", None)
        self.vocab_size = config.vocab_size
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(
            [OrthrusDecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.gradient_checkpointing = False
        self._inv_freq = None

    def inv_freq(self, device) -> torch.Tensor:
        if self._inv_freq is None or self._inv_freq.device != torch.device(device):
            self._inv_freq = ops.rope_inv_freq(self.config.head_dim, _theta(self.config), device)
        return self._inv_freq

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values: KVCache | None = None, inputs_embeds=None, use_cache: bool | None = None,
                cache_position=None, is_diffusion_pass: bool = False, ar_seq_len: int | None = None,
                flex_block_mask: "DualViewMask | None" = None, tree_lo: torch.Tensor | None = None,
                **kwargs) -> "ModelOutput":
        if (input_ids is None) == (inputs_embeds is None):
            raise ValueError("pass exactly one of input_ids or inputs_embeds")
        if past_key_values is not None and not isinstance(past_key_values, KVCache):
            raise ValueError("past_key_values must be this package's KVCache (exported as DynamicCache)")
        x = inputs_embeds if inputs_embeds is not None else self.embed_tokens(input_ids)
        B, T, _ = x.shape
        if use_cache and past_key_values is None:
            past_key_values = KVCache(self.config)
        cache = past_key_values
        seen = cache.get_seq_length() if cache is not None else 0
        if position_ids is None and cache_position is not None:
            position_ids = cache_position[None]
        positions = _positions_of(position_ids, B, T, seen, x.device)
        if attention_mask is not None and attention_mask.dim() == 4:
            if tree_lo is not None:
                raise ValueError("pass a 4-D mask or tree_lo, not both")
            if is_diffusion_pass:
                if flex_block_mask is None:
                    flex_block_mask = dense_mask_to_dual(attention_mask, ar_seq_len, T)
            else:
                tree_lo = tree_mask_to_lo(attention_mask, seen, T).to(x.device)
        if is_diffusion_pass:
            if cache is None or ar_seq_len is None:
                raise ValueError("the diffusion pass needs the AR cache (past_key_values) and ar_seq_len")
            if seen != ar_seq_len:
                raise ValueError(f"AR cache holds {seen} positions, expected {ar_seq_len}")
            if tree_lo is not None:
                raise ValueError("tree masks belong to AR verification passes")
            mode = "dual" if flex_block_mask is not None else "draft"
        else:
            mode = "ar"
            if cache is not None and not use_cache:
                raise ValueError("an AR pass over a cache must append to it (use_cache=True)")
            if tree_lo is not None:
                if cache is None or B != 1:
                    raise ValueError("tree verification runs on a cache, batch 1")
                mode = "tree"
        if cache is not None:
            cache.allocate(B, x.dtype, x.device)
            cache.reserve(seen + T)
        if mode == "dual" and torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            from orthrus_training_b200.objective import diffusion_states

            hidden = diffusion_states(self, x.reshape(B * T, -1), cache, positions, flex_block_mask)
            hidden = hidden.view(B, T, -1)
        else:
            with torch.no_grad():
                kv = cache.buffers() if cache is not None else None
                offsets = cache.offsets(B) if cache is not None else None
                hidden = self.run_layers(x, positions, mode, kv=kv, offsets=offsets, ar_len=ar_seq_len,
                                         block_mask=flex_block_mask, tree_lo=tree_lo)
        if cache is not None and mode in ("ar", "tree"):
            cache.length = seen + T
        return ModelOutput(last_hidden_state=hidden, past_key_values=cache if use_cache else None,
                           hidden_states=(hidden,))

    @torch.no_grad()
    def run_layers(self, x, positions, mode: str, *, kv=None, offsets=None, ar_len=None,
                   limit2=None, block_mask=None, tree_lo=None):
        """The decoder stack over x [B, T, d] at positions [B, T] (int64) -> final-norm hidden.

        mode "ar":    AR view; with kv (per-layer [B, Hkv, cap, D] buffers) the new K/V are written
                      at rows offsets[b] + t and queries attend causally over rows < offsets[b]+t+1
                      (a verification or plain greedy pass); without kv, plain causal attention.
        mode "draft": diffusion view over kv rows < offsets[b] plus the block's own keys
                      [0, limit2[b]) (the generation-time draft, orthrus/modeling_orthrus.py:469-481).
        mode "dual":  diffusion view with the training mask (block_mask) over kv rows < ar_len.
        mode "tree":  AR view writing the new K/V like "ar"; query t sees kv rows
                      < offsets[b] + 1 and rows [offsets[b] + tree_lo[t], offsets[b] + t + 1).
        The residual adds ride in the o / down projection epilogues.
        """
        cfg = self.config
        B, T, d = x.shape
        eps = cfg.rms_norm_eps
        inv = self.inv_freq(x.device)
        diffusion = mode not in ("ar", "tree")
        x = x.reshape(B * T, d).contiguous()
        for i, layer in enumerate(self.layers[: cfg.num_hidden_layers]):
            attn = layer.self_attn
            h = ops.rms_norm(x, layer.input_layernorm.weight, eps)
            o = attn.attend(h, positions, mode, kv=kv[i] if kv is not None else None, offsets=offsets,
                            ar_len=ar_len, limit2=limit2, block_mask=block_mask, tree_lo=tree_lo,
                            inv_freq=inv)
            x = _project(o, attn.view_weights(diffusion)[3], residual=x)
            h = ops.rms_norm(x, layer.post_attention_layernorm.weight, eps)
            x = _project(layer.mlp.activation(h), layer.mlp.down_proj.weight, residual=x)
        x = ops.rms_norm(x, self.norm.weight, eps)
        return x.view(B, T, d)


@dataclass
class ModelOutput:
    logits: torch.Tensor | None = None
    last_hidden_state: torch.Tensor | None = None
    past_key_values: KVCache | None = None
    hidden_states: tuple = ()


@dataclass
class GenerationStats:
    """Forward-pass accounting of one diffusion-mode generation (orthrus/modeling_orthrus.py:299-312)."""

    new_tokens: int = 0
    accepted: list[int] = field(default_factory=list)

    @property
    def cycles(self) -> int:
        return len(self.accepted)

    @property
    def forward_passes(self) -> int:
        return 1 + 2 * self.cycles


def tree_mask_to_lo(mask: torch.Tensor, seen: int, T: int) -> torch.Tensor:
    """int32 [T] branch starts of a dense tree-verification mask [1, 1, T, seen + T] (the form
    orthrus/decoding.py:222-231 builds): every query sees the whole prefix and the root, and among
    the other new tokens exactly a contiguous run [lo, t] ending at itself. Raises otherwise."""
    m = mask.detach().to("cpu", torch.bool)
    if m.shape != (1, 1, T, seen + T):
        raise ValueError(f"tree mask must be [1, 1, {T}, {seen + T}], got {tuple(m.shape)}")
    m = m[0, 0]
    if not bool(m[:, : seen + 1].all()):
        raise ValueError("a tree mask shows every query the prefix and the root")
    lo = torch.ones(T, dtype=torch.int32)
    for t in range(1, T):
        row = m[t, seen + 1:]
        visible = torch.nonzero(row).flatten() + 1
        start = int(visible.min()) if visible.numel() else t + 1
        if visible.numel() == 0 or int(visible.max()) != t or visible.numel() != t - start + 1:
            raise ValueError("each tree-mask query must see a contiguous run of new tokens ending at itself")
        lo[t] = start
    if bool(m[0, seen + 1:].any()):
        raise ValueError("the root sees no other new token")
    return lo


def dense_mask_to_dual(mask: torch.Tensor, ar_len: int, T: int) -> "DualViewMask":
    """The dual-view mask object of a dense 4-D boolean mask [1, 1, T, ar_len + T] of the form
    orthrus/decoding.py:463-481 builds for packed draft blocks: the T queries form consecutive
    blocks of K; every query of block b sees the AR keys [0, anchor_b) and all K keys of its own
    block, nothing else. Checks that form (anchors non-decreasing) and raises ValueError otherwise."""
    m = mask.detach().to("cpu", torch.bool)
    if m.shape != (1, 1, T, ar_len + T):
        raise ValueError(f"a dual-view mask must be [1, 1, {T}, {ar_len + T}], got {tuple(m.shape)}")
    m = m[0, 0]
    own, ar = m[:, ar_len:], m[:, :ar_len]
    K = int(own[0].sum())
    if K < 1 or T % K != 0:
        raise ValueError("the new keys of a dual-view mask form equal blocks")
    blocks = torch.arange(T) // K
    if not torch.equal(own, blocks[:, None] == blocks[None, :]):
        raise ValueError("each query of a dual-view mask sees exactly its own block among the new keys")
    anchors = ar.sum(1).view(T // K, K)
    if not bool((anchors == anchors[:, :1]).all()):
        raise ValueError("all queries of a block see the same AR prefix")
    anchors = anchors[:, 0]
    prefix = torch.arange(ar_len)[None, :] < anchors.repeat_interleave(K)[:, None]
    if not torch.equal(ar, prefix):
        raise ValueError("the AR keys a query sees form a prefix [0, anchor)")
    if bool((anchors[1:] < anchors[:-1]).any()):
        raise ValueError("dual-view anchors must be non-decreasing")
    return DualViewMask(anchors[None].to(mask.device), ar_len, K)


class DualViewMask:
    """The dual-pass training mask (orthrus/modeling_orthrus.py:58-74) as the attention kernels use
    it: per-row sorted anchors plus the per-anchor tile map. ``mask_mod`` evaluates the reference's
    definition for inspection (a query of block b sees AR keys strictly before anchors[:, b] and
    every key of its own block)."""

    def __init__(self, anchors: torch.Tensor, ar_len: int, block_size: int):
        self.anchors = anchors
        self.ar_len = ar_len
        self.block_size = block_size
        self.num_blocks = anchors.shape[1]
        self._tilemap = None

    def mask_mod(self, batch, head, q_idx, kv_idx):
        blocks = self.num_blocks
        block = (q_idx // self.block_size).clamp(max=blocks - 1)
        ar_visible = (kv_idx < self.ar_len) & (kv_idx < self.anchors[batch, block])
        same = (kv_idx >= self.ar_len) & ((kv_idx - self.ar_len) // self.block_size
                                          == q_idx // self.block_size)
        return ar_visible | same

    @property
    def tilemap(self) -> torch.Tensor:
        """int32 [B, tiles of 128 queries, 4]: (source-1 tiles, visible source-1 keys, source-2
        key range), computed on the device (orthrus_attn_tilemap)."""
        if self._tilemap is None:
            self._tilemap = ops.attention_tilemap(self.anchors, self.block_size, self.ar_len)
        return self._tilemap


def build_block_mask(anchors: torch.Tensor, ar_len: int, block_size: int) -> DualViewMask:
    """Dual-pass mask for training (orthrus/modeling_orthrus.py:58-74)."""
    return DualViewMask(anchors, ar_len, block_size)


def diffusion_attention(q, k, v, block_mask: DualViewMask) -> torch.Tensor:
    """Masked attention of the diffusion view over cat([AR keys, block keys])
    (orthrus/modeling_orthrus.py:77-85): q [B, Hq, Q, hd], k/v [B, Hkv, ar_len + Q, hd] ->
    [B, Hq, Q, hd]. Runs the dual-view kernel (tcgen05 for bf16 with hd 64/128)."""
    ar = block_mask.ar_len
    hd = q.shape[-1]
    D = hd if hd in (64, 128) else padded_head_dim(hd)
    pad = (lambda t: torch.nn.functional.pad(t, (0, D - hd))) if D != hd else (lambda t: t)
    qp = pad(q).contiguous()
    kp, vp = pad(k).contiguous(), pad(v).contiguous()
    o, _ = ops.attention_fwd(qp, kp[:, :, :ar], vp[:, :, :ar], kp[:, :, ar:], vp[:, :, ar:],
                             mask=MASK_DUAL, hd=hd, scale=hd ** -0.5,
                             anchors=block_mask.anchors, block=block_mask.block_size, want_lse=False)
    return o.transpose(1, 2)


@torch.no_grad()
def copy_diff_from_ar(model: nn.Module) -> None:
    """Warm-start every diffusion twin from its frozen AR counterpart (orthrus/modeling_orthrus.py:88-94)."""
    for module in model.modules():
        if isinstance(module, OrthrusAttention):
            for name in DIFF_MODULES:
                getattr(module, f"{name}_diff").load_state_dict(getattr(module, name).state_dict())


def freeze_to_diffusion(model: nn.Module) -> list[nn.Parameter]:
    """Freeze the AR backbone; return the trainable diffusion parameters (orthrus/modeling_orthrus.py:97-104)."""
    trainable = []
    for name, param in model.named_parameters():
        param.requires_grad_(any(f".{m}_diff." in name for m in DIFF_MODULES))
        if param.requires_grad:
            trainable.append(param)
    return trainable


def truncate_cache(cache: KVCache, length: int) -> None:
    """Drop cached positions >= length (orthrus/modeling_orthrus.py:107-111): on the device cache this
    only moves the committed length."""
    excess = cache.get_seq_length() - length
    if excess > 0:
        cache.crop(-excess)


class OrthrusLM(nn.Module):
    """Qwen3 with the Orthrus diffusion twins (orthrus/modeling_orthrus.py:315-534)."""

    _tied_weights_keys = {"lm_head.weight": "model.embed_tokens.weight"}

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.model = OrthrusModel(config)
        self.vocab_size = config.vocab_size
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if getattr(config, "tie_word_embeddings", True):
            self.lm_head.weight = self.model.embed_tokens.weight
        self.init_weights()

    # -- weights ------------------------------------------------------------------------------

    @torch.no_grad()
    def init_weights(self, std: float | None = None) -> None:
        """Random init of a Qwen3 model: normal(0, initializer_range) weights, unit norms."""
        std = std if std is not None else getattr(self.config, "initializer_range", 0.02)
        for name, p in self.named_parameters():
            if name.endswith("norm.weight") or ".q_norm" in name or ".k_norm" in name or \
                    "layernorm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std)

    @property
    def is_gradient_checkpointing(self) -> bool:
        return self.model.gradient_checkpointing

    def gradient_checkpointing_enable(self, kwargs=None) -> None:
        self.model.gradient_checkpointing = True

    def inv_freq(self, device) -> torch.Tensor:
        return self.model.inv_freq(device)

    def packed_qkv(self, layer: int, diffusion: bool) -> torch.Tensor:
        """[q; k; v] projection weights of a layer's view as one [(Hq+2Hkv) hd, d] matrix, cached
        for inference (rebuilt when a weight changes)."""
        return self.model.layers[layer].self_attn.packed_qkv(diffusion)

    def _packed_mlp(self, layer: int) -> torch.Tensor:
        return self.model.layers[layer].mlp.packed_gate_up()

    # -- forward ------------------------------------------------------------------------------

    def forward(
        self,
        input_ids: torch.LongTensor | None = None,
        attention_mask: torch.Tensor | None = None,
        position_ids: torch.LongTensor | None = None,
        past_key_values: KVCache | None = None,
        inputs_embeds: torch.FloatTensor | None = None,
        labels: torch.LongTensor | None = None,
        use_cache: bool | None = None,
        cache_position: torch.LongTensor | None = None,
        logits_to_keep: int | torch.Tensor = 0,
        is_diffusion_pass: bool = False,
        ar_seq_len: int | None = None,
        flex_block_mask: DualViewMask | None = None,
        tree_lo: torch.Tensor | None = None,
        **kwargs,
    ) -> ModelOutput:
        """OrthrusLM.forward (orthrus/modeling_orthrus.py:327-362): the decoder stack
        (OrthrusModel.forward), then fp32 logits of the last `logits_to_keep` positions (all when
        0) or of the given indices.

        Tree verification (orthrus/decoding.py:208-241): an AR pass whose new tokens are a root and
        several branches, each token seeing the cached prefix, the root and its own branch up to
        itself. Give either ``tree_lo`` (int32 [T]: the index among the new tokens where each
        token's branch begins, >= 1) or the reference's dense 4-D boolean mask [1, 1, T, seen + T],
        which is checked to have that form and converted."""
        out = self.model(input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                         past_key_values=past_key_values, inputs_embeds=inputs_embeds, use_cache=use_cache,
                         cache_position=cache_position, is_diffusion_pass=is_diffusion_pass,
                         ar_seq_len=ar_seq_len, flex_block_mask=flex_block_mask, tree_lo=tree_lo, **kwargs)
        hidden = out.last_hidden_state
        if isinstance(logits_to_keep, int):
            keep = hidden[:, -logits_to_keep:] if logits_to_keep else hidden
        else:
            keep = hidden[:, logits_to_keep]
        with torch.no_grad():
            logits = self.lm_logits(keep.detach())
        return ModelOutput(logits=logits, last_hidden_state=hidden, past_key_values=out.past_key_values,
                           hidden_states=(hidden,))

    def lm_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        shape = hidden.shape[:-1]
        h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
        w = self.lm_head.weight
        if h.dtype == torch.bfloat16:
            logits = ops.gemm(h, w, out_dtype=torch.float32)
        else:
            logits = ops.gemm(h, w)
        return logits.view(*shape, -1)

    def lm_argmax(self, hidden: torch.Tensor) -> torch.Tensor:
        """Greedy pick of every row of hidden [..., d]: int64 [rows], the argmax of lm_logits(hidden)
        (lowest index on ties). bf16 rows take the LM-head argmax kernel, which computes the same
        fp32 logits tiles and never writes them."""
        h = hidden.reshape(-1, hidden.shape[-1])
        w = self.lm_head.weight
        if h.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and h.shape[-1] % 64 == 0:
            return ops.lmhead_argmax(h, w)
        return ops.argmax_rows(self.lm_logits(h).reshape(h.shape[0], -1))

    def run_layers(self, x, positions, mode: str, **kwargs):
        """The fused layer loop of OrthrusModel.run_layers (used by the device decode loop)."""
        return self.model.run_layers(x, positions, mode, **kwargs)

    # -- generation ---------------------------------------------------------------------------

    @torch.inference_mode()
    def generate(self, input_ids, max_new_tokens=None, max_length=None, temperature=0.0, top_k=20,
                 top_p=0.8, eos_token_id=None, streamer=None, use_diffusion_mode=True, **kwargs):
        """OrthrusLM.generate (orthrus/modeling_orthrus.py:364-402), greedy."""
        eos_token_id = eos_token_id if eos_token_id is not None else self.config.eos_token_id
        max_new_tokens = max_new_tokens or (max_length - input_ids.shape[1])
        if not use_diffusion_mode:
            from orthrus_training_b200.decoding import ar_generate_batch

            return ar_generate_batch(self, input_ids, max_new_tokens, eos_token_id)
        output, _ = self.diffusion_generate(input_ids, max_new_tokens, temperature=temperature,
                                            top_k=top_k, top_p=top_p, eos_token_id=eos_token_id,
                                            streamer=streamer)
        return output

    @torch.inference_mode()
    def diffusion_generate(self, input_ids, max_new_tokens, temperature=0.0, top_k=20, top_p=0.8,
                           eos_token_id=None, streamer=None):
        """Project K tokens in parallel, verify them with the AR view, keep the agreed prefix
        (orthrus/modeling_orthrus.py:404-534) with the cycle state on the device, greedy by default.
        Batch size 1 here, as the reference; decoding.block_decode takes batches. With a temperature
        (>= 1e-5) the drafts and the AR view are sampled through the reference's top-k / top-p
        filter and the drafts kept by exact rejection sampling (:437-449,498-511); the draws come
        from a Philox seed taken from torch's default generator, so torch.manual_seed fixes them."""
        if input_ids.shape[0] != 1:
            raise ValueError("diffusion_generate supports batch size 1")
        from orthrus_training_b200.decoding import block_decode

        sampler = None
        if temperature >= 1e-5:
            seed = int(torch.randint(0, 2 ** 62, (1,)).item())
            sampler = ops.SamplingParams(float(temperature), int(top_k), float(top_p), seed)
        eos = {eos_token_id} if isinstance(eos_token_id, int) else set(eos_token_id or ())
        result = block_decode(self, [input_ids[0].tolist()], max_new_tokens, eos, sampler=sampler)
        tokens = result.tokens[0]
        out = torch.tensor([input_ids[0].tolist() + tokens], device=input_ids.device)
        stats = GenerationStats(new_tokens=len(tokens), accepted=result.accepted[0])
        if streamer is not None:
            streamer.put(input_ids)
            if tokens:
                streamer.put(torch.tensor(tokens))
            streamer.end()
        return out, stats
