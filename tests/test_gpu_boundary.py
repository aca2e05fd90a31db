"""The module-level drop-in surface on the GPU (orthrus/modeling_orthrus.py:107-296): OrthrusModel
and OrthrusAttention forwards with the reference's signatures, the cache's DynamicCache surface,
and the dense dual-view mask form, checked against the fused paths the training step and the
decoder use."""

import pytest
import torch
from conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _golden(dtype=torch.float32):
    from test_gpu_model import _load

    g = load_golden("config1.pt")
    return _load(g, dtype), g


def _states_through_the_backbone(model, input_ids, anchors):
    """The teacher and student hidden states obtained the way orthrus/objective.py:275-295 obtains
    them: the backbone's forward with a cache, then a diffusion pass over that cache with the
    dual-view block mask (the teacher call without gradients, the student call with them)."""
    from orthrus_training_b200.modeling_orthrus import build_block_mask

    K, mask_id = model.config.block_size, model.config.mask_token_id
    L = input_ids.shape[1]
    with torch.no_grad():
        teacher = model.model(input_ids=input_ids, use_cache=True)
    positions = anchors[:, :, None] + torch.arange(K, device=anchors.device)
    block_ids = torch.full_like(positions, mask_id)
    block_ids[:, :, 0] = input_ids.gather(1, anchors)
    student = model.model(input_ids=block_ids.flatten(1), position_ids=positions.flatten(1),
                          past_key_values=teacher.past_key_values, use_cache=False, is_diffusion_pass=True,
                          ar_seq_len=L, flex_block_mask=build_block_mask(anchors, L, K)).last_hidden_state
    return student, teacher.last_hidden_state


def test_backbone_forward_matches_model_states_with_gradients():
    from orthrus_training_b200 import objective as ob

    model, g = _golden()
    c = g["case"]
    ids, anchors = c["input_ids"].to(DEV), c["anchors"].to(DEV)
    s_mod, t_mod = _states_through_the_backbone(model, ids, anchors)
    assert s_mod.requires_grad  # the diffusion pass backpropagates into the twins
    s_fun, t_fun = ob.model_states(model, ids, anchors)
    assert torch.allclose(t_mod, t_fun, atol=1e-5)
    assert torch.allclose(s_mod.detach(), s_fun.detach(), atol=1e-5)
    weights = torch.randn(s_fun.shape, generator=torch.Generator().manual_seed(0)).to(DEV)
    twins = [p for n, p in model.named_parameters() if "_diff." in n]
    g_mod = torch.autograd.grad((s_mod * weights).sum(), twins)
    g_fun = torch.autograd.grad((s_fun * weights).sum(), twins)
    for a, b in zip(g_mod, g_fun):
        assert (a - b).abs().max().item() <= 1e-4 * b.abs().max().item() + 1e-7


def test_layer_by_layer_forward_equals_the_fused_stack():
    """Calling the decoder layers one at a time (each appending to its own layer of the cache), as
    transformers' generation loop does, gives the fused loop's hidden states and cache, for an AR
    prefill, an AR step and a generation-time diffusion pass."""
    from orthrus_training_b200.kv_cache import KVCache

    model, g = _golden()
    backbone = model.model
    ids = g["case"]["input_ids"][:1, :96].to(DEV)
    fused_cache = KVCache(model.config)
    fused = backbone(input_ids=ids, use_cache=True, past_key_values=fused_cache).last_hidden_state

    cache = KVCache(model.config)
    pos = torch.arange(ids.shape[1], device=DEV)[None]
    x = backbone.embed_tokens(ids)
    with torch.no_grad():
        for layer in backbone.layers:
            x = layer(x, attention_mask=None, position_embeddings=None, past_key_values=cache, position_ids=pos)
        x = backbone.norm(x)
    assert torch.allclose(x, fused, atol=1e-5)
    assert [cache.get_seq_length(i) for i in range(len(backbone.layers))] == [96] * len(backbone.layers)
    for (k1, v1), (k2, v2) in zip(cache.buffers(), fused_cache.buffers()):
        assert torch.allclose(k1[:, :, :96], k2[:, :, :96], atol=1e-5)
        assert torch.allclose(v1[:, :, :96], v2[:, :, :96], atol=1e-5)

    # one more AR token, then a diffusion draft over the 97-position cache
    nxt = torch.tensor([[5]], device=DEV)
    step_fused = backbone(input_ids=nxt, use_cache=True, past_key_values=fused_cache).last_hidden_state
    with torch.no_grad():
        y = backbone.embed_tokens(nxt)
        for layer in backbone.layers:
            y = layer(y, past_key_values=cache, position_ids=torch.tensor([[96]], device=DEV))
        y = backbone.norm(y)
    assert torch.allclose(y, step_fused, atol=1e-5)
    K = model.config.block_size
    block = torch.full((1, K), model.config.mask_token_id, device=DEV)
    block[0, 0] = 7
    bpos = torch.arange(97, 97 + K, device=DEV)[None]
    with torch.no_grad():
        d_fused = backbone(input_ids=block, position_ids=bpos, past_key_values=fused_cache, use_cache=False,
                           is_diffusion_pass=True, ar_seq_len=97).last_hidden_state
        z = backbone.embed_tokens(block)
        for layer in backbone.layers:
            z = layer(z, past_key_values=cache, position_ids=bpos, is_diffusion_pass=True, ar_seq_len=97)
        z = backbone.norm(z)
    assert torch.allclose(z, d_fused, atol=1e-5)


def test_dense_dual_mask_equals_the_block_mask():
    """A diffusion pass under the dense 4-D mask of packed draft blocks (AR keys before each block's
    anchor plus the block's own keys) equals the pass under the dual-view block mask."""
    from orthrus_training_b200.modeling_orthrus import DualViewMask, dense_mask_to_dual

    model, g = _golden()
    ids = g["case"]["input_ids"][:1, :200].to(DEV)
    K, total = model.config.block_size, ids.shape[1]
    anchors = torch.tensor([[20, 64, 65, 130]], device=DEV)
    T = anchors.shape[1] * K
    blk = torch.arange(T, device=DEV) // K
    ar_keys = torch.arange(total, device=DEV)[None] < anchors[0, blk][:, None]
    mask = torch.cat([ar_keys, blk[:, None] == blk[None, :]], 1)[None, None]
    conv = dense_mask_to_dual(mask, total, T)
    assert conv.block_size == K and conv.anchors.tolist() == anchors.tolist()
    positions = (anchors[0][:, None] + torch.arange(K, device=DEV)).reshape(1, -1)
    block = torch.full((1, T), model.config.mask_token_id, device=DEV)
    block[0, ::K] = ids[0, anchors[0]]
    outs = []
    for kw in ({"attention_mask": mask}, {"flex_block_mask": DualViewMask(anchors, total, K)}):
        from orthrus_training_b200.kv_cache import KVCache

        cache = KVCache(model.config)
        model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        with torch.no_grad():
            outs.append(model(input_ids=block, position_ids=positions, past_key_values=cache, use_cache=False,
                              is_diffusion_pass=True, ar_seq_len=total, **kw).logits)
    assert torch.equal(outs[0], outs[1])
    bad = mask.clone()
    bad[0, 0, 3, total + K] = True  # a query of block 0 sees a key of block 1
    with pytest.raises(ValueError):
        dense_mask_to_dual(bad, total, T)


def test_foreign_cache_objects_are_refused():
    from transformers import DynamicCache as HFDynamicCache

    model, g = _golden()
    ids = g["case"]["input_ids"][:1, :16].to(DEV)
    with pytest.raises(ValueError):
        model.model(input_ids=ids, past_key_values=HFDynamicCache(), use_cache=True)
