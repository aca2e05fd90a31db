"""Parity at the workload configurations themselves, on the GPU, through the C ABI:

- one row of the Qwen3-0.6B-shape training step (28 layers, 16/8 heads of 128, 2048 tokens,
  32 anchors, K = 32): the bf16 orthrus_loss forward + backward against the fp32 oracle on the
  same bf16-rounded weights (orthrus/objective.py:395-453);
- the dual-view attention sweep shapes (L in {2048, 8192}, K in {32, 64}, A in {32, 64}, 16/8
  heads, hd 128): forward and backward against an fp32 dense-mask computation on the GPU
  (orthrus/objective.py:160-198, orthrus/modeling_orthrus.py:58-85);
- fp32 block decoding of the Qwen3-0.6B layer shape against the oracle's plain greedy decoding on
  the CPU (orthrus/modeling_orthrus.py:404-534, orthrus/evaluate.py:59-76): token identical;
- more block rows than sequence positions (A * K > L) through the fused q|k|v + RoPE projection.

Tolerances (stated by the dual-view path's contract): bf16 loss within 1e-2 relative; bf16
attention outputs and gradients within 2e-2 max-abs; bf16 twin gradients within the reference's
own bf16-vs-fp32 gradient error (about 3 % relative, cosine 0.9996, README.md:243-244) with a 2x
margin: 6 % relative and cosine >= 0.999 over all twins; fp32 decoding exact.
"""

import math

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _oracle_params(model) -> dict:
    params = {k: v.detach().float().cpu().requires_grad_("_diff." in k)
              for k, v in model.state_dict().items()}
    params["lm_head.weight"] = params["model.embed_tokens.weight"]
    return params


def _perturb_twins(model, seed: int, scale: float = 0.02) -> None:
    """Seeded noise on the diffusion twins (scaled by each tensor's mean magnitude) so the
    student's gradients are generic rather than those of an exact copy of the teacher."""
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "_diff." in name:
                noise = torch.randn(p.shape, generator=gen) * scale * (p.float().abs().mean().item() + 1e-3)
                p.add_(noise.to(p.device, p.dtype))


def test_config2_one_row_bf16_step_matches_oracle():
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar, freeze_to_diffusion
    from orthrus_training_b200.objective import orthrus_loss, sample_anchors
    from orthrus_training_b200.synthetic import packed_rows, qwen3_06b_config

    cfg = qwen3_06b_config(32, 151669)
    torch.manual_seed(1)
    with torch.device(DEV):
        model = OrthrusLM(cfg).to(torch.bfloat16)
    copy_diff_from_ar(model)
    _perturb_twins(model, seed=100)
    freeze_to_diffusion(model)
    ids, mask = packed_rows(1, 2048, 151669, seed=1, ids="zipf", doc="prompt_response")
    anchors, valid = sample_anchors(mask, 32, 32, torch.Generator().manual_seed(1))
    loss, stats = orthrus_loss(model, ids.to(DEV), mask.to(DEV), anchors.to(DEV), valid.to(DEV),
                               kl_chunk_size=4096)
    loss.backward()
    torch.cuda.synchronize()

    params = _oracle_params(model)
    ref, ref_stats = O.orthrus_loss(params, O.OracleConfig.from_hf(cfg), ids, mask, anchors, valid)
    ref.backward()

    got, want = loss.item(), ref.item()
    assert abs(got - want) <= 1e-2 * abs(want), (got, want)
    assert int(stats["tokens"]) == int(ref_stats["tokens"])
    assert stats["tokens_by_offset"].cpu().tolist() == ref_stats["tokens_by_offset"].tolist()
    kbo, rkbo = stats["kl_by_offset"].float().cpu(), ref_stats["kl_by_offset"].float()
    assert (kbo - rkbo).abs().max().item() <= 2e-2 * rkbo.abs().max().item()
    # top-1 agreement may flip only where the two top logits are within bf16 rounding
    assert abs(int(stats["agree"]) - int(ref_stats["agree"])) <= max(2, int(ref_stats["tokens"]) // 100)

    diffs, refs, dots, n_got = 0.0, 0.0, 0.0, 0.0
    for name, p in model.named_parameters():
        if "_diff." not in name:
            continue
        g, r = p.grad.float().cpu(), params[name].grad
        assert torch.isfinite(g).all(), name
        diffs += (g - r).pow(2).sum().item()
        refs += r.pow(2).sum().item()
        dots += (g * r).sum().item()
        n_got += g.pow(2).sum().item()
    rel = math.sqrt(diffs / refs)
    cos = dots / math.sqrt(refs * n_got)
    print(f"config-2 row: loss {got:.6f} vs {want:.6f}; twin gradients rel {rel:.4f} cos {cos:.6f}")
    assert rel <= 0.06 and cos >= 0.999, (rel, cos)


def _dense_dual_reference(q, k1, v1, k2, v2, anchors, K, dout, scale, chunk=1024):
    """fp32 dual-view attention and its backward from the dense mask: query t of block
    b = t // K sees source-1 keys j < anchors[b] and the K source-2 keys of its own block.
    Returns o [B, Tq, Hq, hd], dq [B, Hq, Tq, hd], dk2 / dv2 [B, Hkv, Tq, hd]."""
    B, Hq, Tq, hd = q.shape
    Hkv, L = k1.shape[1], k1.shape[2]
    G = Hq // Hkv
    o = torch.empty(B, Tq, Hq, hd, device=q.device)
    dq = torch.empty(B, Hq, Tq, hd, device=q.device)
    dk2 = torch.zeros(B, Hkv, Tq, hd, device=q.device)
    dv2 = torch.zeros_like(dk2)
    for b in range(B):
        for h in range(Hkv):
            heads = slice(h * G, (h + 1) * G)
            kc = torch.cat([k1[b, h], k2[b, h]], 0).float()
            vc = torch.cat([v1[b, h], v2[b, h]], 0).float()
            for t0 in range(0, Tq, chunk):
                t = torch.arange(t0, min(Tq, t0 + chunk), device=q.device)
                blk = t // K
                see1 = torch.arange(L, device=q.device)[None] < anchors[b, blk][:, None]
                see2 = (torch.arange(Tq, device=q.device)[None] // K) == blk[:, None]
                allowed = torch.cat([see1, see2], 1)
                qs = q[b, heads, t].float()                         # [G, n, hd]
                s = (qs @ kc.t()) * scale
                s = s.masked_fill(~allowed[None], float("-inf"))
                p = torch.softmax(s, -1)
                out = p @ vc                                        # [G, n, hd]
                o[b, t, heads] = out.transpose(0, 1)
                do = dout[b, t, heads].float().transpose(0, 1)      # [G, n, hd]
                dp = do @ vc.t()
                delta = (do * out).sum(-1, keepdim=True)
                ds = p * (dp - delta)
                dq[b, heads, t] = (ds @ kc) * scale
                ds2, p2 = ds[:, :, L:], p[:, :, L:]
                dk2[b, h] += torch.einsum("gnk,gnd->kd", ds2, qs) * scale
                dv2[b, h] += torch.einsum("gnk,gnd->kd", p2, do)
    return o, dq, dk2, dv2


@pytest.mark.parametrize("L,K,A", [(2048, 32, 32), (2048, 32, 64), (2048, 64, 32), (2048, 64, 64),
                                   (8192, 32, 32), (8192, 32, 64), (8192, 64, 32), (8192, 64, 64)])
def test_sweep_shape_dual_view_attention_vs_fp32(L, K, A):
    from orthrus_training_b200 import ops

    B, Hq, Hkv, hd = (2 if L <= 2048 else 1), 16, 8, 128
    gen = torch.Generator(device=DEV).manual_seed(L + 7 * K + A)
    Tq = A * K
    rnd = lambda *s: torch.randn(*s, device=DEV, generator=gen).bfloat16()  # noqa: E731
    q, k1, v1, k2, v2 = rnd(B, Hq, Tq, hd), rnd(B, Hkv, L, hd), rnd(B, Hkv, L, hd), rnd(B, Hkv, Tq, hd), \
        rnd(B, Hkv, Tq, hd)
    anchors = torch.stack([torch.randperm(L - K, device=DEV, generator=gen)[:A].add(1).sort().values
                           for _ in range(B)])
    scale = 1.0 / math.sqrt(hd)
    o, lse = ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=hd, scale=scale, anchors=anchors, block=K)
    dout = rnd(B, Tq, Hq, hd)
    dq, dk2, dv2 = ops.attention_bwd(q, k1, v1, k2, v2, anchors, K, o, lse, dout, hd=hd, scale=scale)
    ro, rdq, rdk, rdv = _dense_dual_reference(q, k1, v1, k2, v2, anchors, K, dout, scale)
    for name, got, want in (("o", o.float(), ro), ("dq", dq, rdq), ("dk2", dk2, rdk), ("dv2", dv2, rdv)):
        err = (got - want).abs().max().item()
        assert err <= 2e-2, (name, err)
    from orthrus_training_b200 import _lib

    assert _lib.device_error(0) == 0


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (16, 4)])
def test_own_block_key_gradients_of_32_key_blocks(Hq, Hkv):
    """dK / dV of the own-block keys with 32-key blocks (the HBM-bound 32 x 32 kernel) for two and
    four query heads per KV head, against the fp32 dense-mask backward: relative to the largest
    gradient, within the bf16 rounding of P and dS."""
    from orthrus_training_b200 import _lib, ops

    B, L, K, A, hd = 2, 1024, 32, 24, 128
    gen = torch.Generator(device=DEV).manual_seed(Hq * 31 + Hkv)
    Tq = A * K
    rnd = lambda *s: torch.randn(*s, device=DEV, generator=gen).bfloat16()  # noqa: E731
    q, k1, v1, k2, v2 = rnd(B, Hq, Tq, hd), rnd(B, Hkv, L, hd), rnd(B, Hkv, L, hd), rnd(B, Hkv, Tq, hd), \
        rnd(B, Hkv, Tq, hd)
    anchors = torch.stack([torch.randperm(L - K, device=DEV, generator=gen)[:A].add(1).sort().values
                           for _ in range(B)])
    scale = 1.0 / math.sqrt(hd)
    o, lse = ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=hd, scale=scale, anchors=anchors, block=K)
    dout = rnd(B, Tq, Hq, hd)
    _, dk2, dv2 = ops.attention_bwd(q, k1, v1, k2, v2, anchors, K, o, lse, dout, hd=hd, scale=scale)
    _, _, rdk, rdv = _dense_dual_reference(q, k1, v1, k2, v2, anchors, K, dout, scale)
    for name, got, want in (("dk2", dk2, rdk), ("dv2", dv2, rdv)):
        err = (got - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item(), (name, err, want.abs().max().item())
    assert _lib.device_error(0) == 0


def test_06b_fp32_block_decode_equals_oracle_greedy():
    """fp32, Qwen3-0.6B layer shape with 2 layers, random init: block decoding with the model's
    own drafts and with scripted drafts (the oracle's greedy continuation, 5 % of tokens edited)
    both give exactly the oracle's plain greedy tokens."""
    from transformers import Qwen3Config

    from orthrus_training_b200.decoding import block_decode
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar
    from orthrus_training_b200.synthetic import zipf_ids

    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=2,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                      rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=4096)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size = 32
    cfg.mask_token_id = 151669
    torch.manual_seed(2)
    with torch.device(DEV):
        model = OrthrusLM(cfg).float()
    copy_diff_from_ar(model)
    new = 64
    prompt = zipf_ids(np.random.default_rng(2), 200, 151669).tolist()
    params = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    params["lm_head.weight"] = params["model.embed_tokens.weight"]
    want = O.ar_generate(params, O.OracleConfig.from_hf(cfg), torch.tensor([prompt]), new)
    got = block_decode(model, [prompt], new)
    assert got.tokens[0] == want
    K = cfg.block_size
    rng = np.random.default_rng(5)
    table = torch.zeros(1, new, K - 1, dtype=torch.int64)
    for i in range(new):
        row = [t if rng.random() >= 0.05 else int(rng.integers(0, 151669)) for t in want[i + 1: i + K]]
        table[0, i, : len(row)] = torch.tensor(row, dtype=torch.int64)
    scripted = block_decode(model, [prompt], new, draft_table=table.to(DEV))
    assert scripted.tokens[0] == want
    assert sum(scripted.passes) < sum(got.passes)  # the scripted drafts were accepted


def _bf16_small(seed=0):
    from transformers import Qwen3Config

    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar, freeze_to_diffusion

    cfg = Qwen3Config(vocab_size=2048, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-6,
                      rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=4096)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size = 32
    cfg.mask_token_id = 2047
    torch.manual_seed(seed)
    with torch.device(DEV):
        model = OrthrusLM(cfg).to(torch.bfloat16)
    copy_diff_from_ar(model)
    _perturb_twins(model, seed=101, scale=0.2)
    freeze_to_diffusion(model)
    return model, cfg


def test_more_block_rows_than_positions_through_the_fused_projection():
    """A * K = 1024 block rows over a 512-token row (blocks overlap), the shape of the reference's
    training recipe (256 anchors x 32 over 2048 tokens): the fused q|k|v + RoPE projection takes
    explicit positions, so its table needs only the largest position, not one row per block row."""
    from orthrus_training_b200.objective import orthrus_loss, sample_anchors
    from orthrus_training_b200.synthetic import packed_rows

    model, cfg = _bf16_small()
    ids, mask = packed_rows(1, 512, 2047, seed=4, ids="uniform", doc="short")
    anchors, valid = sample_anchors(mask, 32, 32, torch.Generator().manual_seed(4))
    assert anchors.shape[1] * 32 > 512
    loss, stats = orthrus_loss(model, ids.to(DEV), mask.to(DEV), anchors.to(DEV), valid.to(DEV),
                               kl_chunk_size=1024)
    loss.backward()
    params = _oracle_params(model)
    ref, ref_stats = O.orthrus_loss(params, O.OracleConfig.from_hf(cfg), ids, mask, anchors, valid)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-2 * abs(ref.item()), (loss.item(), ref.item())
    assert int(stats["tokens"]) == int(ref_stats["tokens"])
    for name, p in model.named_parameters():
        if "_diff." in name:
            r = params[name].grad
            err = (p.grad.float().cpu() - r).abs().max().item()
            assert err <= 5e-2 * r.abs().max().item() + 1e-6, (name, err)
    from orthrus_training_b200 import _lib

    assert _lib.device_error(0) == 0


def test_rope_position_past_the_table_is_reported():
    """A block position beyond the RoPE table is clamped (the access stays in bounds) and reported
    through ORTHRUS_ERR_BOUNDS in the device error word."""
    from orthrus_training_b200 import _lib, ops

    B, Q, Hq, Hkv, d = 1, 128, 4, 2, 256
    gen = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(B * Q, d, device=DEV, generator=gen).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * 128, d, device=DEV, generator=gen) * 0.05).bfloat16()
    qn = torch.ones(128, device=DEV, dtype=torch.bfloat16)
    inv = ops.rope_inv_freq(128, 1e6, DEV)
    rope = ops.rope_table(inv, 256)
    positions = torch.arange(Q, device=DEV)[None].clone()
    assert _lib.device_error(0) == 0
    ops.linear_qkv_rope(x, w, qn, qn, rope, B, Q, Hq, Hkv, 1e-6, positions=positions, keep=True)
    assert _lib.device_error(0) == 0  # every position inside the table
    positions[0, 77] = 256 + 5
    ops.linear_qkv_rope(x, w, qn, qn, rope, B, Q, Hq, Hkv, 1e-6, positions=positions, keep=True)
    assert _lib.device_error(0) == _lib.ERR_BOUNDS  # read and cleared
    assert _lib.device_error(0) == 0


def test_bounded_wait_runs_out_and_the_context_stays_usable():
    """A wait that nothing satisfies runs out after its limit (1 ms here), records
    ORTHRUS_ERR_TIMEOUT, drains the TMA copy it issued and frees its TMEM; the next tensor-core
    kernels then run normally."""
    from orthrus_training_b200 import _lib, ops

    lib = _lib.lib()
    tile = torch.randn(64, 64, device=DEV).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _lib.device_error(0) == 0
    st = lib.orthrus_selftest_bounded_wait(tile.data_ptr(), 1_000_000, status.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert status.item() == 1 | 2 | 4
    assert _lib.device_error(0) == _lib.ERR_TIMEOUT
    a = torch.randn(512, 256, device=DEV).bfloat16()
    b = torch.randn(384, 256, device=DEV).bfloat16()
    c = ops.gemm(a, b, out_dtype=torch.float32)
    assert (c - a.float() @ b.float().t()).abs().max().item() < 1e-2
    assert _lib.device_error(0) == 0
