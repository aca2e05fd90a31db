"""The decode passes' split-key attention (bf16, hd 128, blocks of <= 64 rows per sequence over a
KV cache): against dense fp32 attention for the causal-over-cache and draft masks, and row for row
bit-identical to one-row calls, which is what keeps block decoding lossless (GPU)."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from orthrus_training_b200 import ops

    return ops


def _case(B, Hq, Hkv, Tq, cap, seed):
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    q = torch.randn(B, Hq, Tq, 128, generator=g).to(bf)
    kc = torch.randn(B, Hkv, cap, 128, generator=g).to(bf)
    vc = torch.randn(B, Hkv, cap, 128, generator=g).to(bf)
    k2 = torch.randn(B, Hkv, Tq, 128, generator=g).to(bf)
    v2 = torch.randn(B, Hkv, Tq, 128, generator=g).to(bf)
    return q, kc, vc, k2, v2


@pytest.mark.parametrize("Tq,offsets", [(32, [0, 100, 371, 640]), (1, [5, 127, 128, 700]), (64, [64, 3, 250, 600])])
def test_causal_over_the_cache_matches_dense_attention(Tq, offsets):
    B, Hq, Hkv, cap = len(offsets), 16, 8, 704
    q, kc, vc, _, _ = _case(B, Hq, Hkv, Tq, cap, seed=Tq)
    off = torch.tensor(offsets, dtype=torch.int32)
    o, _ = _ops().attention_fwd(q.to(DEV), kc.to(DEV), vc.to(DEV), mask=0, hd=128, scale=128 ** -0.5,
                                offset=off.to(DEV), want_lse=False)
    t = torch.arange(Tq)[None, :, None]
    key = torch.arange(cap)[None, None, :]
    mask = key <= (off[:, None, None] + t)
    ref = O.masked_attention(q.float(), kc.float(), vc.float(), mask)
    err = (o.float().cpu().transpose(1, 2) - ref).abs().max().item()
    assert err <= 2e-2, err


@pytest.mark.parametrize("Tq", [32, 16])
def test_draft_mask_matches_dense_attention(Tq):
    B, Hq, Hkv, cap = 3, 16, 8, 600
    q, kc, vc, k2, v2 = _case(B, Hq, Hkv, Tq, cap, seed=7 + Tq)
    off = torch.tensor([130, 0, 511], dtype=torch.int32)
    limit2 = torch.tensor([Tq, 5, 1], dtype=torch.int32)
    o, _ = _ops().attention_fwd(q.to(DEV), kc.to(DEV), vc.to(DEV), k2.to(DEV), v2.to(DEV), mask=2, hd=128,
                                scale=128 ** -0.5, offset=off.to(DEV), limit2=limit2.to(DEV), want_lse=False)
    keys = torch.cat([kc, k2], 2).float()
    vals = torch.cat([vc, v2], 2).float()
    kv = torch.arange(cap + Tq)[None, None, :]
    mask = ((kv < off[:, None, None]) | ((kv >= cap) & (kv - cap < limit2[:, None, None]))).expand(B, Tq, -1)
    ref = O.masked_attention(q.float(), keys, vals, mask)
    err = (o.float().cpu().transpose(1, 2) - ref).abs().max().item()
    assert err <= 2e-2, err


def test_a_block_pass_equals_one_row_passes_bit_for_bit():
    """Row t of a 32-row causal pass at offset o equals the one-row pass at offset o + t, and a
    draft row equals itself alone: nothing a row computes depends on the other rows."""
    B, Hq, Hkv, Tq, cap = 2, 16, 8, 32, 900
    q, kc, vc, k2, v2 = [x.to(DEV) for x in _case(B, Hq, Hkv, Tq, cap, seed=99)]
    off = torch.tensor([250, 805], dtype=torch.int32, device=DEV)
    ops = _ops()
    full, _ = ops.attention_fwd(q, kc, vc, mask=0, hd=128, scale=128 ** -0.5, offset=off, want_lse=False)
    lim = torch.tensor([Tq, 17], dtype=torch.int32, device=DEV)
    dfull, _ = ops.attention_fwd(q, kc, vc, k2, v2, mask=2, hd=128, scale=128 ** -0.5, offset=off, limit2=lim,
                                 want_lse=False)
    for t in range(Tq):
        one, _ = ops.attention_fwd(q[:, :, t:t + 1].contiguous(), kc, vc, mask=0, hd=128, scale=128 ** -0.5,
                                   offset=off + t, want_lse=False)
        assert torch.equal(one[:, 0], full[:, t]), t
        done, _ = ops.attention_fwd(q[:, :, t:t + 1].contiguous(), kc, vc, k2, v2, mask=2, hd=128,
                                    scale=128 ** -0.5, offset=off, limit2=lim, want_lse=False)
        assert torch.equal(done[:, 0], dfull[:, t]), t


@pytest.mark.parametrize("R", [1, 32, 300, 1024])
def test_lmhead_argmax_equals_the_argmax_of_the_logits(R):
    """Greedy decoding picks tokens with the LM-head argmax kernel (no logits written); plain greedy
    paths take argmax_rows of the fp32 logits. Both must agree row for row (lossless decoding)."""
    ops = _ops()
    g = torch.Generator().manual_seed(R)
    V, d = 151936, 1024
    w = (torch.randn(V, d, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    h = torch.randn(R, d, generator=g).to(torch.bfloat16).to(DEV)
    h[0] = h[-1]  # a repeated row
    want = ops.argmax_rows(ops.gemm(h, w, out_dtype=torch.float32))
    got = ops.lmhead_argmax(h, w)
    assert torch.equal(got, want)
    # a tie: two vocabulary rows equal, the lower index wins
    w2 = w.clone()
    w2[5000] = w2[123456] = h[0] * 4
    assert ops.lmhead_argmax(h[:1], w2).item() == ops.argmax_rows(ops.gemm(h[:1], w2, out_dtype=torch.float32)).item() == 5000
