"""Opt-in document mask for packed rows (off by default, as in the reference, whose rows attend
across conversation boundaries: orthrus/objective.py:155 runs SDPA is_causal over the whole row and
orthrus/modeling_orthrus.py:58-74 lets a block see every AR key before its anchor).

The mask is not part of the reference, so its dense references here are the oracle's masks
(causal, dense_block_mask) narrowed by the document starts, in fp32 on the CPU."""

import math

import pytest
import torch

import oracle as O

DEV = "cuda"


def _starts_from_boundaries(B, L, seed, n=3, forced=()):
    """int32 [B, L] document starts from n random boundaries per row (position 0 always one) and
    the (row, position) boundaries in `forced`."""
    g = torch.Generator().manual_seed(seed)
    out = torch.zeros(B, L, dtype=torch.int32)
    for b in range(B):
        marks = torch.zeros(L, dtype=torch.int32)
        extra = [p for r, p in forced if r == b]
        for p in torch.randperm(L - 1, generator=g)[:n].add(1).tolist() + extra:
            marks[p] = p
        out[b] = marks.cummax(0).values
    return out


def test_document_starts_of_packed_conversations():
    from orthrus_training_b200.objective import document_starts

    mask = torch.tensor([[0, 0, 1, 1, 0, 0, 0, 1, 1, 1, 0, 1],   # two conversations, a third begins
                         [1, 1, 0, 1, 1, 1, 1, 0, 0, 1, 0, 0],   # a row opening inside a response
                         [0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0],   # no response: one document
                         [1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1]],  # one response across the row
                        dtype=torch.bool)
    want = torch.tensor([[0, 0, 0, 0, 4, 4, 4, 4, 4, 4, 10, 10],
                         [0, 0, 2, 2, 2, 2, 2, 7, 7, 7, 10, 10],
                         [0] * 12,
                         [0] * 12], dtype=torch.int32)
    got = document_starts(mask)
    assert got.dtype == torch.int32 and torch.equal(got, want)
    # monotone per row, never past the position itself
    pos = torch.arange(12, dtype=torch.int32)
    assert bool((got <= pos).all()) and bool((got[:, 1:] >= got[:, :-1]).all())


def test_document_starts_match_the_synthetic_packer():
    """On rows made by the synthetic packer (prompt then response, documents back to back) every
    start is a position where a prompt follows a response, or 0."""
    from orthrus_training_b200.objective import document_starts
    from orthrus_training_b200.synthetic import packed_rows

    _, mask = packed_rows(3, 512, 1023, seed=5, ids="uniform", doc="short")
    starts = document_starts(mask)
    m = mask.to(torch.bool)
    for b in range(3):
        for p in sorted(set(starts[b].tolist())):
            assert p == 0 or (bool(m[b, p - 1]) and not bool(m[b, p]))
        assert len(set(starts[b].tolist())) > 1  # short documents: several per row


def _causal_doc_mask(starts, T):
    """bool [B, T, T]: key c visible to query t when starts[t] <= c <= t."""
    t = torch.arange(T)[:, None]
    c = torch.arange(T)[None, :]
    return (c <= t)[None] & (c[None] >= starts[:, :, None].long())


def _dual_doc_mask(anchors, starts, L, K):
    """dense_block_mask narrowed to the anchor's document on the AR side."""
    base = O.dense_block_mask(anchors, L, K)
    Tq = anchors.shape[1] * K
    block = torch.arange(Tq) // K
    lo = starts.long().gather(1, anchors[:, block].clamp(max=L - 1))  # [B, Tq]
    kv = torch.arange(L + Tq)[None, None, :]
    return base & ((kv >= L) | (kv >= lo[:, :, None]))


def _ops():
    from orthrus_training_b200 import ops

    return ops


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hd", [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float32, 32)])
def test_causal_attention_keeps_to_the_document(dtype, hd):
    B, Hq, Hkv, T = 2, 4, 2, 333
    g = torch.Generator().manual_seed(hd + 1)
    q, k, v = [torch.randn(B, h, T, hd, generator=g).to(dtype).float() for h in (Hq, Hkv, Hkv)]
    starts = _starts_from_boundaries(B, T, seed=hd, n=4)
    o, _ = _ops().attention_fwd(q.to(DEV).to(dtype), k.to(DEV).to(dtype), v.to(DEV).to(dtype),
                                mask=0, hd=hd, scale=1 / math.sqrt(hd), doc_start=starts.to(DEV))
    ref = O.masked_attention(q, k, v, _causal_doc_mask(starts, T))
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert (o.float().cpu().transpose(1, 2) - ref).abs().max().item() <= tol


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hd,L,A,K", [(torch.bfloat16, 128, 600, 8, 32),
                                             (torch.bfloat16, 128, 700, 12, 16),
                                             (torch.float32, 32, 120, 5, 8)])
def test_dual_view_attention_keeps_to_the_anchor_document(dtype, hd, L, A, K):
    from test_gpu_attention import _dual_case

    B, Hq, Hkv = 2, 4, 2
    ts, anchors = _dual_case(B, Hq, Hkv, L, A, K, hd, dtype, seed=L + A + 1)
    # two blocks whose anchor opens a document: their AR prefix is empty
    forced = [(0, int(anchors[0, 1])), (1, int(anchors[1, 0]))]
    starts = _starts_from_boundaries(B, L, seed=L, n=5, forced=forced)
    assert int(starts[0, anchors[0, 1]]) == int(anchors[0, 1])
    Tq = A * K
    dev = [t.to(DEV).to(dtype) for t in ts]
    scale = 1.0 / math.sqrt(hd)
    o, lse = _ops().attention_fwd(dev[0], dev[1], dev[2], dev[3], dev[4], mask=1, hd=hd, scale=scale,
                                  anchors=anchors.to(DEV), block=K, doc_start=starts.to(DEV))
    g = torch.Generator().manual_seed(3)
    dout = torch.randn(B, Tq, Hq, hd, generator=g).to(dtype).float()
    q, k1, v1, k2, v2 = [t.clone().requires_grad_(True) for t in ts]
    ref = O.masked_attention(q, torch.cat([k1, k2], 2), torch.cat([v1, v2], 2),
                             _dual_doc_mask(anchors, starts, L, K))
    ref.backward(dout.transpose(1, 2))
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    got = o.float().cpu().transpose(1, 2)
    assert (got - ref.detach()).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    dq, dk, dv = _ops().attention_bwd(dev[0], dev[1], dev[2], dev[3], dev[4], anchors.to(DEV), K, o,
                                      lse, dout.to(DEV).to(dtype), hd=hd, scale=scale,
                                      doc_start=starts.to(DEV))
    for name, a, r in (("dq", dq, q.grad), ("dk", dk, k2.grad), ("dv", dv, v2.grad)):
        a = a[..., :hd].cpu()
        err = (a - r).abs().max().item()
        assert err <= (3e-2 if dtype == torch.bfloat16 else 2e-5) * max(1.0, r.abs().max().item()), (name, err)


@pytest.mark.gpu
def test_single_document_rows_equal_the_unmasked_kernels():
    """All starts 0: the masked kernels are bit-identical to the reference mask's."""
    from test_gpu_attention import _dual_case

    B, Hq, Hkv, L, A, K, hd = 2, 4, 2, 600, 8, 32, 128
    ts, anchors = _dual_case(B, Hq, Hkv, L, A, K, hd, torch.bfloat16, seed=21)
    dev = [t.to(DEV).to(torch.bfloat16) for t in ts]
    zero = torch.zeros(B, L, dtype=torch.int32, device=DEV)
    kw = dict(mask=1, hd=hd, scale=hd ** -0.5, anchors=anchors.to(DEV), block=K)
    o0, l0 = _ops().attention_fwd(*dev, **kw)
    o1, l1 = _ops().attention_fwd(*dev, **kw, doc_start=zero)
    assert torch.equal(o0, o1) and torch.equal(l0, l1)
    dout = torch.randn_like(o0)
    g0 = _ops().attention_bwd(*dev, anchors.to(DEV), K, o0, l0, dout, hd=hd, scale=hd ** -0.5)
    g1 = _ops().attention_bwd(*dev, anchors.to(DEV), K, o1, l1, dout, hd=hd, scale=hd ** -0.5,
                              doc_start=zero)
    assert all(torch.equal(a, b) for a, b in zip(g0, g1))
    q = torch.randn(B, Hq, L, hd, device=DEV, dtype=torch.bfloat16)
    c0, _ = _ops().attention_fwd(q, dev[1], dev[2], mask=0, hd=hd, scale=hd ** -0.5)
    c1, _ = _ops().attention_fwd(q, dev[1], dev[2], mask=0, hd=hd, scale=hd ** -0.5, doc_start=zero)
    assert torch.equal(c0, c1)


@pytest.mark.gpu
def test_later_documents_do_not_see_earlier_ones_through_the_model():
    """With the mask on, changing the tokens of a row's first conversation leaves the teacher's
    states of the later conversations, and the student's states of blocks anchored there, exactly
    as they were; with it off (the reference) they change."""
    from test_gpu_model import _bf16_tiny

    from orthrus_training_b200.objective import document_starts, model_states

    model, cfg = _bf16_tiny(seed=4)
    L, K = 256, cfg.block_size
    g = torch.Generator().manual_seed(8)
    ids = torch.randint(0, cfg.vocab_size - 1, (2, L), generator=g)
    mask = torch.zeros(2, L, dtype=torch.bool)
    mask[:, 40:100] = True    # first conversation: prompt 0..39, response 40..99
    mask[:, 130:200] = True   # second: prompt from 100
    ids2 = ids.clone()
    ids2[:, 5:90] = torch.randint(0, cfg.vocab_size - 1, (2, 85), generator=g)
    anchors = torch.tensor([[20, 60, 110, 150, 210], [30, 70, 120, 160, 220]])
    ids, ids2, mask, anchors = ids.to(DEV), ids2.to(DEV), mask.to(DEV), anchors.to(DEV)
    starts = document_starts(mask)
    assert starts[0, 150].item() == 100
    late = anchors[0] >= 100  # blocks anchored in the second conversation or later
    with torch.no_grad():
        s1, t1 = model_states(model, ids, anchors, doc_start=starts)
        s2, t2 = model_states(model, ids2, anchors, doc_start=document_starts(mask))
        u1, v1 = model_states(model, ids, anchors)
        u2, v2 = model_states(model, ids2, anchors)
    assert torch.equal(t1[:, 100:], t2[:, 100:])
    rows = s1.view(2, -1, K, s1.shape[-1])
    rows2 = s2.view(2, -1, K, s2.shape[-1])
    assert torch.equal(rows[:, late], rows2[:, late])
    assert not torch.equal(v1[:, 100:], v2[:, 100:])
    assert not torch.equal(u1.view_as(rows)[:, late], u2.view_as(rows)[:, late])


@pytest.mark.gpu
def test_training_step_with_the_document_mask_runs_and_defaults_off():
    from test_gpu_model import _bf16_tiny
    from test_gpu_train_step import _micro_batches

    from orthrus_training_b200.train_step import Trainer

    for flag in (False, True):
        model, _ = _bf16_tiny(seed=6)
        trainer = Trainer(model, lr=1e-3, total_steps=4, num_anchors=8, kl_chunk_size=256, seed=2,
                          document_mask=flag)
        batches = [(i.to(DEV), m.to(DEV)) for i, m in _micro_batches(77, 1)]
        out = trainer.step(batches)
        assert torch.isfinite(out["loss"]).item()
        if not flag:
            loss_off = out["loss"].item()
        else:
            assert out["loss"].item() != loss_off  # short packed documents: the mask matters
    assert Trainer.__init__.__kwdefaults__["document_mask"] is False
