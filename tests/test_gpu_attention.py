"""Dual-view attention, q/k norm + RoPE prologue and the decode step kernels vs the oracle (GPU)."""

import math

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from orthrus_training_b200 import ops

    return ops


def _anchors(B, A, L, K, seed):
    g = torch.Generator().manual_seed(seed)
    rows = [torch.randperm(L - K, generator=g)[:A].add(1).sort().values for _ in range(B)]
    return torch.stack(rows)


def _dual_case(B, Hq, Hkv, L, A, K, hd, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    Tq = A * K
    q = torch.randn(B, Hq, Tq, hd, generator=g)
    k1 = torch.randn(B, Hkv, L, hd, generator=g)
    v1 = torch.randn(B, Hkv, L, hd, generator=g)
    k2 = torch.randn(B, Hkv, Tq, hd, generator=g)
    v2 = torch.randn(B, Hkv, Tq, hd, generator=g)
    anchors = _anchors(B, A, L, K, seed)
    ts = [t.to(dtype).float() for t in (q, k1, v1, k2, v2)]
    return ts, anchors


def _oracle_dual(ts, anchors, L, K, grad_out=None):
    q, k1, v1, k2, v2 = [t.clone().requires_grad_(True) for t in ts]
    mask = O.dense_block_mask(anchors, L, K)
    out = O.masked_attention(q, torch.cat([k1, k2], 2), torch.cat([v1, v2], 2), mask)
    grads = None
    if grad_out is not None:
        out.backward(grad_out)
        grads = (q.grad, k2.grad, v2.grad)
    return out.detach(), grads


@pytest.mark.parametrize("dtype,hd,L,A,K", [(torch.bfloat16, 128, 300, 8, 32),
                                             (torch.bfloat16, 128, 700, 12, 16),
                                             (torch.bfloat16, 64, 260, 4, 64),
                                             (torch.float32, 32, 120, 5, 8)])
def test_dual_view_attention_forward_backward(dtype, hd, L, A, K):
    B, Hq, Hkv = 2, 4, 2
    ts, anchors = _dual_case(B, Hq, Hkv, L, A, K, hd, dtype, seed=L + A)
    Tq = A * K
    D = hd if hd >= 64 else hd
    dev = [t.to(DEV).to(dtype) for t in ts]
    scale = 1.0 / math.sqrt(hd)
    o, lse = _ops().attention_fwd(dev[0], dev[1], dev[2], dev[3], dev[4], mask=1, hd=hd, scale=scale,
                                  anchors=anchors.to(DEV), block=K)
    g = torch.Generator().manual_seed(7)
    dout = torch.randn(B, Tq, Hq, hd, generator=g).to(dtype).float()
    ref, (rdq, rdk, rdv) = _oracle_dual(ts, anchors, L, K, grad_out=dout.transpose(1, 2))
    got = o.float().cpu().transpose(1, 2)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert (got - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    dq, dk, dv = _ops().attention_bwd(dev[0], dev[1], dev[2], dev[3], dev[4], anchors.to(DEV), K, o,
                                      lse, dout.to(DEV).to(dtype), hd=hd, scale=scale)
    for name, a, r in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        a = a[..., :hd].cpu()
        err = (a - r).abs().max().item()
        assert err <= (3e-2 if dtype == torch.bfloat16 else 2e-5) * max(1.0, r.abs().max().item()), (name, err)


def test_dual_view_rescale_in_some_rows_of_a_warp():
    """The forward raises a row's reference max (and rescales its O accumulator in TMEM) only when
    a tile max exceeds it by 2^8. Here the rows of the first block see one AR key and an own block
    with large scores, so they rescale, while the rows of the next block (same warp) do not: the
    rescale must still be correct when only part of a warp needs it."""
    B, Hq, Hkv, L, A, K, hd = 1, 4, 2, 300, 8, 16, 128
    dtype = torch.bfloat16
    ts, _ = _dual_case(B, Hq, Hkv, L, A, K, hd, dtype, seed=11)
    anchors = torch.tensor([[1, 40, 80, 120, 160, 200, 240, 280]])
    k2 = ts[3].clone()
    k2[:, :, :K] *= 6.0  # the own block of the first anchor: scores about 6x larger
    ts = [ts[0], ts[1], ts[2], k2.to(dtype).float(), ts[4]]
    dev = [t.to(DEV).to(dtype) for t in ts]
    o, _ = _ops().attention_fwd(dev[0], dev[1], dev[2], dev[3], dev[4], mask=1, hd=hd,
                                scale=1.0 / math.sqrt(hd), anchors=anchors.to(DEV), block=K)
    ref, _ = _oracle_dual(ts, anchors, L, K)
    got = o.float().cpu().transpose(1, 2)
    assert (got - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    from orthrus_training_b200 import _lib

    assert _lib.device_error(0) == 0


@pytest.mark.parametrize("dtype,hd", [(torch.bfloat16, 128), (torch.float32, 32), (torch.bfloat16, 64)])
def test_teacher_causal_attention(dtype, hd):
    B, Hq, Hkv, T = 2, 4, 2, 333
    g = torch.Generator().manual_seed(hd)
    q, k, v = [torch.randn(B, h, T, hd, generator=g).to(dtype).float() for h in (Hq, Hkv, Hkv)]
    o, lse = _ops().attention_fwd(q.to(DEV).to(dtype), k.to(DEV).to(dtype), v.to(DEV).to(dtype),
                                  mask=0, hd=hd, scale=1 / math.sqrt(hd))
    ref = O.masked_attention(q, k, v, None, causal=True)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert (o.float().cpu().transpose(1, 2) - ref).abs().max().item() <= tol


def _tree_lo(branches):
    return [1] + [1 + sum(branches[:g]) for g, n in enumerate(branches) for _ in range(n)]


@pytest.mark.parametrize("dtype,hd,offsets,branches", [
    (torch.bfloat16, 128, [150], [5, 3, 6]),            # tensor-core path, one query tile
    (torch.bfloat16, 128, [97, 260], [70, 60, 69]),     # two query tiles, per-row offsets
    (torch.bfloat16, 64, [33], [31]),                   # one branch: the causal verification
    (torch.float32, 64, [150, 40], [5, 3, 6]),          # CUDA-core path
])
def test_tree_mask_attention(dtype, hd, offsets, branches):
    """Tree verification (mask TREE): the new tokens sit in the cache at rows offset[b] + t;
    query t sees rows < offset[b] + 1 and its own branch [offset[b] + lo[t], offset[b] + t + 1).
    Against the dense-mask oracle: bf16 2e-2, fp32 1e-5."""
    B, Hq, Hkv = len(offsets), 4, 2
    lo = _tree_lo(branches)
    T = len(lo)
    cap = max(offsets) + T + 40
    g = torch.Generator().manual_seed(T + hd)
    q = torch.randn(B, Hq, T, hd, generator=g).to(dtype).float()
    k = torch.randn(B, Hkv, cap, hd, generator=g).to(dtype).float()
    v = torch.randn(B, Hkv, cap, hd, generator=g).to(dtype).float()
    mask = torch.zeros(B, T, cap, dtype=torch.bool)
    for b, off in enumerate(offsets):
        for t in range(T):
            mask[b, t, : off + 1] = True
            mask[b, t, off + lo[t]: off + t + 1] = True
    ref = O.masked_attention(q.double(), k.double(), v.double(), mask).float()
    kd, vd = k.to(DEV).to(dtype), v.to(DEV).to(dtype)
    o, _ = _ops().attention_fwd(q.to(DEV).to(dtype), kd, vd, kd, vd, mask=3, hd=hd, scale=hd ** -0.5,
                                offset=torch.tensor(offsets, dtype=torch.int32, device=DEV),
                                limit2=torch.tensor(lo, dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    got = o.float().cpu().permute(0, 2, 1, 3)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert (got - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())


def test_tree_mask_needs_branch_starts():
    q = torch.zeros(1, 2, 4, 64, device=DEV).bfloat16()
    k = torch.zeros(1, 2, 16, 64, device=DEV).bfloat16()
    off = torch.tensor([3], dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        _ops().attention_fwd(q, k, k, k, k, mask=3, hd=64, scale=0.125, offset=off)
    with pytest.raises(ValueError):
        _ops().attention_fwd(q, k, k, k, k, mask=3, hd=64, scale=0.125, offset=off,
                             limit2=torch.ones(3, dtype=torch.int32, device=DEV))


def test_tilemap_matches_mask():
    anchors = torch.tensor([[3, 10, 30, 200], [1, 2, 36, 500]])
    tm = _ops().attention_tilemap(anchors.to(DEV), 32, 400).cpu()
    assert tm.shape == (2, 1, 4)
    assert tm[0, 0].tolist() == [2, 200, 0, 128]
    assert tm[1, 0].tolist() == [4, 400, 0, 128]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_qkv_prep_matches_oracle(dtype):
    B, T, Hq, Hkv, hd = 2, 37, 4, 2, 32
    D = 64
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * hd, generator=g).to(dtype)
    pos = torch.randint(0, 2000, (B, T), generator=g)
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).to(dtype)
    inv = _ops().rope_inv_freq(hd, 1e6, DEV)
    q, k, v, rstd = _ops().qkv_prep(qkv.to(DEV), pos.to(DEV), inv, qw.to(DEV), kw.to(DEV), B, T, Hq, Hkv,
                                    hd, D, 1e-6, want_rstd=True)
    x = qkv.view(B, T, -1)
    rq = O.rms_norm(x[..., :Hq * hd].view(B, T, Hq, hd), qw, 1e-6).transpose(1, 2)
    rk = O.rms_norm(x[..., Hq * hd:(Hq + Hkv) * hd].view(B, T, Hkv, hd), kw, 1e-6).transpose(1, 2)
    cos, sin = O.rope_cos_sin(pos, hd, 1e6, dtype)
    rq, rk = O.apply_rope(rq, cos, sin), O.apply_rope(rk, cos, sin)
    rv = x[..., (Hq + Hkv) * hd:].view(B, T, Hkv, hd).transpose(1, 2)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (q[..., :hd].float().cpu() - rq.float()).abs().max().item() <= tol * 4
    assert (k[..., :hd].float().cpu() - rk.float()).abs().max().item() <= tol * 4
    assert torch.equal(v[..., :hd].cpu(), rv)
    assert (q[..., hd:] == 0).all() and (k[..., hd:] == 0).all()


def test_qkv_prep_backward_matches_autograd():
    B, T, Hq, Hkv, hd, D = 2, 19, 4, 2, 32, 64
    g = torch.Generator().manual_seed(4)
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * hd, generator=g)
    pos = torch.randint(0, 500, (B, T), generator=g)
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    gq = torch.randn(B, Hq, T, hd, generator=g)
    gk = torch.randn(B, Hkv, T, hd, generator=g)
    gv = torch.randn(B, Hkv, T, hd, generator=g)
    inv = _ops().rope_inv_freq(hd, 1e6, DEV)
    _, _, _, rstd = _ops().qkv_prep(qkv.to(DEV), pos.to(DEV), inv, qw.to(DEV), kw.to(DEV), B, T, Hq, Hkv,
                                    hd, D, 1e-6, want_rstd=True)
    pad = lambda t: torch.nn.functional.pad(t, (0, D - hd)).to(DEV)
    dqkv, dqw, dkw = _ops().qkv_prep_backward(qkv.to(DEV), pos.to(DEV), inv, qw.to(DEV), kw.to(DEV), rstd,
                                              pad(gq), pad(gk), pad(gv), B, T, Hq, Hkv, hd, D)
    x = qkv.clone().requires_grad_(True)
    qw_, kw_ = qw.clone().requires_grad_(True), kw.clone().requires_grad_(True)
    xv = x.view(B, T, -1)
    cos, sin = O.rope_cos_sin(pos, hd, 1e6)
    rq = O.apply_rope(O.rms_norm(xv[..., :Hq * hd].view(B, T, Hq, hd), qw_, 1e-6).transpose(1, 2), cos, sin)
    rk = O.apply_rope(O.rms_norm(xv[..., Hq * hd:(Hq + Hkv) * hd].view(B, T, Hkv, hd), kw_, 1e-6).transpose(1, 2),
                      cos, sin)
    rv = xv[..., (Hq + Hkv) * hd:].view(B, T, Hkv, hd).transpose(1, 2)
    ((rq * gq).sum() + (rk * gk).sum() + (rv * gv).sum()).backward()
    assert torch.allclose(dqkv.cpu(), x.grad, rtol=1e-4, atol=1e-5)
    assert torch.allclose(dqw.cpu(), qw_.grad, rtol=1e-4, atol=1e-4)
    assert torch.allclose(dkw.cpu(), kw_.grad, rtol=1e-4, atol=1e-4)


def test_qkv_prep_backward_bf16_0_6b_heads_matches_autograd():
    """bf16 at the Qwen3-0.6B head layout (16 / 8 heads of 128: the pipelined backward kernel),
    67 rows per sequence so the warps' row counts are ragged, against fp32 autograd of the same
    bf16 inputs with the bf16-rounded rotary table the kernel uses."""
    B, T, Hq, Hkv, hd, D = 2, 67, 16, 8, 128, 128
    g = torch.Generator().manual_seed(8)
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * hd, generator=g).bfloat16()
    pos = torch.randint(0, 2000, (B, T), generator=g)
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16()
    gq = torch.randn(B, Hq, T, hd, generator=g)
    gk = torch.randn(B, Hkv, T, hd, generator=g)
    gv = torch.randn(B, Hkv, T, hd, generator=g)
    inv = _ops().rope_inv_freq(hd, 1e6, DEV)
    _, _, _, rstd = _ops().qkv_prep(qkv.to(DEV), pos.to(DEV), inv, qw.to(DEV), kw.to(DEV), B, T, Hq, Hkv,
                                    hd, D, 1e-6, want_rstd=True)
    dqkv, dqw, dkw = _ops().qkv_prep_backward(qkv.to(DEV), pos.to(DEV), inv, qw.to(DEV), kw.to(DEV), rstd,
                                              gq.to(DEV), gk.to(DEV), gv.to(DEV), B, T, Hq, Hkv, hd, D)
    x = qkv.float().requires_grad_(True)
    qw_, kw_ = qw.float().requires_grad_(True), kw.float().requires_grad_(True)
    xv = x.view(B, T, -1)
    cos, sin = O.rope_cos_sin(pos, hd, 1e6, torch.bfloat16)
    cos, sin = cos.float(), sin.float()
    rq = O.apply_rope(O.rms_norm(xv[..., :Hq * hd].view(B, T, Hq, hd), qw_, 1e-6).transpose(1, 2), cos, sin)
    rk = O.apply_rope(O.rms_norm(xv[..., Hq * hd:(Hq + Hkv) * hd].view(B, T, Hkv, hd), kw_, 1e-6).transpose(1, 2),
                      cos, sin)
    rv = xv[..., (Hq + Hkv) * hd:].view(B, T, Hkv, hd).transpose(1, 2)
    ((rq * gq).sum() + (rk * gk).sum() + (rv * gv).sum()).backward()
    got, want = dqkv.float().cpu(), x.grad
    assert (got - want).abs().max().item() <= 1e-2 * want.abs().max().item()
    # the v part is the incoming gradient rounded to bf16
    assert torch.equal(dqkv.cpu().view(B, T, -1)[..., (Hq + Hkv) * hd:],
                       gv.transpose(1, 2).reshape(B, T, Hkv * hd).bfloat16())
    assert (dqw.cpu() - qw_.grad).abs().max().item() <= 1e-3 * qw_.grad.abs().max().item()
    assert (dkw.cpu() - kw_.grad).abs().max().item() <= 1e-3 * kw_.grad.abs().max().item()


def test_argmax_lowest_index_on_ties():
    x = torch.zeros(3, 151936, device=DEV)
    x[0, 5] = x[0, 99] = 1.0
    x[1, 151935] = 2.0
    x[2, :] = -1.0
    assert _ops().argmax_rows(x).tolist() == [5, 151935, 0]
    r = torch.randn(17, 1003, device=DEV)
    assert torch.equal(_ops().argmax_rows(r), r.argmax(-1))


def _accept_reference(drafts, ar, block_len, eos):
    """decoding._verify / _advance for one sequence (orthrus/decoding.py:336-369)."""
    accepted = 0
    while accepted < block_len - 1 and drafts[accepted] == ar[accepted]:
        accepted += 1
        if drafts[accepted - 1] in eos:
            break
    return accepted, ar[accepted]


def test_verify_accept_kernel_matches_reference_rules():
    B, K, V = 6, 8, 50
    g = torch.Generator().manual_seed(0)
    truth = torch.randint(0, V, (B, K), generator=g)
    drafts = truth[:, :-1].clone()
    for b, j in enumerate([0, 2, 7, 3, 5, 1]):
        if j < K - 1:
            drafts[b, j] = (drafts[b, j] + 1) % V
    eos = torch.tensor([int(truth[3, 1])])
    logits = torch.full((B, K, V), -5.0)
    logits.scatter_(2, truth[..., None], 5.0)
    verify_ids = torch.cat([torch.zeros(B, 1, dtype=torch.long), drafts], 1)
    start = torch.tensor([10, 10, 10, 10, 10, 14], dtype=torch.int32)
    max_len = torch.tensor([100, 100, 100, 100, 100, 18], dtype=torch.int32)
    dev = lambda t: t.to(DEV)
    st, an, dn = dev(start.clone()), dev(torch.zeros(B, dtype=torch.long)), dev(torch.zeros(B, dtype=torch.uint8))
    out, out_len = dev(torch.zeros(B, 64, dtype=torch.long)), dev(torch.zeros(B, dtype=torch.int32))
    log, cyc = dev(torch.zeros(B, 8, dtype=torch.int32)), dev(torch.zeros(B, dtype=torch.int32))
    ar = dev(torch.zeros(B, K, dtype=torch.long))
    _ops().decode_verify_accept(dev(logits), dev(verify_ids), ar, dev(eos), dev(max_len), st, an, dn, out,
                                out_len, log, cyc)
    torch.cuda.synchronize()
    assert torch.equal(ar.cpu(), truth)
    for b in range(B):
        block_len = min(K, int(max_len[b]) - int(start[b]))
        acc, bonus = _accept_reference(drafts[b].tolist(), truth[b].tolist(), block_len, set(eos.tolist()))
        assert log[b, 0].item() == acc
        kept = drafts[b, :acc].tolist()
        if any(t in eos.tolist() for t in kept):
            cut = next(i for i, t in enumerate(kept) if t in eos.tolist())
            assert out[b, :out_len[b]].tolist() == kept[:cut + 1] and dn[b].item() == 1
            continue
        ns = int(start[b]) + acc + 1
        assert st[b].item() == ns and an[b].item() == bonus
        expect = kept + ([bonus] if ns < int(max_len[b]) else [])
        assert out[b, :out_len[b]].tolist() == expect
        assert dn[b].item() == int(ns >= int(max_len[b]) - 1)
