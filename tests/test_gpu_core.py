"""GEMM and fused LM-head + KL kernels against the oracle / an fp32 torch reference (GPU only)."""

import pytest
import torch
from conftest import load_golden

import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from orthrus_training_b200 import ops

    return ops


def _ref_mm(a, b, b_kn=False):
    bb = b.double() if b_kn else b.double().t()
    return (a.double() @ bb).float()


@pytest.mark.parametrize("M,N,K,b_kn", [(300, 512, 320, False), (129, 384, 192, True),
                                        (64, 1024, 4096, False), (257, 1024, 3072, True),
                                        (1000, 256, 64, False)])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemm_bf16_tcgen05(M, N, K, b_kn, out_f32):
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    b = torch.randn(K, N, device=DEV, generator=g).bfloat16() if b_kn else torch.randn(
        N, K, device=DEV, generator=g).bfloat16()
    c = _ops().gemm(a, b, b_kn=b_kn, out_dtype=torch.float32 if out_f32 else torch.bfloat16)
    torch.cuda.synchronize()
    ref = _ref_mm(a, b, b_kn)
    err = (c.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= (1e-5 if out_f32 else 8e-3) * scale + 1e-3, (err, scale)


def test_gemm_bf16_is_batch_invariant():
    g = torch.Generator(device=DEV).manual_seed(0)
    w = torch.randn(1024, 3072, device=DEV, generator=g).bfloat16()
    x = torch.randn(300, 3072, device=DEV, generator=g).bfloat16()
    full = _ops().gemm(x, w, out_dtype=torch.float32)
    for rows in (1, 7, 32, 129):
        part = _ops().gemm(x[:rows].contiguous(), w, out_dtype=torch.float32)
        assert torch.equal(part, full[:rows])


def test_gemm_simt_fp32_exact_and_batch_invariant():
    g = torch.Generator(device=DEV).manual_seed(1)
    w = torch.randn(777, 1536, device=DEV, generator=g)
    x = torch.randn(97, 1536, device=DEV, generator=g)
    full = _ops().gemm(x, w)
    ref = _ref_mm(x, w)
    assert torch.allclose(full, ref, rtol=1e-5, atol=1e-4)
    for rows in (1, 5, 32):
        assert torch.equal(_ops().gemm(x[:rows].contiguous(), w), full[:rows])


def _bf16(t):
    return t.bfloat16().float()


@pytest.mark.parametrize("M,N,K", [(300, 512, 320), (16384 // 8, 4096, 1024), (129, 1024, 3072),
                                   (1000, 384, 72)])
def test_fused_linear_store_and_residual(M, N, K):
    """orthrus_linear_bf16 (persistent tcgen05 kernel) against fp32 torch: ragged M, N with a
    half-empty last tile (384 = 256 + 128), K not a multiple of 64. Store: one rounding of the fp32
    product; residual: the fp32 sum rounded once (torch.addmm with beta = 1)."""
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    r = torch.randn(M, N, device=DEV, generator=g).bfloat16()
    ref = x.double() @ w.double().t()
    y = _ops().linear(x, w)
    yr = _ops().linear(x, w, residual=r)
    torch.cuda.synchronize()
    # fp32 accumulation in another order: compare within a bf16 rounding of the result
    assert (y.double() - ref).abs().max().item() <= 8e-3 * ref.abs().max().item() + 1e-3
    ref_r = ref + r.double()
    assert (yr.double() - ref_r).abs().max().item() <= 8e-3 * ref_r.abs().max().item() + 1e-3
    # the epilogue rounds once: residual form equals rounding (fp32 product + residual)
    prod = (x.float() @ w.float().t())
    assert (yr.float() - (prod + r.float()).bfloat16().float()).abs().max().item() <= \
        2e-2 * ref_r.abs().max().item()


@pytest.mark.parametrize("M,F,K", [(300, 256, 320), (2048, 3072, 1024), (77, 768, 256)])
def test_fused_linear_swiglu_matches_silu_mul(M, F, K):
    """SwiGLU epilogue against the unfused path silu_mul(x @ [gate; up]^T): the same roundings
    (gate and up to bf16, silu to bf16, product to bf16), so the two agree to one bf16 ulp of the
    inputs' accumulation-order differences."""
    g = torch.Generator(device=DEV).manual_seed(M + F)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2 * F, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    h = _ops().linear_swiglu(x, w)
    gu = (x.double() @ w.double().t()).float()
    gate, up = _bf16(gu[:, :F]), _bf16(gu[:, F:])
    ref = _bf16(_bf16(torch.nn.functional.silu(gate)) * up)
    torch.cuda.synchronize()
    err = (h.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err
    # agreement with the two-kernel path on the same GPU (GEMM then orthrus_swiglu_fwd)
    two = _ops().silu_mul(_ops().linear(x, w))
    assert (h.float() - two.float()).abs().max().item() <= 2e-2 * ref.abs().max().item()


@pytest.mark.parametrize("B,L,K,Hq,Hkv", [(2, 256, 1024, 16, 8), (1, 384, 320, 4, 2), (3, 128, 256, 6, 1)])
def test_fused_qkv_rope_matches_the_prologue(B, L, K, Hq, Hkv):
    """q|k|v GEMM with the q/k RMSNorm + RoPE prologue in its epilogue against the two-kernel path
    through the same GEMM mainloop (orthrus_linear_bf16 store, then orthrus_qkv_prep_fwd): the
    same fp32 accumulators and the same arithmetic, so bit-identical outputs are expected; and
    against an fp32 torch restatement of the prologue within bf16 rounding."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(B * L + K)
    H = Hq + 2 * Hkv
    x = torch.randn(B * L, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(H * 128, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    qn = (1 + 0.2 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    kn = (1 + 0.2 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    inv = ops.rope_inv_freq(128, 1_000_000.0, torch.device(DEV))
    rope = ops.rope_table(inv, L)
    q, k, v = ops.linear_qkv_rope(x, w, qn, kn, rope, B, L, Hq, Hkv, 1e-6)
    pos = torch.arange(L, device=DEV).repeat(B).view(B, L)
    rq, rk, rv, _ = ops.qkv_prep(ops.linear(x, w), pos, inv, qn, kn, B, L, Hq, Hkv, 128, 128, 1e-6)
    torch.cuda.synchronize()
    for got, ref in ((q, rq), (k, rk), (v, rv)):
        assert got.shape == ref.shape
        assert torch.equal(got, ref), (got.float() - ref.float()).abs().max().item()
    # fp32 restatement: RMSNorm per head, weight, rotate_half RoPE, bf16 roundings between steps
    qkv = (x.float() @ w.float().t()).bfloat16().float().view(B, L, H, 128)
    ang = torch.arange(L, device=DEV).float()[:, None] * inv[None]
    cos, sin = ang.cos().bfloat16().float(), ang.sin().bfloat16().float()
    cos, sin = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)

    def prep(t, wn):
        t = (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().float()
        t = (t * wn.float()).bfloat16().float()
        rot = torch.cat([-t[..., 64:], t[..., :64]], -1)
        return t * cos[None, :, None] + rot * sin[None, :, None]

    ref_q = prep(qkv[:, :, :Hq], qn).permute(0, 2, 1, 3)
    ref_k = prep(qkv[:, :, Hq:Hq + Hkv], kn).permute(0, 2, 1, 3)
    ref_v = qkv[:, :, Hq + Hkv:].permute(0, 2, 1, 3)
    for got, ref in ((q, ref_q), (k, ref_k), (v, ref_v)):
        assert (got.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("B,Q,K,Hq,Hkv", [(2, 256, 1024, 16, 8), (1, 384, 320, 4, 2)])
def test_fused_qkv_rope_keep_for_the_trainable_view(B, Q, K, Hq, Hkv):
    """The trainable view's form: RoPE at given positions (anchor + offset per block), and the q / k
    columns of the projection and rstd kept for the backward; all bit-identical to the projection
    kernel followed by the prologue kernel."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(Q + K + Hq)
    H = Hq + 2 * Hkv
    L = 2048
    x = torch.randn(B * Q, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(H * 128, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    qn = (1 + 0.2 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    kn = (1 + 0.2 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    inv = ops.rope_inv_freq(128, 1_000_000.0, torch.device(DEV))
    rope = ops.rope_table(inv, L)
    blocks = Q // 32
    anchors = torch.randint(1, L - 32, (B, blocks), device=DEV, generator=g).sort(-1).values
    pos = (anchors[:, :, None] + torch.arange(32, device=DEV)).reshape(B, Q).contiguous()
    q, k, v, qkv, rstd = ops.linear_qkv_rope(x, w, qn, kn, rope, B, Q, Hq, Hkv, 1e-6, positions=pos,
                                             keep=True)
    proj = ops.linear(x, w)
    rq, rk, rv, rr = ops.qkv_prep(proj, pos, inv, qn, kn, B, Q, Hq, Hkv, 128, 128, 1e-6, want_rstd=True)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
    assert torch.equal(qkv[:, : (Hq + Hkv) * 128], proj[:, : (Hq + Hkv) * 128])
    assert torch.equal(rstd, rr.view_as(rstd))
    from orthrus_training_b200 import _lib
    assert _lib.device_error(0) == 0


def test_rope_table_matches_sincos():
    ops = _ops()
    inv = ops.rope_inv_freq(128, 1_000_000.0, torch.device(DEV))
    cos, sin = ops.rope_table(inv, 300)
    ang = torch.arange(300, device=DEV, dtype=torch.float64)[:, None] * inv.double()[None]
    assert (cos.float() - ang.cos().float()).abs().max().item() <= 4e-3
    assert (sin.float() - ang.sin().float()).abs().max().item() <= 4e-3


@pytest.mark.parametrize("M,F,K", [(8192 // 16, 3072, 1024), (300, 256, 320)])
def test_fused_linear_swiglu_keep(M, F, K):
    """The SwiGLU form that also writes [gate | up]: the activation equals the plain SwiGLU form
    and the kept projection equals the store form (same mainloop, same roundings: bit-identical)."""
    g = torch.Generator(device=DEV).manual_seed(M + F)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2 * F, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    y, gu = _ops().linear_swiglu(x, w, keep_gate_up=True)
    torch.cuda.synchronize()
    assert torch.equal(y, _ops().linear_swiglu(x, w))
    assert torch.equal(gu, _ops().linear(x, w))


def test_student_mlp_backward_through_the_fused_swiglu():
    """dh of the fused gate/up + SwiGLU equals the autograd of F.linear + the activation kernels."""
    from orthrus_training_b200 import objective as ob

    g = torch.Generator(device=DEV).manual_seed(11)
    h = torch.randn(640, 256, device=DEV, generator=g).bfloat16().requires_grad_(True)
    w = (torch.randn(2 * 384, 256, device=DEV, generator=g) / 16).bfloat16()
    dact = torch.randn(640, 384, device=DEV, generator=g).bfloat16()
    ob._GateUpSwiGLU.apply(h, w).backward(dact)
    fused = h.grad.clone()
    h.grad = None
    ob._SwiGLU.apply(torch.nn.functional.linear(h, w)).backward(dact)
    ref = h.grad
    assert (fused.float() - ref.float()).abs().max().item() <= 2e-2 * ref.float().abs().max().item()


def test_fused_linear_rejects_bad_shapes():
    x = torch.randn(8, 64, device=DEV).bfloat16()
    with pytest.raises(ValueError):
        _ops().linear(x, torch.randn(100, 64, device=DEV).bfloat16())  # N not a multiple of 128
    with pytest.raises(ValueError):
        _ops().linear_swiglu(x, torch.randn(2 * 100, 64, device=DEV).bfloat16())


def _lmhead_case(n, m, V, d, dtype, seed, weighted):
    g = torch.Generator().manual_seed(seed)
    student = torch.randn(n, d, generator=g)
    teacher = torch.randn(m, d, generator=g)
    index = torch.randint(0, m, (n,), generator=g).sort().values
    weight = torch.randn(V, d, generator=g) * 0.5
    rw = torch.rand(n, generator=g) if weighted else None
    if dtype == torch.bfloat16:  # the oracle sees the same bf16-rounded inputs
        student, teacher, weight = student.bfloat16().float(), teacher.bfloat16().float(), \
            weight.bfloat16().float()
    return student, teacher, index, weight, rw


@pytest.mark.parametrize("kind", ["plain", "weighted"])
def test_lmhead_kl_fp32_matches_reference_kat(kind):
    """The reference's own known-answer case (tests/test_objective.py:16-38) through the fp32
    kernels: total / per-row KL 1e-5 relative, gradient 1e-4, agreement exact."""
    k = load_golden("kl_kat.pt")[kind]
    rw = k["row_weight"]
    total, kl, agree, grad, _, _ = _ops().lmhead_kl(
        k["student"].to(DEV), k["teacher"].to(DEV), k["index"].to(DEV), k["weight"].to(DEV),
        None if rw is None else rw.to(DEV))
    torch.cuda.synchronize()
    assert torch.allclose(total.cpu(), k["total"], rtol=1e-5, atol=1e-5)
    assert torch.allclose(kl.cpu(), k["kl_rows"], rtol=1e-5, atol=1e-6)
    assert torch.equal(agree.cpu(), k["agree"])
    assert torch.allclose(grad.cpu(), k["grad"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("n,m,V,d,weighted", [(300, 200, 1000, 128, False), (517, 300, 5003, 192, True)])
def test_lmhead_kl_bf16_matches_oracle(n, m, V, d, weighted):
    s, t, idx, w, rw = _lmhead_case(n, m, V, d, torch.bfloat16, n + V, weighted)
    offsets = torch.arange(n) % 7
    total, kl, agree, grad, kbo, abo = _ops().lmhead_kl(
        s.bfloat16().to(DEV), t.bfloat16().to(DEV), idx.to(DEV), w.bfloat16().to(DEV),
        None if rw is None else rw.to(DEV), offsets.to(DEV), 7, chunk_rows=256)
    torch.cuda.synchronize()
    r_total, r_kl, r_agree, r_grad = O.fused_linear_forward_kl(s, t, idx, w, rw)
    assert abs(total.item() - r_total.item()) <= 1e-2 * abs(r_total.item())
    assert (kl.cpu() - r_kl).abs().max().item() <= 2e-2 * r_kl.abs().max().item() + 1e-3
    assert (agree.cpu() == r_agree).float().mean().item() >= 0.99
    assert (grad.float().cpu() - r_grad).abs().max().item() <= 2e-2 * r_grad.abs().max().item()
    r_kbo = torch.zeros(7).index_add_(0, offsets, r_kl)
    assert torch.allclose(kbo.cpu(), r_kbo, rtol=2e-2, atol=1e-3)
    assert torch.equal(abo.cpu(), torch.bincount(offsets[agree.cpu()], minlength=7))


def test_lmhead_kl_fp32_matches_oracle_ragged():
    s, t, idx, w, rw = _lmhead_case(203, 77, 517, 40, torch.float32, 3, True)
    total, kl, agree, grad, _, _ = _ops().lmhead_kl(s.to(DEV), t.to(DEV), idx.to(DEV), w.to(DEV),
                                                    rw.to(DEV), chunk_rows=64)
    torch.cuda.synchronize()
    r_total, r_kl, r_agree, r_grad = O.fused_linear_forward_kl(s, t, idx, w, rw)
    assert torch.allclose(total.cpu(), r_total, rtol=1e-5)
    assert torch.allclose(kl.cpu(), r_kl, rtol=1e-5, atol=1e-6)
    assert torch.equal(agree.cpu(), r_agree)
    assert torch.allclose(grad.cpu(), r_grad, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("n,m,chunk_rows", [(1536, 1100, 4096), (3000, 3000, 2048)])
def test_lmhead_kl_bf16_full_vocab_vs_torch_fp32(n, m, chunk_rows):
    """0.6B LM-head shape (V = 151936, d = 1024) against an fp32 torch computation on the GPU. The
    second case gives every persistent CTA several (row tile, vocabulary split) units in both passes
    and splits the student rows into two chunks."""
    V, d = 151936, 1024
    g = torch.Generator(device=DEV).manual_seed(5)
    s = torch.randn(n, d, device=DEV, generator=g).bfloat16()
    t = torch.randn(m, d, device=DEV, generator=g).bfloat16()
    idx = torch.randint(0, m, (n,), device=DEV, generator=g).sort().values
    w = (torch.randn(V, d, device=DEV, generator=g) * 0.05).bfloat16()
    total, kl, agree, grad, _, _ = _ops().lmhead_kl(s, t, idx, w, chunk_rows=chunk_rows)
    ls = s.float() @ w.float().t()
    lt = t.float() @ w.float().t()
    lpt = lt.log_softmax(-1)[idx]
    lps = ls.log_softmax(-1)
    r_kl = (lpt.exp() * (lpt - lps)).sum(-1)
    r_agree = ls.argmax(-1) == lt.argmax(-1)[idx]
    r_grad = ((lps.exp() - lpt.exp()).bfloat16().float() @ w.float())
    assert abs(total.item() - r_kl.sum().item()) <= 1e-2 * r_kl.sum().item()
    assert (kl - r_kl).abs().max().item() <= 2e-2 * r_kl.abs().max().item()
    assert (agree == r_agree).float().mean().item() >= 0.99
    assert (grad.float() - r_grad).abs().max().item() <= 2e-2 * r_grad.abs().max().item() + 1e-4


def test_lmhead_kl_deterministic():
    s, t, idx, w, rw = _lmhead_case(400, 250, 3000, 128, torch.bfloat16, 9, True)
    args = (s.bfloat16().to(DEV), t.bfloat16().to(DEV), idx.to(DEV), w.bfloat16().to(DEV), rw.to(DEV))
    a = _ops().lmhead_kl(*args)
    b = _ops().lmhead_kl(*args)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and torch.equal(a[3], b[3])


def test_no_device_error_left():
    from orthrus_training_b200 import _lib

    assert _lib.device_error(0) == 0


def test_device_prefetcher_delivers_the_host_batches():
    """Micro-batches reach the device one ahead of use, with the host order and contents."""
    import numpy as np

    from orthrus_training_b200.data_io import DevicePrefetcher, batches

    rng = np.random.default_rng(1)
    ids = rng.integers(0, 1000, size=(20, 64), dtype=np.int32)
    mask = (rng.random((20, 64)) < 0.5).astype(np.uint8)
    host = list(batches(ids, mask, 4, 5, 0))
    got = list(DevicePrefetcher(batches(ids, mask, 4, 5, 0), DEV))
    assert [g[0] for g in got] == [h[0] for h in host]
    for (_, gi, gm), (_, hi, hm) in zip(got, host):
        assert gi.is_cuda and torch.equal(gi.cpu(), hi) and torch.equal(gm.cpu(), hm)
