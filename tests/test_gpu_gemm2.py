"""The projection GEMM on CTA pairs (orthrus_gemm2_bf16, tcgen05 cta_group::2) against fp32 torch:
every operand layout of the forward, dX and dW forms, the residual epilogue, ragged sizes and
run-to-run determinism."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(*shape, seed, scale=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, device=DEV, generator=g) * scale).bfloat16()


# (1024, 2048, 8192) and (256, 512, 4096) fill less than one wave of SM pairs and are split over K
@pytest.mark.parametrize("M,N,K", [(512, 256, 128), (300, 96, 200), (1000, 1024, 3072), (256, 512, 64),
                                   (2048, 1024, 2048), (1024, 2048, 8192), (256, 512, 4096)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm2_layouts_match_fp32(M, N, K, a_t, b_t):
    from orthrus_training_b200 import ops

    if a_t and M % 8:
        pytest.skip("a transposed A needs M to be a multiple of 8")
    a = _rand(*((K, M) if a_t else (M, K)), seed=M + K)
    b = _rand(*((K, N) if b_t else (N, K)), seed=N + 3 * K, scale=0.05)
    got = ops.gemm2(a, b, a_t=a_t, b_t=b_t)
    A = a.float().t() if a_t else a.float()
    B = b.float() if b_t else b.float().t()
    ref = A @ B
    err = (got.float() - ref).abs().max().item()
    assert err <= 8e-3 * ref.abs().max().item(), err
    again = ops.gemm2(a, b, a_t=a_t, b_t=b_t)
    assert torch.equal(got, again)


@pytest.mark.parametrize("M,N,K,b_t", [(512, 256, 128, False), (300, 96, 200, True), (2048, 1024, 3072, False),
                                       (256, 512, 4096, False)])
def test_gemm2_residual_epilogue(M, N, K, b_t):
    from orthrus_training_b200 import _lib as lib_

    if (M, N, K) == (256, 512, 4096):
        assert lib_.lib().orthrus_gemm2_workspace_bytes(M, N, K) > 0  # the split-K path
    from orthrus_training_b200 import _lib, ops

    a = _rand(M, K, seed=1)
    b = _rand(*((K, N) if b_t else (N, K)), seed=2, scale=0.05)
    r = _rand(M, N, seed=3)
    got = ops.gemm2(a, b, b_t=b_t, residual=r)
    ref = r.float() + a.float() @ (b.float() if b_t else b.float().t())
    err = (got.float() - ref).abs().max().item()
    assert err <= 8e-3 * ref.abs().max().item(), err
    assert _lib.device_error(0) == 0


@pytest.mark.parametrize("M,d,F", [(1000, 256, 512), (8192, 1024, 3072)])
def test_swiglu_backward_epilogue_matches_the_separate_kernels(M, d, F):
    """[dgate | dup] from the GEMM epilogue equals silu_mul_backward(gate_up, dy @ W_down) up to
    the accumulation order of dact (one bf16 unit in its rounding)."""
    from orthrus_training_b200 import _lib, ops

    dy, w_down, gu = _rand(M, d, seed=11), _rand(d, F, seed=12, scale=0.05), _rand(M, 2 * F, seed=13)
    got = ops.gemm2_swiglu_backward(dy, w_down, gu)
    dact = (dy.float() @ w_down.float()).bfloat16()
    ref = ops.silu_mul_backward(gu, dact).float()
    err = (got.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err
    # with dact from the same GEMM (stored, same k order) the two paths agree bit for bit
    same = ops.silu_mul_backward(gu, ops.gemm2(dy, w_down, b_t=True))
    assert torch.equal(got, same)
    assert _lib.device_error(0) == 0


def test_rmsnorm_backward_adds_the_residual_gradient():
    from orthrus_training_b200 import ops

    x, w = _rand(777, 1024, seed=21), (1 + 0.1 * _rand(1024, seed=22).float()).bfloat16()
    dy, dres = _rand(777, 1024, seed=23), _rand(777, 1024, seed=24)
    _, rstd = ops.rms_norm(x, w, 1e-6, want_rstd=True)
    got = ops.rms_norm_backward(x, w, rstd, dy, dres=dres).float()
    ref = ops.rms_norm_backward(x, w, rstd, dy).float() + dres.float()
    assert (got - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


@pytest.mark.parametrize("K", [64, 192, 1024, 3072])
@pytest.mark.parametrize("epi,N", [("store", 1024), ("store", 4096), ("residual", 1024), ("swiglu", 1536),
                                   ("swiglu", 3072)])
def test_skinny_projection_rows_do_not_depend_on_the_row_count(epi, N, K):
    """The few-row projection kernel of the inference passes gives a row the same bits whatever the
    row count of the call (1 row, a 32-row block, 300 and 5000 rows: all three tile widths and both
    row-slot sizes occur), for K of one k-block, of a partial four-k-block box, and the model's
    1024 and 3072; and the same bits as the persistent 128 x 256 kernel, so a pass may take either
    by its row count without breaking the batch invariance of decoding."""
    from orthrus_training_b200 import ops

    x = _rand(5000, K, seed=K)
    w = _rand(2 * N if epi == "swiglu" else N, K, seed=7, scale=0.03)
    r = _rand(5000, N, seed=9) if epi == "residual" else None

    def run(rows, skinny=True):
        if epi == "swiglu":
            return ops.linear_swiglu(x[:rows], w, skinny=skinny)
        return ops.linear(x[:rows], w, residual=None if r is None else r[:rows], skinny=skinny)

    full = run(5000)
    for rows in (1, 32, 300):
        assert torch.equal(run(rows), full[:rows]), rows
    assert torch.equal(run(5000, skinny=False), full)
    assert torch.equal(run(32, skinny=False), full[:32])


def test_pair_mode_of_the_fused_projection_kernel_matches_one_cta():
    """The fused-epilogue projection kernel on CTA pairs (the training step's launch form) against
    its one-CTA form: store, residual and SwiGLU through the pair flag; the q|k|v + prologue and
    the kept SwiGLU forms at training sizes (which take the pair form) against the one-CTA store
    kernel followed by the prologue / activation."""
    from orthrus_training_b200 import _lib, ops

    M, K = 4096, 1024
    x = _rand(M, K, seed=31)
    w = _rand(1024, K, seed=32, scale=0.03)
    r = _rand(M, 1024, seed=33)
    for res in (None, r):
        a, b = ops.linear(x, w, residual=res), ops.linear(x, w, residual=res, pair=True)
        assert (a.float() - b.float()).abs().max().item() <= 1e-2 * a.float().abs().max().item()
    wg = _rand(2 * 1536, K, seed=34, scale=0.03)
    a, b = ops.linear_swiglu(x, wg), ops.linear_swiglu(x, wg, pair=True)
    assert (a.float() - b.float()).abs().max().item() <= 2e-2 * a.float().abs().max().item()
    y, gu = ops.linear_swiglu(x, wg, keep_gate_up=True)
    assert torch.equal(y, b) and torch.equal(gu, ops.linear(x, wg, pair=True))
    B, L, Hq, Hkv = 2, 2048, 16, 8
    xq = _rand(B * L, K, seed=35)
    wq = _rand((Hq + 2 * Hkv) * 128, K, seed=36, scale=0.03)
    qn = (1 + 0.2 * _rand(128, seed=37).float()).bfloat16()
    inv = ops.rope_inv_freq(128, 1e6, DEV)
    rope = ops.rope_table(inv, L)
    q, k, v = ops.linear_qkv_rope(xq, wq, qn, qn, rope, B, L, Hq, Hkv, 1e-6)
    pos = torch.arange(L, device=DEV).repeat(B).view(B, L)
    rq, rk, rv, _ = ops.qkv_prep(ops.linear(xq, wq, pair=True), pos, inv, qn, qn, B, L, Hq, Hkv, 128, 128, 1e-6)
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
    print("pair vs one-CTA store bit-identical:", torch.equal(ops.linear(x, w), ops.linear(x, w, pair=True)))
    assert _lib.device_error(0) == 0
