"""Stand-alone cases of the hot kernels at the shapes of one Qwen3-0.6B training row group.

``python -m orthrus_training_b200.kernel_cases <case> [--iters N] [--warmup W]`` runs one case on
``cuda:0`` and prints, per entry point, its CUDA-event time per call and its algorithmic
throughput (the FLOP counts of ``ops.attention_flops`` and of the LM-head GEMMs). The same cases,
with small ``--iters``, are the programs the ncu captures profile: each keeps a few GB on the
device and launches its kernels a handful of times.

Cases (B = 8 rows of 2048 tokens, 16 query / 8 KV heads of 128, A = 32 anchors, K = 32):
  causal   teacher attention forward, causal over 2048 keys       (orthrus/objective.py:155)
  dual     dual-view attention forward, Tq = A*K queries over the AR prefix and own blocks
                                                                   (orthrus/objective.py:163)
  dualbwd  dual-view attention forward, then backward (dQ; dK/dV of the own-block keys)
  lmhead   fused LM head + KL of one step: 7936 = 8 * 32 * 31 student rows against 7936 teacher
           rows, V = 151936, d = 1024                              (orthrus/objective.py:338-392)
  prologue q/k RMSNorm + RoPE + head-major scatter of the teacher's fused q|k|v projection
           (16384 rows of 32 heads x 128), forward and backward    (orthrus/objective.py:136-143)
  linear   the teacher layer's projections at 16384 rows (d = 1024, q|k|v 4096, o 2048 -> 1024, gate|up
           2 x 3072, down 3072 -> 1024), each through torch / cuBLAS (plus orthrus_qkv_prep_fwd or
           orthrus_swiglu_fwd) and through the fused persistent kernels orthrus_linear_qkv_rope_bf16
           and orthrus_linear_bf16
                                                                   (orthrus/objective.py:136-149)
  sweep    dual-view attention forward + backward over L in {1024, 2048, 4096, 8192}, K in
           {16, 32, 64}, A in {8, 32, 64} (batch filling 16384 query tokens, capped at 65536 keys
           per head), and the fused LM head + KL over N in {4096, 16384, 65536} student rows
"""

from __future__ import annotations

import argparse
import math

import torch

from . import ops

B, HQ, HKV, L, A, K, HD = 8, 16, 8, 2048, 32, 32, 128
LM_N, LM_M, LM_V, LM_D = B * A * (K - 1), B * A * (K - 1), 151936, 1024


def _attention_inputs(gen, dev):
    Tq = A * K
    q = torch.randn(B, HQ, Tq, HD, device=dev, generator=gen).bfloat16()
    k1 = torch.randn(B, HKV, L, HD, device=dev, generator=gen).bfloat16()
    v1 = torch.randn(B, HKV, L, HD, device=dev, generator=gen).bfloat16()
    k2 = torch.randn(B, HKV, Tq, HD, device=dev, generator=gen).bfloat16()
    v2 = torch.randn(B, HKV, Tq, HD, device=dev, generator=gen).bfloat16()
    anchors = torch.stack([torch.randperm(L - K, device=dev, generator=gen)[:A].add(1).sort().values
                           for _ in range(B)])
    return q, k1, v1, k2, v2, anchors


def _time(fn, iters: int, warmup: int) -> float:
    """Milliseconds per call of ``fn``: CUDA events around ``iters`` back-to-back calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run(case: str, iters: int, warmup: int) -> dict:
    """{entry point: {"ms_per_call", "tflops"}} for one case."""
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    sc = 1.0 / math.sqrt(HD)
    timed = []  # (name, fn, algorithmic FLOPs per call)
    if case == "causal":
        q = torch.randn(B, HQ, L, HD, device=dev, generator=gen).bfloat16()
        k = torch.randn(B, HKV, L, HD, device=dev, generator=gen).bfloat16()
        v = torch.randn_like(k)
        timed.append(("attn_fwd_causal", lambda: ops.attention_fwd(q, k, v, mask=0, hd=HD, scale=sc),
                      ops.attention_flops(0, B, HQ, L, HD)))
    elif case in ("dual", "dualbwd"):
        q, k1, v1, k2, v2, anchors = _attention_inputs(gen, dev)
        fwd = lambda: ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=HD, scale=sc, anchors=anchors, block=K)
        flops = float(ops.attention_flops(1, B, HQ, A * K, HD, anchors, K, L))
        timed.append(("attn_fwd_dual", fwd, flops))
        if case == "dualbwd":
            o, lse = fwd()
            dout = torch.randn(B, A * K, HQ, HD, device=dev, generator=gen).bfloat16()
            timed.append(("attn_bwd_dual",
                          lambda: ops.attention_bwd(q, k1, v1, k2, v2, anchors, K, o, lse, dout, hd=HD, scale=sc),
                          1.5 * flops))
    elif case == "lmhead":
        s = torch.randn(LM_N, LM_D, device=dev, generator=gen).bfloat16()
        t = torch.randn(LM_M, LM_D, device=dev, generator=gen).bfloat16()
        idx = torch.randint(0, LM_M, (LM_N,), device=dev, generator=gen).sort().values
        w = (torch.randn(LM_V, LM_D, device=dev, generator=gen) * 0.05).bfloat16()
        # logits of the student and unique teacher rows once each, plus the grad GEMM diff @ W
        timed.append(("lmhead_kl", lambda: ops.lmhead_kl(s, t, idx, w),
                      2.0 * LM_D * LM_V * (2 * LM_N + LM_M)))
    elif case == "prologue":
        rows, H = B * L, HQ + 2 * HKV
        qkv = torch.randn(rows, H * HD, device=dev, generator=gen).bfloat16()
        pos = torch.arange(L, device=dev).repeat(B)
        inv = ops.rope_inv_freq(HD, 1_000_000.0, dev)
        qw = (1 + 0.1 * torch.randn(HD, device=dev, generator=gen)).bfloat16()
        kw = (1 + 0.1 * torch.randn(HD, device=dev, generator=gen)).bfloat16()
        q, k, v, rstd = ops.qkv_prep(qkv, pos, inv, qw, kw, B, L, HQ, HKV, HD, HD, 1e-6, want_rstd=True)
        dq, dk, dv = (torch.randn(t.shape, device=dev, generator=gen) for t in (q, k, v))
        nbytes = 2 * rows * H * HD * 2  # bf16 in and out
        timed.append(("qkv_prep_fwd", lambda: ops.qkv_prep(qkv, pos, inv, qw, kw, B, L, HQ, HKV, HD, HD, 1e-6),
                      nbytes))
        timed.append(("qkv_prep_bwd", lambda: ops.qkv_prep_backward(qkv, pos, inv, qw, kw, rstd, dq, dk, dv, B, L,
                                                                    HQ, HKV, HD, HD),
                      rows * H * HD * (2 + 4 + 2)))
    elif case == "linear":
        rows, d, ff, hq = B * L, 1024, 3072, HQ * HD
        x = torch.randn(rows, d, device=dev, generator=gen).bfloat16()
        o = torch.randn(rows, hq, device=dev, generator=gen).bfloat16()
        a = torch.randn(rows, ff, device=dev, generator=gen).bfloat16()
        w_qkv = (torch.randn((HQ + 2 * HKV) * HD, d, device=dev, generator=gen) * 0.03).bfloat16()
        w_o = (torch.randn(d, hq, device=dev, generator=gen) * 0.02).bfloat16()
        w_gu = (torch.randn(2 * ff, d, device=dev, generator=gen) * 0.03).bfloat16()
        w_d = (torch.randn(d, ff, device=dev, generator=gen) * 0.02).bfloat16()
        fl = lambda n, k: 2.0 * rows * n * k
        pos = torch.arange(L, device=dev).repeat(B).view(B, L)
        inv = ops.rope_inv_freq(HD, 1_000_000.0, dev)
        rope = ops.rope_table(inv, L)
        qw = (1 + 0.1 * torch.randn(HD, device=dev, generator=gen)).bfloat16()
        kw = (1 + 0.1 * torch.randn(HD, device=dev, generator=gen)).bfloat16()
        timed += [
            ("qkv_prologue_cublas", lambda: ops.qkv_prep(x @ w_qkv.t(), pos, inv, qw, kw, B, L, HQ, HKV, HD, HD,
                                                         1e-6), fl(w_qkv.shape[0], d)),
            ("qkv_prologue_fused", lambda: ops.linear_qkv_rope(x, w_qkv, qw, kw, rope, B, L, HQ, HKV, 1e-6),
             fl(w_qkv.shape[0], d)),
        ]
        timed += [
            ("qkv_cublas", lambda: x @ w_qkv.t(), fl(w_qkv.shape[0], d)),
            ("qkv_fused", lambda: ops.linear(x, w_qkv), fl(w_qkv.shape[0], d)),
            ("o_residual_cublas", lambda: torch.addmm(x, o, w_o.t()), fl(d, hq)),
            ("o_residual_fused", lambda: ops.linear(o, w_o, residual=x), fl(d, hq)),
            ("gate_up_cublas", lambda: x @ w_gu.t(), fl(2 * ff, d)),
            ("gate_up_swiglu_cublas", lambda: ops.silu_mul(x @ w_gu.t()), fl(2 * ff, d)),
            ("gate_up_swiglu_fused", lambda: ops.linear_swiglu(x, w_gu), fl(2 * ff, d)),
            ("down_residual_cublas", lambda: torch.addmm(x, a, w_d.t()), fl(d, ff)),
            ("down_residual_fused", lambda: ops.linear(a, w_d, residual=x), fl(d, ff)),
        ]
    else:
        raise ValueError(f"unknown case {case!r}")
    out = {}
    for name, fn, work in timed:
        ms = _time(fn, iters, warmup)
        if case == "prologue":  # HBM-bound: work is bytes moved
            out[name] = {"ms_per_call": round(ms, 4), "gbs": round(work / (ms / 1e3) / 1e9, 1)}
        else:
            out[name] = {"ms_per_call": round(ms, 4), "tflops": round(work / (ms / 1e3) / 1e12, 1)}
    return out


def sweep(iters: int, warmup: int):
    """Yields one record per configuration as it is measured: attention (dual view, fwd and bwd),
    then LM head + KL."""
    dev = torch.device("cuda", 0)
    sc = 1.0 / math.sqrt(HD)
    for L1 in (1024, 2048, 4096, 8192):
        for K1 in (16, 32, 64):
            for A1 in (8, 32, 64):
                if A1 * K1 > L1:
                    continue
                B1 = max(1, min(16384 // (A1 * K1), 65536 // L1))
                gen = torch.Generator(device=dev).manual_seed(L1 + K1 + A1)
                Tq = A1 * K1
                q = torch.randn(B1, HQ, Tq, HD, device=dev, generator=gen).bfloat16()
                k1 = torch.randn(B1, HKV, L1, HD, device=dev, generator=gen).bfloat16()
                v1 = torch.randn_like(k1)
                k2 = torch.randn(B1, HKV, Tq, HD, device=dev, generator=gen).bfloat16()
                v2 = torch.randn_like(k2)
                anchors = torch.stack([torch.randperm(L1 - K1, device=dev, generator=gen)[:A1].add(1).sort().values
                                       for _ in range(B1)])
                fwd = lambda: ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=HD, scale=sc, anchors=anchors,
                                                block=K1)
                flops = float(ops.attention_flops(1, B1, HQ, Tq, HD, anchors, K1, L1))
                o, lse = fwd()
                dout = torch.randn(B1, Tq, HQ, HD, device=dev, generator=gen).bfloat16()
                bwd = lambda: ops.attention_bwd(q, k1, v1, k2, v2, anchors, K1, o, lse, dout, hd=HD, scale=sc)
                tf, tb = _time(fwd, iters, warmup), _time(bwd, iters, warmup)
                yield {"case": "attention", "L": L1, "K": K1, "A": A1, "B": B1, "query_tokens": B1 * Tq,
                       "fwd_ms": round(tf, 4), "fwd_tflops": round(flops / tf / 1e9, 1),
                       "bwd_ms": round(tb, 4), "bwd_tflops": round(1.5 * flops / tb / 1e9, 1)}
                del q, k1, v1, k2, v2, o, lse, dout
    for n in (4096, 16384, 65536):
        gen = torch.Generator(device=dev).manual_seed(n)
        s = torch.randn(n, LM_D, device=dev, generator=gen).bfloat16()
        t = torch.randn(n, LM_D, device=dev, generator=gen).bfloat16()
        idx = torch.arange(n, device=dev)
        w = (torch.randn(LM_V, LM_D, device=dev, generator=gen) * 0.05).bfloat16()
        ms = _time(lambda: ops.lmhead_kl(s, t, idx, w), max(1, iters // 4), max(1, warmup // 2))
        flops = 2.0 * LM_D * LM_V * (2 * n + n)
        yield {"case": "lmhead_kl", "N": n, "teacher_rows": n, "ms": round(ms, 3),
               "tflops": round(flops / ms / 1e9, 1)}
        del s, t, w


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=["causal", "dual", "dualbwd", "lmhead", "prologue", "linear", "sweep"])
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args()
    if args.case == "sweep":
        import json

        for rec in sweep(args.iters, args.warmup):
            print(json.dumps(rec), flush=True)
        return
    for name, rec in run(args.case, args.iters, args.warmup).items():
        rate = f"{rec['gbs']} GB/s" if "gbs" in rec else f"{rec['tflops']} TF/s algorithmic"
        print(f"{name}: {rec['ms_per_call']:.3f} ms/call, {rate}", flush=True)
    from . import _lib
    err = _lib.device_error(0)
    print("device error word", err)
    if err:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
