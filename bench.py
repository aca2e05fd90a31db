"""Benchmark of the Orthrus dual-view training step (Qwen3-0.6B shape) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline metric, train input tok/s): per GPU one micro-batch of 8 packed rows x 2048
tokens (seed 1 + rank), 32 anchors per row, block K = 32, bf16, random-init Qwen3-0.6B-shape
weights; a step = frozen causal teacher pass + diffusion-view forward/backward + fused LM-head KL +
gradient all-reduce of the twins (N > 1) + clip + AdamW. Weak scaling: rows per GPU fixed.
Synthetic data stand in for the reference's private dataset: rows of ~300-token prompts plus
Geometric(mean 690) responses, Zipf(1.1) ids.

Prints one JSON line (rank 0). `value` is measured with each step's rows already resident in HBM;
`e2e` runs the same steps through the public API with the rows copied from pinned host memory and
the loss read back every step. The activations of a step are far larger than the 126 MB L2, so no
flush is needed between steps.

--impl reference times the reference algorithm's CPU implementation (the fp32 CPU port in oracle/)
on the host cores: each step is one 2048-token row of the same workload.
"""

from __future__ import annotations

import argparse
import datetime
import gc
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, SEQ, ANCHORS, BLOCK = 8, 2048, 32, 32
MASK_TOKEN, REAL_VOCAB = 151669, 151669
METRIC = "train input tok/s (Qwen3-0.6B dual-view step)"


def qwen3_06b_config():
    from orthrus_training_b200.synthetic import qwen3_06b_config as cfg06b

    return cfg06b(BLOCK, MASK_TOKEN)


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region. The sampler
    is started ahead of the region (nvidia-smi takes a while to start on a box of eight GPUs) and
    only the samples stamped between mark_start() and mark_end() are summarised."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.start = self.end = None

    def mark_start(self):
        self.start = datetime.datetime.now()

    def mark_end(self):
        self.end = datetime.datetime.now()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                stamp = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                if (self.start and stamp < self.start) or (self.end and stamp > self.end):
                    continue
                clock, mx = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            sm.append(clock)
            for name, val in zip(names, parts[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_rows(seed: int):
    from orthrus_training_b200.synthetic import packed_rows

    return packed_rows(ROWS, SEQ, REAL_VOCAB, seed, ids="zipf", doc="prompt_response")


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def cpu_params(cfg, seed: int = 1) -> dict:
    """Random-init fp32 parameters of the workload's model for the CPU port (twins trainable)."""
    g = torch.Generator().manual_seed(seed)
    d, inter, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qd, kvd = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd
    params = {}
    emb = torch.randn(cfg.vocab_size, d, generator=g) * 0.02
    params["model.embed_tokens.weight"] = emb
    params["lm_head.weight"] = emb
    params["model.norm.weight"] = torch.ones(d)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        for suf in ("", "_diff"):
            for n, shape in (("q_proj", (qd, d)), ("k_proj", (kvd, d)), ("v_proj", (kvd, d)),
                             ("o_proj", (d, qd))):
                params[f"{p}self_attn.{n}{suf}.weight"] = (torch.randn(*shape, generator=g) * 0.02
                                                           ).requires_grad_(bool(suf))
            params[f"{p}self_attn.q_norm{suf}.weight"] = torch.ones(hd).requires_grad_(bool(suf))
            params[f"{p}self_attn.k_norm{suf}.weight"] = torch.ones(hd).requires_grad_(bool(suf))
        for n, shape in (("gate_proj", (inter, d)), ("up_proj", (inter, d)), ("down_proj", (d, inter))):
            params[f"{p}mlp.{n}.weight"] = torch.randn(*shape, generator=g) * 0.02
        params[f"{p}input_layernorm.weight"] = torch.ones(d)
        params[f"{p}post_attention_layernorm.weight"] = torch.ones(d)
    return params


def cpu_baseline_sample() -> dict:
    """The reference algorithm on the host cores: orthrus_loss forward + backward of one row of
    the workload through the fp32 CPU port (oracle/), all host threads, one timed run after the
    parameters are built (about 10-30 s of CPU work)."""
    import oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = qwen3_06b_config()
    ocfg = O.OracleConfig.from_hf(cfg)
    params = cpu_params(cfg)
    ids, mask = make_rows(1)
    ids, mask = ids[:1], mask[:1]
    anchors, valid = O.sample_anchors(mask, BLOCK, ANCHORS, torch.Generator().manual_seed(0))
    t0 = time.perf_counter()
    loss, _ = O.orthrus_loss(params, ocfg, ids, mask, anchors, valid)
    loss.backward()
    sec = time.perf_counter() - t0
    return {"value": round(SEQ / sec, 2), "unit": "input tok/s", "cores": threads, "kind": "port",
            "sample": f"1 row x {SEQ} tokens, {ANCHORS} anchors, K={BLOCK}: fp32 orthrus_loss "
                      f"fwd+bwd through the CPU port of the reference algorithm ({sec:.1f} s)"}


def run_decode(args):
    """--decode: parallel block decoding of the 0.6B shape (random init). For each batch size,
    prompts of U[128, 512] Zipf ids, 512 new tokens, K = 32:
    - plain: the diffusion drafts of a random-init model are rejected, so every cycle commits one
      token (TPF below 1 is expected and is not a quality figure);
    - scripted: the drafts are the greedy continuation with seeded edits (the device analogue of
      the reference tests' ScriptedBackend), which exercises accept / rollback; the output must
      equal the plain run's tokens.
    Under torchrun every rank decodes its own prompts on its own GPU (replicas, no collective on
    the data path); `value` is the tokens of all ranks over the slowest rank's device time.
    One JSON line per configuration; achieved HBM bandwidth per pass = (weights + the KV read at
    the mean context) / time per pass. A CPU line times the reference algorithm (the oracle port,
    fp32) on a bounded sample."""
    import numpy as np

    from orthrus_training_b200.decoding import block_decode
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar
    from orthrus_training_b200.synthetic import zipf_ids

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    dtype = torch.bfloat16 if args.decode_dtype == "bf16" else torch.float32
    torch.manual_seed(2)
    cfg = qwen3_06b_config()
    with torch.device(dev):
        model = OrthrusLM(cfg).to(dtype)
    copy_diff_from_ar(model)
    model.eval()
    K, new = BLOCK, args.decode_new
    L, Hkv, hd = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
    esize = 2 if dtype == torch.bfloat16 else 4
    weight_bytes = sum(p.numel() for n, p in model.named_parameters()
                       if not any(f".{m}_diff." in n for m in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                                 "q_norm", "k_norm"))) * esize
    kv_per_token = 2 * L * Hkv * hd * esize
    pk = peaks()

    def timed_decode(prompts, **kw):
        barrier(world)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        res = block_decode(model, prompts, new, **kw)
        e1.record()
        torch.cuda.synchronize(dev)
        return res, e0.elapsed_time(e1) / 1e3

    def total_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return float(t.item())

    with torch.inference_mode():
        block_decode(model, [[1, 2, 3, 4] * 40], 16)  # kernel set-up outside the timed runs
    for batch in args.decode_batch:
        rng = np.random.default_rng(2 + batch + 1000 * rank)
        prompts = [zipf_ids(rng, int(rng.integers(128, 513)), REAL_VOCAB).tolist() for _ in range(batch)]
        with torch.inference_mode():
            # one untimed call of each kind with the timed calls' shapes first: lazy kernel loading,
            # the decode state's allocation and the capture of its cycle (reused by the timed call
            # with the same shapes) stay outside the timed calls
            block_decode(model, prompts, new)
            block_decode(model, prompts, new, draft_table=torch.zeros(batch, new, K - 1, dtype=torch.int64,
                                                                    device=dev))
            plain, plain_s = timed_decode(prompts)
            ref = plain.tokens
            # scripted drafts: the true continuation after each anchor, 5 % of tokens edited
            table = torch.zeros(batch, new, K - 1, dtype=torch.int64)
            erng = np.random.default_rng(7 + batch + 1000 * rank)
            for b, toks in enumerate(ref):
                for i in range(new):
                    nxt = toks[i + 1: i + K]
                    row = [t if erng.random() >= 0.05 else int(erng.integers(0, REAL_VOCAB)) for t in nxt]
                    table[b, i, : len(row)] = torch.tensor(row, dtype=torch.int64)
            scripted, scripted_s = timed_decode(prompts, draft_table=table.to(dev))
        lossless = total_over_ranks(float(scripted.tokens == ref)) == world
        for name, res, dev_s in (("plain", plain, plain_s), ("scripted", scripted, scripted_s)):
            # time the replayed cycles only; a plain cycle runs two model passes (draft, verify),
            # a scripted one only the verify pass (its drafts come from the table)
            model_passes = 2 if name == "plain" else 1
            per_pass = max_over_ranks(res.steady_seconds / max(model_passes * res.steady_cycles, 1), world)
            seconds = max_over_ranks(dev_s - res.prefill_seconds, world)
            gen = total_over_ranks(float(res.total_tokens))
            passes = total_over_ranks(float(sum(res.passes)))
            mean_ctx = sum(len(p) for p in prompts) / batch + new / 2
            pass_bytes = weight_bytes + kv_per_token * mean_ctx * batch
            gbs = pass_bytes / per_pass / 1e9
            line = {
                "metric": "decode tok/s (Qwen3-0.6B-shape Orthrus block decode, greedy)", "mode": name,
                "value": round(gen / seconds, 1), "unit": "generated tok/s", "n_gpus": world,
                "scaling": "weak", "batch_per_gpu": batch, "new_tokens": new, "K": K,
                "dtype": args.decode_dtype, "tpf": round(gen / max(passes, 1), 3),
                "mean_accepted": round(sum(sum(a) for a in res.accepted) / max(sum(res.cycles), 1), 3),
                "ms_per_pass": round(per_pass * 1e3, 4), "model_passes_per_cycle": model_passes,
                "hbm": {"bytes_per_pass": int(pass_bytes), "achieved_gbs": round(gbs, 1),
                        "peak_gbs": pk["hbm_gbs"], "frac": round(gbs / pk["hbm_gbs"], 4)},
                "lossless_vs_plain_greedy": bool(lossless) if name == "scripted" else True,
                "timing": "CUDA events around each rank's decode call (prefill excluded), max over ranks",
                "data": "synthetic Zipf(1.1) prompts, random-init weights",
            }
            if rank == 0:
                emit(json.dumps(line))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        ocfg = O.OracleConfig.from_hf(cfg)
        params = {k: v.detach() for k, v in cpu_params(cfg, seed=2).items()}
        prompt = torch.tensor([zipf_ids(np.random.default_rng(2), 128, REAL_VOCAB).tolist()])
        t0 = time.perf_counter()
        with torch.no_grad():
            toks, _ = O.diffusion_generate(params, ocfg, prompt, 8)
        sec = time.perf_counter() - t0
        emit(json.dumps({"metric": "decode tok/s (reference algorithm on the host cores)",
                          "value": round(8 / sec, 3), "unit": "generated tok/s", "cores": threads,
                          "kind": "port", "sample": f"batch 1, 128-token prompt, 8 new tokens, K={BLOCK}, "
                                                     f"fp32 diffusion_generate of the CPU port ({sec:.1f} s)"}))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()

def run_decode_cycle_profile(args):
    """--decode-cycle-profile B: the decode state of B prompts after prefill, one eager draft +
    verify cycle timed with CUDA events (mean of 4), then one more cycle between
    torch.cuda.profiler.start() / stop(), so `ncu --profile-from-start off` lists exactly the
    launches of one cycle."""
    import numpy as np

    from orthrus_training_b200 import ops
    from orthrus_training_b200.decoding import _DecodeState, block_decode
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar
    from orthrus_training_b200.synthetic import zipf_ids

    batch = args.decode_cycle_profile
    dev = torch.device("cuda", 0)
    torch.manual_seed(2)
    cfg = qwen3_06b_config()
    with torch.device(dev):
        model = OrthrusLM(cfg).to(torch.bfloat16)
    copy_diff_from_ar(model)
    model.eval()
    rng = np.random.default_rng(2 + batch)
    prompts = [zipf_ids(rng, int(rng.integers(128, 513)), REAL_VOCAB).tolist() for _ in range(batch)]
    with torch.inference_mode():
        block_decode(model, prompts, 8)
        st = _DecodeState.for_prompts(model, prompts, 64, set())
        for b, p in enumerate(prompts):  # prefill each prompt into its slice of the cache
            x = model.model.embed_tokens(torch.tensor([p], device=dev))
            pos = torch.arange(len(p), device=dev)[None]
            kv_b = [(k[b: b + 1], v[b: b + 1]) for k, v in st.kv]
            hidden = model.run_layers(x, pos, "ar", kv=kv_b, offsets=torch.zeros(1, dtype=torch.int32, device=dev))
            st.anchor[b] = ops.argmax_rows(model.lm_logits(hidden[:, -1:]).reshape(1, -1))[0]
        st.out_len.fill_(1)
        st.cycle_once()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(4):
            st.cycle_once()
        e1.record()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.start()
        st.cycle_once()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
    emit(json.dumps({"decode_cycle_profile": batch, "eager_ms_per_cycle": round(e0.elapsed_time(e1) / 4, 3),
                     "note": "eager launches (no CUDA graph); one cycle = draft pass + verify pass"}))


# --- isolated kernel cases (--kernel-case) -----------------------------------------------------
#
# Each hot entry point alone at the shapes of one training micro-batch (8 rows x 2048 tokens,
# 16 query / 8 KV heads of 128, 32 anchors, K = 32), timed with CUDA events per call. With small
# --steps these are also the programs the ncu captures profile: each keeps a few GB on the device
# and launches its kernels a handful of times.
#   causal   teacher attention forward, causal over 2048 keys          (orthrus/objective.py:155)
#   dual     dual-view attention forward, A*K queries over the AR prefix and own blocks (:163)
#   dualbwd  dual-view attention forward, then backward (dQ; dK/dV of the own-block keys)
#   lmhead   fused LM head + KL of one step: 7936 = 8 * 32 * 31 student rows against 7936 teacher
#            rows, V = 151936, d = 1024                                   (:338-392)
#   prologue q/k RMSNorm + RoPE + head-major scatter of the teacher's q|k|v projection, fwd + bwd
#   linear   the projections of a layer at 16384 rows through torch (cuBLAS) and through this
#            library's tcgen05 kernels                                    (:136-149)
#   linear2  every projection GEMM of the step (forward with residual, dX, dW) through cuBLAS and
#            through the CTA-pair kernel orthrus_gemm2_bf16
#   decode_proj the projections of a decode pass (32 and 1024 rows) on the persistent and the
#            128 x 64-tile kernels (weight bytes streamed per call)
#   sweep    dual-view attention fwd + bwd over L in {1024..8192}, K in {16, 32, 64}, A in
#            {8, 32, 64} (batch filling 16384 query tokens, at most 65536 keys per head), and the
#            fused LM head + KL over N in {4096, 16384, 65536} student rows

KC_HQ, KC_HKV, KC_HD = 16, 8, 128
KC_LM_N = ROWS * ANCHORS * (BLOCK - 1)
KC_LM_V, KC_LM_D = 151936, 1024


def _kc_time(fn, iters: int, warmup: int) -> float:
    """Milliseconds per call of fn: CUDA events around `iters` back-to-back calls."""
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


def _kc_time_graph(fn, iters: int, warmup: int) -> float:
    """Milliseconds per call of fn with `iters` calls captured in one CUDA graph and replayed, for
    kernels shorter than the host's per-call cost of the Python wrapper (back-to-back eager calls
    would time the host)."""
    for _ in range(max(warmup, 1)):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(iters):
            fn()
    graph.replay()  # the first replay uploads the graph
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _kc_dual_inputs(gen, dev, B, L, A, K):
    Tq = A * K
    rnd = lambda *shape: torch.randn(*shape, device=dev, generator=gen).bfloat16()  # noqa: E731
    q = rnd(B, KC_HQ, Tq, KC_HD)
    k1, v1 = rnd(B, KC_HKV, L, KC_HD), rnd(B, KC_HKV, L, KC_HD)
    k2, v2 = rnd(B, KC_HKV, Tq, KC_HD), rnd(B, KC_HKV, Tq, KC_HD)
    anchors = torch.stack([torch.randperm(L - K, device=dev, generator=gen)[:A].add(1).sort().values
                           for _ in range(B)])
    return q, k1, v1, k2, v2, anchors


def kernel_case(case: str, iters: int, warmup: int) -> dict:
    """{entry point: {"ms_per_call", "tflops" or "gbs"}} for one case."""
    import math

    from orthrus_training_b200 import ops

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    B, L, A, K, HQ, HKV, HD = ROWS, SEQ, ANCHORS, BLOCK, KC_HQ, KC_HKV, KC_HD
    sc = 1.0 / math.sqrt(HD)
    rnd = lambda *shape, scale=1.0: (torch.randn(*shape, device=dev, generator=gen) * scale).bfloat16()  # noqa
    timed = []  # (name, fn, algorithmic work per call, "tflops" | "gbs")
    if case == "causal":
        q, k, v = rnd(B, HQ, L, HD), rnd(B, HKV, L, HD), rnd(B, HKV, L, HD)
        timed.append(("attn_fwd_causal", lambda: ops.attention_fwd(q, k, v, mask=0, hd=HD, scale=sc),
                      ops.attention_flops(0, B, HQ, L, HD), "tflops"))
    elif case in ("dual", "dualbwd"):
        q, k1, v1, k2, v2, anchors = _kc_dual_inputs(gen, dev, B, L, A, K)
        fwd = lambda: ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=HD, scale=sc, anchors=anchors,  # noqa
                                        block=K)
        flops = float(ops.attention_flops(1, B, HQ, A * K, HD, anchors, K, L))
        timed.append(("attn_fwd_dual", fwd, flops, "tflops"))
        if case == "dualbwd":
            o, lse = fwd()
            dout = rnd(B, A * K, HQ, HD)
            timed.append(("attn_bwd_dual", lambda: ops.attention_bwd(q, k1, v1, k2, v2, anchors, K, o, lse, dout,
                                                                     hd=HD, scale=sc), 1.5 * flops, "tflops"))
    elif case == "lmhead":
        n = m = KC_LM_N
        s, t = rnd(n, KC_LM_D), rnd(m, KC_LM_D)
        idx = torch.randint(0, m, (n,), device=dev, generator=gen).sort().values
        w = rnd(KC_LM_V, KC_LM_D, scale=0.05)
        # logits of the student and unique teacher rows once each, plus the grad GEMM diff @ W
        timed.append(("lmhead_kl", lambda: ops.lmhead_kl(s, t, idx, w),
                      2.0 * KC_LM_D * KC_LM_V * (2 * n + m), "tflops"))
    elif case == "prologue":
        rows, H = B * L, HQ + 2 * HKV
        qkv = rnd(rows, H * HD)
        pos = torch.arange(L, device=dev).repeat(B)
        inv = ops.rope_inv_freq(HD, 1_000_000.0, dev)
        qw, kw = (1 + rnd(HD, scale=0.1).float()).bfloat16(), (1 + rnd(HD, scale=0.1).float()).bfloat16()
        q, k, v, rstd = ops.qkv_prep(qkv, pos, inv, qw, kw, B, L, HQ, HKV, HD, HD, 1e-6, want_rstd=True)
        dq, dk, dv = (torch.randn(t.shape, device=dev, generator=gen) for t in (q, k, v))
        timed.append(("qkv_prep_fwd", lambda: ops.qkv_prep(qkv, pos, inv, qw, kw, B, L, HQ, HKV, HD, HD, 1e-6),
                      2 * rows * H * HD * 2, "gbs"))  # bf16 in and out
        timed.append(("qkv_prep_bwd", lambda: ops.qkv_prep_backward(qkv, pos, inv, qw, kw, rstd, dq, dk, dv, B, L,
                                                                    HQ, HKV, HD, HD),
                      rows * H * HD * (2 + 4 + 2), "gbs"))
    elif case == "rownorm":
        # RMSNorm forward and backward (with the residual gradient) at the teacher's 16384 x 1024;
        # four input sets (about 270 MB) rotate so that no call finds its rows in L2
        import itertools

        rows, d = B * L, 1024
        sets = [(rnd(rows, d), rnd(rows, d), rnd(rows, d)) for _ in range(4)]  # x, dy, residual grad
        w = (1 + rnd(d, scale=0.1).float()).bfloat16()
        rstds = [ops.rms_norm(x, w, 1e-6, want_rstd=True)[1] for x, _, _ in sets]
        turn = itertools.count()

        def norm_fwd():
            return ops.rms_norm(sets[next(turn) % 4][0], w, 1e-6)

        def norm_bwd():
            i = next(turn) % 4
            x, dy, dres = sets[i]
            return ops.rms_norm_backward(x, w, rstds[i], dy, dres=dres)

        # timed as graph replays: an eager call of the wrapper costs the host longer than the kernel
        timed.append(("rmsnorm_fwd", norm_fwd, 2 * rows * d * 2, "gbs", _kc_time_graph))  # x in, y out
        timed.append(("rmsnorm_bwd_add", norm_bwd, 4 * rows * d * 2, "gbs", _kc_time_graph))  # x, dy, dres in; dx out
    elif case == "linear":
        rows, d, ff, hq = B * L, 1024, 3072, HQ * HD
        x, o, a = rnd(rows, d), rnd(rows, hq), rnd(rows, ff)
        w_qkv = rnd((HQ + 2 * HKV) * HD, d, scale=0.03)
        w_o, w_gu, w_d = rnd(d, hq, scale=0.02), rnd(2 * ff, d, scale=0.03), rnd(d, ff, scale=0.02)
        fl = lambda n, k: 2.0 * rows * n * k  # noqa: E731
        pos = torch.arange(L, device=dev).repeat(B).view(B, L)
        inv = ops.rope_inv_freq(HD, 1_000_000.0, dev)
        rope = ops.rope_table(inv, L)
        qw, kw = (1 + rnd(HD, scale=0.1).float()).bfloat16(), (1 + rnd(HD, scale=0.1).float()).bfloat16()
        nq = w_qkv.shape[0]
        timed += [
            ("qkv_prologue_cublas", lambda: ops.qkv_prep(x @ w_qkv.t(), pos, inv, qw, kw, B, L, HQ, HKV, HD, HD,
                                                         1e-6), fl(nq, d), "tflops"),
            ("qkv_prologue_fused", lambda: ops.linear_qkv_rope(x, w_qkv, qw, kw, rope, B, L, HQ, HKV, 1e-6),
             fl(nq, d), "tflops"),
            ("qkv_cublas", lambda: x @ w_qkv.t(), fl(nq, d), "tflops"),
            ("qkv_fused", lambda: ops.linear(x, w_qkv), fl(nq, d), "tflops"),
            ("o_residual_cublas", lambda: torch.addmm(x, o, w_o.t()), fl(d, hq), "tflops"),
            ("o_residual_fused", lambda: ops.linear(o, w_o, residual=x), fl(d, hq), "tflops"),
            ("gate_up_cublas", lambda: x @ w_gu.t(), fl(2 * ff, d), "tflops"),
            ("gate_up_swiglu_cublas", lambda: ops.silu_mul(x @ w_gu.t()), fl(2 * ff, d), "tflops"),
            ("gate_up_swiglu_fused", lambda: ops.linear_swiglu(x, w_gu), fl(2 * ff, d), "tflops"),
            ("down_residual_cublas", lambda: torch.addmm(x, a, w_d.t()), fl(d, ff), "tflops"),
            ("down_residual_fused", lambda: ops.linear(a, w_d, residual=x), fl(d, ff), "tflops"),
        ]
    elif case == "linear2":
        # every cuBLAS projection of the step against the CTA-pair kernel (forward with the
        # residual, dX = dY W, dW = dY^T X), teacher rows 16384 and trainable-view rows 8192
        d, ff, hq, qkv_n = 1024, 3072, HQ * HD, (HQ + 2 * HKV) * HD
        T_, S_ = B * L, B * A * K
        w_o, w_d = rnd(d, hq, scale=0.02), rnd(d, ff, scale=0.02)
        w_gu, w_qkv = rnd(2 * ff, d, scale=0.03), rnd(qkv_n, d, scale=0.03)
        xt_o, xt_a, rt = rnd(T_, hq), rnd(T_, ff), rnd(T_, d)
        xs_o, xs_a, rs = rnd(S_, hq), rnd(S_, ff), rnd(S_, d)
        dys, dgu, dqkv, hs = rnd(S_, d), rnd(S_, 2 * ff), rnd(S_, qkv_n), rnd(S_, d)
        fl = lambda m, n, k: 2.0 * m * n * k  # noqa: E731
        pairs = [
            ("o_residual_16384", lambda: torch.addmm(rt, xt_o, w_o.t()),
             lambda: ops.gemm2(xt_o, w_o, residual=rt), fl(T_, d, hq)),
            ("down_residual_16384", lambda: torch.addmm(rt, xt_a, w_d.t()),
             lambda: ops.gemm2(xt_a, w_d, residual=rt), fl(T_, d, ff)),
            ("o_residual_8192", lambda: torch.addmm(rs, xs_o, w_o.t()),
             lambda: ops.gemm2(xs_o, w_o, residual=rs), fl(S_, d, hq)),
            ("down_residual_8192", lambda: torch.addmm(rs, xs_a, w_d.t()),
             lambda: ops.gemm2(xs_a, w_d, residual=rs), fl(S_, d, ff)),
            ("down_dx_8192", lambda: dys @ w_d, lambda: ops.gemm2(dys, w_d, b_t=True), fl(S_, ff, d)),
            ("gate_up_dx_8192", lambda: dgu @ w_gu, lambda: ops.gemm2(dgu, w_gu, b_t=True), fl(S_, d, 2 * ff)),
            ("o_dx_8192", lambda: dys @ w_o, lambda: ops.gemm2(dys, w_o, b_t=True), fl(S_, hq, d)),
            ("o_dw_8192", lambda: dys.t() @ xs_o, lambda: ops.gemm2(dys, xs_o, a_t=True, b_t=True), fl(d, hq, S_)),
            ("qkv_dx_8192", lambda: dqkv @ w_qkv, lambda: ops.gemm2(dqkv, w_qkv, b_t=True), fl(S_, d, qkv_n)),
            ("qkv_dw_8192", lambda: dqkv.t() @ hs, lambda: ops.gemm2(dqkv, hs, a_t=True, b_t=True),
             fl(qkv_n, d, S_)),
        ]
        for name, ref_fn, own_fn, work in pairs:
            timed += [(name + "_cublas", ref_fn, work, "tflops"), (name + "_pair", own_fn, work, "tflops")]
    elif case == "decode_proj":
        # the projections of one decode pass (32 rows per sequence: batch 1 and 32) on the
        # persistent 128 x 256-tile kernel and on the 128 x 64-tile kernel
        d, ff, hq, qkv_n = 1024, 3072, HQ * HD, (HQ + 2 * HKV) * HD
        w_qkv, w_o = rnd(qkv_n, d, scale=0.03), rnd(d, hq, scale=0.02)
        w_gu, w_d = rnd(2 * ff, d, scale=0.03), rnd(d, ff, scale=0.02)
        for rows in (32, 1024):
            x, o, a, r = rnd(rows, d), rnd(rows, hq), rnd(rows, ff), rnd(rows, d)
            for sk in (False, True):
                tag = f"{rows}_{'skinny' if sk else 'persistent'}"
                # bytes of weights streamed per call: what bounds a pass of a few rows
                timed += [
                    (f"qkv_{tag}", lambda x=x, sk=sk: ops.linear(x, w_qkv, skinny=sk), w_qkv.numel() * 2, "gbs"),
                    (f"o_res_{tag}", lambda o=o, r=r, sk=sk: ops.linear(o, w_o, residual=r, skinny=sk),
                     w_o.numel() * 2, "gbs"),
                    (f"gate_up_swiglu_{tag}", lambda x=x, sk=sk: ops.linear_swiglu(x, w_gu, skinny=sk),
                     w_gu.numel() * 2, "gbs"),
                    (f"down_res_{tag}", lambda a=a, r=r, sk=sk: ops.linear(a, w_d, residual=r, skinny=sk),
                     w_d.numel() * 2, "gbs"),
                ]
    else:
        raise ValueError(f"unknown kernel case {case!r}")
    out = {}
    for name, fn, work, unit, *how in timed:
        ms = (how[0] if how else _kc_time)(fn, iters, warmup)
        rate = work / (ms / 1e3) / (1e9 if unit == "gbs" else 1e12)
        out[name] = {"ms_per_call": round(ms, 4), unit: round(float(rate), 1)}
    return out


def kernel_sweep(iters: int, warmup: int):
    """Yields one record per configuration as it is measured: dual-view attention forward and
    backward, then the fused LM head + KL."""
    import math

    from orthrus_training_b200 import ops

    dev = torch.device("cuda", 0)
    sc = 1.0 / math.sqrt(KC_HD)
    for L1 in (1024, 2048, 4096, 8192):
        for K1 in (16, 32, 64):
            for A1 in (8, 32, 64):
                if A1 * K1 > L1:
                    continue
                B1 = max(1, min(16384 // (A1 * K1), 65536 // L1))
                gen = torch.Generator(device=dev).manual_seed(L1 + K1 + A1)
                Tq = A1 * K1
                q, k1, v1, k2, v2, anchors = _kc_dual_inputs(gen, dev, B1, L1, A1, K1)
                fwd = lambda: ops.attention_fwd(q, k1, v1, k2, v2, mask=1, hd=KC_HD, scale=sc,  # noqa: E731
                                                anchors=anchors, block=K1)
                flops = float(ops.attention_flops(1, B1, KC_HQ, Tq, KC_HD, anchors, K1, L1))
                o, lse = fwd()
                dout = torch.randn(B1, Tq, KC_HQ, KC_HD, device=dev, generator=gen).bfloat16()
                bwd = lambda: ops.attention_bwd(q, k1, v1, k2, v2, anchors, K1, o, lse, dout,  # noqa: E731
                                                hd=KC_HD, scale=sc)
                tf, tb = _kc_time(fwd, iters, warmup), _kc_time(bwd, iters, warmup)
                yield {"case": "attention", "L": L1, "K": K1, "A": A1, "B": B1, "query_tokens": B1 * Tq,
                       "fwd_ms": round(tf, 4), "fwd_tflops": round(flops / tf / 1e9, 1),
                       "bwd_ms": round(tb, 4), "bwd_tflops": round(1.5 * flops / tb / 1e9, 1)}
                del q, k1, v1, k2, v2, o, lse, dout
    for n in (4096, 16384, 65536):
        gen = torch.Generator(device=dev).manual_seed(n)
        s = torch.randn(n, KC_LM_D, device=dev, generator=gen).bfloat16()
        t = torch.randn(n, KC_LM_D, device=dev, generator=gen).bfloat16()
        idx = torch.arange(n, device=dev)
        w = (torch.randn(KC_LM_V, KC_LM_D, device=dev, generator=gen) * 0.05).bfloat16()
        ms = _kc_time(lambda: ops.lmhead_kl(s, t, idx, w), max(1, iters // 4), max(1, warmup // 2))
        flops = 2.0 * KC_LM_D * KC_LM_V * (2 * n + n)
        yield {"case": "lmhead_kl", "N": n, "teacher_rows": n, "ms": round(ms, 3),
               "tflops": round(flops / ms / 1e9, 1)}
        del s, t, w


def run_kernel_case(args) -> None:
    """--kernel-case NAME: one isolated case on cuda:0 (--steps calls after --warmup), one JSON
    line per entry point (per configuration for the sweep); exits 1 if the device error word is
    set afterwards."""
    from orthrus_training_b200 import _lib

    torch.cuda.set_device(0)
    if args.kernel_case == "sweep":
        for rec in kernel_sweep(args.steps, args.warmup):
            emit(json.dumps(rec))
    else:
        for name, rec in kernel_case(args.kernel_case, args.steps, args.warmup).items():
            emit(json.dumps({"kernel_case": args.kernel_case, "entry_point": name, **rec}))
    err = _lib.device_error(0)
    if err:
        emit(json.dumps({"device_error": err}))
        raise SystemExit(1)


def step_roofline(cfg, kernels: dict, steps: int, ms_per_step: float, pk: dict) -> dict:
    """The whole step against its algorithmic work per GPU: projection GEMMs of the teacher
    (forward over every token) and of the diffusion view (forward, dX, and dW of the twins only),
    plus the attention and LM-head FLOPs the kernels counted in the breakdown pass."""
    d, inter, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers
    qkv = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * cfg.head_dim * d
    o = d * cfg.num_attention_heads * cfg.head_dim
    per_layer = qkv + o + 3 * d * inter
    teacher_tokens, student_tokens = ROWS * SEQ, ROWS * ANCHORS * BLOCK
    linear = 2.0 * L * (teacher_tokens * per_layer + 2 * student_tokens * per_layer
                        + student_tokens * (qkv + o))
    # the projections are counted in `linear` above, whichever kernel ran them
    kernel_flops = sum(v["flops"] for k, v in kernels.items() if not k.startswith("proj_")) / steps
    total = linear + kernel_flops
    achieved = total / (ms_per_step / 1e3) / 1e12
    return {"tflop_per_step": round(total / 1e12, 2), "achieved": round(achieved, 1),
            "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops_sustained"], 4), "peak_kind": "sustained"}


def run_reference(args):
    """--impl reference: the reference algorithm's CPU implementation timed on the host cores."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = qwen3_06b_config()
    ocfg = O.OracleConfig.from_hf(cfg)
    params = cpu_params(cfg)
    ids, mask = make_rows(1)
    times = []
    for step in range(args.warmup + args.steps):
        r = step % ROWS
        row_ids, row_mask = ids[r: r + 1], mask[r: r + 1]
        anchors, valid = O.sample_anchors(row_mask, BLOCK, ANCHORS, torch.Generator().manual_seed(step))
        t0 = time.perf_counter()
        loss, _ = O.orthrus_loss(params, ocfg, row_ids, row_mask, anchors, valid)
        loss.backward()
        for v in params.values():
            v.grad = None
        if step >= args.warmup:
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    value = SEQ / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "input tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "Qwen3-0.6B-shape dual-view train step, one "
                                        "2048-token row per step on the host cores",
                                        "rows": 1, "seq_len": SEQ, "anchors": ANCHORS, "block": BLOCK},
        "cpu_baseline": {"value": value, "unit": "input tok/s", "cores": threads, "kind": "port",
                         "sample": f"1 row x {SEQ} tokens per step, fp32 orthrus_loss fwd+bwd"},
        "e2e": {"value": value, "unit": "input tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(json.dumps(line))


def run_ours(args):
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    from orthrus_training_b200 import _lib, ops
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar
    from orthrus_training_b200.data_io import DevicePrefetcher
    from orthrus_training_b200.train_step import Trainer

    torch.manual_seed(1)
    cfg = qwen3_06b_config()
    with torch.device(dev):
        model = OrthrusLM(cfg).to(torch.bfloat16)
    copy_diff_from_ar(model)
    group = None
    trainer = Trainer(model, lr=1e-4, total_steps=1000, num_anchors=ANCHORS, kl_chunk_size=4096,
                      seed=1, world=world, rank=rank, group=group, layers_per_bucket=args.layers_per_bucket)
    ids, mask = make_rows(1 + rank)
    ids_dev, mask_dev = ids.to(dev), mask.to(dev)
    resident = torch.cuda.Event()  # the device-resident rows are complete from here on
    resident.record()
    h2d = ids.numel() * ids.element_size() + mask.numel() * mask.element_size()

    with ClockSampler(local) as clocks:  # started during the warm-up, summarised over the timed steps
        for _ in range(args.warmup):
            trainer.step([(ids_dev, mask_dev)], ready=resident)
        barrier(world)
        # Python's cyclic garbage collector stays off through the timed loops (collected once here
        # and re-enabled after them), so a collection pause of the host never lands in a timed step
        gc.collect()
        gc.disable()

        # device-resident inputs: the headline number, nothing else recorded in the timed region
        launches0 = _lib.launch_count()
        barrier(world)
        clocks.mark_start()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for i in range(args.steps):
            last = i == args.steps - 1
            if last:  # the last timed step is the one `ncu --profile-from-start off` captures
                torch.cuda.profiler.start()
            out = trainer.step([(ids_dev, mask_dev)], ready=resident)
            if last:
                torch.cuda.profiler.stop()
        e1.record()
        barrier(world)
        clocks.mark_end()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    launches = (_lib.launch_count() - launches0) // max(args.steps, 1)
    loss = float(out["loss"])

    # the same steps again with CUDA events around every entry point (on its launching stream)
    # for the per-kernel breakdown, kept out of the headline number. Recording ~1700 events a step
    # makes the host the slower side, and an event pair would then also time the host's gap before
    # the launch; so each step starts behind a ~60 ms device sleep that lets the host queue the
    # whole step first, and the pairs time device work only.
    ops.TIMER = ops.KernelTimer()
    barrier(world)
    for _ in range(args.steps):
        torch.cuda._sleep(100_000_000)
        trainer.step([(ids_dev, mask_dev)], ready=resident)
    barrier(world)
    kernels = ops.TIMER.summary()
    ops.TIMER = None

    comm = None
    if world > 1:
        # the same steps without the gradient all-reduce: the difference is the communication the
        # backward does not hide (every rank skips it, so all ranks still take the same collectives)
        trainer.buckets.world = 1
        barrier(world)
        c0, c1 = torch.cuda.Event(True), torch.cuda.Event(True)
        c0.record()
        for _ in range(args.steps):
            trainer.step([(ids_dev, mask_dev)], ready=resident)
        c1.record()
        barrier(world)
        trainer.buckets.world = world
        ms_nocomm = max_over_ranks(c0.elapsed_time(c1), world)
        grad_bytes = sum(p.numel() * p.element_size() for p in trainer.params)
        comm = {"ms_per_step_without_allreduce": round(ms_nocomm / args.steps, 3),
                "exposed_ms_per_step": round((ms - ms_nocomm) / args.steps, 3),
                "allreduce_bytes_per_step": grad_bytes, "collective": "NCCL all-reduce (AVG) of the twin "
                f"gradients, one bucket per {args.layers_per_bucket} layers, launched from grad hooks during "
                "the backward"}

    # end to end through the public API: host rows through DevicePrefetcher (pinned buffers, a
    # copy stream one micro-batch ahead), every step's loss read back to the host. A training
    # loop logs step i's loss once step i + 1 is queued, so the read does not drain the device
    # between steps; the last loss is read before the end event.
    barrier(world)
    f0, f1 = torch.cuda.Event(True), torch.cuda.Event(True)
    f0.record()
    feed = DevicePrefetcher(((i, ids, mask) for i in range(args.steps)), dev)
    pending = None
    for _, b_ids, b_mask in feed:
        o = trainer.step([(b_ids, b_mask)], ready=feed.ready)
        if pending is not None:
            float(pending)
        pending = o["loss"]
    float(pending)
    f1.record()
    barrier(world)
    gc.enable()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1), world)

    tokens = ROWS * SEQ * world * args.steps
    value = tokens / (ms / 1e3)
    pk = peaks()
    dominant = max(kernels.items(), key=lambda kv: kv[1]["ms"]) if kernels else None
    roofline = None
    if dominant:
        name, rec = dominant
        per_launch_ms = rec["ms"] / rec["launches"]
        achieved = rec["flops"] / rec["launches"] / (per_launch_ms / 1e3) / 1e12
        # the kernel is timed inside seconds of back-to-back steps: the sustained peak applies
        peak = pk["bf16_tflops_sustained"]
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.exists():
            traffic = json.loads(tfile.read_text()).get(name)
        roofline = {"bound": "tensor", "kernel": name, "achieved": round(achieved, 1),
                    "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                    "traffic": traffic, "peak_source": pk["source"], "peak_kind": "sustained",
                    "ms_per_launch": round(per_launch_ms, 4), "launches_per_step": rec["launches"] // args.steps}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "input tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded packed rows, Zipf(1.1) ids, random-init weights)",
        "config": {"workload": "Qwen3-0.6B-shape dual-view train step: 8 rows x 2048 tokens per GPU, "
                               "32 anchors/row, K=32, teacher pass + diffusion fwd/bwd + fused "
                               "LM-head KL + AdamW on the twins", "global_batch": ROWS * world,
                   "seq_len": SEQ, "parallelism": f"dp{world}",
                   "l2": "inputs and activations exceed the 126 MB L2 (no flush needed)"},
        "e2e": {"value": round(tokens / (ms_e2e / 1e3), 1), "unit": "input tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "step_roofline": step_roofline(cfg, kernels, args.steps, ms / args.steps, pk),
        "kernels": {k: {"launches_per_step": v["launches"] // args.steps,
                        "ms_per_step": round(v["ms"] / args.steps, 3),
                        "tflops": round(v["flops"] / (v["ms"] / 1e3) / 1e12, 1) if v["ms"] else None}
                    for k, v in sorted(kernels.items(), key=lambda kv: -kv[1]["ms"])},
        # step time not inside any library entry point: torch's AdamW, clipping, gathers and the
        # gaps between launches
        "unattributed_ms_per_step": round(ms / args.steps - sum(v["ms"] for v in kernels.values()) / args.steps, 3),
        "loss": round(loss, 5),
        "clocks": clocks.summary(),
    }
    if comm is not None:
        line["comm"] = comm
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample()
    err = _lib.device_error(local)
    if err:
        line["device_error"] = err
    if rank == 0:
        emit(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


_RESULT_FD: int | None = None  # the process's original stdout while a run is in progress


def emit(line: str) -> None:
    """Prints a result line on the original stdout, which carries nothing else during a run."""
    sys.stdout.flush()
    if _RESULT_FD is None:
        print(line, flush=True)
    else:
        os.write(_RESULT_FD, (line + "\n").encode())


def main():
    global _RESULT_FD
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers-per-bucket", type=int, default=4,
                    help="decoder layers per gradient all-reduce bucket (N > 1)")
    ap.add_argument("--decode", action="store_true", help="measure parallel block decoding instead")
    ap.add_argument("--decode-batch", type=int, nargs="+", default=[1, 32])
    ap.add_argument("--decode-new", type=int, default=512)
    ap.add_argument("--decode-dtype", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--decode-cycle-profile", type=int, default=None, metavar="BATCH",
                    help="run one eager draft + verify cycle at this batch between profiler start / stop "
                         "(for ncu --profile-from-start off) and print its CUDA-event time")
    ap.add_argument("--kernel-case", default=None,
                    choices=["causal", "dual", "dualbwd", "lmhead", "prologue", "rownorm", "linear", "linear2",
                             "decode_proj", "sweep"],
                    help="time one hot entry point alone (--steps calls after --warmup)")
    args = ap.parse_args()
    if args.warmup < 3 and args.kernel_case is None:
        raise SystemExit("--warmup must be >= 3")
    # native libraries may print on file descriptor 1 (NCCL's version banner at communicator
    # set-up): send all of that to stderr so stdout holds only the JSON result line
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    try:
        if args.kernel_case is not None:
            run_kernel_case(args)
        elif args.decode_cycle_profile is not None:
            run_decode_cycle_profile(args)
        elif args.decode:
            run_decode(args)
        elif args.impl == "reference":
            run_reference(args)
        else:
            run_ours(args)
    finally:
        sys.stdout.flush()
        os.dup2(_RESULT_FD, 1)
        os.close(_RESULT_FD)
        _RESULT_FD = None


if __name__ == "__main__":
    main()
