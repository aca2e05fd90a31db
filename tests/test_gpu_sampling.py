"""Sampled decoding on the device (GPU): the Philox generator, the top-k / top-p filter against the
reference's own distributions (tests/golden/sampling.pt, pinned to the oracle on the CPU), the
rejection-sampling cycle's output distribution, and the decode loop end to end."""

import pytest
import torch
from conftest import load_golden

import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from orthrus_training_b200 import ops

    return ops


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors of its authors' distribution."""
    M = 0xFFFFFFFF
    cases = [([0, 0, 0, 0, 0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
             ([M, M, M, M, M, M], [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
             ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344, 0xA4093822, 0x299F31D0],
              [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1])]

    def as_i32(words):
        return [w - (1 << 32) if w >= (1 << 31) else w for w in words]

    ck = torch.tensor([as_i32(c) for c, _ in cases], dtype=torch.int32, device=DEV)
    out = _ops().philox4x32_10(ck).cpu().tolist()
    assert out == [as_i32(w) for _, w in cases]


def _params(c, seed=0):
    return _ops().SamplingParams(c["temperature"], c["top_k"], c["top_p"], seed)


def _full(probs, ids, V):
    return torch.zeros(probs.shape[0], V, device=probs.device).scatter(1, ids, probs)


def test_filter_matches_the_reference_distributions():
    g = load_golden("sampling.pt")
    V = g["vocab"]
    for c in g["cases"]:
        params = _params(c)
        for logits, want in ((c["prefill_last"][None], c["first_probs"]), (c["draft_logits"], c["draft_probs"]),
                             (c["verify_logits"], c["ar_probs"])):
            vals, ids = _ops().sample_candidates(logits.to(DEV), params)
            got = _full(_ops().sample_probs(vals, params), ids, V).cpu()
            assert torch.equal(got > 0, want > 0), (c["top_k"], c["top_p"])  # the same tokens kept
            assert (got - want).abs().max().item() <= 2e-6


def _cycle_state(B, K, cap, start=10, max_new=100):
    i32, i64 = torch.int32, torch.int64
    return dict(
        max_len=torch.full((B,), start + max_new, dtype=i32, device=DEV),
        start=torch.full((B,), start, dtype=i32, device=DEV),
        anchor=torch.full((B,), 3, dtype=i64, device=DEV),
        done=torch.zeros(B, dtype=torch.uint8, device=DEV),
        out=torch.zeros(B, cap, dtype=i64, device=DEV),
        out_len=torch.ones(B, dtype=i32, device=DEV),
        log=torch.zeros(B, 8, dtype=i32, device=DEV),
        cycle=torch.zeros(B, dtype=i32, device=DEV),
        verify=torch.zeros(B, K, dtype=i64, device=DEV))


@pytest.mark.parametrize("case", [0, 2, 3, 5, 7])
def test_rejection_cycle_emits_the_verify_distribution(case):
    """Whatever the drafts' distribution q, the first token a cycle commits after the anchor is
    distributed as the verify pass's p_0 (exact rejection sampling), and draft 0 is kept with
    probability sum_x min(p_0(x), q_0(x)). 200k replicas of one cycle, each with its own draws."""
    g = load_golden("sampling.pt")
    c, V, K = g["cases"][case], g["vocab"], g["block_size"]
    ops = _ops()
    params = _params(c, seed=1234 + case)
    B = 200_000
    dv, di = ops.sample_candidates(c["draft_logits"].to(DEV), params)
    pv, pi = ops.sample_candidates(c["verify_logits"].to(DEV), params)
    C = dv.shape[-1]
    dv, di = dv.expand(B, K - 1, C).contiguous(), di.expand(B, K - 1, C).contiguous()
    pv, pi = pv.expand(B, K, C).contiguous(), pi.expand(B, K, C).contiguous()
    s = _cycle_state(B, K, cap=K + 4)
    qprob = torch.zeros(B, K - 1, C, device=DEV)
    ops.decode_sample_draft(dv, di, params, s["cycle"], s["anchor"], s["done"], s["verify"], qprob)
    ops.decode_sample_accept(pv, pi, qprob, di, params, s["verify"], None, s["max_len"], s["start"],
                             s["anchor"], s["done"], s["out"], s["out_len"], s["log"], s["cycle"])
    first = s["out"][:, 1].cpu()
    accepted = s["log"][:, 0].cpu()
    p0 = O.sampling_probs(c["verify_logits"], c["temperature"], c["top_k"], c["top_p"])[0].double()
    q0 = O.sampling_probs(c["draft_logits"], c["temperature"], c["top_k"], c["top_p"])[0].double()
    freq = torch.bincount(first, minlength=V).double() / B
    sigma = (p0 * (1 - p0) / B).sqrt()
    assert bool(((freq - p0).abs() <= 5 * sigma + 1e-4).all()), (freq - p0).abs().max().item()
    keep0 = torch.minimum(p0, q0).sum().item()
    rate = (accepted >= 1).double().mean().item()
    assert abs(rate - keep0) <= 5 * (keep0 * (1 - keep0) / B) ** 0.5 + 1e-4
    # the drafts are distributed as q_0 and every commit advanced the cache by accepted + 1
    dfreq = torch.bincount(s["verify"][:, 1].cpu(), minlength=V).double() / B
    assert bool(((dfreq - q0).abs() <= 5 * (q0 * (1 - q0) / B).sqrt() + 1e-4).all())
    assert torch.equal(s["start"].cpu(), 10 + accepted.to(torch.int32) + 1)


def _tiny():
    from test_gpu_model import _load

    g = load_golden("tiny_decode.pt")
    return _load(g), g


def test_top_1_sampling_is_greedy_decoding():
    """With top_k = 1 every distribution is a point mass on the argmax: the sampled cycle (draws
    and all) must reproduce greedy decoding token for token and cycle for cycle."""
    from orthrus_training_b200.decoding import block_decode

    model, g = _tiny()
    ops = _ops()
    for c in g["cases"]:
        greedy = block_decode(model, [c["prompt"]], c["max_new"], set(c["eos"]))
        sampled = block_decode(model, [c["prompt"]], c["max_new"], set(c["eos"]),
                               sampler=ops.SamplingParams(0.7, 1, 0.8, seed=5))
        assert sampled.tokens == greedy.tokens == [c["diffusion"]]
        assert sampled.accepted == greedy.accepted


def test_sampled_decoding_is_reproducible_from_its_seed():
    from orthrus_training_b200.decoding import block_decode

    model, g = _tiny()
    ops = _ops()
    V = g["config"]["vocab_size"]
    prompts = [c["prompt"] for c in g["cases"]]
    runs = [block_decode(model, prompts, 40, sampler=ops.SamplingParams(1.0, 20, 0.9, seed=s), use_graph=graph)
            for s, graph in ((11, True), (11, False), (12, True))]
    assert runs[0].tokens == runs[1].tokens  # graph replay == eager, same draws
    assert runs[0].accepted == runs[1].accepted
    assert runs[0].tokens != runs[2].tokens  # another seed, other draws
    for r in runs:
        for toks, acc in zip(r.tokens, r.accepted):
            assert len(toks) == 40 and all(0 <= t < V for t in toks)
            assert 1 + sum(a + 1 for a in acc) >= 40  # every cycle commits accepted + 1 tokens
    # the model-level entry point draws its seed from torch's default generator
    prompt = torch.tensor([prompts[0]], device=DEV)
    torch.manual_seed(3)
    a, sa = model.diffusion_generate(prompt, 24, temperature=0.8, top_k=20, top_p=0.9)
    torch.manual_seed(3)
    b, sb = model.diffusion_generate(prompt, 24, temperature=0.8, top_k=20, top_p=0.9)
    assert torch.equal(a, b) and sa.accepted == sb.accepted and a.shape[1] == len(prompts[0]) + 24


def test_sampler_refuses_what_the_device_filter_cannot_hold():
    ops = _ops()
    logits = torch.randn(2, 300, device=DEV)
    for bad in (ops.SamplingParams(0.0, 20, 0.8), ops.SamplingParams(1.0, 0, 0.8),
                ops.SamplingParams(1.0, ops.SAMPLE_MAX_TOP_K + 1, 0.8), ops.SamplingParams(1.0, 20, 0.0)):
        with pytest.raises(ValueError):
            ops.sample_candidates(logits, bad)
