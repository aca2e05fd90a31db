"""The CPU oracle reproduces the reference's outputs stored in tests/golden (pins the oracle)."""

import pytest
import torch
from conftest import load_golden, oracle_config

import oracle as O


@pytest.mark.parametrize("kind", ["plain", "weighted"])
def test_fused_kl_kat(kind):
    g = load_golden("kl_kat.pt")[kind]
    total, kl, agree, grad = O.fused_linear_forward_kl(
        g["student"], g["teacher"], g["index"], g["weight"], g["row_weight"])
    assert torch.allclose(total, g["total"], rtol=1e-5, atol=1e-5)
    assert torch.allclose(kl, g["kl_rows"], rtol=1e-5, atol=1e-6)
    assert torch.equal(agree, g["agree"])
    assert torch.allclose(grad, g["grad"], rtol=1e-4, atol=1e-6)


def test_block_mask_kat():
    g = load_golden("mask_kat.pt")
    dense = O.dense_block_mask(g["anchors"], g["seq_len"], g["block"])
    assert torch.equal(dense, g["mask"])


@pytest.mark.parametrize("fixture,case", [("config1.pt", "case"), ("config1.pt", "many_anchors"),
                                          ("tiny_model.pt", "case")])
def test_model_states_and_loss(fixture, case):
    g = load_golden(fixture)
    cfg = oracle_config(g["config"])
    c = g[case]
    gen = torch.Generator().manual_seed(c["anchor_seed"])
    anchors, valid = O.sample_anchors(c["assistant_mask"], cfg.block_size, c["num_anchors"], gen)
    assert torch.equal(anchors, c["anchors"]) and torch.equal(valid, c["valid"])
    params = {k: v.clone() for k, v in g["params"].items()}
    student, teacher = O.model_states(params, cfg, c["input_ids"], anchors)
    assert torch.allclose(teacher, c["teacher"], atol=1e-5, rtol=1e-5)
    assert torch.allclose(student, c["student"], atol=1e-5, rtol=1e-5)
    for gamma, ref in c["losses"].items():
        p = {k: (v.clone().requires_grad_("_diff." in k)) for k, v in g["params"].items()}
        p["lm_head.weight"] = p["model.embed_tokens.weight"] if torch.equal(
            g["params"]["lm_head.weight"], g["params"]["model.embed_tokens.weight"]) else p[
            "lm_head.weight"]
        loss, stats = O.orthrus_loss(p, cfg, c["input_ids"], c["assistant_mask"], anchors, valid,
                                     gamma=gamma)
        loss.backward()
        assert torch.allclose(loss, ref["loss"], rtol=1e-5, atol=1e-6)
        for key in ("tokens", "agree", "agree_by_offset", "tokens_by_offset"):
            assert torch.equal(stats[key], ref["stats"][key]), key
        for key in ("kl_sum", "weighted_kl_sum", "weight_sum", "valid_anchors"):
            assert torch.allclose(stats[key], ref["stats"][key], rtol=1e-5, atol=1e-6), key
        # offset 0 sums KLs of nearly identical distributions: rounding dominates, so an absolute
        # floor of 1e-5 on top of the relative 1e-5
        assert torch.allclose(stats["kl_by_offset"], ref["stats"]["kl_by_offset"], rtol=1e-5,
                              atol=1e-5)
        for name, grad in ref["grads"].items():
            assert p[name].grad is not None, name
            assert torch.allclose(p[name].grad, grad, rtol=1e-4, atol=1e-6), name
        assert all(p[n].grad is None for n in p if "_diff." not in n)


def test_decode_greedy_and_lossless():
    g = load_golden("tiny_decode.pt")
    cfg = oracle_config(g["config"])
    for c in g["cases"]:
        out, accepted = O.diffusion_generate(g["params"], cfg, torch.tensor([c["prompt"]]),
                                             c["max_new"], set(c["eos"]))
        assert out[0, len(c["prompt"]):].tolist() == c["diffusion"]
        assert accepted == c["accepted"]
        assert O.ar_generate(g["params"], cfg, torch.tensor([c["prompt"]]), c["max_new"]) == c["ar"]


def test_decode_scripted_drafts_accept_and_rollback():
    g = load_golden("tiny_decode.pt")
    cfg = oracle_config(g["config"])
    for s in g["scripted"]:
        plen = len(s["prompt"])
        table = s["table"]
        tokens, accepted, passes = O.decode_base(
            g["params"], cfg, s["prompt"], s["max_new"], set(s["eos"]),
            drafts=lambda start, n: table[start - plen][: n - 1])
        assert tokens == s["tokens"] and accepted == s["accepted"] and passes == s["passes"]


def test_decode_eos_stop():
    g = load_golden("tiny_decode.pt")
    cfg = oracle_config(g["config"])
    e = g["eos_case"]
    out, accepted = O.diffusion_generate(g["params"], cfg, torch.tensor([e["prompt"]]),
                                         e["max_new"], set(e["eos"]))
    assert out[0, len(e["prompt"]):].tolist() == e["tokens"] and accepted == e["accepted"]


def test_config1_decode():
    g = load_golden("config1_decode.pt")
    cfg = oracle_config(g["config"])
    for c in g["cases"]:
        out, accepted = O.diffusion_generate(g["params"], cfg, torch.tensor([c["prompt"]]),
                                             c["max_new"])
        assert out[0, len(c["prompt"]):].tolist() == c["diffusion"] == c["ar"]
        assert accepted == c["accepted"]


def test_sampling_filter_and_rejection_rule():
    """sampling_probs and rejection_accept against the reference's own sampled cycle (the
    distributions its `pick` handed to torch.multinomial, its uniforms, accepted count and bonus
    distribution; tests/golden/sampling.pt)."""
    g = load_golden("sampling.pt")
    for c in g["cases"]:
        knobs = (c["temperature"], c["top_k"], c["top_p"])
        assert torch.equal(O.sampling_probs(c["prefill_last"][None], *knobs), c["first_probs"])
        assert torch.equal(O.sampling_probs(c["draft_logits"], *knobs), c["draft_probs"])
        assert torch.equal(O.sampling_probs(c["verify_logits"], *knobs), c["ar_probs"])
        n = c["draft_tokens"].numel()
        uniforms = torch.tensor(c["uniforms"] + [1.0] * (n - len(c["uniforms"])))
        accepted, target = O.rejection_accept(c["draft_tokens"], c["draft_probs"], c["ar_probs"], uniforms)
        assert accepted == c["accepted"]
        assert torch.equal(target, c["target"])
