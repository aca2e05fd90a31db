"""The drop-in modules on the GPU against the reference's golden outputs and the oracle:
model_states / orthrus_loss (fp32 exact path and bf16 tensor-core path) and decoding."""

import math

import pytest
import torch
from conftest import load_golden, oracle_config

import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _hf_config(c: dict):
    from transformers import Qwen3Config

    cfg = Qwen3Config(vocab_size=c["vocab_size"], hidden_size=c["hidden_size"],
                      intermediate_size=c["intermediate_size"], num_hidden_layers=c["num_layers"],
                      num_attention_heads=c["num_heads"], num_key_value_heads=c["num_kv_heads"],
                      head_dim=c["head_dim"], rms_norm_eps=c["rms_norm_eps"],
                      rope_theta=c["rope_theta"], tie_word_embeddings=True,
                      max_position_embeddings=4096)
    cfg.rope_parameters = {"rope_theta": c["rope_theta"], "rope_type": "default"}
    cfg.block_size = c["block_size"]
    cfg.mask_token_id = c["mask_token_id"]
    return cfg


def _load(g: dict, dtype=torch.float32):
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, freeze_to_diffusion

    cfg = _hf_config(g["config"])
    with torch.device(DEV):
        model = OrthrusLM(cfg)
    params = g["params"]
    untied = not torch.equal(params["lm_head.weight"], params["model.embed_tokens.weight"])
    if untied:
        model.lm_head.weight = torch.nn.Parameter(torch.empty_like(model.lm_head.weight))
    sd = {k: v for k, v in params.items() if k != "lm_head.weight" or untied}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing)
    model = model.to(dtype)
    freeze_to_diffusion(model)
    return model


@pytest.mark.parametrize("fixture,case", [("config1.pt", "case"), ("config1.pt", "many_anchors"),
                                          ("tiny_model.pt", "case")])
def test_fp32_states_and_loss_match_reference(fixture, case):
    """fp32 path: states 1e-5, loss 1e-5 relative, twin gradients 1e-4 (the reference's own
    tolerances, tests/test_objective.py:59-99)."""
    from orthrus_training_b200 import objective as ob

    g = load_golden(fixture)
    c = g[case]
    model = _load(g)
    ids, mask = c["input_ids"].to(DEV), c["assistant_mask"].to(DEV)
    anchors, valid = c["anchors"].to(DEV), c["valid"].to(DEV)
    student, teacher = ob.model_states(model, ids, anchors)
    assert torch.allclose(teacher.cpu(), c["teacher"], atol=2e-5, rtol=1e-5)
    assert torch.allclose(student.detach().cpu(), c["student"], atol=2e-5, rtol=1e-5)
    for gamma, ref in c["losses"].items():
        model.zero_grad(set_to_none=True)
        loss, stats = ob.orthrus_loss(model, ids, mask, anchors, valid, kl_chunk_size=64, gamma=gamma)
        loss.backward()
        assert torch.allclose(loss.cpu(), ref["loss"], rtol=1e-5, atol=1e-6)
        for key in ("tokens", "agree", "agree_by_offset", "tokens_by_offset"):
            assert torch.equal(stats[key].cpu(), ref["stats"][key]), key
        for key in ("kl_sum", "weighted_kl_sum", "weight_sum"):
            assert torch.allclose(stats[key].cpu(), ref["stats"][key], rtol=1e-5, atol=1e-6), key
        assert torch.allclose(stats["kl_by_offset"].cpu(), ref["stats"]["kl_by_offset"], rtol=1e-5,
                              atol=1e-5)
        named = dict(model.named_parameters())
        for name, grad in ref["grads"].items():
            assert torch.allclose(named[name].grad.cpu(), grad, rtol=1e-4, atol=1e-6), name
        assert all(p.grad is None for n, p in named.items() if "_diff." not in n)


def test_reference_states_module_path_matches_functional():
    from orthrus_training_b200 import objective as ob

    g = load_golden("config1.pt")
    c = g["case"]
    model = _load(g)
    s1, t1 = ob.model_states(model, c["input_ids"].to(DEV), c["anchors"].to(DEV))
    s2, t2 = ob.reference_states(model, c["input_ids"].to(DEV), c["anchors"].to(DEV))
    assert torch.allclose(t1, t2, atol=1e-5) and torch.allclose(s1.detach(), s2, atol=1e-5)


def _bf16_tiny(seed=0):
    from transformers import Qwen3Config

    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar, freeze_to_diffusion

    cfg = Qwen3Config(vocab_size=2048, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True,
                      max_position_embeddings=4096)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size = 32
    cfg.mask_token_id = 2047
    torch.manual_seed(seed)
    with torch.device("cuda", torch.cuda.current_device()):  # the rank's own GPU under spawn
        model = OrthrusLM(cfg).to(torch.bfloat16)
    copy_diff_from_ar(model)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "_diff." in n and "norm" not in n:
                p.add_(torch.randn_like(p) * 0.004)
    freeze_to_diffusion(model)
    return model, cfg


def test_bf16_tensor_core_step_matches_oracle():
    """bf16 path (tcgen05 attention, fused LM-head KL) vs the fp32 oracle on the same bf16-rounded
    weights: loss within 1e-2 relative, twin gradients within 5e-2 of their scale."""
    from orthrus_training_b200 import objective as ob
    from orthrus_training_b200.synthetic import packed_rows

    model, cfg = _bf16_tiny()
    ids, mask = packed_rows(2, 512, 2047, seed=3, ids="uniform", doc="short")
    anchors, valid = ob.sample_anchors(mask, 32, 8, torch.Generator().manual_seed(0))
    loss, stats = ob.orthrus_loss(model, ids.to(DEV), mask.to(DEV), anchors.to(DEV), valid.to(DEV),
                                  kl_chunk_size=256)
    loss.backward()
    params = {k: v.detach().float().cpu().requires_grad_("_diff." in k)
              for k, v in model.state_dict().items()}
    params["lm_head.weight"] = params["model.embed_tokens.weight"]
    ref, ref_stats = O.orthrus_loss(params, O.OracleConfig.from_hf(cfg), ids, mask, anchors, valid)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-2 * abs(ref.item()), (loss.item(), ref.item())
    assert int(stats["tokens"]) == int(ref_stats["tokens"])
    for n, p in model.named_parameters():
        if "_diff." in n:
            r = params[n].grad
            err = (p.grad.float().cpu() - r).abs().max().item()
            assert err <= 5e-2 * r.abs().max().item() + 1e-6, (n, err, r.abs().max().item())


def test_decode_matches_reference_golden():
    """fp32: block decode == reference diffusion_generate == plain greedy (token identical), with
    the reference's accepted counts."""
    from orthrus_training_b200.decoding import block_decode

    g = load_golden("tiny_decode.pt")
    model = _load(g)
    for c in g["cases"]:
        res = block_decode(model, [c["prompt"]], c["max_new"], set(c["eos"]))
        assert res.tokens[0] == c["diffusion"] == c["ar"]
        assert res.accepted[0] == c["accepted"]
    e = g["eos_case"]
    out, stats = model.diffusion_generate(torch.tensor([e["prompt"]], device=DEV), e["max_new"],
                                          eos_token_id=e["eos"])
    assert out[0, len(e["prompt"]):].tolist() == e["tokens"]


def test_decode_scripted_drafts_accept_and_rollback():
    """Scripted drafts (the true continuation with one edit per block) exercise accept and the
    on-device cache rollback; the trace equals the reference decode's."""
    from orthrus_training_b200.decoding import block_decode

    g = load_golden("tiny_decode.pt")
    model = _load(g)
    K = g["config"]["block_size"]
    for s in g["scripted"]:
        table = torch.tensor([row + [0] * (K - 1 - len(row)) for row in s["table"]], dtype=torch.long)
        res = block_decode(model, [s["prompt"]], s["max_new"], set(s["eos"]),
                           draft_table=table[None].to(DEV))
        assert res.tokens[0] == s["tokens"]
        assert res.accepted[0] == s["accepted"]
        assert res.passes[0] == s["passes"]


def test_batched_decode_equals_single_sequences():
    from orthrus_training_b200.decoding import block_decode

    g = load_golden("config1_decode.pt")
    model = _load(g)
    prompts = [c["prompt"] for c in g["cases"]] + [g["cases"][0]["prompt"][:20]]
    batch = block_decode(model, prompts, 48)
    for b, p in enumerate(prompts):
        single = block_decode(model, [p], 48)
        assert batch.tokens[b] == single.tokens[0]
    for b, c in enumerate(g["cases"]):
        assert batch.tokens[b] == c["ar"]


def test_backend_decode_and_ar_decode_api():
    from orthrus_training_b200 import decoding as D

    g = load_golden("tiny_decode.pt")
    model = _load(g)
    c = g["cases"][0]
    gen = D.decode(D.ModelBackend(model, c["prompt"]), D.Strategy("base"), len(c["prompt"]),
                   c["max_new"], set())
    assert gen.tokens == c["diffusion"] and gen.accepted == c["accepted"]
    ar = D.ar_decode(D.ModelBackend(model, c["prompt"]), len(c["prompt"]), c["max_new"], set())
    assert ar.tokens == c["ar"] and ar.forward_passes == c["max_new"]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_lossless_block_decode_06b_layers(dtype):
    """Qwen3-0.6B layer shape (hidden 1024, 16/8 heads, hd 128, vocab 151936), 2 layers, random
    init: block decoding equals plain greedy decoding of the same model token for token."""
    from transformers import Qwen3Config

    from orthrus_training_b200.decoding import ar_generate_batch, block_decode
    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar

    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=2,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                      rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=4096)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size = 32
    cfg.mask_token_id = 151669
    torch.manual_seed(2)
    with torch.device(DEV):
        model = OrthrusLM(cfg).to(dtype)
    copy_diff_from_ar(model)
    prompt = torch.randint(0, 151669, (150,), generator=torch.Generator().manual_seed(2)).tolist()
    res = block_decode(model, [prompt], 64)
    ref = ar_generate_batch(model, torch.tensor([prompt], device=DEV), 64)[0, 150:].tolist()
    assert res.tokens[0] == ref


def test_block_decode_reuses_its_captured_cycle_across_calls():
    """A second call with other prompts of the same shapes replays the first call's captured cycle
    on the reset state: its tokens equal a fresh decode's, and so do the first prompts' again."""
    from orthrus_training_b200 import decoding as D

    g = load_golden("config1_decode.pt")
    model = _load(g)
    p1 = [c["prompt"] for c in g["cases"]]
    p2 = [p[3:] + p[:3] for p in p1]  # other prompts, same lengths
    D.clear_decode_cache()
    fresh2 = D.block_decode(model, p2, 40)
    D.clear_decode_cache()
    first = D.block_decode(model, p1, 40)
    assert len(D._STATE_CACHE) == 1
    second = D.block_decode(model, p2, 40)
    again = D.block_decode(model, p1, 40)
    assert len(D._STATE_CACHE) == 1
    assert second.tokens == fresh2.tokens and second.accepted == fresh2.accepted
    assert again.tokens == first.tokens
    D.clear_decode_cache()
