"""Generate the golden fixtures in this folder by running the reference implementation.

Run in a container that has the reference checked out (it is pure Python):

    python tests/golden/make_golden.py <reference checkout>          # every fixture
    python tests/golden/make_golden.py <reference checkout> data     # data_batches.pt only
    python tests/golden/make_golden.py <reference checkout> sampling # sampling.pt only

It imports the reference's own modules (orthrus.modeling_orthrus, orthrus.objective,
orthrus.decoding, orthrus.evaluate) and stores seeded inputs together with the reference outputs,
plus the torch and transformers versions they were made with. The fixtures pin the CPU oracle
(tests/test_oracle_golden.py) and the CUDA path (tests/test_gpu_*.py). Nothing at test time reads
the reference itself.
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))


def _versions() -> dict:
    import transformers

    return {"torch": torch.__version__, "transformers": transformers.__version__}


def make_model(mo, *, vocab, hidden, inter, layers, heads, kv_heads, head_dim, block, mask_id,
               theta, seed, eos=None):
    from transformers import Qwen3Config

    config = Qwen3Config(
        vocab_size=vocab,
        hidden_size=hidden,
        intermediate_size=inter,
        num_hidden_layers=layers,
        num_attention_heads=heads,
        num_key_value_heads=kv_heads,
        head_dim=head_dim,
        max_position_embeddings=4096,
        tie_word_embeddings=True,
        rms_norm_eps=1e-6,
        rope_theta=theta,
        eos_token_id=eos if eos is not None else [vocab - 2],
    )
    config.rope_parameters = {"rope_theta": theta, "rope_type": "default"}
    config.block_size = block
    config.mask_token_id = mask_id
    config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = mo.OrthrusLM(config).float()
    mo.copy_diff_from_ar(model)
    mo.freeze_to_diffusion(model)
    return model


def perturb_twins(model, seed: int, scale: float = 0.02) -> None:
    """Seeded noise on the diffusion twins, so the student differs from the teacher and the KL is
    well conditioned (copy_diff_from_ar alone makes student ~= teacher)."""
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "_diff." in name:
                p.add_(torch.randn(p.shape, generator=gen) * scale * (p.abs().mean() + 1e-3))


def config_dict(model) -> dict:
    c = model.config
    return {
        "vocab_size": c.vocab_size,
        "hidden_size": c.hidden_size,
        "intermediate_size": c.intermediate_size,
        "num_layers": c.num_hidden_layers,
        "num_heads": c.num_attention_heads,
        "num_kv_heads": c.num_key_value_heads,
        "head_dim": c.head_dim,
        "rms_norm_eps": c.rms_norm_eps,
        "rope_theta": float(c.rope_parameters["rope_theta"]),
        "block_size": c.block_size,
        "mask_token_id": c.mask_token_id,
    }


def state(model) -> dict:
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    sd.setdefault("lm_head.weight", sd["model.embed_tokens.weight"])
    return sd


def kl_kat(ob) -> dict:
    """tests/test_objective.py:16-38 inputs through FusedLinearForwardKL."""
    out = {}
    for weighted in (False, True):
        torch.manual_seed(0)
        student = torch.randn(37, 16, requires_grad=True)
        teacher = torch.randn(11, 16)
        index = torch.randint(0, 11, (37,)).sort().values
        weight = torch.randn(50, 16)
        row_weight = torch.rand(37) if weighted else None
        total, kl_rows, agree = ob.FusedLinearForwardKL.apply(
            student, teacher, index, weight, 8, False, row_weight
        )
        total.backward()
        out["weighted" if weighted else "plain"] = {
            "student": student.detach(),
            "teacher": teacher,
            "index": index,
            "weight": weight,
            "row_weight": row_weight,
            "total": total.detach(),
            "kl_rows": kl_rows,
            "agree": agree,
            "grad": student.grad.detach(),
        }
    return out


def mask_kat(mo) -> dict:
    """tests/test_modeling.py:8-23: the dual-pass mask evaluated densely."""
    seq_len, block = 40, 4
    anchors = torch.tensor([[3, 10, 30], [1, 2, 36]])
    mask = mo.build_block_mask(anchors, seq_len, block)
    q = torch.arange(anchors.shape[1] * block)[:, None]
    k = torch.arange(seq_len + anchors.shape[1] * block)[None, :]
    dense = torch.stack([
        mask.mask_mod(torch.tensor(b), torch.tensor(0), q.expand(-1, k.shape[1]),
                      k.expand(q.shape[0], -1))
        for b in range(anchors.shape[0])
    ])
    return {"anchors": anchors, "seq_len": seq_len, "block": block, "mask": dense}


def training_case(mo, ob, model, ids, mask, num_anchors, anchor_seed) -> dict:
    gen = torch.Generator().manual_seed(anchor_seed)
    anchors, valid = ob.sample_anchors(mask, model.config.block_size, num_anchors, gen)
    student, teacher = ob.reference_states(model, ids, anchors)
    fstudent, fteacher = ob.model_states(model, ids, anchors)
    case = {
        "input_ids": ids,
        "assistant_mask": mask,
        "anchors": anchors,
        "valid": valid,
        "anchor_seed": anchor_seed,
        "num_anchors": num_anchors,
        "student": student.detach(),
        "teacher": teacher.detach(),
        "functional_student": fstudent.detach(),
        "losses": {},
    }
    for gamma in (0.0, 2.0):
        model.zero_grad(set_to_none=True)
        loss, stats = ob.orthrus_loss(model, ids, mask, anchors, valid, kl_chunk_size=64,
                                      gamma=gamma)
        loss.backward()
        grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()
                 if p.grad is not None}
        case["losses"][gamma] = {
            "loss": loss.detach(),
            "stats": {k: v.detach().clone() for k, v in stats.items()},
            "grads": grads,
        }
    model.zero_grad(set_to_none=True)
    return case


def config1(mo, ob) -> dict:
    """Tiny Qwen3 plumbing workload: 2 layers, hidden 128, 4q/2kv heads, hd 32, MLP 384, tied vocab
    1024, K=8, 2 rows x 256 tokens of short documents, 4 anchors per row."""
    from orthrus_training_b200.synthetic import packed_rows

    model = make_model(mo, vocab=1024, hidden=128, inter=384, layers=2, heads=4, kv_heads=2,
                       head_dim=32, block=8, mask_id=1023, theta=1e6, seed=0)
    perturb_twins(model, seed=100)
    ids, mask = packed_rows(2, 256, 1023, seed=0, ids="uniform", doc="short")
    case = training_case(mo, ob, model, ids, mask, num_anchors=4, anchor_seed=0)
    many = training_case(mo, ob, model, ids, mask, num_anchors=24, anchor_seed=1)
    return {"config": config_dict(model), "params": state(model), "case": case,
            "many_anchors": many}


def reference_test_model(mo, ob) -> dict:
    """The reference tests' tiny model (tests/conftest.py:11-33) and batch (tests/test_objective.py
    _batch: 2 rows x 48, 12 overlapping anchor slots)."""
    model = make_model(mo, vocab=512, hidden=64, inter=128, layers=2, heads=4, kv_heads=2,
                       head_dim=16, block=8, mask_id=511, theta=1e6, seed=0, eos=[510, 509])
    perturb_twins(model, seed=101)
    torch.manual_seed(0)
    ids = torch.randint(0, 500, (2, 48))
    mask = torch.zeros(2, 48, dtype=torch.bool)
    mask[:, 12:] = True
    mask[1, 30:36] = False
    case = training_case(mo, ob, model, ids, mask, num_anchors=12, anchor_seed=0)
    return {"config": config_dict(model), "params": state(model), "case": case}


def lively_model(mo):
    """tests/test_decoding.py:32-45: untied random lm_head, non-norm weights x10."""
    model = make_model(mo, vocab=512, hidden=64, inter=128, layers=2, heads=4, kv_heads=2,
                       head_dim=16, block=8, mask_id=511, theta=1e6, seed=0, eos=[510, 509])
    model.eval()
    generator = torch.Generator().manual_seed(0)
    with torch.no_grad():
        model.lm_head.weight = torch.nn.Parameter(
            torch.randn(model.lm_head.weight.shape, generator=generator))
        for name, param in model.model.layers.named_parameters():
            if "norm" not in name:
                param.mul_(10)
    return model


def scripted_table(reference, block_size, edit=None):
    """tests/test_decoding.py:127-142."""
    table = []
    for i in range(len(reference)):
        truth = (reference[i + 1: i + block_size + 1] + [7] * block_size)[:block_size]
        j, kind = 1 + i % 5, i % 3 if edit is None else edit
        if kind == 0:
            drafts = truth[:j] + [(truth[j] + 1) % 500] + truth[j + 1:]
        elif kind == 1:
            drafts = truth[:j] + truth[j + 1:]
        else:
            drafts = truth[:j] + [(truth[j] + 3) % 500] + truth[j:]
        table.append(drafts[: block_size - 1])
    return table


def decode_cases(mo, dec, ev) -> dict:
    model = lively_model(mo)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    sd["lm_head.weight"] = model.lm_head.weight.detach().clone()
    cases = []
    for seed in range(4):
        prompt = torch.randint(0, 500, (9,), generator=torch.Generator().manual_seed(seed)).tolist()
        out, stats = model.diffusion_generate(torch.tensor([prompt]), 40, eos_token_id=[])
        ar, _ = ev.ar_generate(model, torch.tensor([prompt]), 40, set())
        cases.append({"prompt": prompt, "max_new": 40, "eos": [],
                      "diffusion": out[0, len(prompt):].tolist(),
                      "accepted": list(stats.accepted), "ar": ar})
    # scripted drafts exercise accept / rollback (tests/test_decoding.py:145-178)
    from orthrus.decoding import Hypothesis, ModelBackend, Strategy

    class ScriptedBackend(ModelBackend):
        def __init__(self, model, prompt_ids, table):
            super().__init__(model, prompt_ids)
            self.table, self.prompt_len = table, len(prompt_ids)

        def draft(self, start, anchor, block_len, confidence):
            self._timed("draft", block_len, lambda: None)
            tokens = self.table[start - self.prompt_len][: block_len - 1]
            return Hypothesis(None, list(tokens), [0.9] * len(tokens) if confidence else None)

    scripted = []
    for seed, new, stop_at in ((11, 60, None), (5, 50, 23)):
        prompt = torch.randint(0, 500, (9,), generator=torch.Generator().manual_seed(seed)).tolist()
        free = dec.ar_decode(ModelBackend(model, prompt), len(prompt), new, set()).tokens
        eos = set() if stop_at is None else {free[stop_at]}
        table = scripted_table(free, model.config.block_size)
        gen = dec.decode(ScriptedBackend(model, prompt, table), Strategy("base"), len(prompt),
                         new, eos)
        scripted.append({"prompt": prompt, "max_new": new, "eos": sorted(eos), "table": table,
                         "tokens": gen.tokens, "accepted": gen.accepted,
                         "passes": gen.forward_passes, "free": free})
    eos_case = None
    prompt = torch.randint(0, 500, (7,), generator=torch.Generator().manual_seed(3)).tolist()
    free, _ = model.diffusion_generate(torch.tensor([prompt]), 30, eos_token_id=[])
    stop = int(free[0, len(prompt) + 5])
    out, stats = model.diffusion_generate(torch.tensor([prompt]), 30, eos_token_id=[stop])
    eos_case = {"prompt": prompt, "max_new": 30, "eos": [stop],
                "tokens": out[0, len(prompt):].tolist(), "accepted": list(stats.accepted)}
    return {"config": config_dict(model), "params": sd, "cases": cases, "scripted": scripted,
            "eos_case": eos_case}


STRATEGY_SPECS = [  # tests/test_decoding.py:20-29
    {"name": "base"},
    {"name": "tail-s0", "kind": "tail", "shifts": [0]},
    {"name": "tail-tree", "kind": "tail", "shifts": [1, 0, -1, -2]},
    {"name": "tail-x2", "kind": "tail", "shifts": [1, 0, -1], "max_tail_passes": 2},
    {"name": "tail-gated", "kind": "tail", "shifts": [0], "min_tail": 3, "min_expected": 2.5},
    {"name": "reuse-tree", "kind": "reuse", "shifts": [1, 0, -1, -2]},
]


def _prompt(seed: int, length: int = 9) -> list[int]:
    return torch.randint(0, 500, (length,), generator=torch.Generator().manual_seed(seed)).tolist()


def _trace(gen) -> dict:
    return {"tokens": list(gen.tokens), "eos": bool(gen.eos), "passes": dict(gen.passes),
            "input_tokens": dict(gen.input_tokens), "accepted": list(gen.accepted),
            "branch": list(gen.branch), "tails": [list(t) for t in gen.tails]}


def strategy_cases(mo, dec) -> dict:
    """orthrus.decoding traces on the lively tiny model (the weights of tiny_decode.pt) for every
    strategy of tests/test_decoding.py: real decoding with its draft tables
    (test_replay_from_draft_table_matches_real_decoding), scripted drafts with each edit kind and
    an EOS (test_tail_strategies_*, test_eos_inside_a_tail_*), a draft table cut into chunks of 4
    blocks (test_draft_table_matches_decoding_drafts) and one tree verification."""
    model = lively_model(mo)
    strategies = dec.parse_strategies(STRATEGY_SPECS)
    K = model.config.block_size

    class ScriptedBackend(dec.ModelBackend):
        def __init__(self, model, prompt_ids, table):
            super().__init__(model, prompt_ids)
            self.table, self.prompt_len = table, len(prompt_ids)

        def draft(self, start, anchor, block_len, confidence):
            self._timed("draft", block_len, lambda: None)
            tokens = self.table[start - self.prompt_len][: block_len - 1]
            return dec.Hypothesis(None, list(tokens), [0.9] * len(tokens) if confidence else None)

    real = []
    for seed in range(3):
        prompt, new = _prompt(20 + seed), 40
        eos = {_prompt(100 + seed, 1)[0]}
        traces = {st.name: _trace(dec.decode(dec.ModelBackend(model, prompt), st, len(prompt), new, eos))
                  for st in strategies}
        reference = traces["base"]["tokens"]
        drafts, confidence = dec.draft_table(model, prompt, reference, new)
        real.append({"prompt": prompt, "max_new": new, "eos": sorted(eos), "traces": traces,
                     "drafts": torch.from_numpy(drafts), "confidence": torch.from_numpy(confidence)})
    scripted = []
    for seed, new, edit, stop_at in ((11, 60, None, None), (12, 60, 0, None), (12, 60, 1, None),
                                     (12, 60, 2, None), (5, 50, None, 23)):
        prompt = _prompt(seed)
        free = dec.ar_decode(dec.ModelBackend(model, prompt), len(prompt), new, set()).tokens
        eos = set() if stop_at is None else {free[stop_at]}
        table = scripted_table(free, K, edit)
        traces = {st.name: _trace(dec.decode(ScriptedBackend(model, prompt, table), st, len(prompt), new, eos))
                  for st in strategies}
        scripted.append({"prompt": prompt, "max_new": new, "edit": edit, "eos": sorted(eos),
                         "free": free, "table": table, "traces": traces})
    prompt, new = _prompt(2), 30
    reference = dec.ar_decode(dec.ModelBackend(model, prompt), len(prompt), new, set()).tokens
    drafts, confidence = dec.draft_table(model, prompt, reference, new, chunk_blocks=4)
    chunked = {"prompt": prompt, "max_new": new, "reference": reference,
               "drafts": torch.from_numpy(drafts), "confidence": torch.from_numpy(confidence)}
    prompt = _prompt(3)
    g = torch.Generator().manual_seed(7)
    hyps = [dec.Hypothesis(sh, torch.randint(0, 500, (n,), generator=g).tolist())
            for sh, n in ((1, 5), (0, 3), (-1, 6))]
    tree = dec.ModelBackend(model, prompt)
    root = tree.prefill()
    preds = tree.verify("tail", len(prompt), root, hyps)
    tree_case = {"prompt": prompt, "root": root, "hypotheses": [(h.shift, h.tokens) for h in hyps],
                 "preds": preds}
    return {"config": config_dict(model), "strategies": STRATEGY_SPECS, "real": real,
            "scripted": scripted, "chunked": chunked, "tree": tree_case}


def config1_decode(mo, ev) -> dict:
    """Config-1 shape (hd 32, K=8), lively weights: diffusion_generate == ar_generate."""
    model = make_model(mo, vocab=1024, hidden=128, inter=384, layers=2, heads=4, kv_heads=2,
                       head_dim=32, block=8, mask_id=1023, theta=1e6, seed=0)
    perturb_twins(model, seed=100)
    model.eval()
    generator = torch.Generator().manual_seed(1)
    with torch.no_grad():  # lively variant (tests/test_decoding.py:32-45) so outputs do not collapse
        model.lm_head.weight = torch.nn.Parameter(
            torch.randn(model.lm_head.weight.shape, generator=generator))
        for name, param in model.model.layers.named_parameters():
            if "norm" not in name:
                param.mul_(10)
    cases = []
    for seed in range(2):
        prompt = torch.randint(0, 1023, (37,), generator=torch.Generator().manual_seed(seed))
        out, stats = model.diffusion_generate(prompt[None], 48, eos_token_id=[])
        ar, _ = ev.ar_generate(model, prompt[None], 48, set())
        cases.append({"prompt": prompt.tolist(), "max_new": 48,
                      "diffusion": out[0, 37:].tolist(), "accepted": list(stats.accepted),
                      "ar": ar})
    sd = state(model)
    sd["lm_head.weight"] = model.lm_head.weight.detach().clone()
    return {"config": config_dict(model), "params": sd, "cases": cases}


class _FakeLogits:
    """Stands in for OrthrusLM.forward inside the reference's diffusion_generate: returns fixed
    logits per call kind (prefill, diffusion draft, verify) and stops the run at the second draft,
    so exactly one sampled cycle runs through the reference's own code."""

    class Stop(Exception):
        pass

    def __init__(self, config, prefill, draft, verify):
        self.config = config
        self.logits = {"prefill": prefill, "draft": draft, "verify": verify}
        self.drafts = 0

    def __call__(self, input_ids=None, is_diffusion_pass=False, **kwargs):
        from types import SimpleNamespace

        if is_diffusion_pass:
            self.drafts += 1
            if self.drafts > 1:
                raise self.Stop()
            return SimpleNamespace(logits=self.logits["draft"][None, : input_ids.shape[1]])
        kind = "prefill" if kwargs.get("position_ids") is None else "verify"
        return SimpleNamespace(logits=self.logits[kind][None, : input_ids.shape[1]])


def sampling_cases(mo) -> dict:
    """The reference's sampled decoding (orthrus/modeling_orthrus.py:437-449,498-511) on fixed
    logits: the distributions `pick` hands to torch.multinomial, the uniforms of the rejection
    test, the accepted count and the bonus token's distribution of one cycle."""
    from transformers import Qwen3Config

    V, K, P = 96, 8, 5
    cfg = Qwen3Config(vocab_size=V, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=32)
    cfg.block_size, cfg.mask_token_id = K, V - 1
    cases = []
    settings = [(0.7, 20, 0.8), (1.0, 5, 1.0), (1.3, 12, 0.9), (0.5, 40, 0.95), (0.9, 1, 0.8)]
    for n, (temperature, top_k, top_p) in enumerate(settings * 3):
        g = torch.Generator().manual_seed(1000 + n)
        base = torch.randn(K, V, generator=g) * 2
        prefill = torch.randn(P, V, generator=g) * 2
        draft = base + torch.randn(K, V, generator=g) * (0.3 + 0.3 * (n % 3))
        verify = base + torch.randn(K, V, generator=g) * 0.3
        if n % 5 == 4:  # integer logits: ties at the top_k-th value
            draft, verify = draft.round(), verify.round()
        multinomial, rand, stats = [], [], []
        orig_multinomial, orig_rand, orig_stats = torch.multinomial, torch.rand, mo.GenerationStats

        def rec_multinomial(probs, num, *a, **k):
            out = orig_multinomial(probs, num, *a, **k)
            multinomial.append((probs.clone(), out.clone()))
            return out

        def rec_rand(*a, **k):
            out = orig_rand(*a, **k)
            rand.append(float(out))
            return out

        class RecStats(orig_stats):
            def __init__(self, *a, **k):
                super().__init__(*a, **k)
                stats.append(self)

        torch.manual_seed(77 + n)
        torch.multinomial, torch.rand, mo.GenerationStats = rec_multinomial, rec_rand, RecStats
        try:
            fake = _FakeLogits(cfg, prefill, draft, verify)
            mo.OrthrusLM.diffusion_generate(fake, torch.zeros(1, P, dtype=torch.long), 64,
                                            temperature=temperature, top_k=top_k, top_p=top_p)
        except _FakeLogits.Stop:
            pass
        finally:
            torch.multinomial, torch.rand, mo.GenerationStats = orig_multinomial, orig_rand, orig_stats
        (_, _), (q, d), (p, _), (target, _) = multinomial[:4]
        cases.append({"temperature": temperature, "top_k": top_k, "top_p": top_p,
                      "prefill_last": prefill[-1].clone(), "draft_logits": draft[: K - 1].clone(),
                      "verify_logits": verify.clone(), "first_probs": multinomial[0][0].clone(),
                      "draft_probs": q.view(K - 1, V).clone(), "draft_tokens": d.view(-1).clone(),
                      "ar_probs": p.view(K, V).clone(), "uniforms": rand, "accepted": stats[0].accepted[0],
                      "target": target.clone()})
    return {"vocab": V, "block_size": K, "cases": cases}


def data_batches(data) -> dict:
    """The reference's micro-batch order (orthrus/data.py:89-103) for a few (seed, epoch, start)."""
    import numpy as np

    rng = np.random.default_rng(123)
    ids = rng.integers(0, 1000, size=(37, 16), dtype=np.int32)
    mask = (rng.random((37, 16)) < 0.5).astype(np.uint8)
    cases = []
    for seed, epoch, bs, start in ((0, 0, 4, 0), (3, 1, 5, 2), (7, 2, 8, 1)):
        out = [(i, x.clone(), m.clone()) for i, x, m in data.batches(ids, mask, bs, seed, epoch, start)]
        cases.append({"seed": seed, "epoch": epoch, "batch_size": bs, "start": start,
                      "index": [o[0] for o in out], "ids": [o[1] for o in out], "mask": [o[2] for o in out]})
    return {"ids": torch.from_numpy(ids), "mask": torch.from_numpy(mask), "cases": cases}


def main(reference: str, only: str | None = None) -> None:
    sys.path.insert(0, reference)
    from orthrus import decoding as dec
    from orthrus import evaluate as ev
    from orthrus import modeling_orthrus as mo
    from orthrus import objective as ob

    from orthrus import data

    torch.set_num_threads(4)
    meta = _versions()
    if only == "sampling":
        torch.save({"meta": meta, **sampling_cases(mo)}, HERE / "sampling.pt")
        return
    torch.save({"meta": meta, **data_batches(data)}, HERE / "data_batches.pt")
    if only == "data":
        return
    torch.save({"meta": meta, **strategy_cases(mo, dec)}, HERE / "tiny_strategies.pt")
    if only == "strategies":
        return
    torch.save({"meta": meta, **sampling_cases(mo)}, HERE / "sampling.pt")
    torch.save({"meta": meta, **kl_kat(ob)}, HERE / "kl_kat.pt")
    torch.save({"meta": meta, **mask_kat(mo)}, HERE / "mask_kat.pt")
    torch.save({"meta": meta, **config1(mo, ob)}, HERE / "config1.pt")
    torch.save({"meta": meta, **reference_test_model(mo, ob)}, HERE / "tiny_model.pt")
    torch.save({"meta": meta, **decode_cases(mo, dec, ev)}, HERE / "tiny_decode.pt")
    torch.save({"meta": meta, **config1_decode(mo, ev)}, HERE / "config1_decode.pt")
    print("golden fixtures written to", HERE, meta)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden.py <reference checkout> [data]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else None)
