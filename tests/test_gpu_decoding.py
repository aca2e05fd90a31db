"""Decoding strategies on the GPU against the reference's own traces (tests/golden/
tiny_strategies.pt, written by orthrus.decoding on the lively tiny model whose weights are in
tiny_decode.pt): real decoding with every strategy, scripted drafts, tree verification with its
cache commit, and draft_table. Token-for-token and pass-for-pass equality (fp32 path)."""

import pytest
import torch
from conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _model():
    from test_gpu_model import _load

    return _load(load_golden("tiny_decode.pt"))


def _dec():
    from orthrus_training_b200 import decoding

    return decoding


def _trace(gen) -> dict:
    return {"tokens": gen.tokens, "passes": gen.passes, "accepted": gen.accepted,
            "branch": gen.branch, "tails": [list(t) for t in gen.tails]}


def _golden_trace(t) -> dict:
    return {k: t[k] for k in ("tokens", "passes", "accepted", "branch", "tails")}


@pytest.fixture(scope="module")
def setup():
    return _model(), load_golden("tiny_strategies.pt")


def test_real_decoding_of_every_strategy_matches_the_reference(setup):
    model, g = setup
    D = _dec()
    for case in g["real"]:
        for st in D.parse_strategies(g["strategies"]):
            gen = D.decode(D.ModelBackend(model, case["prompt"]), st, len(case["prompt"]),
                           case["max_new"], set(case["eos"]))
            assert _trace(gen) == _golden_trace(case["traces"][st.name]), st.name
            assert gen.input_tokens == case["traces"][st.name]["input_tokens"], st.name


def test_scripted_drafts_with_every_strategy_match_the_reference(setup):
    """Drafts from a table with one edit per block (substitution, skipped or spurious token):
    tail passes repair them through tree verification and the cache commit of a non-first branch."""
    model, g = setup
    D = _dec()

    class Scripted(D.ModelBackend):
        def __init__(self, model, prompt, table):
            super().__init__(model, prompt)
            self.table, self.prompt_len = table, len(prompt)

        def draft(self, start, anchor, block_len, confidence):
            self._timed("draft", block_len, lambda: None)
            tokens = self.table[start - self.prompt_len][: block_len - 1]
            return D.Hypothesis(None, list(tokens), [0.9] * len(tokens) if confidence else None)

    for case in g["scripted"]:
        for st in D.parse_strategies(g["strategies"]):
            gen = D.decode(Scripted(model, case["prompt"], case["table"]), st, len(case["prompt"]),
                           case["max_new"], set(case["eos"]))
            assert _trace(gen) == _golden_trace(case["traces"][st.name]), (case["edit"], st.name)


def test_tree_verification_matches_the_reference_and_separate_chains(setup):
    model, g = setup
    D = _dec()
    c = g["tree"]
    hyps = [D.Hypothesis(sh, toks) for sh, toks in c["hypotheses"]]
    tree = D.ModelBackend(model, c["prompt"])
    root = tree.prefill()
    assert root == c["root"]
    preds = tree.verify("tail", len(c["prompt"]), root, hyps)
    assert preds == c["preds"]
    for i, h in enumerate(hyps):
        chain = D.ModelBackend(model, c["prompt"])
        chain.prefill()
        assert chain.verify("tail", len(c["prompt"]), root, [h])[0] == preds[i]
    tree.commit(2, 4)  # the root and 4 tokens of the third branch stay
    chain = D.ModelBackend(model, c["prompt"])
    chain.prefill()
    chain.verify("tail", len(c["prompt"]), root, [hyps[2]])
    chain.commit(0, 4)
    n = len(c["prompt"]) + 1 + 4
    assert tree.cache.get_seq_length() == chain.cache.get_seq_length() == n
    for (ka, va), (kb, vb) in zip(tree.cache.buffers(), chain.cache.buffers()):
        assert torch.allclose(ka[:, :, :n], kb[:, :, :n], atol=1e-5)
        assert torch.allclose(va[:, :, :n], vb[:, :, :n], atol=1e-5)


def test_dense_tree_mask_through_the_model_forward(setup):
    """The reference's calling form: a dense 4-D tree mask to OrthrusLM.forward gives the same
    predictions as the tree_lo form the backend uses."""
    model, g = setup
    D = _dec()
    c = g["tree"]
    prompt = c["prompt"]
    branches = [toks for _, toks in c["hypotheses"]]
    tokens = [c["root"]] + [t for b in branches for t in b]
    depth = [0] + [i + 1 for b in branches for i in range(len(b))]
    group = torch.tensor([-1] + [j for j, b in enumerate(branches) for _ in b])
    level = torch.tensor(depth)
    tree = (group[None, :] == -1) | ((group[:, None] == group[None, :]) & (level[None, :] <= level[:, None]))
    mask = torch.cat([torch.ones(len(tokens), len(prompt), dtype=torch.bool), tree], 1)[None, None]
    backend = D.ModelBackend(model, prompt)
    backend.prefill()
    logits = model(input_ids=torch.tensor([tokens], device=DEV),
                   position_ids=torch.tensor([[len(prompt) + d for d in depth]], device=DEV),
                   attention_mask=mask.to(DEV), past_key_values=backend.cache, use_cache=True).logits[0]
    preds = logits.argmax(-1).tolist()
    offs, at = [], 1
    for b in branches:
        offs.append(at)
        at += len(b)
    assert [[preds[0]] + preds[o: o + len(b)] for o, b in zip(offs, branches)] == c["preds"]


def test_draft_table_matches_the_reference(setup):
    model, g = setup
    D = _dec()
    c = g["chunked"]
    drafts, conf = D.draft_table(model, c["prompt"], c["reference"], c["max_new"], chunk_blocks=4)
    assert torch.equal(torch.from_numpy(drafts), c["drafts"])
    assert torch.allclose(torch.from_numpy(conf), c["confidence"], atol=1e-5)
    for case in g["real"]:
        reference = case["traces"]["base"]["tokens"]
        drafts, conf = D.draft_table(model, case["prompt"], reference, case["max_new"])
        assert torch.equal(torch.from_numpy(drafts), case["drafts"])
        assert torch.allclose(torch.from_numpy(conf), case["confidence"], atol=1e-5)


def test_tree_verification_runs_the_ar_view_when_the_twins_differ():
    """Tree verification is an AR pass: with diffusion twins that differ from the AR weights, the
    tree's predictions still equal separate AR chains (a pass on the twins would not)."""
    D = _dec()
    model = _model()
    with torch.no_grad():
        g = torch.Generator(device=DEV).manual_seed(3)
        for n, p in model.named_parameters():
            if "_diff." in n:
                p.add_(torch.randn(p.shape, device=DEV, generator=g) * p.abs().mean())
    prompt = list(range(3, 14))
    hyps = [D.Hypothesis(1, [5, 9, 2, 7]), D.Hypothesis(0, [11, 4]), D.Hypothesis(-1, [8, 8, 1])]
    tree = D.ModelBackend(model, prompt)
    root = tree.prefill()
    preds = tree.verify("tail", len(prompt), root, hyps)
    for i, h in enumerate(hyps):
        chain = D.ModelBackend(model, prompt)
        chain.prefill()
        assert chain.verify("tail", len(prompt), root, [h])[0] == preds[i]
