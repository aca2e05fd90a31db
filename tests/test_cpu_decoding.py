"""Host side of the decoding strategies (no GPU): strategy rules, tail hypotheses, the tree-mask
conversion, and replays through OracleBackend that must reproduce the reference's own traces of
real and scripted decoding (tests/golden/tiny_strategies.pt, written by the reference's
orthrus.decoding)."""

import pytest
import torch

from conftest import load_golden


def _dec():
    from orthrus_training_b200 import decoding

    return decoding


def _trace(gen) -> dict:
    return {"tokens": gen.tokens, "passes": gen.passes, "accepted": gen.accepted,
            "branch": gen.branch, "tails": [list(t) for t in gen.tails]}


def _golden_trace(t) -> dict:
    return {k: t[k] for k in ("tokens", "passes", "accepted", "branch", "tails")}


def test_strategy_rules():
    D = _dec()
    for bad in ({"kind": "tail", "shifts": (2,)}, {"kind": "sideways"}, {"shifts": ()},
                {"shifts": (0, 0)}, {"kind": "tail", "min_tail": 0},
                {"kind": "reuse", "oracle_min_tokens": 2}):
        with pytest.raises(ValueError):
            D.Strategy("s", **bad)
    with pytest.raises(ValueError):
        D.parse_strategies([{"name": "x"}, {"name": "x"}])
    assert D.Strategy("g", kind="tail", min_expected=1.5).needs_confidence
    assert not D.Strategy("g", kind="reuse", min_expected=1.5).needs_confidence


def test_tail_hypotheses_and_expected_tokens():
    D = _dec()
    src = D.Hypothesis(None, [40, 41, 42, 43, 44, 45, 46], [0.9, 0.8, 0.7, 0.6, 0.5, 0.4, 0.3])
    # drafts[1] = 41 was rejected: insertion keeps it, substitution drops it, deletions drop more
    hyps = D.tail_hypotheses(src, accepted=1, shifts=(0, 1, -1, -3), room=4)
    assert [(h.shift, h.tokens) for h in hyps] == [(0, [42, 43, 44, 45]), (1, [41, 42, 43, 44]),
                                                   (-1, [43, 44, 45, 46]), (-3, [45, 46])]
    assert hyps[0].confidence == [0.7, 0.6, 0.5, 0.4]
    # duplicates of an earlier shift's tokens and empty tails are dropped
    rep = D.Hypothesis(None, [5, 5, 5, 5, 5])
    assert [h.shift for h in D.tail_hypotheses(rep, 0, (1, 0, -1), 2)] == [1]
    assert D.tail_hypotheses(src, accepted=6, shifts=(0, -1), room=3) == []
    assert D.tail_hypotheses(src, accepted=1, shifts=(0,), room=0) == []
    assert D.expected_tokens(D.Hypothesis(0, [1, 2, 3], [0.5, 0.5, 1.0])) == pytest.approx(2.0)
    assert D.expected_tokens(D.Hypothesis(0, [1])) == 1.0


def test_tree_mask_conversion():
    from orthrus_training_b200.modeling_orthrus import tree_mask_to_lo

    seen, branches = 6, [3, 2, 4]
    T = 1 + sum(branches)
    group = [-1] + [g for g, n in enumerate(branches) for _ in range(n)]
    level = [0] + [i + 1 for n in branches for i in range(n)]
    g, lv = torch.tensor(group), torch.tensor(level)
    tree = (g[None, :] == -1) | ((g[:, None] == g[None, :]) & (lv[None, :] <= lv[:, None]))
    mask = torch.cat([torch.ones(T, seen, dtype=torch.bool), tree], 1)[None, None]
    assert tree_mask_to_lo(mask, seen, T).tolist() == [1, 1, 1, 1, 4, 4, 6, 6, 6, 6]
    causal = torch.ones(T, seen + T, dtype=torch.bool).tril(seen)[None, None]
    assert tree_mask_to_lo(causal, seen, T).tolist() == [1] * T
    broken = mask.clone()
    broken[0, 0, 5, seen + 1] = True  # a token of branch 1 sees into branch 0
    with pytest.raises(ValueError):
        tree_mask_to_lo(broken, seen, T)
    hidden_prefix = mask.clone()
    hidden_prefix[0, 0, 3, 2] = False
    with pytest.raises(ValueError):
        tree_mask_to_lo(hidden_prefix, seen, T)


def test_replay_reproduces_the_reference_real_decoding():
    """OracleBackend replays of every strategy from the reference's draft tables equal the traces
    of the reference's real decoding of the same outputs (pass counts, accepted, branches, tails)."""
    D = _dec()
    g = load_golden("tiny_strategies.pt")
    strategies = D.parse_strategies(g["strategies"])
    K = g["config"]["block_size"]
    for case in g["real"]:
        reference = case["traces"]["base"]["tokens"]
        rows = [row[row >= 0].tolist() for row in case["drafts"]]
        conf = case["confidence"].tolist()
        for st in strategies:
            oracle = D.OracleBackend(len(case["prompt"]), reference, rows, conf, K)
            got = D.decode(oracle, st, len(case["prompt"]), case["max_new"], set(case["eos"]))
            assert _trace(got) == _golden_trace(case["traces"][st.name]), st.name


def test_replay_reproduces_the_reference_scripted_decoding():
    D = _dec()
    g = load_golden("tiny_strategies.pt")
    strategies = D.parse_strategies(g["strategies"])
    K = g["config"]["block_size"]
    for case in g["scripted"]:
        eos = set(case["eos"])
        free = case["free"]
        reference = free[: free.index(case["eos"][0]) + 1] if eos else free
        conf = [[0.9] * len(row) for row in case["table"]]
        for st in strategies:
            oracle = D.OracleBackend(len(case["prompt"]), reference, case["table"], conf, K)
            got = D.decode(oracle, st, len(case["prompt"]), case["max_new"], eos)
            assert _trace(got) == _golden_trace(case["traces"][st.name]), (case["edit"], st.name)
            assert got.tokens == reference


def test_replay_gates_and_errors():
    """oracle_min_tokens gates a tail pass on what it would keep; replay-only on real backends;
    a replay that leaves the reference output raises."""
    D = _dec()
    g = load_golden("tiny_strategies.pt")
    case = g["scripted"][0]
    K = g["config"]["block_size"]
    free = case["free"]
    conf = [[0.9] * len(row) for row in case["table"]]
    plain = D.decode(D.OracleBackend(len(case["prompt"]), free, case["table"], conf, K),
                     D.Strategy("t", kind="tail", shifts=(1, 0, -1)), len(case["prompt"]), 60, set())
    gated = D.decode(D.OracleBackend(len(case["prompt"]), free, case["table"], conf, K),
                     D.Strategy("t", kind="tail", shifts=(1, 0, -1), oracle_min_tokens=4),
                     len(case["prompt"]), 60, set())
    assert gated.tokens == plain.tokens == free
    assert all(t[2] + 1 >= 4 for t in gated.tails)
    assert gated.passes.get("tail", 0) <= plain.passes.get("tail", 0)

    class NoPeek:
        pass

    with pytest.raises(ValueError):
        D._gate_open(D.Strategy("t", kind="tail", oracle_min_tokens=2),
                        [D.Hypothesis(0, [1, 2])], NoPeek(), 0)
    oracle = D.OracleBackend(3, [7, 8, 9], [[8, 9]], None, 3)
    with pytest.raises(RuntimeError):
        oracle.draft(3, 99, 3, False)
