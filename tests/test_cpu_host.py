"""Host-side logic of the drop-in modules against the oracle and the reference's golden traces."""

import pytest
import torch
from conftest import load_golden

import oracle as O
from orthrus_training_b200 import decoding as D
from orthrus_training_b200 import objective as ob
from orthrus_training_b200.train_step import anchor_rng, lr_scale


def test_sample_anchors_match_reference_fixture():
    g = load_golden("config1.pt")
    for case in ("case", "many_anchors"):
        c = g[case]
        gen = torch.Generator().manual_seed(c["anchor_seed"])
        anchors, valid = ob.sample_anchors(c["assistant_mask"], g["config"]["block_size"],
                                           c["num_anchors"], gen)
        assert torch.equal(anchors, c["anchors"]) and torch.equal(valid, c["valid"])


def test_anchor_edge_cases():
    """tests/test_objective.py:116-136 semantics: few candidates, no assistant tokens."""
    mask = torch.zeros(3, 64, dtype=torch.bool)
    mask[0, 10:50] = True
    mask[1, 5:9] = True
    gen = torch.Generator().manual_seed(1)
    anchors, valid = ob.sample_anchors(mask, 8, 16, gen)
    assert anchors.shape == (3, 16)
    assert valid[0].all() and mask[0, anchors[0]].all() and (anchors[0, 1:] > anchors[0, :-1]).all()
    assert valid[1].sum() == 4 and mask[1, anchors[1, :4]].all()
    assert not valid[2].any()
    assert (anchors >= 1).all() and (anchors <= 64 - 8).all()
    keep = ob.supervision_mask(torch.tensor([[False] * 6 + [True] * 6 + [False] * 8]),
                               torch.tensor([[5, 10]]), torch.tensor([[True, True]]), 4)
    assert keep.tolist() == [[[True, True, True], [True, False, False]]]


@pytest.mark.parametrize("seed", range(6))
def test_sample_anchors_equal_the_oracle_draws(seed):
    """One generator state gives the oracle's anchors (the reference's per-row boolean gather and
    randperm) for dense, sparse, empty and shorter-than-slots candidate rows."""
    g = torch.Generator().manual_seed(seed)
    L, K, A = 160, 8, 12
    density = torch.tensor([0.9, 0.3, 0.0, 0.04, 0.6])[:, None]
    mask = torch.rand(5, L, generator=g) < density
    mask[3, :] = False
    mask[3, [7, 40, 41]] = True  # three candidates for twelve slots
    ours = ob.sample_anchors(mask, K, A, torch.Generator().manual_seed(100 + seed))
    ref = O.sample_anchors(mask, K, A, torch.Generator().manual_seed(100 + seed))
    assert torch.equal(ours[0], ref[0]) and torch.equal(ours[1], ref[1])


def test_position_weights_and_lr_schedule():
    assert ob.position_weights(32, 0.0) is None
    assert torch.allclose(ob.position_weights(32, 4.0), O.position_weights(32, 4.0))
    for step in (0, 3, 49, 50, 51, 500, 999, 1000, 2000):
        assert lr_scale(step, 50, 1000, 0.1) == pytest.approx(O.lr_scale(step, 50, 1000, 0.1))


def test_anchor_rng_is_keyed():
    a = torch.randperm(100, generator=anchor_rng(42, 0, 7, device="cpu"))
    b = torch.randperm(100, generator=anchor_rng(42, 0, 7, device="cpu"))
    c = torch.randperm(100, generator=anchor_rng(42, 0, 8, device="cpu"))
    assert torch.equal(a, b) and not torch.equal(a, c)


def test_strategy_validation():
    with pytest.raises(ValueError):
        D.Strategy("x", kind="tail", shifts=(2,))
    with pytest.raises(ValueError):
        D.Strategy("x", kind="other")
    with pytest.raises(ValueError):
        D.parse_strategies([{"name": "a"}, {"name": "a"}])
    assert D.Strategy("g", kind="tail", min_expected=2).needs_confidence


class ReplayBackend:
    """AR predictions from a fixed greedy output, drafts from a table: the host-side cycle
    (decode / _verify / _advance) without a model."""

    def __init__(self, prompt_len, reference, table, block_size):
        self.prompt_len, self.reference, self.table = prompt_len, reference, table
        self.block_size = block_size
        self.passes, self.input_tokens, self.seconds = {}, {}, {}

    def _count(self, kind, n):
        self.passes[kind] = self.passes.get(kind, 0) + 1
        self.input_tokens[kind] = self.input_tokens.get(kind, 0) + n

    def prefill(self):
        self._count("prefill", self.prompt_len)
        return self.reference[0]

    def draft(self, start, anchor, block_len, confidence):
        self._count("draft", block_len)
        return D.Hypothesis(None, list(self.table[start - self.prompt_len][: block_len - 1]))

    def verify(self, kind, start, root, hypotheses):
        i = start - self.prompt_len
        self._count(kind, 1 + len(hypotheses[0].tokens))
        ref = self.reference
        return [[ref[i + 1 + d] if i + 1 + d < len(ref) else -1
                 for d in range(len(hypotheses[0].tokens) + 1)]]

    def commit(self, best, accepted):
        pass


def test_decode_cycle_reproduces_reference_scripted_traces():
    g = load_golden("tiny_decode.pt")
    K = g["config"]["block_size"]
    for s in g["scripted"]:
        backend = ReplayBackend(len(s["prompt"]), s["free"], s["table"], K)
        gen = D.decode(backend, D.Strategy("base"), len(s["prompt"]), s["max_new"], set(s["eos"]))
        assert gen.tokens == s["tokens"]
        assert gen.accepted == s["accepted"]
        assert gen.forward_passes == s["passes"]


def test_ar_decode_cycle():
    ref = [5, 6, 7, 8, 9, 10]
    backend = ReplayBackend(3, ref, [[0] * 7] * 10, 8)
    gen = D.ar_decode(backend, 3, 6, set())
    assert gen.tokens == ref and gen.forward_passes == 6
    gen = D.ar_decode(ReplayBackend(3, ref, [[0] * 7] * 10, 8), 3, 6, {8})
    assert gen.tokens == [5, 6, 7, 8] and gen.eos


def test_cache_has_the_dynamic_cache_surface():
    """KVCache(config=...) allocates on its first write like DynamicCache; update() appends one
    layer and returns its committed keys / values; lengths are per layer; crop() truncates all
    (orthrus/modeling_orthrus.py:107-111,162-166)."""
    from transformers import Qwen3Config

    from orthrus_training_b200.kv_cache import KVCache
    from orthrus_training_b200.modeling_orthrus import DynamicCache, truncate_cache

    cfg = Qwen3Config(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=16)
    assert DynamicCache is KVCache
    cache = DynamicCache(config=cfg)
    assert not cache.allocated and cache.get_seq_length() == 0
    k = torch.randn(1, 1, 5, 16, dtype=torch.float64)
    v = torch.randn(1, 1, 5, 16, dtype=torch.float64)
    keys, values = cache.update(k, v, 0)
    assert cache.allocated and cache.dtype == torch.float64
    assert torch.equal(keys, k) and torch.equal(values, v)
    assert cache.get_seq_length(0) == 5 and cache.get_seq_length(1) == 0
    cache.update(k, v, 1)
    cache.update(k[:, :, :2], v[:, :, :2], 0)
    assert torch.equal(cache.layers[0].keys, torch.cat([k, k[:, :, :2]], 2))
    truncate_cache(cache, 4)
    assert [cache.get_seq_length(i) for i in range(2)] == [4, 4]
    cache.crop(-1)
    assert cache.layers[1].values.shape == (1, 1, 3, 16)
    big = torch.randn(1, 1, 2000, 16, dtype=torch.float64)
    cache.update(big, big, 0)  # grows past the initial capacity, keeping the committed rows
    assert cache.get_seq_length(0) == 2003 and torch.equal(cache.layers[0].keys[:, :, :3], k[:, :, :3])
    with pytest.raises(ValueError):
        cache.update(k.float(), v.float(), 0)  # the cache holds float64
