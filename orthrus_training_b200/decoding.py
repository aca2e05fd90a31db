"""Orthrus parallel block decoding on the Blackwell kernels: drop-in for orthrus/decoding.py (the
base, tail and reuse strategies with tree verification, plain greedy, replay from a draft table,
draft_table) plus a batched, device-resident decode loop for the base strategy.

``block_decode`` keeps every piece of the cycle state on the GPU: per-sequence committed cache
length (``start``), anchor token, done flag, output buffer, accepted counts. One cycle is

    draft pass  (diffusion view over [anchor, mask x K-1], orthrus_attn_fwd mask DRAFT)
    orthrus_decode_draft          -> verify ids [anchor, argmax drafts]
    verify pass (AR view, writes K/V rows [start, start+K) of the cache, causal)
    orthrus_decode_verify_accept  -> greedy longest-prefix accept, bonus token, start += accepted+1

with fixed shapes, so after a warm-up cycle it is captured once as a CUDA graph and replayed; the
host reads the done flags only every few cycles. Rolling the cache back is the ``start`` update:
rows past it are dead and the next verification overwrites them.

Losslessness: the GEMMs and attention kernels give per-row results independent of how many rows a
pass has, so the verification logits of a position equal the logits a one-token greedy pass
computes there, and the output equals plain greedy decoding token for token.
"""

from __future__ import annotations

import dataclasses
import time
from collections import Counter
from dataclasses import dataclass, field

import torch

from orthrus_training_b200 import ops
from orthrus_training_b200.kv_cache import KVCache

KINDS = ("base", "tail", "reuse")


@dataclass(frozen=True)
class Strategy:
    """A decoding strategy (orthrus/decoding.py:41-70): base, tail (extra tree-verified passes over
    the rejected tail) or reuse (the rejected tail rides along in the next verification)."""

    name: str
    kind: str = "base"
    shifts: tuple[int, ...] = (0,)
    min_tail: int = 1
    min_expected: float = 0.0
    max_tail_passes: int = 1
    oracle_min_tokens: int = 0

    def __post_init__(self):
        shifts = tuple(int(s) for s in self.shifts)
        object.__setattr__(self, "shifts", shifts)
        if self.kind not in KINDS:
            raise ValueError(f"strategy {self.name}: kind must be one of {KINDS}")
        if not shifts or len(set(shifts)) != len(shifts) or max(shifts) > 1:
            raise ValueError(f"strategy {self.name}: shifts must be distinct and <= 1")
        if self.min_tail < 1 or self.max_tail_passes < 1:
            raise ValueError(f"strategy {self.name}: min_tail and max_tail_passes must be >= 1")
        if self.oracle_min_tokens and self.kind != "tail":
            raise ValueError(f"strategy {self.name}: oracle_min_tokens needs kind tail")

    @property
    def needs_confidence(self) -> bool:
        return self.kind == "tail" and self.min_expected > 0

    def to_dict(self) -> dict:
        return {**dataclasses.asdict(self), "shifts": list(self.shifts)}


def parse_strategies(specs: list[dict]) -> list[Strategy]:
    strategies = [Strategy(**spec) for spec in specs]
    names = [s.name for s in strategies]
    if len(set(names)) != len(names):
        raise ValueError(f"strategy names must be unique: {names}")
    return strategies


@dataclass
class Hypothesis:
    """A continuation to verify (orthrus/decoding.py:82-86): shift None for the fresh drafts of a
    block, else the tail shift it was cut with; confidence = diffusion probability of each token."""

    shift: int | None
    tokens: list[int]
    confidence: list[float] | None = None


def tail_hypotheses(source: Hypothesis, accepted: int, shifts: tuple[int, ...],
                    room: int) -> list[Hypothesis]:
    """Tails after a rejection (orthrus/decoding.py:89-107). source.tokens[accepted] lost to the
    AR token (the bonus); the shift-s continuation of the bonus is source.tokens[accepted + 1 - s:]
    (s = 0 substitution, 1 insertion, -j deletion of j spurious drafts), at most `room` tokens.
    Empty continuations and repeats of an earlier shift's tokens are left out; order is kept."""
    out: list[Hypothesis] = []
    seen: set[tuple[int, ...]] = set()
    for shift in shifts:
        begin = accepted + 1 - shift
        tokens = list(source.tokens[begin: begin + room])
        if not tokens or tuple(tokens) in seen:
            continue
        seen.add(tuple(tokens))
        conf = None if source.confidence is None else list(source.confidence[begin: begin + room])
        out.append(Hypothesis(shift, tokens, conf))
    return out


def expected_tokens(hypothesis: Hypothesis) -> float:
    """1 + sum_j prod_{i <= j} confidence_i: the tokens a verification of the hypothesis keeps in
    expectation, the confidences taken as independent acceptance probabilities
    (orthrus/decoding.py:110-116)."""
    total = prefix = 1.0
    for p in hypothesis.confidence or ():
        prefix *= p
        total += prefix
    return total


@dataclass
class Generation:
    """One decoded output with its pass accounting (orthrus/decoding.py:119-142). tails holds per
    tail pass (cycle, shift of the kept hypothesis, accepted, hypotheses, longest hypothesis)."""

    strategy: str
    tokens: list[int] = field(default_factory=list)
    eos: bool = False
    accepted: list[int] = field(default_factory=list)
    branch: list[int | None] = field(default_factory=list)
    tails: list = field(default_factory=list)
    passes: dict = field(default_factory=dict)
    input_tokens: dict = field(default_factory=dict)
    seconds: dict = field(default_factory=dict)

    @property
    def forward_passes(self) -> int:
        return sum(self.passes.values())

    @property
    def tpf(self) -> float:
        return len(self.tokens) / max(self.forward_passes, 1)


class ModelBackend:
    """Forward passes of an OrthrusLM, batch 1, greedy, with per-kind pass / token / time counts
    (orthrus/decoding.py:145-264). The AR cache holds the committed prefix; the anchor is not in
    it yet. Several hypotheses are verified in one pass with the tree mask of the attention
    kernels (orthrus_attn_fwd mask TREE); commit() moves the kept branch's cache rows behind the
    root and drops the rest."""

    def __init__(self, model, prompt_ids: list[int], record_drafts: bool = False):
        self.model = model
        self.device = next(model.parameters()).device
        self.block_size = model.config.block_size
        self.mask_token_id = model.config.mask_token_id
        self.prompt = torch.tensor([prompt_ids], device=self.device)
        dtype = next(model.parameters()).dtype
        self.cache = KVCache(model.config, batch=1, capacity=len(prompt_ids) + 64,
                             device=self.device, dtype=dtype)
        self.passes, self.input_tokens, self.seconds = Counter(), Counter(), Counter()
        self.record_drafts = record_drafts
        self.drafts: dict[int, list[int]] = {}
        self._layout: tuple[int, list[int]] | None = None

    def _timed(self, kind: str, tokens: int, run):
        begin = time.perf_counter()
        result = run()  # ends in a host read of the argmax, which synchronises the device
        self.seconds[kind] += time.perf_counter() - begin
        self.passes[kind] += 1
        self.input_tokens[kind] += tokens
        return result

    def prefill(self) -> int:
        def run():
            out = self.model(input_ids=self.prompt, past_key_values=self.cache, use_cache=True,
                             logits_to_keep=1)
            return int(ops.argmax_rows(out.logits[0]).item())

        return self._timed("prefill", self.prompt.shape[1], run)

    def draft(self, start: int, anchor: int, block_len: int, confidence: bool) -> Hypothesis:
        def run():
            block = torch.full((1, block_len), self.mask_token_id, dtype=torch.long,
                               device=self.device)
            block[0, 0] = anchor
            positions = torch.arange(start, start + block_len, device=self.device)[None]
            logits = self.model(input_ids=block, position_ids=positions, past_key_values=self.cache,
                                use_cache=False, is_diffusion_pass=True, ar_seq_len=start).logits[0, :-1]
            tokens = ops.argmax_rows(logits.contiguous())
            probs = None
            if confidence:
                probs = torch.softmax(logits.float(), -1).gather(-1, tokens[:, None])[:, 0].tolist()
            return Hypothesis(None, tokens.tolist(), probs)

        drafts = self._timed("draft", block_len, run)
        if self.record_drafts:
            self.drafts[start] = drafts.tokens
        return drafts

    def verify(self, kind: str, start: int, root: int, hypotheses: list[Hypothesis]) -> list:
        """AR pass over the root (position `start`) and every hypothesis after it, all written to
        the cache at rows start + index; one hypothesis is a causal chain, several a tree (each
        token sees the prefix, the root and its own branch up to itself, at position start +
        depth). Returns per hypothesis the AR argmax after the root and after each of its tokens
        (orthrus/decoding.py:208-241)."""
        branches = [list(h.tokens) for h in hypotheses]
        tokens = [root] + [t for b in branches for t in b]
        depth = [0] + [i + 1 for b in branches for i in range(len(b))]
        begins, at = [], 1
        for b in branches:
            begins.append(at)
            at += len(b)
        lo = [1] + [begin for begin, b in zip(begins, branches) for _ in b] if len(branches) > 1 else None

        def run():
            ids = torch.tensor([tokens], device=self.device)
            positions = torch.tensor([[start + d for d in depth]], device=self.device)
            tree_lo = None if lo is None else torch.tensor(lo, dtype=torch.int32, device=self.device)
            self.cache.reserve(start + len(tokens))
            logits = self.model(input_ids=ids, position_ids=positions, past_key_values=self.cache,
                                use_cache=True, tree_lo=tree_lo).logits[0]
            return ops.argmax_rows(logits.contiguous()).tolist()

        preds = self._timed(kind, len(tokens), run)
        self._layout = (start, begins)
        return [[preds[0]] + preds[begin: begin + len(b)] for begin, b in zip(begins, branches)]

    def commit(self, best: int, accepted: int) -> None:
        """Keep the prefix, the root and the first `accepted` tokens of hypothesis `best` of the
        last verification (orthrus/decoding.py:243-264): a length update when that hypothesis
        followed the root, else its K/V rows are first copied behind the root in every layer."""
        start, begins = self._layout
        src = start + begins[best]
        if src != start + 1 and accepted > 0:
            dst = slice(start + 1, start + 1 + accepted)
            for k, v in self.cache.buffers():
                k[:, :, dst] = k[:, :, src: src + accepted].clone()
                v[:, :, dst] = v[:, :, src: src + accepted].clone()
        self.cache.crop(start + 1 + accepted)


class OracleBackend:
    """Greedy decoding replayed without a model (orthrus/decoding.py:267-333): AR predictions come
    from the reference output, drafts from a draft table (row i: the drafts of the block anchored
    at reference[i]). Exact when real decoding produced the reference with these drafts."""

    def __init__(self, prompt_len: int, reference: list[int], drafts: list[list[int]],
                 confidence: list[list[float]] | None, block_size: int):
        self.prompt_len, self.reference, self.block_size = prompt_len, list(reference), block_size
        self.drafts, self.confidence = drafts, confidence
        self.passes, self.input_tokens, self.seconds = Counter(), Counter(), Counter()

    def _count(self, kind: str, tokens: int) -> None:
        self.passes[kind] += 1
        self.input_tokens[kind] += tokens

    def _index(self, start: int, token: int) -> int:
        i = start - self.prompt_len
        if not 0 <= i < len(self.reference) or self.reference[i] != token:
            raise RuntimeError(f"replay left the reference output at position {start}")
        return i

    def prefill(self) -> int:
        self._count("prefill", self.prompt_len)
        return self.reference[0]

    def draft(self, start: int, anchor: int, block_len: int, confidence: bool) -> Hypothesis:
        i = self._index(start, anchor)
        tokens = list(self.drafts[i][: block_len - 1])
        if len(tokens) != block_len - 1 or min(tokens, default=0) < 0:
            raise RuntimeError(f"draft table has no block of {block_len} at position {start}")
        probs = list(self.confidence[i][: block_len - 1]) if confidence else None
        self._count("draft", block_len)
        return Hypothesis(None, tokens, probs)

    def verify(self, kind: str, start: int, root: int, hypotheses: list[Hypothesis]) -> list:
        i = self._index(start, root)
        self._count(kind, 1 + sum(len(h.tokens) for h in hypotheses))
        ref = self.reference
        # the prediction after depth d is the reference token there; past the end: never accepted
        return [[ref[i + 1 + d] if i + 1 + d < len(ref) else -1 for d in range(len(h.tokens) + 1)]
                for h in hypotheses]

    def commit(self, best: int, accepted: int) -> None:
        pass

    def peek(self, start: int, hypotheses: list[Hypothesis]) -> int:
        """Tokens a verification at `start` would keep (most accepted + 1), without a pass."""
        i = start - self.prompt_len
        most = 0
        for h in hypotheses:
            n = 0
            while (n < len(h.tokens) and i + 1 + n < len(self.reference)
                   and h.tokens[n] == self.reference[i + 1 + n]):
                n += 1
            most = max(most, n)
        return most + 1


def _verify(backend, kind, start, root, hypotheses, eos):
    """Verify and keep the hypothesis with the most accepted tokens, the first on ties; acceptance
    ends after an accepted EOS (orthrus/decoding.py:336-351). Returns (index, accepted, bonus)."""
    preds = backend.verify(kind, start, root, hypotheses)
    best, best_accepted = 0, -1
    for index, (hyp, pred) in enumerate(zip(hypotheses, preds)):
        n = 0
        while n < len(hyp.tokens) and hyp.tokens[n] == pred[n]:
            n += 1
            if hyp.tokens[n - 1] in eos:
                break
        if n > best_accepted:
            best, best_accepted = index, n
    backend.commit(best, best_accepted)
    return best, best_accepted, preds[best][best_accepted]


def _advance(gen, start, kept, bonus, eos, max_length):
    """Append the accepted tokens and the AR bonus (orthrus/decoding.py:354-369); returns
    (finished, position of the new anchor)."""
    for i, token in enumerate(kept):
        if token in eos:
            gen.tokens.extend(kept[: i + 1])
            gen.eos = True
            return True, start + i + 1
    gen.tokens.extend(kept)
    start += len(kept) + 1
    if start < max_length:
        gen.tokens.append(bonus)
        if bonus in eos:
            gen.eos = True
            return True, start
    return start >= max_length - 1, start


def _worth_a_pass(strategy: Strategy, hypotheses: list[Hypothesis], backend, start: int) -> bool:
    """The tail-pass gate (orthrus/decoding.py:372-381): a long enough hypothesis, enough expected
    tokens when min_expected is set, and for replay-only strategies enough tokens kept."""
    if not hypotheses or max(len(h.tokens) for h in hypotheses) < strategy.min_tail:
        return False
    if strategy.min_expected > 0 and max(map(expected_tokens, hypotheses)) < strategy.min_expected:
        return False
    if strategy.oracle_min_tokens:
        if not hasattr(backend, "peek"):
            raise ValueError(f"strategy {strategy.name} (oracle_min_tokens) is replay-only")
        return backend.peek(start, hypotheses) >= strategy.oracle_min_tokens
    return True


def _finish(gen, backend):
    gen.passes = dict(backend.passes)
    gen.input_tokens = dict(backend.input_tokens)
    gen.seconds = dict(backend.seconds)
    return gen


def decode(backend, strategy: Strategy, prompt_len: int, max_new_tokens: int, eos: set[int]) -> Generation:
    """Greedy Orthrus decoding with `strategy` on a ModelBackend or OracleBackend
    (orthrus/decoding.py:391-429). Each cycle drafts a block and verifies it together with the
    stale tails (reuse); a rejection then yields tail hypotheses that a tail strategy verifies in
    up to max_tail_passes extra passes, or that reuse carries into the next verification."""
    gen = Generation(strategy.name)
    max_length = prompt_len + max_new_tokens
    gen.tokens.append(backend.prefill())
    gen.eos = done = gen.tokens[-1] in eos
    start = prompt_len  # position of the anchor gen.tokens[-1], not in the cache yet
    stale: list[Hypothesis] = []
    while not done and start < max_length - 1:
        block_len = min(backend.block_size, max_length - start)
        root = gen.tokens[-1]
        fresh = backend.draft(start, root, block_len, strategy.needs_confidence)
        hypotheses = [fresh] + [h for h in stale if h.tokens != fresh.tokens]
        best, accepted, bonus = _verify(backend, "verify", start, root, hypotheses, eos)
        kept = hypotheses[best]
        gen.accepted.append(accepted)
        gen.branch.append(kept.shift)
        done, start = _advance(gen, start, kept.tokens[:accepted], bonus, eos, max_length)
        stale, tail_passes = [], 0
        while strategy.kind != "base" and not done and accepted < len(kept.tokens):
            tails = tail_hypotheses(kept, accepted, strategy.shifts, max_length - 1 - start)
            if strategy.kind == "reuse":
                stale = tails
                break
            if tail_passes == strategy.max_tail_passes or not _worth_a_pass(strategy, tails, backend, start):
                break
            tail_passes += 1
            best, accepted, bonus = _verify(backend, "tail", start, gen.tokens[-1], tails, eos)
            kept = tails[best]
            gen.tails.append((len(gen.accepted) - 1, kept.shift, accepted, len(tails),
                              max(len(h.tokens) for h in tails)))
            done, start = _advance(gen, start, kept.tokens[:accepted], bonus, eos, max_length)
    return _finish(gen, backend)


def ar_decode(backend, prompt_len: int, max_new_tokens: int, eos: set[int]) -> Generation:
    """Plain greedy AR decoding through the same backend, one pass per token (orthrus/decoding.py:432-444)."""
    gen = Generation("ar")
    gen.tokens.append(backend.prefill())
    start = prompt_len
    while gen.tokens[-1] not in eos and len(gen.tokens) < max_new_tokens:
        (pred,) = backend.verify("ar", start, gen.tokens[-1], [Hypothesis(None, [])])
        backend.commit(0, 0)
        gen.tokens.append(pred[0])
        start += 1
    gen.eos = gen.tokens[-1] in eos
    return _finish(gen, backend)


@torch.inference_mode()
def draft_table(model, prompt_ids: list[int], reference: list[int], max_new_tokens: int,
                chunk_blocks: int = 64):
    """Diffusion drafts at every anchor of a reference output, as decoding draws them after
    committing reference[: i + 1] (orthrus/decoding.py:447-503): row i holds the block_size - 1
    drafts of the block anchored at reference[i] (fewer where max_new_tokens cuts the block).

    One AR pass caches the whole output; full blocks then go chunk_blocks at a time through one
    diffusion pass with the dual-view training mask (orthrus_attn_fwd mask DUAL: AR keys before
    the anchor, the block's own keys), short blocks one by one. Returns numpy (drafts int32,
    confidence float32), both [len(reference), block_size - 1], padded with -1 and 0."""
    from orthrus_training_b200.modeling_orthrus import DualViewMask

    dev = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    K, mask_id = model.config.block_size, model.config.mask_token_id
    P, max_length = len(prompt_ids), len(prompt_ids) + max_new_tokens
    full = torch.tensor([list(prompt_ids) + list(reference)], device=dev)
    total = full.shape[1]
    cache = KVCache(model.config, batch=1, capacity=total + 8, device=dev, dtype=dtype)
    model(input_ids=full, past_key_values=cache, use_cache=True, logits_to_keep=1)
    drafts = torch.full((len(reference), K - 1), -1, dtype=torch.int32)
    confidence = torch.zeros((len(reference), K - 1), dtype=torch.float32)

    def run(anchors: list[int], block_len: int) -> None:
        n = len(anchors)
        a = torch.tensor(anchors, device=dev)
        ids = torch.full((n, block_len), mask_id, dtype=torch.long, device=dev)
        ids[:, 0] = full[0, a]
        positions = (a[:, None] + torch.arange(block_len, device=dev)).view(1, -1)
        logits = model(input_ids=ids.view(1, -1), position_ids=positions, past_key_values=cache,
                       use_cache=False, is_diffusion_pass=True, ar_seq_len=total,
                       flex_block_mask=DualViewMask(a[None], total, block_len)).logits[0]
        logits = logits.view(n, block_len, -1)[:, :-1].contiguous()
        tokens = ops.argmax_rows(logits.view(-1, logits.shape[-1])).view(n, block_len - 1)
        probs = torch.softmax(logits.float(), -1).gather(-1, tokens[..., None])[..., 0]
        rows = (a - P).cpu()
        drafts[rows, : block_len - 1] = tokens.to(torch.int32).cpu()
        confidence[rows, : block_len - 1] = probs.cpu()

    starts = range(P, min(P + len(reference), max_length - 1))
    full_blocks = [s for s in starts if s + K <= max_length]
    for i in range(0, len(full_blocks), chunk_blocks):
        run(full_blocks[i: i + chunk_blocks], K)
    for s in starts:
        if s + K > max_length:
            run([s], max_length - s)
    return drafts.numpy(), confidence.numpy()


# --- batched device-resident decoding ----------------------------------------------------------


@dataclass
class BlockDecodeResult:
    tokens: list[list[int]]
    accepted: list[list[int]]
    cycles: list[int]
    passes: list[int]
    seconds: float
    prefill_seconds: float
    steady_seconds: float = 0.0  # the replayed cycles only (after prefill, set-up and capture)
    steady_cycles: int = 0       # batched cycles replayed in steady_seconds

    @property
    def total_tokens(self) -> int:
        return sum(len(t) for t in self.tokens)

    @property
    def tpf(self) -> float:
        return self.total_tokens / max(sum(self.passes), 1)


class _DecodeState:
    """Static device buffers of a batched decode (fixed shapes, so one cycle can be graph-captured)."""

    def __init__(self, model, prompts, max_new_tokens, eos, draft_table):
        cfg = model.config
        dev = next(model.parameters()).device
        dtype = next(model.parameters()).dtype
        self.model, self.dev, self.K = model, dev, cfg.block_size
        B = len(prompts)
        self.B = B
        plens = [len(p) for p in prompts]
        self.max_len = torch.tensor([p + max_new_tokens for p in plens], dtype=torch.int32, device=dev)
        cap = max(plens) + max_new_tokens + self.K + 8
        self.cache = KVCache(cfg, batch=B, capacity=cap, device=dev, dtype=dtype)
        self.kv = self.cache.buffers()
        self.start = torch.tensor(plens, dtype=torch.int32, device=dev)
        self.prompt_len = torch.tensor(plens, dtype=torch.int32, device=dev)
        self.anchor = torch.zeros(B, dtype=torch.int64, device=dev)
        self.done = torch.zeros(B, dtype=torch.uint8, device=dev)
        self.out = torch.zeros(B, max_new_tokens + self.K + 1, dtype=torch.int64, device=dev)
        self.out_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.log = torch.zeros(B, max_new_tokens + 1, dtype=torch.int32, device=dev)
        self.cycle = torch.zeros(B, dtype=torch.int32, device=dev)
        self.eos = torch.tensor(sorted(eos), dtype=torch.int64, device=dev) if eos else None
        self.verify_ids = torch.zeros(B, self.K, dtype=torch.int64, device=dev)
        self.ar_tokens = torch.zeros(B, self.K, dtype=torch.int64, device=dev)
        self.block_ids = torch.full((B, self.K), cfg.mask_token_id, dtype=torch.int64, device=dev)
        self.arange = torch.arange(self.K, device=dev, dtype=torch.int64)
        self.draft_table = draft_table  # [B, rows, K-1] int64 or None (scripted drafts)

    def cycle_once(self):
        """One draft + verify + accept cycle on the current stream (no host synchronisation)."""
        model, B, K = self.model, self.B, self.K
        positions = (self.start.to(torch.int64)[:, None] + self.arange[None]).contiguous()
        if self.draft_table is None:
            self.block_ids[:, 0] = self.anchor
            x = model.model.embed_tokens(self.block_ids)
            limit2 = torch.clamp(self.max_len - self.start, 1, K).to(torch.int32)
            hidden = model.run_layers(x, positions, "draft", kv=self.kv, offsets=self.start,
                                      limit2=limit2)
            logits = model.lm_logits(hidden)
            ops.decode_draft(logits, self.anchor, self.done, self.verify_ids)
        else:
            row = (self.start - self.prompt_len).clamp(0, self.draft_table.shape[1] - 1).to(torch.int64)
            drafts = self.draft_table[torch.arange(B, device=self.dev), row]
            self.verify_ids[:, 0] = self.anchor
            self.verify_ids[:, 1:] = drafts
        x = model.model.embed_tokens(self.verify_ids)
        hidden = model.run_layers(x, positions, "ar", kv=self.kv, offsets=self.start)
        logits = model.lm_logits(hidden)
        ops.decode_verify_accept(logits, self.verify_ids, self.ar_tokens, self.eos, self.max_len,
                                 self.start, self.anchor, self.done, self.out, self.out_len, self.log,
                                 self.cycle)


@torch.inference_mode()
def block_decode(model, prompts: list[list[int]], max_new_tokens: int, eos=(), *, draft_table=None,
                 use_graph: bool = True, check_every: int = 4) -> BlockDecodeResult:
    """Greedy Orthrus decoding of a batch of prompts with the cycle state on the device.

    draft_table: optional int64 [B, max_new_tokens, K-1]; row i replaces the diffusion drafts of
    the block anchored at prompt_len + i (scripted drafts that exercise accept / rollback, the
    device counterpart of the reference tests' ScriptedBackend)."""
    eos = set(eos)
    st = _DecodeState(model, prompts, max_new_tokens, eos, draft_table)
    B, dev = st.B, st.dev
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    # prefill each prompt into its slice of the batched cache
    for b, p in enumerate(prompts):
        ids = torch.tensor([p], device=dev)
        x = model.model.embed_tokens(ids)
        pos = torch.arange(len(p), device=dev)[None]
        kv_b = [(k[b: b + 1], v[b: b + 1]) for k, v in st.kv]
        zero = torch.zeros(1, dtype=torch.int32, device=dev)
        hidden = model.run_layers(x, pos, "ar", kv=kv_b, offsets=zero)
        tok = ops.argmax_rows(model.lm_logits(hidden[:, -1:]).reshape(1, -1))
        st.anchor[b] = tok[0]
        st.out[b, 0] = tok[0]
    st.out_len.fill_(1)
    if st.eos is not None:
        st.done |= torch.isin(st.anchor, st.eos).to(torch.uint8)
    st.done |= (st.start >= st.max_len - 1).to(torch.uint8)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    graph = None
    if use_graph:
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            # warm-up cycles on a throwaway copy of the state would change it, so the first real
            # cycle runs eagerly (allocations, kernel attribute setup) and the next ones replay
            st.cycle_once()
        torch.cuda.current_stream(dev).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            st.cycle_once()
        # capture recorded but did not run the cycle
    cycles_run = 1 if use_graph else 0
    torch.cuda.synchronize(dev)
    t_steady = time.perf_counter()
    first_steady = cycles_run
    max_cycles = max_new_tokens + 1
    while cycles_run < max_cycles:
        if int(st.done.min().item()) == 1:
            break
        for _ in range(check_every):
            if graph is not None:
                graph.replay()
            else:
                st.cycle_once()
            cycles_run += 1
    torch.cuda.synchronize(dev)
    t2 = time.perf_counter()
    out_len = st.out_len.tolist()
    out = st.out.tolist()
    cyc = st.cycle.tolist()
    log = st.log.tolist()
    tokens = [out[b][: min(out_len[b], max_new_tokens)] for b in range(B)]
    accepted = [log[b][: cyc[b]] for b in range(B)]
    return BlockDecodeResult(tokens=tokens, accepted=accepted, cycles=cyc,
                             passes=[1 + 2 * c for c in cyc], seconds=t2 - t0,
                             prefill_seconds=t1 - t0, steady_seconds=t2 - t_steady,
                             steady_cycles=cycles_run - first_steady)


@torch.inference_mode()
def ar_generate_batch(model, input_ids: torch.Tensor, max_new_tokens: int, eos=()):
    """Plain greedy decoding with the AR view (orthrus/evaluate.py:59-76), batch 1, on the device
    path: one verification pass of one token per step."""
    eos = {eos} if isinstance(eos, int) else set(eos or ())
    prompt = input_ids[0].tolist()
    backend = ModelBackend(model, prompt)
    gen = ar_decode(backend, len(prompt), max_new_tokens, eos)
    return torch.tensor([prompt + gen.tokens], device=input_ids.device)
