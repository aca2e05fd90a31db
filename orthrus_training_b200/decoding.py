"""Orthrus parallel block decoding on the Blackwell kernels: drop-in for orthrus/decoding.py (the
base, tail and reuse strategies with tree verification, plain greedy, replay from a draft table,
draft_table) plus a batched, device-resident decode loop for the base strategy.

Decoding with a strategy is a small state machine (``_Decoder``) over a backend that offers four
calls, the protocol of orthrus/decoding.py:145-333:

    prefill()                                  -> first generated token (the first anchor)
    draft(start, anchor, block_len, confidence) -> Hypothesis of the block's drafts
    verify(kind, start, root, hypotheses)       -> per hypothesis, the AR argmax after the root
                                                   and after each of its tokens
    commit(best, accepted)                      -> keep the root and `accepted` tokens of one

``ModelBackend`` runs an OrthrusLM on the device (several hypotheses share one pass through the
TREE mask of the attention kernels); ``OracleBackend`` replays a strategy without the model from
a reference output and a draft table. The bookkeeping rules are fixed by the reference's traces
(kept pass for pass): the hypothesis with the most accepted tokens wins and the first listed wins
ties, acceptance stops after an accepted EOS, the AR token after the accepted run (the bonus) is
always kept, and a tail pass happens only while the strategy's gate allows it.

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
import functools
import itertools
import operator
import time
from collections import Counter
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch

from orthrus_training_b200 import ops
from orthrus_training_b200.kv_cache import KVCache

KINDS = ("base", "tail", "reuse")


# --- strategies and hypotheses -----------------------------------------------------------------


@dataclass(frozen=True)
class Strategy:
    """One decoding strategy, configured by the reference's fields (orthrus/decoding.py:41-70):

    kind               base: draft then verify; tail: after a rejection, verify the rest of the
                       block behind the bonus in extra passes; reuse: carry that rest into the
                       next block's verification instead
    shifts             the tail hypotheses, in tie-breaking order (0 substitution, 1 insertion,
                       -j deletion of j drafts)
    min_tail           a tail pass needs a hypothesis of at least this many tokens
    min_expected       ... and, when > 0, an expected kept-token count of at least this
    max_tail_passes    tail passes per cycle
    oracle_min_tokens  replay only: a tail pass only when it would keep at least this many tokens
    """

    name: str
    kind: str = "base"
    shifts: tuple[int, ...] = (0,)
    min_tail: int = 1
    min_expected: float = 0.0
    max_tail_passes: int = 1
    oracle_min_tokens: int = 0

    def __post_init__(self):
        object.__setattr__(self, "shifts", tuple(int(s) for s in self.shifts))
        problem = next(self._problems(), None)
        if problem is not None:
            raise ValueError(f"decoding strategy {self.name!r}: {problem}")

    def _problems(self):
        if self.kind not in KINDS:
            yield f"kind {self.kind!r} is not one of {', '.join(KINDS)}"
        if not self.shifts:
            yield "at least one tail shift is needed"
        elif len(set(self.shifts)) < len(self.shifts):
            yield f"tail shifts repeat: {self.shifts}"
        elif max(self.shifts) > 1:
            yield f"a tail shift above 1 has no meaning: {self.shifts}"
        if self.min_tail < 1:
            yield f"min_tail is {self.min_tail}, it must be at least 1"
        if self.max_tail_passes < 1:
            yield f"max_tail_passes is {self.max_tail_passes}, it must be at least 1"
        if self.oracle_min_tokens and self.kind != "tail":
            yield "oracle_min_tokens gates tail passes, so the kind must be 'tail'"

    @property
    def needs_confidence(self) -> bool:
        """Whether drafts must carry their probabilities (the min_expected gate of a tail pass)."""
        return self.kind == "tail" and self.min_expected > 0

    def to_dict(self) -> dict:
        out = dataclasses.asdict(self)
        out["shifts"] = list(self.shifts)
        return out


def parse_strategies(specs: list[dict]) -> list[Strategy]:
    """Strategies from their field dicts; names must be distinct."""
    strategies = [Strategy(**spec) for spec in specs]
    repeated = sorted(n for n, c in Counter(s.name for s in strategies).items() if c > 1)
    if repeated:
        raise ValueError(f"strategy names must be distinct; repeated: {repeated}")
    return strategies


@dataclass
class Hypothesis:
    """A continuation to verify (orthrus/decoding.py:82-86): shift None for a block's fresh
    drafts, else the tail shift it was cut with; confidence: the diffusion probability of each
    token, when the strategy needs it."""

    shift: int | None
    tokens: list[int]
    confidence: list[float] | None = None


def tail_hypotheses(source: Hypothesis, accepted: int, shifts: tuple[int, ...],
                    room: int) -> list[Hypothesis]:
    """Continuations of the bonus after source.tokens[accepted] lost to it (orthrus/decoding.py:
    89-107): for shift s the tokens from index accepted + 1 - s on, at most `room` of them.
    An empty continuation, or one equal to an earlier shift's, is not a hypothesis."""
    kept: dict[tuple[int, ...], Hypothesis] = {}
    for shift in shifts:
        cut = slice(accepted + 1 - shift, accepted + 1 - shift + room)
        tokens = tuple(source.tokens[cut])
        if tokens and tokens not in kept:
            conf = None if source.confidence is None else list(source.confidence[cut])
            kept[tokens] = Hypothesis(shift, list(tokens), conf)
    return list(kept.values())


def expected_tokens(hypothesis: Hypothesis) -> float:
    """Tokens a verification of the hypothesis keeps in expectation when each confidence is an
    independent acceptance probability: 1 (the bonus) + the sum of the running products
    (orthrus/decoding.py:110-116). Summed left to right from 1, the order the gate's threshold
    comparison was pinned with."""
    running = itertools.accumulate(hypothesis.confidence or (), operator.mul)
    return functools.reduce(operator.add, running, 1.0)


@dataclass
class Generation:
    """One decoded output and its pass accounting, with the reference's fields
    (orthrus/decoding.py:119-142): accepted and branch per cycle (branch: None for the fresh
    drafts, else the shift of a reused tail), tails per tail pass (cycle, shift of the kept
    hypothesis, accepted, number of hypotheses, longest hypothesis), and per pass kind the
    passes, input tokens and host-synchronised seconds."""

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


# --- backends ------------------------------------------------------------------------------------


class _PassLedger:
    """Per-kind pass, input-token and time counts shared by the backends."""

    def __init__(self):
        self.passes, self.input_tokens, self.seconds = Counter(), Counter(), Counter()

    def _count(self, kind: str, tokens: int) -> None:
        self.passes[kind] += 1
        self.input_tokens[kind] += tokens

    @contextmanager
    def _pass(self, kind: str, tokens: int):
        began = time.perf_counter()
        yield
        self.seconds[kind] += time.perf_counter() - began
        self._count(kind, tokens)


def _tree_layout(hypotheses: list[Hypothesis]):
    """Verification input of a root plus hypotheses: the new tokens after the root, each token's
    depth below the root, where each hypothesis begins among the new tokens (the root is 0), and,
    for more than one hypothesis, each token's branch start (the tree mask's int32 form)."""
    starts = list(itertools.accumulate((len(h.tokens) for h in hypotheses[:-1]), initial=1))
    tokens, depth, branch_lo = [], [0], [1]
    for begin, h in zip(starts, hypotheses):
        tokens += h.tokens
        depth += range(1, len(h.tokens) + 1)
        branch_lo += [begin] * len(h.tokens)
    return tokens, depth, starts, (branch_lo if len(hypotheses) > 1 else None)


class ModelBackend(_PassLedger):
    """An OrthrusLM decoding one prompt greedily on the device, the backend of
    orthrus/decoding.py:145-264. The cache holds the committed prefix; the newest token (the
    anchor) enters it only with the next verification. Hypotheses verified together share one
    pass under the TREE mask of the attention kernels; commit() moves the kept branch's K/V rows
    behind the root when it was not the first branch."""

    def __init__(self, model, prompt_ids: list[int], record_drafts: bool = False):
        super().__init__()
        self.model = model
        self.device = next(model.parameters()).device
        self.block_size = model.config.block_size
        self.mask_token_id = model.config.mask_token_id
        self.prompt = torch.tensor([prompt_ids], device=self.device)
        dtype = next(model.parameters()).dtype
        self.cache = KVCache(model.config, batch=1, capacity=len(prompt_ids) + 64,
                             device=self.device, dtype=dtype)
        self.record_drafts = record_drafts
        self.drafts: dict[int, list[int]] = {}
        self._last: tuple[int, list[int]] | None = None  # (root position, hypothesis starts)

    def _timed(self, kind: str, tokens: int, run):
        """Runs `run` as one counted, timed pass of `kind` (the hook a scripted subclass such as
        the reference tests' ScriptedBackend calls)."""
        with self._pass(kind, tokens):
            return run()

    def _argmax(self, logits: torch.Tensor) -> torch.Tensor:
        return ops.argmax_rows(logits.reshape(-1, logits.shape[-1]).contiguous())

    def prefill(self) -> int:
        with self._pass("prefill", self.prompt.shape[1]):
            out = self.model(input_ids=self.prompt, past_key_values=self.cache, use_cache=True,
                             logits_to_keep=1)
            return int(self._argmax(out.logits[0]).item())  # the host read ends the timed pass

    def draft(self, start: int, anchor: int, block_len: int, confidence: bool) -> Hypothesis:
        """The diffusion view over [anchor, mask x (block_len - 1)] at positions start.. : the
        drafts for positions start + 1 .. start + block_len - 1."""
        with self._pass("draft", block_len):
            ids = torch.full((1, block_len), self.mask_token_id, dtype=torch.long, device=self.device)
            ids[0, 0] = anchor
            pos = torch.arange(start, start + block_len, device=self.device)[None]
            logits = self.model(input_ids=ids, position_ids=pos, past_key_values=self.cache,
                                use_cache=False, is_diffusion_pass=True, ar_seq_len=start).logits[0, :-1]
            best = self._argmax(logits)
            probs = None
            if confidence:
                probs = torch.softmax(logits.float(), -1).gather(-1, best[:, None])[:, 0].tolist()
            hyp = Hypothesis(None, best.tolist(), probs)
        if self.record_drafts:
            self.drafts[start] = hyp.tokens
        return hyp

    def verify(self, kind: str, start: int, root: int, hypotheses: list[Hypothesis]) -> list:
        """One AR pass over the root (position `start`) and every hypothesis behind it, all written
        to the cache at rows start + their index; each token sits at position start + its depth
        and sees the prefix, the root and its own branch up to itself. Returns per hypothesis the
        AR argmax after the root and after each of its tokens (orthrus/decoding.py:208-241)."""
        new, depth, starts, branch_lo = _tree_layout(hypotheses)
        with self._pass(kind, 1 + len(new)):
            ids = torch.tensor([[root] + new], device=self.device)
            pos = torch.tensor([depth], device=self.device) + start
            tree_lo = None if branch_lo is None else torch.tensor(branch_lo, dtype=torch.int32,
                                                                  device=self.device)
            self.cache.reserve(start + ids.shape[1])
            logits = self.model(input_ids=ids, position_ids=pos, past_key_values=self.cache,
                                use_cache=True, tree_lo=tree_lo).logits[0]
            preds = self._argmax(logits).tolist()
        self._last = (start, starts)
        return [[preds[0]] + preds[b: b + len(h.tokens)] for b, h in zip(starts, hypotheses)]

    def commit(self, best: int, accepted: int) -> None:
        """Keeps the prefix, the root and the first `accepted` tokens of hypothesis `best` of the
        last verification (orthrus/decoding.py:243-264)."""
        root_at, starts = self._last
        kept_from = root_at + starts[best]
        if accepted and kept_from != root_at + 1:  # not directly behind the root: move its rows
            dst = slice(root_at + 1, root_at + 1 + accepted)
            src = slice(kept_from, kept_from + accepted)
            for k, v in self.cache.buffers():
                k[:, :, dst] = k[:, :, src].clone()
                v[:, :, dst] = v[:, :, src].clone()
        self.cache.crop(root_at + 1 + accepted)


class OracleBackend(_PassLedger):
    """Greedy decoding replayed without a model (orthrus/decoding.py:267-333): the AR argmax at
    every position is the reference output's next token, and drafts come from a draft table
    (row i: the drafts of the block anchored at reference[i]). A replay is exact when real
    decoding produced that output and drew those drafts."""

    def __init__(self, prompt_len: int, reference: list[int], drafts: list[list[int]],
                 confidence: list[list[float]] | None, block_size: int):
        super().__init__()
        self.prompt_len, self.block_size = prompt_len, block_size
        self.reference = list(reference)
        self.drafts, self.confidence = drafts, confidence

    def _row(self, position: int, token: int) -> int:
        """Index of `position` in the reference output, checking that it holds `token`."""
        row = position - self.prompt_len
        if row < 0 or row >= len(self.reference) or self.reference[row] != token:
            raise RuntimeError(f"the replay no longer follows the reference output (position {position})")
        return row

    def _after(self, row: int, n: int) -> list[int]:
        """The reference tokens after row, n + 1 of them, -1 (never accepted) past its end."""
        tail = self.reference[row + 1: row + 2 + n]
        return tail + [-1] * (n + 1 - len(tail))

    def prefill(self) -> int:
        self._count("prefill", self.prompt_len)
        return self.reference[0]

    def draft(self, start: int, anchor: int, block_len: int, confidence: bool) -> Hypothesis:
        row = self._row(start, anchor)
        tokens = list(self.drafts[row][: block_len - 1])
        if len(tokens) < block_len - 1 or any(t < 0 for t in tokens):
            raise RuntimeError(f"the draft table holds no full block of {block_len} at position {start}")
        probs = list(self.confidence[row][: block_len - 1]) if confidence else None
        self._count("draft", block_len)
        return Hypothesis(None, tokens, probs)

    def verify(self, kind: str, start: int, root: int, hypotheses: list[Hypothesis]) -> list:
        row = self._row(start, root)
        self._count(kind, 1 + sum(len(h.tokens) for h in hypotheses))
        return [self._after(row, len(h.tokens)) for h in hypotheses]

    def commit(self, best: int, accepted: int) -> None:
        pass

    def peek(self, start: int, hypotheses: list[Hypothesis]) -> int:
        """Tokens a verification at `start` would keep (the longest accepted run + the bonus),
        without counting a pass."""
        row = start - self.prompt_len
        truth = self.reference[row + 1:]
        runs = (sum(1 for _ in itertools.takewhile(lambda pair: pair[0] == pair[1], zip(h.tokens, truth)))
                for h in hypotheses)
        return max(runs, default=0) + 1


# --- the decoding state machine ------------------------------------------------------------------


def _accepted_run(tokens: list[int], preds: list[int], eos: set[int]) -> int:
    """Leading tokens equal to the AR argmax before them, ending after an accepted EOS."""
    n = 0
    for token, pred in zip(tokens, preds):
        if token != pred:
            break
        n += 1
        if token in eos:
            break
    return n


def _gate_open(strategy: Strategy, hypotheses: list[Hypothesis], backend, start: int) -> bool:
    """Whether a tail pass over `hypotheses` is worth it (orthrus/decoding.py:372-381): a long
    enough hypothesis, enough expected tokens when min_expected is set, and for a replay-only
    strategy enough tokens actually kept."""
    if not hypotheses or max(len(h.tokens) for h in hypotheses) < strategy.min_tail:
        return False
    if strategy.min_expected > 0 and max(expected_tokens(h) for h in hypotheses) < strategy.min_expected:
        return False
    if strategy.oracle_min_tokens:
        peek = getattr(backend, "peek", None)
        if peek is None:
            raise ValueError(f"strategy {strategy.name!r} gates on oracle_min_tokens, which only a "
                             f"replay backend (one with peek) can evaluate")
        return peek(start, hypotheses) >= strategy.oracle_min_tokens
    return True


class _Decoder:
    """One greedy Orthrus generation (orthrus/decoding.py:391-429) as a state machine over a
    backend: `anchor_at` is the position of the newest token (the anchor, not in the cache yet),
    `limit` the first position past the output, `pending` the previous block's rejected tails
    that a reuse strategy verifies again."""

    def __init__(self, backend, strategy: Strategy, prompt_len: int, max_new_tokens: int, eos):
        self.backend, self.strategy, self.eos = backend, strategy, eos
        self.limit = prompt_len + max_new_tokens
        self.anchor_at = prompt_len
        self.gen = Generation(strategy.name)
        self.finished = False
        self.pending: list[Hypothesis] = []

    def run(self) -> Generation:
        first = self.backend.prefill()
        self.gen.tokens.append(first)
        self.finished = self.gen.eos = first in self.eos
        while not self.finished and self.anchor_at < self.limit - 1:
            self._cycle()
        return _with_accounting(self.gen, self.backend)

    def _select(self, kind: str, hypotheses: list[Hypothesis]) -> tuple[Hypothesis, int]:
        """Verifies the hypotheses behind the current anchor, keeps the one with the longest
        accepted run (the first listed on ties), appends its run and the bonus."""
        preds = self.backend.verify(kind, self.anchor_at, self.gen.tokens[-1], hypotheses)
        runs = [_accepted_run(h.tokens, p, self.eos) for h, p in zip(hypotheses, preds)]
        best = max(range(len(runs)), key=runs.__getitem__)  # max() keeps the first maximum
        self.backend.commit(best, runs[best])
        self._extend(hypotheses[best].tokens[: runs[best]], preds[best][runs[best]])
        return hypotheses[best], runs[best]

    def _extend(self, run: list[int], bonus: int) -> None:
        """Appends an accepted run and the AR bonus behind it (orthrus/decoding.py:354-369): the
        output ends at an EOS in the run, at an EOS bonus, or when the next anchor would leave no
        room for a block."""
        gen = self.gen
        for i, token in enumerate(run):
            if token in self.eos:
                gen.tokens += run[: i + 1]
                gen.eos = self.finished = True
                self.anchor_at += i + 1
                return
        gen.tokens += run
        self.anchor_at += len(run) + 1
        if self.anchor_at < self.limit:
            gen.tokens.append(bonus)
            if bonus in self.eos:
                gen.eos = self.finished = True
                return
        self.finished = self.anchor_at >= self.limit - 1

    def _cycle(self) -> None:
        strategy, backend = self.strategy, self.backend
        block_len = min(backend.block_size, self.limit - self.anchor_at)
        fresh = backend.draft(self.anchor_at, self.gen.tokens[-1], block_len, strategy.needs_confidence)
        candidates = [fresh, *(h for h in self.pending if h.tokens != fresh.tokens)]
        kept, accepted = self._select("verify", candidates)
        self.gen.accepted.append(accepted)
        self.gen.branch.append(kept.shift)
        self.pending = []
        if strategy.kind == "base":
            return
        tail_passes = 0
        while not self.finished and accepted < len(kept.tokens):
            tails = tail_hypotheses(kept, accepted, strategy.shifts, self.limit - 1 - self.anchor_at)
            if strategy.kind == "reuse":
                self.pending = tails
                return
            if tail_passes >= strategy.max_tail_passes or not _gate_open(strategy, tails, backend,
                                                                          self.anchor_at):
                return
            tail_passes += 1
            kept, accepted = self._select("tail", tails)
            self.gen.tails.append((len(self.gen.accepted) - 1, kept.shift, accepted, len(tails),
                                   max(len(h.tokens) for h in tails)))


def _with_accounting(gen: Generation, backend) -> Generation:
    gen.passes = dict(backend.passes)
    gen.input_tokens = dict(backend.input_tokens)
    gen.seconds = dict(backend.seconds)
    return gen


def decode(backend, strategy: Strategy, prompt_len: int, max_new_tokens: int, eos: set[int]) -> Generation:
    """Greedy Orthrus decoding with `strategy` on a ModelBackend or OracleBackend
    (orthrus/decoding.py:391-429)."""
    return _Decoder(backend, strategy, prompt_len, max_new_tokens, set(eos)).run()


def ar_decode(backend, prompt_len: int, max_new_tokens: int, eos: set[int]) -> Generation:
    """Plain greedy decoding through the same backend, one verification of the newest token per
    generated token (orthrus/decoding.py:432-444): the reference for losslessness."""
    gen = Generation("ar")
    position, token = prompt_len, backend.prefill()
    gen.tokens.append(token)
    while token not in eos and len(gen.tokens) < max_new_tokens:
        token = backend.verify("ar", position, token, [Hypothesis(None, [])])[0][0]
        backend.commit(0, 0)
        gen.tokens.append(token)
        position += 1
    gen.eos = token in eos
    return _with_accounting(gen, backend)


@torch.inference_mode()
def draft_table(model, prompt_ids: list[int], reference: list[int], max_new_tokens: int,
                chunk_blocks: int = 64):
    """The diffusion drafts decoding would draw at every anchor of a reference output, each
    after committing reference[: i + 1] (orthrus/decoding.py:447-503): row i holds the
    block_size - 1 drafts of the block anchored at reference[i] (fewer where max_new_tokens cuts
    the block). Returns numpy (drafts int32, confidence float32), [len(reference), block_size - 1],
    padded with -1 and 0.

    One AR pass caches the prompt and the whole output. The anchors are then grouped into passes:
    full blocks chunk_blocks at a time, each pass one diffusion forward over all its blocks under
    the dual-view mask (orthrus_attn_fwd mask DUAL: AR keys strictly before each block's anchor,
    plus the block's own keys), and each block that max_new_tokens cuts short in a pass of its own.
    """
    from orthrus_training_b200.modeling_orthrus import DualViewMask

    dev = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    K, mask_id = model.config.block_size, model.config.mask_token_id
    P = len(prompt_ids)
    limit = P + max_new_tokens
    sequence = torch.tensor([list(prompt_ids) + list(reference)], device=dev)
    total = sequence.shape[1]
    cache = KVCache(model.config, batch=1, capacity=total + 8, device=dev, dtype=dtype)
    model(input_ids=sequence, past_key_values=cache, use_cache=True, logits_to_keep=1)

    anchors = range(P, min(P + len(reference), limit - 1))
    full = [a for a in anchors if a + K <= limit]
    passes = [(full[i: i + chunk_blocks], K) for i in range(0, len(full), chunk_blocks)]
    passes += [([a], limit - a) for a in anchors if a + K > limit]

    drafts = torch.full((len(reference), K - 1), -1, dtype=torch.int32)
    confidence = torch.zeros((len(reference), K - 1), dtype=torch.float32)
    for group, width in passes:
        at = torch.tensor(group, device=dev)
        ids = torch.full((len(group), width), mask_id, dtype=torch.long, device=dev)
        ids[:, 0] = sequence[0, at]
        pos = (at[:, None] + torch.arange(width, device=dev)).reshape(1, -1)
        out = model(input_ids=ids.reshape(1, -1), position_ids=pos, past_key_values=cache, use_cache=False,
                    is_diffusion_pass=True, ar_seq_len=total,
                    flex_block_mask=DualViewMask(at[None], total, width))
        logits = out.logits[0].view(len(group), width, -1)[:, :-1].contiguous()
        best = ops.argmax_rows(logits.view(-1, logits.shape[-1])).view(len(group), width - 1)
        prob = torch.softmax(logits.float(), -1).gather(-1, best[..., None])[..., 0]
        rows = (at - P).cpu()
        drafts[rows, : width - 1] = best.to(torch.int32).cpu()
        confidence[rows, : width - 1] = prob.cpu()
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
    """Static device buffers of a batched decode (fixed shapes, so one cycle can be graph-captured).
    The buffers depend on the batch size, the cache capacity and the decode settings only; reset()
    loads a new set of prompts into them, so a captured cycle can be replayed for later calls."""

    def __init__(self, model, B, cap, max_new_tokens, eos, table_rows=None, sampler=None):
        cfg = model.config
        dev = next(model.parameters()).device
        dtype = next(model.parameters()).dtype
        self.model, self.dev, self.K = model, dev, cfg.block_size
        self.B, self.cap, self.max_new = B, cap, max_new_tokens
        self.max_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.cache = KVCache(cfg, batch=B, capacity=cap, device=dev, dtype=dtype)
        self.kv = self.cache.buffers()
        self.start = torch.zeros(B, dtype=torch.int32, device=dev)
        self.prompt_len = torch.zeros(B, dtype=torch.int32, device=dev)
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
        # scripted drafts: [B, rows, K-1] int64, or None
        self.draft_table = (torch.zeros(B, table_rows, self.K - 1, dtype=torch.int64, device=dev)
                            if table_rows is not None else None)
        # sampled decoding: the draft distributions q of the cycle's drafts, over their candidates
        self.sampler = sampler
        if sampler is not None:
            if table_rows is not None:
                raise ValueError("scripted drafts have no draft distribution to sample against")
            C = sampler.candidates(cfg.vocab_size)
            self.draft_probs = torch.zeros(B, self.K - 1, C, dtype=torch.float32, device=dev)

    @staticmethod
    def capacity(prompts, max_new_tokens, K) -> int:
        """KV rows per sequence, rounded up to 128 so that calls with similar prompts share one state."""
        need = max(len(p) for p in prompts) + max_new_tokens + K + 8
        return -(-need // 128) * 128

    @classmethod
    def for_prompts(cls, model, prompts, max_new_tokens, eos, draft_table=None, sampler=None):
        K = model.config.block_size
        st = cls(model, len(prompts), cls.capacity(prompts, max_new_tokens, K), max_new_tokens, eos,
                 None if draft_table is None else draft_table.shape[1], sampler)
        st.reset(prompts, draft_table)
        return st

    def reset(self, prompts, draft_table=None):
        """Loads a new batch of prompts (the KV cache rows are rewritten by their prefill)."""
        plens = torch.tensor([len(p) for p in prompts], dtype=torch.int32)
        self.max_len.copy_(plens + self.max_new)
        self.start.copy_(plens)
        self.prompt_len.copy_(plens)
        for t in (self.anchor, self.done, self.out, self.out_len, self.log, self.cycle):
            t.zero_()
        if self.draft_table is not None:
            self.draft_table.copy_(draft_table)

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
            if self.sampler is None:
                ops.decode_draft_ids(model.lm_argmax(hidden), self.anchor, self.done, self.verify_ids)
            else:
                logits = model.lm_logits(hidden)
                draft_vals, draft_ids = ops.sample_candidates(logits[:, : K - 1], self.sampler)
                ops.decode_sample_draft(draft_vals, draft_ids, self.sampler, self.cycle, self.anchor,
                                        self.done, self.verify_ids, self.draft_probs)
        else:
            row = (self.start - self.prompt_len).clamp(0, self.draft_table.shape[1] - 1).to(torch.int64)
            drafts = self.draft_table[torch.arange(B, device=self.dev), row]
            self.verify_ids[:, 0] = self.anchor
            self.verify_ids[:, 1:] = drafts
        x = model.model.embed_tokens(self.verify_ids)
        hidden = model.run_layers(x, positions, "ar", kv=self.kv, offsets=self.start)
        if self.sampler is None:
            ops.decode_accept_ids(model.lm_argmax(hidden), self.verify_ids, self.eos, self.max_len,
                                  self.start, self.anchor, self.done, self.out, self.out_len, self.log,
                                  self.cycle)
        else:
            vals, ids = ops.sample_candidates(model.lm_logits(hidden), self.sampler)
            ops.decode_sample_accept(vals, ids, self.draft_probs, draft_ids, self.sampler,
                                     self.verify_ids, self.eos, self.max_len, self.start, self.anchor,
                                     self.done, self.out, self.out_len, self.log, self.cycle)


_STATE_CACHE: dict = {}  # insertion-ordered: the least recently used state is evicted first
_STATE_CACHE_SIZE = 2  # e.g. plain and scripted drafts over the same prompts


def clear_decode_cache() -> None:
    """Drops the decode states and captured cycles kept for reuse by block_decode."""
    _STATE_CACHE.clear()


@torch.inference_mode()
def block_decode(model, prompts: list[list[int]], max_new_tokens: int, eos=(), *, draft_table=None,
                 use_graph: bool = True, check_every: int = 4,
                 sampler: ops.SamplingParams | None = None) -> BlockDecodeResult:
    """Orthrus decoding of a batch of prompts with the cycle state on the device: greedy, or with
    `sampler` exact rejection sampling of the drafts (orthrus/modeling_orthrus.py:498-511).

    draft_table: optional int64 [B, max_new_tokens, K-1]; row i replaces the diffusion drafts of
    the block anchored at prompt_len + i (scripted drafts that exercise accept / rollback, the
    device counterpart of the reference tests' ScriptedBackend)."""
    eos = set(eos)
    K = model.config.block_size
    cap = _DecodeState.capacity(prompts, max_new_tokens, K)
    rows = None if draft_table is None else draft_table.shape[1]
    # a state and its captured cycle are reused by later calls with the same shapes and settings
    # (and the same weight tensors): the capture is host work of about a tenth of a second
    key = (id(model), tuple(p.data_ptr() for p in model.parameters()), len(prompts), cap, max_new_tokens,
           tuple(sorted(eos)), rows, sampler)
    entry = _STATE_CACHE.pop(key, None) if use_graph else None
    if entry is None:
        while len(_STATE_CACHE) >= _STATE_CACHE_SIZE:  # free the oldest state before allocating one
            _STATE_CACHE.pop(next(iter(_STATE_CACHE)))
        st, graph = _DecodeState(model, len(prompts), cap, max_new_tokens, eos, rows, sampler), None
    else:
        st, graph = entry
    st.reset(prompts, draft_table)
    B, dev = st.B, st.dev
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    # prefill each prompt into its slice of the batched cache
    firsts = []
    for b, p in enumerate(prompts):
        ids = torch.tensor([p], device=dev)
        x = model.model.embed_tokens(ids)
        pos = torch.arange(len(p), device=dev)[None]
        kv_b = [(k[b: b + 1], v[b: b + 1]) for k, v in st.kv]
        zero = torch.zeros(1, dtype=torch.int32, device=dev)
        hidden = model.run_layers(x, pos, "ar", kv=kv_b, offsets=zero)
        if sampler is None:
            tok = model.lm_argmax(hidden[:, -1:])
            st.anchor[b] = tok[0]
            st.out[b, 0] = tok[0]
        else:
            firsts.append(model.lm_logits(hidden[:, -1:]).reshape(1, -1))
    if sampler is not None:  # one draw per sequence, counted by its index
        vals, ids = ops.sample_candidates(torch.cat(firsts), sampler)
        tok = ops.sample_rows(vals, ids, sampler)
        st.anchor.copy_(tok)
        st.out[:, 0] = tok
    st.out_len.fill_(1)
    if st.eos is not None:
        st.done |= torch.isin(st.anchor, st.eos).to(torch.uint8)
    st.done |= (st.start >= st.max_len - 1).to(torch.uint8)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    cycles_run = 0
    if use_graph and graph is None:
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
        cycles_run = 1
    if use_graph:
        _STATE_CACHE[key] = (st, graph)
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
