"""Orthrus parallel block decoding on the Blackwell kernels: drop-in for orthrus/decoding.py (base
strategy and plain greedy) plus a batched, device-resident decode loop.

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
    """A decoding strategy (orthrus/decoding.py:41-70). The device path implements kind "base"."""

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
    shift: int | None
    tokens: list[int]
    confidence: list[float] | None = None


@dataclass
class Generation:
    """One decoded output with its pass accounting (orthrus/decoding.py:119-142)."""

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
    it yet. Verification of several hypotheses (tree masks) is not implemented yet."""

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
        self._layout = None

    def _timed(self, kind: str, tokens: int, run):
        begin = time.perf_counter()
        result = run()
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
        if len(hypotheses) != 1:
            raise NotImplementedError("tree verification of several hypotheses is not implemented")
        tokens = [root] + list(hypotheses[0].tokens)

        def run():
            ids = torch.tensor([tokens], device=self.device)
            positions = torch.arange(start, start + len(tokens), device=self.device)[None]
            self.cache.reserve(start + len(tokens))
            logits = self.model(input_ids=ids, position_ids=positions, past_key_values=self.cache,
                                use_cache=True).logits[0]
            return ops.argmax_rows(logits.contiguous()).tolist()

        preds = self._timed(kind, len(tokens), run)
        self._layout = start
        return [preds]

    def commit(self, best: int, accepted: int) -> None:
        """Keep the root and the first `accepted` tokens of the verified chain (a length update)."""
        self.cache.crop(self._layout + 1 + accepted)


def _verify(backend, kind, start, root, hypotheses, eos):
    """Greedy accept of one chain: acceptance ends after an accepted EOS (orthrus/decoding.py:336-351)."""
    preds = backend.verify(kind, start, root, hypotheses)
    tokens, pred = hypotheses[0].tokens, preds[0]
    accepted = 0
    while accepted < len(tokens) and tokens[accepted] == pred[accepted]:
        accepted += 1
        if tokens[accepted - 1] in eos:
            break
    backend.commit(0, accepted)
    return 0, accepted, pred[accepted]


def _advance(gen, start, kept, bonus, eos, max_length):
    """Append the accepted tokens and the AR bonus (orthrus/decoding.py:354-369)."""
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


def _finish(gen, backend):
    gen.passes = dict(backend.passes)
    gen.input_tokens = dict(backend.input_tokens)
    gen.seconds = dict(backend.seconds)
    return gen


def decode(backend, strategy: Strategy, prompt_len: int, max_new_tokens: int, eos: set[int]) -> Generation:
    """Greedy Orthrus decoding with the base strategy (orthrus/decoding.py:391-429)."""
    if strategy.kind != "base":
        raise NotImplementedError("tail / reuse strategies are not implemented on the device path")
    gen = Generation(strategy.name)
    max_length = prompt_len + max_new_tokens
    gen.tokens.append(backend.prefill())
    gen.eos = done = gen.tokens[-1] in eos
    start = prompt_len
    while not done and start < max_length - 1:
        block_len = min(backend.block_size, max_length - start)
        root = gen.tokens[-1]
        hypotheses = [backend.draft(start, root, block_len, strategy.needs_confidence)]
        _, accepted, bonus = _verify(backend, "verify", start, root, hypotheses, eos)
        gen.accepted.append(accepted)
        gen.branch.append(None)
        done, start = _advance(gen, start, hypotheses[0].tokens[:accepted], bonus, eos, max_length)
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
