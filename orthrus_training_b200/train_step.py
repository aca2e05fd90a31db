"""One optimizer step of Orthrus training, data-parallel over the GPUs of one node.

Reference: the step body of orthrus/train.py:336-375 (gradient accumulation over micro-batches,
clip_grad_norm_(1.0), skip the update when the norm is not finite, AdamW on the twins, LambdaLR
with linear warmup + cosine to min_lr_ratio, lr_scale :71-76) and anchor_rng (:79-82).

Data parallelism (new; the reference trains on one GPU): one process per GPU, disjoint packed rows
per rank, and one collective, an all-reduce (average) of the trainable diffusion-view gradients
only. The gradients live in one flat buffer per decoder layer; a post-accumulate-grad hook launches
that layer's all-reduce as soon as its six twin gradients of the last micro-batch are complete,
so communication overlaps the backward of the layers below. The frozen weights never move. The
gradient norm for clipping / skipping is computed after the all-reduce, so every rank takes the
same decision.
"""

from __future__ import annotations

import hashlib
import math

import torch
import torch.distributed as dist

from orthrus_training_b200.objective import (SupervisedLayout, document_starts, orthrus_loss,
                                              sample_anchors, teacher_pass)


def lr_scale(step: int, warmup: int, total: int, min_ratio: float) -> float:
    """Linear warmup then cosine decay to min_ratio (orthrus/train.py:71-76)."""
    if warmup > 0 and step < warmup:
        return (step + 1) / warmup
    progress = min(1.0, max(0.0, (step - warmup) / max(1, total - warmup)))
    return min_ratio + (1.0 - min_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress))


def anchor_rng(seed: int, *keys, device) -> torch.Generator:
    """Generator keyed by (seed, epoch, micro-batch) (orthrus/train.py:79-82)."""
    digest = hashlib.sha256(":".join(map(str, (seed, *keys))).encode()).digest()
    return torch.Generator(device=device).manual_seed(int.from_bytes(digest[:8], "little") >> 1)


class GradBuckets:
    """Flat gradient buffers of the trainable parameters, `layers_per_bucket` decoder layers each,
    with all-reduce hooks: a bucket's all-reduce is launched as soon as its last gradient of the
    step is accumulated. With one rank there is nothing to reduce: the parameters keep no
    preassigned gradient buffers, so the first micro-batch's gradients are stored by autograd as
    they come (no zeroing pass and no accumulating add into a zeroed buffer)."""

    def __init__(self, model, params: list[torch.nn.Parameter], world: int, group=None,
                 layers_per_bucket: int = 1):
        self.world = world
        self.group = group
        self.params = list(params)
        self.buckets = []
        self.armed = False
        if world == 1:
            return
        by_layer: dict[int, list] = {}
        names = {id(p): n for n, p in model.named_parameters()}
        for p in params:
            name = names[id(p)]
            layer = int(name.split("layers.")[1].split(".")[0]) if "layers." in name else -1
            by_layer.setdefault(layer // max(layers_per_bucket, 1) if layer >= 0 else -1, []).append(p)
        self.buckets = []
        for layer in sorted(by_layer, reverse=True):  # backward reaches the last layer first
            ps = by_layer[layer]
            numel = sum(p.numel() for p in ps)
            flat = torch.zeros(numel, dtype=ps[0].dtype, device=ps[0].device)
            off = 0
            for p in ps:
                p.grad = flat[off: off + p.numel()].view_as(p)
                off += p.numel()
            self.buckets.append({"params": ps, "flat": flat, "ready": 0, "handle": None})
        for bucket in self.buckets:
            for p in bucket["params"]:
                p.register_post_accumulate_grad_hook(self._hook(bucket))

    def _hook(self, bucket):
        def fn(param):
            if not self.armed:
                return
            bucket["ready"] += 1
            if bucket["ready"] == len(bucket["params"]):
                bucket["handle"] = dist.all_reduce(bucket["flat"], op=dist.ReduceOp.AVG,
                                                   group=self.group, async_op=True)
        return fn

    def arm(self, on: bool) -> None:
        """Only the last micro-batch of a step all-reduces."""
        self.armed = on and self.world > 1
        for b in self.buckets:
            b["ready"] = 0
            b["handle"] = None

    def wait(self) -> None:
        for b in self.buckets:
            if b["handle"] is not None:
                b["handle"].wait()
                b["handle"] = None
        self.armed = False

    def zero(self) -> None:
        if self.world == 1:
            for p in self.params:
                p.grad = None
            return
        for b in self.buckets:
            b["flat"].zero_()


class PeerLost(RuntimeError):
    """A data-parallel peer left or stopped answering; raised before any collective is launched."""


class PeerMonitor:
    """Host-side liveness of the data-parallel ranks through the process group's key-value store.

    Each rank posts a heartbeat (its step number) before the step's collectives, and a rank that
    leaves posts that it left. Before launching a step's collectives a rank waits until every peer
    has posted the same step; a peer that left, or stayed silent for `timeout_s`, raises PeerLost.
    So no rank launches an all-reduce that a peer will never join (on the GPU that collective
    would otherwise wait for the peer until the process group's own timeout)."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, poll_s: float = 0.005,
                 prefix: str = "orthrus"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.poll_s, self.prefix = timeout_s, poll_s, prefix

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def beat(self, step: int) -> None:
        self.store.set(self._key("step", self.rank), str(step))

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), "1")

    def check(self, step: int) -> None:
        import time

        deadline = time.monotonic() + self.timeout_s
        for peer in range(self.world):
            if peer == self.rank:
                continue
            while True:
                if self.store.check([self._key("left", peer)]):
                    raise PeerLost(f"rank {peer} left before step {step}")
                key = self._key("step", peer)
                if self.store.check([key]) and int(self.store.get(key)) >= step:
                    break
                if time.monotonic() > deadline:
                    raise PeerLost(f"rank {peer} posted no heartbeat for step {step} in {self.timeout_s} s")
                time.sleep(self.poll_s)


class Trainer:
    """Optimizer state and the step of one rank."""

    def __init__(self, model, *, lr=1e-4, betas=(0.9, 0.95), weight_decay=0.0, total_steps=1000,
                 warmup_ratio=0.05, min_lr_ratio=0.1, max_grad_norm=1.0, num_anchors=32,
                 kl_chunk_size=4096, gamma=0.0, seed=42, world=1, rank=0, group=None,
                 check_device_every=50, monitor: PeerMonitor | None = None,
                 document_mask: bool = False, layers_per_bucket: int = 4):
        from orthrus_training_b200.modeling_orthrus import freeze_to_diffusion

        self.model = model
        self.params = freeze_to_diffusion(model)
        self.buckets = GradBuckets(model, self.params, world, group, layers_per_bucket)
        fused = all(p.is_cuda for p in self.params)
        self.optimizer = torch.optim.AdamW(self.params, lr=lr, betas=betas,
                                           weight_decay=weight_decay, fused=fused)
        warmup = int(total_steps * warmup_ratio)
        self.scheduler = torch.optim.lr_scheduler.LambdaLR(
            self.optimizer, lambda s: lr_scale(s, warmup, total_steps, min_lr_ratio))
        self.max_grad_norm = max_grad_norm
        self.num_anchors = num_anchors
        self.kl_chunk_size = kl_chunk_size
        self.gamma = gamma
        self.seed = seed
        self.world, self.rank = world, rank
        self.step_index = 0
        self.fused = fused
        # skipped updates, counted on the device (no host read per step)
        self.skipped = torch.zeros((), dtype=torch.int64, device=self.params[0].device)
        # every this many steps the library's device error word is read (a host sync): a bounded
        # wait that ran out or a clamped out-of-range index then raises instead of passing silently
        self.check_device_every = check_device_every
        self._side = None  # stream of the anchor draw and the supervised layout
        # optional liveness check of the peers before each step's collectives (world > 1)
        self.monitor = monitor
        # attention kept inside each packed conversation (objective.document_starts); off, as in
        # the reference, whose rows attend across conversation boundaries
        self.document_mask = document_mask

    def _prepare(self, model, ids, mask, rng, ready):
        """Queues the teacher pass (it needs the input ids only) and draws the anchors and
        settles the supervised layout on a side stream beside it. Their host reads (candidate
        counts, kept rows, unique targets) then wait only for the side stream's few small
        kernels: with `ready` (an event after which the inputs are complete) those do not wait
        for the previous step's work either, so the device is never drained between steps."""
        main = torch.cuda.current_stream(ids.device)
        if self._side is None:
            self._side = torch.cuda.Stream(ids.device)
        side = self._side
        if ready is None:
            side.wait_stream(main)  # the inputs are complete in the main stream's order
        else:
            side.wait_event(ready)
            main.wait_event(ready)
        doc_start = document_starts(mask) if self.document_mask else None
        teacher = teacher_pass(model, ids, doc_start)
        with torch.cuda.stream(side):
            anchors, valid = sample_anchors(mask, model.config.block_size, self.num_anchors, rng)
            layout = SupervisedLayout(mask, anchors, valid, model.config.block_size, self.gamma)
        main.wait_stream(side)
        # made on the side stream, read on the main one: keep their memory from the side
        # stream's pool until the main stream is done with them
        for t in (anchors, valid, *layout.tensors()):
            t.record_stream(main)
        return anchors, valid, teacher, layout

    def step(self, micro_batches: list[tuple[torch.Tensor, torch.Tensor]], epoch: int = 0,
             indices: list[int] | None = None, ready: torch.cuda.Event | None = None) -> dict:
        """One optimizer step over this rank's micro-batches [(input_ids, assistant_mask), ...]
        (already on the device). `indices` are the micro-batches' indices in the epoch (the keys of
        their anchor generators, as data_io.batches yields them); by default the global
        micro-batch count of this trainer. `ready` is an optional CUDA event after which the
        micro-batches are complete on the device (DevicePrefetcher.ready, or one recorded after
        device-resident inputs were written); without it they are taken as complete in the
        current stream's order. Returns loss, grad_norm and skipped as device tensors (nothing is
        read back to the host)."""
        model = self.model
        accum = len(micro_batches)
        if indices is not None and len(indices) != accum:
            raise ValueError("one index per micro-batch")
        if self.monitor is not None and self.world > 1:
            self.monitor.beat(self.step_index)
            self.monitor.check(self.step_index)  # raises PeerLost before any collective
        self.buckets.zero()
        losses = []
        for j, (ids, mask) in enumerate(micro_batches):
            self.buckets.arm(j == accum - 1)
            if indices is not None:
                index = indices[j]
            else:
                index = (self.step_index * accum + j) * self.world + self.rank  # global micro-batch
            rng = anchor_rng(self.seed, epoch, index, device=ids.device)
            anchors, valid, teacher, layout = self._prepare(model, ids, mask, rng, ready)
            loss, stats = orthrus_loss(model, ids, mask, anchors, valid, self.kl_chunk_size,
                                       gamma=self.gamma, teacher=teacher, layout=layout)
            (loss / accum).backward()
            losses.append(loss.detach())
        self.buckets.wait()
        grad_norm = torch.nn.utils.clip_grad_norm_(self.params, self.max_grad_norm)
        nonfinite = ~torch.isfinite(grad_norm)
        if self.fused:
            # the fused AdamW kernel leaves parameters, moments and step counts untouched when
            # found_inf is 1: the reference's "skip the update if the norm is not finite"
            # (orthrus/train.py:364-368) decided on the device, without reading the norm back
            self.optimizer.found_inf = nonfinite.to(torch.float32)
            self.optimizer.step()
        elif bool(nonfinite):
            pass
        else:
            self.optimizer.step()
        self.skipped += nonfinite.to(torch.int64)
        self.scheduler.step()
        self.step_index += 1
        if self.check_device_every and self.step_index % self.check_device_every == 0:
            from orthrus_training_b200 import _lib

            _lib.raise_on_device_error(grad_norm.device.index or 0)
        return {"loss": torch.stack(losses).mean(), "grad_norm": grad_norm, "skipped": nonfinite}
