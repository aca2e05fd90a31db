"""The optimizer step (orthrus/train.py:336-375) on the GPU: Trainer.step against the reference's
step body restated on the CPU with the oracle's loss, the device-side non-finite skip, and a
bit-exact resume from a checkpoint (the property tests/test_train.py:77-137 pins for the
reference's training loop).

The reference step body, per optimizer step: for each micro-batch, anchors from
anchor_rng(seed, epoch, index) and sample_anchors, (loss / accum).backward(); then
clip_grad_norm_(twins, max_grad_norm); optimizer.step() only when the norm is finite (AdamW,
betas (0.9, 0.95), weight decay 0, on the twins only); scheduler.step() always (LambdaLR with
lr_scale: linear warmup, cosine to min_lr_ratio)."""

import math

import pytest
import torch
from conftest import load_golden

import oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _golden_model(dtype=torch.float32):
    from test_gpu_model import _load

    g = load_golden("config1.pt")
    return _load(g, dtype), g


def _micro_batches(seed: int, n: int = 2):
    from orthrus_training_b200.synthetic import packed_rows

    out = []
    for j in range(n):
        ids, mask = packed_rows(2, 256, 1023, seed=seed + j, ids="uniform", doc="short")
        out.append((ids, mask))
    return out


def test_trainer_step_equals_the_reference_step_body():
    from orthrus_training_b200.objective import sample_anchors
    from orthrus_training_b200.train_step import Trainer, anchor_rng, lr_scale

    model, g = _golden_model()
    cfg = model.config
    K = cfg.block_size
    hp = dict(lr=1e-3, total_steps=10, warmup_ratio=0.2, min_lr_ratio=0.1, max_grad_norm=0.02,
              num_anchors=4, kl_chunk_size=64, seed=3)
    # the reference body on the CPU, from the same starting weights
    params = {k: v.detach().float().cpu().clone().requires_grad_("_diff." in k)
              for k, v in model.state_dict().items()}
    params["lm_head.weight"] = params["model.embed_tokens.weight"]
    frozen_before = {k: v.detach().clone() for k, v in params.items() if not v.requires_grad}
    twins = [params[n] for n, p in model.named_parameters() if "_diff." in n]
    opt = torch.optim.AdamW(twins, lr=hp["lr"], betas=(0.9, 0.95), weight_decay=0.0)
    warmup = int(hp["total_steps"] * hp["warmup_ratio"])
    sched = torch.optim.lr_scheduler.LambdaLR(
        opt, lambda s: lr_scale(s, warmup, hp["total_steps"], hp["min_lr_ratio"]))

    trainer = Trainer(model, **hp)
    ocfg = O.OracleConfig.from_hf(cfg)
    for step in range(2):
        batches = _micro_batches(10 * step)
        indices = [2 * step, 2 * step + 1]
        # reference step body
        for index, (ids, mask) in zip(indices, batches):
            rng = anchor_rng(hp["seed"], 0, index, device=DEV)
            anchors, valid = sample_anchors(mask.to(DEV), K, hp["num_anchors"], rng)
            loss, _ = O.orthrus_loss(params, ocfg, ids, mask, anchors.cpu(), valid.cpu())
            (loss / len(batches)).backward()
        ref_grads = {n: params[n].grad.clone() for n, p in model.named_parameters() if "_diff." in n}
        norm = torch.nn.utils.clip_grad_norm_(twins, hp["max_grad_norm"])
        assert torch.isfinite(norm)
        opt.step()
        sched.step()
        opt.zero_grad(set_to_none=True)
        # the trainer
        out = trainer.step([(i.to(DEV), m.to(DEV)) for i, m in batches], epoch=0, indices=indices)
        assert not bool(out["skipped"])
        assert abs(out["grad_norm"].item() - norm.item()) <= 1e-4 * norm.item()
        # clipped gradients (the norm exceeded max_grad_norm, so clipping scaled them)
        assert norm.item() > hp["max_grad_norm"]
        for n, p in model.named_parameters():
            if "_diff." in n:
                clipped = ref_grads[n] * (hp["max_grad_norm"] / (norm.item() + 1e-6))
                err = (p.grad.cpu() - clipped).abs().max().item()
                assert err <= 1e-4 * clipped.abs().max().item() + 1e-9, (n, err)
        # parameters after the update: AdamW's first steps move each element by about lr, so a
        # sign flip of a near-zero gradient moves it by at most 2 lr; nearly all agree closely
        lr = hp["lr"] * lr_scale(step, warmup, hp["total_steps"], hp["min_lr_ratio"])
        close = total = 0
        for n, p in model.named_parameters():
            if "_diff." in n:
                d = (p.detach().cpu() - params[n].detach()).abs()
                assert d.max().item() <= 2 * lr + 1e-7, (n, d.max().item())
                close += int((d <= 1e-3 * lr).sum())
                total += d.numel()
        assert close >= 0.99 * total, (close, total)
        assert trainer.scheduler.get_last_lr()[0] == pytest.approx(sched.get_last_lr()[0], rel=1e-12)
    # frozen weights never move
    for n, p in model.state_dict().items():
        if n in frozen_before:
            assert torch.equal(p.cpu(), frozen_before[n]), n


def test_nonfinite_gradient_skips_the_update_on_the_device():
    from orthrus_training_b200.train_step import Trainer

    model, _ = _golden_model()
    trainer = Trainer(model, lr=1e-3, total_steps=10, num_anchors=4, kl_chunk_size=64, seed=5)
    batches = [(i.to(DEV), m.to(DEV)) for i, m in _micro_batches(50, 1)]
    trainer.step(batches, indices=[0])  # one normal step, so the optimizer has state
    before = {n: p.detach().clone() for n, p in model.named_parameters() if p.requires_grad}
    state_before = {n: {k: v.clone() for k, v in trainer.optimizer.state[p].items()}
                    for n, p in model.named_parameters() if p.requires_grad}
    lr_before = trainer.scheduler.get_last_lr()[0]
    victim = next(p for n, p in model.named_parameters() if n.endswith("q_proj_diff.weight"))
    handle = victim.register_hook(lambda grad: grad * float("nan"))
    out = trainer.step(batches, indices=[1])
    handle.remove()
    assert bool(out["skipped"]) and not math.isfinite(out["grad_norm"].item())
    assert int(trainer.skipped) == 1
    for n, p in model.named_parameters():
        if p.requires_grad:
            assert torch.equal(p.detach(), before[n]), n
            for k, v in trainer.optimizer.state[p].items():
                assert torch.equal(v, state_before[n][k]), (n, k)
    assert trainer.scheduler.get_last_lr()[0] != lr_before  # the schedule still advances
    out = trainer.step(batches, indices=[2])  # and training continues
    assert not bool(out["skipped"])
    assert any(not torch.equal(p.detach(), before[n]) for n, p in model.named_parameters() if p.requires_grad)


def test_resume_from_a_checkpoint_is_bit_exact(tmp_path):
    """bf16 tensor-core path: three steps straight, against one step, a checkpoint, a fresh model
    and trainer loaded from it, and two more steps; the twins are equal bit for bit."""
    from orthrus_training_b200.data_io import load_checkpoint, save_checkpoint
    from orthrus_training_b200.train_step import Trainer

    hp = dict(lr=1e-3, total_steps=10, warmup_ratio=0.2, num_anchors=8, kl_chunk_size=256, seed=9)
    steps = [[(i.to(DEV), m.to(DEV)) for i, m in _micro_batches(100 + 10 * s, 2)] for s in range(3)]

    def fresh():
        from test_gpu_model import _bf16_tiny

        model, _ = _bf16_tiny(seed=3)
        return model, Trainer(model, **hp)

    model_a, tr_a = fresh()
    for s in range(3):
        tr_a.step(steps[s])
    model_b, tr_b = fresh()
    tr_b.step(steps[0])
    save_checkpoint(tmp_path / "step-1", model_b, tr_b.optimizer, tr_b.scheduler,
                    {"step": tr_b.step_index})
    del model_b, tr_b
    model_c, tr_c = fresh()
    state = load_checkpoint(tmp_path / "step-1", model_c, tr_c.optimizer, tr_c.scheduler)
    tr_c.step_index = state["step"]
    for s in (1, 2):
        tr_c.step(steps[s])
    for (n, a), (_, c) in zip(model_a.named_parameters(), model_c.named_parameters()):
        assert torch.equal(a, c), n


def test_inputs_through_the_prefetcher_with_a_ready_event_step_identically():
    """Trainer.step(..., ready=event) lets the anchor draw and the supervised layout wait for the
    inputs' copy event alone (on a side stream, beside the teacher pass); it gives the same steps,
    bit for bit, as rows already on the device without an event."""
    from orthrus_training_b200.data_io import DevicePrefetcher
    from orthrus_training_b200.train_step import Trainer

    hp = dict(lr=1e-3, total_steps=10, warmup_ratio=0.2, num_anchors=8, kl_chunk_size=256, seed=4)
    host = _micro_batches(300, 3)

    def fresh():
        from test_gpu_model import _bf16_tiny

        model, _ = _bf16_tiny(seed=5)
        return model, Trainer(model, **hp)

    model_a, tr_a = fresh()
    losses_a = [tr_a.step([(i.to(DEV), m.to(DEV))])["loss"] for i, m in host]
    model_b, tr_b = fresh()
    feed = DevicePrefetcher(((j, i, m) for j, (i, m) in enumerate(host)), DEV)
    losses_b = [tr_b.step([(i, m)], ready=feed.ready)["loss"] for _, i, m in feed]
    assert torch.equal(torch.stack(losses_a), torch.stack(losses_b))
    for (n, a), (_, b) in zip(model_a.named_parameters(), model_b.named_parameters()):
        assert torch.equal(a, b), n
