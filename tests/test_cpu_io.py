"""The on-disk formats (packed rows, micro-batch order, twin checkpoints) on the host."""

import json

import numpy as np
import pytest
import torch

from conftest import load_golden


def test_batches_follow_the_reference_order():
    """The reference's own micro-batch order (orthrus/data.py:89-103) for three (seed, epoch,
    start) cases: the same rows, in the same batches, in the same order."""
    from orthrus_training_b200.data_io import batches

    g = load_golden("data_batches.pt")
    ids, mask = g["ids"].numpy(), g["mask"].numpy()
    for case in g["cases"]:
        got = list(batches(ids, mask, case["batch_size"], case["seed"], case["epoch"], case["start"]))
        assert [i for i, _, _ in got] == case["index"]
        for (_, x, m), rx, rm in zip(got, case["ids"], case["mask"]):
            assert x.dtype == torch.int64 and m.dtype == torch.bool
            assert torch.equal(x, rx) and torch.equal(m, rm)


def test_packed_rows_round_trip(tmp_path):
    from orthrus_training_b200.data_io import IDS_FILE, MASK_FILE, load_packed, save_packed

    rng = np.random.default_rng(0)
    ids = rng.integers(0, 151669, size=(6, 32))
    mask = rng.random((6, 32)) < 0.7
    save_packed(tmp_path, ids, mask)
    assert (tmp_path / IDS_FILE).exists() and (tmp_path / MASK_FILE).exists()
    got_ids, got_mask = load_packed(tmp_path)
    assert got_ids.dtype == np.int32 and got_mask.dtype == np.uint8
    assert isinstance(got_ids, np.memmap)
    assert np.array_equal(got_ids, ids) and np.array_equal(got_mask, mask.astype(np.uint8))


def test_incomplete_packed_directory_is_refused(tmp_path):
    from orthrus_training_b200.data_io import IDS_FILE, load_packed

    np.save(tmp_path / IDS_FILE, np.zeros((2, 8), dtype=np.int32))  # the mask was never written
    with pytest.raises(FileNotFoundError):
        load_packed(tmp_path)


def _tiny_model():
    from transformers import Qwen3Config

    from orthrus_training_b200.modeling_orthrus import OrthrusLM, copy_diff_from_ar, freeze_to_diffusion

    cfg = Qwen3Config(vocab_size=96, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=8, tie_word_embeddings=True,
                      max_position_embeddings=256)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size, cfg.mask_token_id = 4, 95
    model = OrthrusLM(cfg)
    copy_diff_from_ar(model)
    return model, freeze_to_diffusion(model)


def test_checkpoint_round_trip(tmp_path):
    """Twin weights, optimizer / scheduler state and progress survive a save and a load into a
    fresh model; the files and tensor names are the reference's (trainable.safetensors holds only
    the *_diff.* parameters)."""
    from safetensors.torch import load_file

    from orthrus_training_b200.data_io import OPTIMIZER, STATE, WEIGHTS, load_checkpoint, save_checkpoint

    torch.manual_seed(0)
    model, params = _tiny_model()
    opt = torch.optim.AdamW(params, lr=1e-3)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: 1.0 / (1 + s))
    for p in params:
        p.grad = torch.randn_like(p)
    opt.step()
    sched.step()
    path = tmp_path / "step-1"
    save_checkpoint(path, model, opt, sched, {"step": 1, "epoch": 0})
    assert sorted(x.name for x in path.iterdir()) == sorted([WEIGHTS, OPTIMIZER, STATE])
    names = set(load_file(path / WEIGHTS))
    assert names and all("_diff." in n for n in names)
    assert json.loads((path / STATE).read_text())["step"] == 1

    torch.manual_seed(1)
    fresh, fparams = _tiny_model()
    fopt = torch.optim.AdamW(fparams, lr=1e-3)
    fsched = torch.optim.lr_scheduler.LambdaLR(fopt, lambda s: 1.0 / (1 + s))
    state = load_checkpoint(path, fresh, fopt, fsched)
    assert state == {"step": 1, "epoch": 0}
    ref = dict(model.named_parameters())
    for n, p in fresh.named_parameters():
        if p.requires_grad:
            assert torch.equal(p, ref[n]), n
    assert fsched.state_dict()["last_epoch"] == sched.state_dict()["last_epoch"]
    assert torch.equal(fopt.state_dict()["state"][0]["exp_avg"], opt.state_dict()["state"][0]["exp_avg"])


def test_checkpoint_of_another_model_is_refused(tmp_path):
    from orthrus_training_b200.data_io import load_checkpoint, save_checkpoint

    model, params = _tiny_model()
    opt = torch.optim.AdamW(params)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: 1.0)
    save_checkpoint(tmp_path / "c", model, opt, sched, {})
    other, _ = _tiny_model()
    for p in other.parameters():
        p.requires_grad_(True)  # a different trainable set
    with pytest.raises(RuntimeError):
        load_checkpoint(tmp_path / "c", other)


def test_export_writes_an_hf_directory(tmp_path):
    """bf16 weights under the reference's names (tied head left out), config with the Orthrus
    fields and auto_map; the weights load back into a fresh model."""
    from safetensors.torch import load_file

    from orthrus_training_b200.data_io import export_model

    torch.manual_seed(0)
    model, _ = _tiny_model()
    modeling = tmp_path / "src.py"
    modeling.write_text("# modeling file\n")
    export_model(model, None, tmp_path / "out", modeling_file=modeling)
    out = tmp_path / "out"
    cfg = json.loads((out / "config.json").read_text())
    assert cfg["auto_map"] == {"AutoModelForCausalLM": "modeling_orthrus.OrthrusLM"}
    assert cfg["block_size"] == 4 and cfg["mask_token_id"] == 95 and cfg["tie_word_embeddings"]
    assert (out / "modeling_orthrus.py").read_text() == "# modeling file\n"
    weights = load_file(out / "model.safetensors")
    assert "lm_head.weight" not in weights and all(v.dtype == torch.bfloat16 for v in weights.values())
    names = set(dict(model.named_parameters())) - {"lm_head.weight"}
    assert names <= set(weights)
    torch.manual_seed(1)
    fresh, _ = _tiny_model()
    missing, unexpected = fresh.load_state_dict({k: v.float() for k, v in weights.items()}, strict=False)
    assert not unexpected and set(missing) <= {"lm_head.weight"}
    for n, p in fresh.named_parameters():
        assert torch.equal(p, dict(model.named_parameters())[n].bfloat16().float()), n

