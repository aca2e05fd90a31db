"""The on-disk formats on either side of the training step, in the reference's layout.

- Packed rows (orthrus/data.py:72-86): ``input_ids.npy`` (int32 [rows, seq_len]) and
  ``assistant_mask.npy`` (uint8, same shape) in one directory, the mask written last so that its
  presence marks a complete set; read memory-mapped.
- Micro-batch order (orthrus/data.py:89-103): one permutation of the rows per (seed, epoch) from
  ``numpy.random.default_rng([seed, epoch])``, cut into consecutive micro-batches, each sorted by
  row id (sequential reads of the memory map), resumable at a micro-batch index. Restated with the
  same generator calls so that a run resumed here sees the rows the reference would have fed.
- Training checkpoints (orthrus/checkpoint.py:27,68-97): a directory holding
  ``trainable.safetensors`` (the diffusion twins under their parameter names),
  ``optimizer.pt`` (optimizer and scheduler state) and ``trainer_state.json``, built in a hidden
  staging directory and swapped in once complete. Checkpoints move between the reference and this
  package unchanged, since the file names and parameter names are the same.

- Model export (orthrus/checkpoint.py:98-105): a Hugging Face model directory with the bf16
  weights (``model.safetensors``, the reference's parameter names, the tied ``lm_head.weight``
  left out), ``config.json`` (the Qwen3 config plus ``block_size`` / ``mask_token_id`` and the
  ``auto_map`` entry to ``modeling_orthrus.OrthrusLM``) and the tokenizer files.

``DevicePrefetcher`` is this package's loader side: it copies each micro-batch into pinned host
buffers and on to the GPU on a copy stream, one micro-batch ahead of the step that consumes it.
"""

from __future__ import annotations

import json
import os
import shutil
from pathlib import Path
from typing import Iterator

import numpy as np
import torch

IDS_FILE, MASK_FILE = "input_ids.npy", "assistant_mask.npy"
WEIGHTS, OPTIMIZER, STATE = "trainable.safetensors", "optimizer.pt", "trainer_state.json"


def save_packed(directory: Path, ids: np.ndarray, mask: np.ndarray) -> None:
    """Writes packed rows; the mask goes last, so its presence marks a complete directory."""
    if ids.shape != mask.shape or ids.ndim != 2:
        raise ValueError(f"ids {ids.shape} and mask {mask.shape} must be the same [rows, seq_len]")
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    np.save(directory / IDS_FILE, ids.astype(np.int32, copy=False))
    np.save(directory / MASK_FILE, mask.astype(np.uint8, copy=False))


def load_packed(directory: Path) -> tuple[np.ndarray, np.ndarray]:
    """Memory-mapped (input_ids int32, assistant_mask uint8) of a packed directory."""
    directory = Path(directory)
    if not (directory / MASK_FILE).exists():
        raise FileNotFoundError(f"{directory} holds no complete packed rows ({MASK_FILE} missing)")
    ids = np.load(directory / IDS_FILE, mmap_mode="r")
    mask = np.load(directory / MASK_FILE, mmap_mode="r")
    if ids.shape != mask.shape or ids.ndim != 2:
        raise ValueError(f"{directory}: ids {ids.shape} and mask {mask.shape} do not match")
    if ids.dtype != np.int32 or mask.dtype != np.uint8:
        raise ValueError(f"{directory}: expected int32 ids and uint8 mask, got {ids.dtype} / {mask.dtype}")
    return ids, mask


def batch_rows(num_rows: int, batch_size: int, seed: int, epoch: int, start: int = 0) -> Iterator[tuple[int, np.ndarray]]:
    """(micro-batch index, sorted row ids) of one epoch from micro-batch ``start`` on."""
    order = np.random.default_rng([seed, epoch]).permutation(num_rows)
    for index in range(start, len(order) // batch_size):
        yield index, np.sort(order[index * batch_size: (index + 1) * batch_size])


def batches(ids: np.ndarray, mask: np.ndarray, batch_size: int, seed: int, epoch: int,
            start: int = 0) -> Iterator[tuple[int, torch.Tensor, torch.Tensor]]:
    """(index, input_ids int64 [batch, seq_len], assistant_mask bool) micro-batches on the host."""
    for index, rows in batch_rows(len(ids), batch_size, seed, epoch, start):
        yield (index, torch.from_numpy(ids[rows].astype(np.int64)),
               torch.from_numpy(mask[rows].astype(np.bool_)))


class DevicePrefetcher:
    """Feeds host micro-batches to one GPU: each is copied into pinned buffers and sent with a
    non-blocking copy on a dedicated stream, one micro-batch ahead. Iterating yields
    (index, ids, mask) already on the device; the consumer's stream waits for the copy, and
    `ready` is the copy's event (Trainer.step(..., ready=...) lets its side stream wait for that
    event alone rather than for everything the consumer's stream has queued)."""

    def __init__(self, host_batches: Iterator[tuple[int, torch.Tensor, torch.Tensor]], device):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DevicePrefetcher feeds a CUDA device")
        self.source = iter(host_batches)
        self.stream = torch.cuda.Stream(self.device)
        self.pending = None
        self.ready = None
        self._issue()

    def _issue(self) -> None:
        item = next(self.source, None)
        if item is None:
            self.pending = None
            return
        index, ids, mask = item
        ids_pin, mask_pin = ids.pin_memory(), mask.pin_memory()
        with torch.cuda.stream(self.stream):
            ids_dev = ids_pin.to(self.device, non_blocking=True)
            mask_dev = mask_pin.to(self.device, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.stream)
        self.pending = (index, ids_dev, mask_dev, done, ids_pin, mask_pin)

    def __iter__(self):
        return self

    def __next__(self):
        if self.pending is None:
            raise StopIteration
        index, ids_dev, mask_dev, done, _, _ = self.pending
        consumer = torch.cuda.current_stream(self.device)
        consumer.wait_event(done)
        ids_dev.record_stream(consumer)
        mask_dev.record_stream(consumer)
        self.ready = done
        self._issue()
        return index, ids_dev, mask_dev


def _trainable(model) -> dict[str, torch.nn.Parameter]:
    return {name: p for name, p in model.named_parameters() if p.requires_grad}


def _publish(staging: Path, path: Path) -> None:
    """Swaps a completed staging directory in at `path`. An older checkpoint there is first moved
    aside and deleted only after the new one is in place, so at every instant `path` is either the
    old complete checkpoint or the new one."""
    retired = None
    if path.exists():
        retired = path.with_name(f".{path.name}.retired-{os.getpid()}")
        shutil.rmtree(retired, ignore_errors=True)
        os.replace(path, retired)
    os.replace(staging, path)
    if retired is not None:
        shutil.rmtree(retired, ignore_errors=True)


def save_checkpoint(path: Path, model, optimizer, scheduler, state: dict) -> None:
    """Writes the trainable twins (safetensors, under their parameter names), the optimizer and
    scheduler state and the progress dict as the reference's checkpoint directory. The files are
    built in a hidden staging directory beside `path` (a name the reference's ``step-*`` listing
    never matches) and flushed to disk before the directory is swapped in."""
    import tempfile

    from safetensors.torch import save_file

    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{path.name}.staging-", dir=path.parent))
    try:
        tensors = {name: p.detach().contiguous() for name, p in _trainable(model).items()}
        save_file(tensors, staging / WEIGHTS)
        torch.save({"optimizer": optimizer.state_dict(), "scheduler": scheduler.state_dict()},
                   staging / OPTIMIZER)
        (staging / STATE).write_text(json.dumps(state, indent=2), encoding="utf-8")
        for name in (WEIGHTS, OPTIMIZER, STATE):
            with open(staging / name, "rb") as f:
                os.fsync(f.fileno())
        _publish(staging, path)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise


def load_checkpoint(path: Path, model, optimizer=None, scheduler=None) -> dict:
    """Loads a checkpoint directory into the model's trainable twins (the stored names must be
    exactly those parameters, with their shapes) and, when given, the optimizer and scheduler.
    Returns the stored progress dict."""
    from safetensors import safe_open

    path = Path(path)
    params = _trainable(model)
    device = next(model.parameters()).device
    with safe_open(str(path / WEIGHTS), framework="pt", device=str(device)) as stored:
        names = set(stored.keys())
        missing, unexpected = sorted(set(params) - names), sorted(names - set(params))
        if missing or unexpected:
            raise RuntimeError(f"{path}: the stored tensors are not the model's trainable parameters "
                               f"(missing {missing[:3]}{'...' if len(missing) > 3 else ''}, "
                               f"unexpected {unexpected[:3]}{'...' if len(unexpected) > 3 else ''})")
        with torch.no_grad():
            for name, param in params.items():
                value = stored.get_tensor(name)
                if value.shape != param.shape:
                    raise RuntimeError(f"{path}: {name} is stored as {tuple(value.shape)}, the model "
                                       f"has {tuple(param.shape)}")
                param.copy_(value)
    if optimizer is not None:
        blob = torch.load(path / OPTIMIZER, map_location=device, weights_only=False)
        optimizer.load_state_dict(blob["optimizer"])
        if scheduler is not None:
            scheduler.load_state_dict(blob["scheduler"])
    return json.loads((path / STATE).read_text(encoding="utf-8"))


def export_model(model, tokenizer, out_dir: Path, modeling_file: Path | None = None) -> None:
    """Writes the model as a Hugging Face directory in the reference's export format. The
    reference also copies its own modeling_orthrus.py beside the weights (the ``auto_map``
    target); pass that file as ``modeling_file`` to do the same."""
    from safetensors.torch import save_file

    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    cfg = model.config
    state = {k: v.detach().to(torch.bfloat16).contiguous().cpu() for k, v in model.state_dict().items()}
    head, embed = model.state_dict().get("lm_head.weight"), model.state_dict().get("model.embed_tokens.weight")
    if getattr(cfg, "tie_word_embeddings", False) and head is not None and embed is not None \
            and head.data_ptr() == embed.data_ptr():
        state.pop("lm_head.weight")  # tied: restored from the embedding on load
    save_file(state, out_dir / "model.safetensors", metadata={"format": "pt"})
    config = cfg.to_dict()
    config["auto_map"] = {"AutoModelForCausalLM": "modeling_orthrus.OrthrusLM"}
    config["torch_dtype"] = "bfloat16"
    for key in ("block_size", "mask_token_id"):
        config[key] = getattr(cfg, key)
    (out_dir / "config.json").write_text(json.dumps(config, indent=2, sort_keys=True), encoding="utf-8")
    if tokenizer is not None:
        tokenizer.save_pretrained(out_dir)
    if modeling_file is not None:
        shutil.copy(modeling_file, out_dir / "modeling_orthrus.py")

