"""Seeded synthetic packed rows with the shapes and value distributions of the workloads.

The reference trains on a private generated dataset; these rows stand in for it with its shape:
packed rows of documents, each a prompt followed by an assistant response, with the assistant
mask covering the response (orthrus/data.py:43-69 packs documents back to back with no document
mask). Ids are drawn from a bounded Zipf law or uniformly, always below the mask token.
"""

from __future__ import annotations

import numpy as np
import torch


def zipf_ids(rng: np.random.Generator, count: int, vocab: int, s: float = 1.1) -> np.ndarray:
    """Ids in [0, vocab) with P(id = k-1) proportional to k^-s (a Zipf law truncated to vocab)."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    cdf = np.cumsum(ranks ** (-s))
    cdf /= cdf[-1]
    return np.searchsorted(cdf, rng.random(count), side="right").clip(0, vocab - 1)


def packed_rows(
    rows: int,
    seq_len: int,
    real_vocab: int,
    seed: int,
    *,
    ids: str = "zipf",
    doc: str = "prompt_response",
) -> tuple[torch.Tensor, torch.Tensor]:
    """(input_ids int64 [rows, seq_len], assistant_mask bool [rows, seq_len]).

    doc="prompt_response": documents of a prompt of U[250, 350] tokens plus a response of
    Geometric(mean 690) tokens capped at seq_len (the production row construction).
    doc="short": documents of U[40, 120] tokens, the first 30% prompt, the rest response (the
    tiny CPU plumbing workload).
    ids="zipf": Zipf(1.1) ids; ids="uniform": uniform ids. All ids are < real_vocab.
    """
    rng = np.random.default_rng(seed)
    input_ids = np.zeros((rows, seq_len), dtype=np.int64)
    mask = np.zeros((rows, seq_len), dtype=bool)
    for r in range(rows):
        pos = 0
        while pos < seq_len:
            if doc == "prompt_response":
                prompt = int(rng.integers(250, 351))
                response = min(int(rng.geometric(1.0 / 690.0)), seq_len)
            else:
                length = int(rng.integers(40, 121))
                prompt = int(length * 0.3)
                response = length - prompt
            end_prompt = min(pos + prompt, seq_len)
            end = min(end_prompt + response, seq_len)
            mask[r, end_prompt:end] = True
            pos = end
        if ids == "zipf":
            input_ids[r] = zipf_ids(rng, seq_len, real_vocab)
        else:
            input_ids[r] = rng.integers(0, real_vocab, seq_len)
    return torch.from_numpy(input_ids), torch.from_numpy(mask)


def qwen3_06b_config(block_size: int = 32, mask_token_id: int = 151669):
    """The Qwen3-0.6B architecture (28 layers, d 1024, 16 query / 8 KV heads of 128, MLP 3072,
    vocabulary 151936 tied) with the Orthrus block size and mask token, for random-init runs."""
    from transformers import Qwen3Config

    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                      num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      rope_theta=1e6, tie_word_embeddings=True)
    cfg.rope_parameters = {"rope_theta": 1e6, "rope_type": "default"}
    cfg.block_size = block_size
    cfg.mask_token_id = mask_token_id
    return cfg
