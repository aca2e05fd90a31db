"""Device-resident KV cache of the AR view, the stand-in for transformers' DynamicCache in the
reference's decode loop (orthrus/modeling_orthrus.py:428,459,489-527).

Per layer one preallocated [B, Hkv, capacity, D] key buffer and one value buffer, written in place
by the q/k prologue kernel at row offset = committed length. Truncation (the rollback after a
rejected draft) only moves the committed length: rows past it are dead and are overwritten by the
next verification pass, so no data moves and no host synchronisation is needed.
"""

from __future__ import annotations

import torch


class _LayerView:
    def __init__(self, cache: "KVCache", layer: int):
        self._cache, self._layer = cache, layer

    @property
    def keys(self) -> torch.Tensor:
        c = self._cache
        return c.k[self._layer][:, :, : c.length, : c.head_dim]

    @property
    def values(self) -> torch.Tensor:
        c = self._cache
        return c.v[self._layer][:, :, : c.length, : c.head_dim]


class KVCache:
    def __init__(self, config, batch: int = 1, capacity: int | None = None, device=None,
                 dtype=torch.bfloat16):
        from orthrus_training_b200.modeling_orthrus import padded_head_dim

        self.config = config
        self.batch = batch
        self.head_dim = config.head_dim
        self.D = padded_head_dim(config.head_dim)
        self.capacity = capacity or 1024
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.dtype = dtype
        n = config.num_hidden_layers
        shape = (batch, config.num_key_value_heads, self.capacity, self.D)
        self.k = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(n)]
        self.v = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(n)]
        self.length = 0
        self._offsets = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self._offsets_len = 0

    # DynamicCache-compatible surface ---------------------------------------------------------
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.length

    def crop(self, max_length: int) -> None:
        """Keep the first max_length positions (negative: drop that many from the end)."""
        self.length = self.length + max_length if max_length < 0 else min(self.length, max_length)

    @property
    def layers(self) -> list[_LayerView]:
        return [_LayerView(self, i) for i in range(len(self.k))]

    # kernel-facing helpers --------------------------------------------------------------------
    def reserve(self, total: int) -> None:
        """Grow every buffer to hold `total` positions (copying the committed rows)."""
        if total <= self.capacity:
            return
        cap = max(total, 2 * self.capacity)
        for lst in (self.k, self.v):
            for i, t in enumerate(lst):
                new = torch.zeros(t.shape[0], t.shape[1], cap, t.shape[3], dtype=t.dtype,
                                  device=t.device)
                new[:, :, : self.capacity] = t
                lst[i] = new
        self.capacity = cap

    def buffers(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        return list(zip(self.k, self.v))

    def keys(self, layer: int) -> torch.Tensor:
        return self.k[layer]

    def values(self, layer: int) -> torch.Tensor:
        return self.v[layer]

    def offsets(self, batch: int) -> torch.Tensor:
        """int32 [batch] committed length per sequence (all equal in the single-length API)."""
        if batch != self.batch:
            raise ValueError(f"cache built for batch {self.batch}, got {batch}")
        if self._offsets_len != self.length:
            self._offsets.fill_(self.length)
            self._offsets_len = self.length
        return self._offsets
