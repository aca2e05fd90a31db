"""Device-resident KV cache of the AR view, with the surface of transformers' DynamicCache that the
reference's modules and decode loop use (orthrus/modeling_orthrus.py:107-111,162-166,257-259,
428-527): ``DynamicCache(config=...)``, ``get_seq_length``, ``update``, ``crop`` and
``layers[i].keys / .values``.

Per layer one preallocated [B, Hkv, capacity, D] key buffer and one value buffer, written in place
by the q/k prologue kernel at row offset = that layer's committed length. Truncation (the rollback
after a rejected draft) only moves the committed lengths: rows past them are dead and are
overwritten by the next verification pass, so no data moves and no host synchronisation is needed.

Like DynamicCache, a cache built from a config alone allocates on its first write, taking the
batch, dtype and device of that write. Each layer keeps its own length, so a model forward that
calls the layers one by one (each appending its keys) and the fused decoder loop (which appends to
every layer at once) leave the cache in the same state.
"""

from __future__ import annotations

import torch


class _LayerView:
    """layers[i] of a DynamicCache: the committed keys / values of one layer, [B, Hkv, len, hd]."""

    def __init__(self, cache: "KVCache", layer: int):
        self._cache, self._layer = cache, layer

    @property
    def keys(self) -> torch.Tensor:
        c = self._cache
        return c.k[self._layer][:, :, : c.lengths[self._layer], : c.head_dim]

    @property
    def values(self) -> torch.Tensor:
        c = self._cache
        return c.v[self._layer][:, :, : c.lengths[self._layer], : c.head_dim]


class KVCache:
    def __init__(self, config, batch: int | None = None, capacity: int | None = None, device=None,
                 dtype=None):
        from orthrus_training_b200.modeling_orthrus import padded_head_dim

        self.config = config
        self.head_dim = config.head_dim
        self.D = padded_head_dim(config.head_dim)
        self.num_layers = config.num_hidden_layers
        self.capacity = capacity or 1024
        self.lengths = [0] * self.num_layers
        self.k: list[torch.Tensor] = []
        self.v: list[torch.Tensor] = []
        self.batch = None
        self._offsets = None
        self._offsets_len = -1
        if batch is not None:
            self.allocate(batch, dtype or torch.bfloat16, device if device is not None else "cuda")

    # allocation -------------------------------------------------------------------------------
    @property
    def allocated(self) -> bool:
        return bool(self.k)

    def allocate(self, batch: int, dtype: torch.dtype, device) -> None:
        """Creates the buffers (once): [batch, Hkv, capacity, D] per layer for keys and values."""
        if self.allocated:
            if batch != self.batch:
                raise ValueError(f"cache holds batch {self.batch}, got {batch}")
            if dtype != self.dtype:
                raise ValueError(f"cache holds {self.dtype}, got {dtype}")
            return
        self.batch, self.dtype, self.device = batch, dtype, torch.device(device)
        shape = (batch, self.config.num_key_value_heads, self.capacity, self.D)
        self.k = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(self.num_layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(self.num_layers)]
        self._offsets = torch.zeros(batch, dtype=torch.int32, device=self.device)

    # DynamicCache-compatible surface ---------------------------------------------------------
    @property
    def length(self) -> int:
        """Committed positions (of layer 0, which every forward writes first)."""
        return self.lengths[0]

    @length.setter
    def length(self, value: int) -> None:
        self.lengths = [int(value)] * self.num_layers

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.lengths[layer_idx]

    def crop(self, max_length: int) -> None:
        """Keeps the first max_length positions of every layer; a negative value counts back from
        the committed length of layer 0, as DynamicCache.crop does."""
        if max_length < 0:
            max_length = max(0, self.lengths[0] + max_length)
        self.lengths = [min(n, max_length) for n in self.lengths]

    @property
    def layers(self) -> list[_LayerView]:
        return [_LayerView(self, i) for i in range(self.num_layers)]

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: dict | None = None):
        """Appends [B, Hkv, T, hd] keys and values to layer `layer_idx` and returns that layer's
        committed keys and values (DynamicCache.update)."""
        B, H, T, hd = key_states.shape
        if hd != self.head_dim or H != self.config.num_key_value_heads:
            raise ValueError(f"cache of {self.config.num_key_value_heads} heads of {self.head_dim}, "
                             f"got {H} of {hd}")
        self.allocate(B, key_states.dtype, key_states.device)
        n = self.lengths[layer_idx]
        self.reserve(n + T)
        self.k[layer_idx][:, :, n: n + T, :hd] = key_states
        self.v[layer_idx][:, :, n: n + T, :hd] = value_states
        self.lengths[layer_idx] = n + T
        view = self.layers[layer_idx]
        return view.keys, view.values

    # kernel-facing helpers --------------------------------------------------------------------
    def reserve(self, total: int) -> None:
        """Grows every buffer to hold `total` positions (copying the committed rows)."""
        if total <= self.capacity:
            return
        cap = max(total, 2 * self.capacity)
        if self.allocated:
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

    def offsets(self, batch: int, layer: int = 0) -> torch.Tensor:
        """int32 [batch] committed length of `layer` per sequence (all sequences share it)."""
        if batch != self.batch:
            raise ValueError(f"cache built for batch {self.batch}, got {batch}")
        n = self.lengths[layer]
        if self._offsets_len != n:
            self._offsets.fill_(n)
            self._offsets_len = n
        return self._offsets
