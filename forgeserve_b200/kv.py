"""Contiguous KV cache (the reference's ContiguousKV, forgeserve/kv.py:10-33).

Same view protocol — `length`, `update(k, v) -> (k_all, v_all)`, `truncate(n)`, and `.k` / `.v` holding every
key and value so far as (B, n_kv, S, head_dim) — but stored as device buffers with spare capacity, so a decode
step writes one slot instead of re-copying the whole cache with torch.cat (kv.py:22-23). The decoder layers
do not call `update`: the RoPE kernel writes the new keys/values straight into the buffer (slots
length .. length + T - 1) and attention reads them there.
"""

from typing import Dict, Optional, Tuple

import torch

_ROW_TABLES: Dict[Tuple[str, int], torch.Tensor] = {}


def row_table(batch: int, device: torch.device) -> torch.Tensor:
    """[0, 1, ..., batch-1] as int64 on `device` (the block table of a per-row cache)."""
    key = (str(device), batch)
    t = _ROW_TABLES.get(key)
    if t is None:
        t = torch.arange(max(batch, 1), dtype=torch.int64, device=device)
        _ROW_TABLES[key] = t
    return t


class ContiguousKV:
    """Per-layer cache for rows that all have the same length."""

    def __init__(self, max_len: Optional[int] = None):
        self._k: Optional[torch.Tensor] = None   # (B, n_kv, capacity, head_dim)
        self._v: Optional[torch.Tensor] = None
        self._len = 0
        self.max_len = max_len                   # growth never allocates more slots than this (when needed fits)

    @property
    def k(self) -> Optional[torch.Tensor]:
        return None if self._k is None else self._k[:, :, : self._len]

    @property
    def v(self) -> Optional[torch.Tensor]:
        return None if self._v is None else self._v[:, :, : self._len]

    @property
    def length(self) -> int:
        return self._len

    @property
    def capacity(self) -> int:
        return 0 if self._k is None else self._k.shape[2]

    def reserve(self, batch: int, n_kv: int, head_dim: int, t_new: int, dtype: torch.dtype,
                device: torch.device) -> int:
        """Make room for t_new more slots; returns the first new slot (the current length)."""
        need = self._len + t_new
        if self._k is not None:
            b, h, cap, d = self._k.shape
            if (b, h, d) != (batch, n_kv, head_dim) or self._k.dtype != dtype or self._k.device != torch.device(device):
                raise ValueError(f"cache holds ({b}, {h}, *, {d}) {self._k.dtype} on {self._k.device}; "
                                 f"got ({batch}, {n_kv}, *, {head_dim}) {dtype} on {device}")
            if need <= cap:
                return self._len
            new_cap = max(need, 2 * cap)
        else:
            new_cap = need
        if self.max_len is not None and need <= self.max_len:
            new_cap = min(new_cap, self.max_len)
        new_cap = -(-new_cap // 16) * 16     # whole 16-slot chunks: the tensor-core attention reads the cache in those
        k = torch.empty(batch, n_kv, new_cap, head_dim, dtype=dtype, device=device)
        v = torch.empty_like(k)
        if self._len:
            k[:, :, : self._len].copy_(self._k[:, :, : self._len])
            v[:, :, : self._len].copy_(self._v[:, :, : self._len])
        self._k, self._v = k, v
        return self._len

    def commit(self, t_new: int) -> None:
        self._len += t_new

    def buffers(self) -> Tuple[torch.Tensor, torch.Tensor]:
        return self._k, self._v

    def update(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append k, v of shape (B, n_kv, T, head_dim); return all keys and values so far."""
        b, h, t, d = k.shape
        start = self.reserve(b, h, d, t, k.dtype, k.device)
        self._k[:, :, start : start + t].copy_(k)
        self._v[:, :, start : start + t].copy_(v)
        self.commit(t)
        return self.k, self.v

    def truncate(self, n: int) -> None:
        """Keep only the first n positions."""
        self._len = max(0, min(n, self._len))


def new_contiguous_cache(n_layers: int, max_len: Optional[int] = None):
    return [ContiguousKV(max_len) for _ in range(n_layers)]
