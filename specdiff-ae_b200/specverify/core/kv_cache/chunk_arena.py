"""Chunk arena for the retrieval working set: the drop-in for
``diffspec.core.kv_cache.chunk_arena``.

Same configuration, arena layout ``[L, 2, 1, H, max_chunks * chunk, D]`` and
public methods as the reference (``chunk_arena.py:16-365``), with the same
slot bookkeeping (Python sets for the evict/add difference, slots taken from
the front of the free list, oldest-first eviction when full), so chunk-to-slot
mappings are identical.  The rows of every added chunk -- all layers, K and V,
all heads -- are copied by ONE ``tv_arena_gather`` launch instead of a
per-chunk, per-layer loop of slice copies (``chunk_arena.py:126-173``).

:func:`arena_page_table` is the zero-copy form for a paged cache: when chunk
boundaries are page-aligned the working set is just the chosen chunks' page
lists laid end to end, which the paged verify-attention kernel reads directly.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from ... import _lib


@dataclass
class ChunkArenaConfig:
    """Configuration for :class:`ChunkArena` (``chunk_arena.py:16-27``)."""
    max_chunks: int = 64
    chunk_size: int = 64
    num_layers: int = 32
    num_heads: int = 32
    head_dim: int = 128
    dtype: torch.dtype = torch.float16
    device: str = "cuda"
    enable_apw: bool = False
    apw_hit_ratio: float = 0.5


class ChunkArena:
    """Contiguous KV arena holding the active top-k chunks."""

    def __init__(self, config: ChunkArenaConfig):
        self.config = config
        self.max_chunks = config.max_chunks
        self.chunk_size = config.chunk_size
        self.num_layers = config.num_layers
        self.num_heads = config.num_heads
        self.head_dim = config.head_dim
        self.device = config.device
        self.dtype = config.dtype
        self.arena_kv = torch.zeros(config.num_layers, 2, 1, config.num_heads, config.max_chunks * config.chunk_size,
                                    config.head_dim, dtype=config.dtype, device=config.device)
        self.chunk_to_offset: Dict[int, int] = {}
        self.active_chunks: List[int] = []
        self.free_offsets: List[int] = list(range(config.max_chunks))
        self.total_updates = 0
        self.total_evictions = 0
        self.total_additions = 0
        self.hit_count = 0
        self.miss_count = 0
        self.enable_apw = config.enable_apw
        self.apw_hit_ratio = config.apw_hit_ratio
        self.apw_enabled_flag = False

    def update_arena(self, new_top_k_chunks: List[int],
                     full_kv_cache: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None) -> torch.Tensor:
        """Differential update; returns the active arena view ``[L, 2, 1, H, n*chunk, D]``."""
        self.total_updates += 1
        new_top_k_chunks = list(new_top_k_chunks)[: self.max_chunks]
        old_set, new_set = set(self.active_chunks), set(new_top_k_chunks)
        to_evict, to_add = old_set - new_set, new_set - old_set
        self.hit_count += len(old_set & new_set)
        self.miss_count += len(to_add)
        for c in to_evict:
            if c in self.chunk_to_offset:
                self.free_offsets.append(self.chunk_to_offset.pop(c))
                self.active_chunks.remove(c)
                self.total_evictions += 1
        if full_kv_cache is not None:
            copies = []
            for c in to_add:
                if not self.free_offsets:
                    if not self.active_chunks:
                        raise RuntimeError("Arena overflow and no chunks to evict")
                    oldest = self.active_chunks.pop(0)
                    self.free_offsets.append(self.chunk_to_offset.pop(oldest))
                slot = self.free_offsets.pop(0)
                self.chunk_to_offset[c] = slot
                self.active_chunks.append(c)
                self.total_additions += 1
                copies.append((c, slot))
            self._gather(copies, full_kv_cache)
        return self.arena_kv[:, :, :, :, : len(self.active_chunks) * self.chunk_size, :]

    def _gather(self, copies: List[Tuple[int, int]], full_kv_cache) -> None:
        """Copy the rows of every (chunk, slot) pair for all layers in one launch."""
        if not copies:
            return
        layers = min(self.num_layers, len(full_kv_cache))
        if layers == 0:
            return
        ks, vs = [], []
        for i in range(layers):
            k, v = full_kv_cache[i]
            k = k.unsqueeze(0) if k.dim() == 3 else k
            v = v.unsqueeze(0) if v.dim() == 3 else v
            if k.size(1) != self.num_heads:
                raise RuntimeError(f"ChunkArena head mismatch: arena_heads={self.num_heads}, "
                                   f"cache_heads={k.size(1)}")
            ks.append(k)
            vs.append(v)
        _lib.require_cuda(self.arena_kv, *ks, *vs)
        ref = ks[0]
        src_len = ref.shape[2]
        for t in ks + vs:
            if (t.stride(1), t.stride(2), t.stride(3), t.shape[2], t.dtype) != \
                    (ref.stride(1), ref.stride(2), 1, src_len, self.dtype):
                raise _lib.SpecVerifyError(-3, "all layers' K/V must share [1, H, S, D] strides, length and the "
                                               "arena dtype")
        dev = self.arena_kv.device
        kp = torch.tensor([t.data_ptr() for t in ks], dtype=torch.int64).to(dev, non_blocking=True)
        vp = torch.tensor([t.data_ptr() for t in vs], dtype=torch.int64).to(dev, non_blocking=True)
        cp = torch.tensor(copies, dtype=torch.int32).to(dev, non_blocking=True)
        a = self.arena_kv
        es = a.element_size()
        st = _lib.load().tv_arena_gather(
            layers, self.num_heads, kp.data_ptr(), vp.data_ptr(), ref.stride(1) * es, ref.stride(2) * es, src_len,
            a.data_ptr(), a.stride(0) * es, a.stride(1) * es, a.stride(3) * es, self.head_dim * es,
            self.chunk_size, a.shape[4], cp.data_ptr(), len(copies), _lib.stream_ptr(dev))
        _lib.check(st, "tv_arena_gather")

    def get_chunk_kv(self, chunk_id: int, layer_idx: int):
        if chunk_id not in self.chunk_to_offset:
            return None
        s = self.chunk_to_offset[chunk_id] * self.chunk_size
        return (self.arena_kv[layer_idx, 0, :, :, s:s + self.chunk_size, :],
                self.arena_kv[layer_idx, 1, :, :, s:s + self.chunk_size, :])

    def get_working_cache(self) -> torch.Tensor:
        return self.arena_kv[:, :, :, :, : len(self.active_chunks) * self.chunk_size, :]

    def get_chunk_mapping(self) -> Dict[int, int]:
        return self.chunk_to_offset.copy()

    def enable_l2_residency(self, stream=None):
        """APW hook kept for API compatibility; marks the flag like the reference
        (``chunk_arena.py:216-257``).  No L2 persistence window is configured."""
        if not self.enable_apw:
            return
        self.apw_enabled_flag = True
        warnings.warn("APW residency hint recorded; no L2 access-policy window is applied.", RuntimeWarning,
                      stacklevel=2)

    def disable_l2_residency(self, stream=None):
        self.apw_enabled_flag = False

    def get_statistics(self) -> Dict:
        total = self.hit_count + self.miss_count
        return {
            "total_updates": self.total_updates,
            "total_evictions": self.total_evictions,
            "total_additions": self.total_additions,
            "hit_count": self.hit_count,
            "miss_count": self.miss_count,
            "hit_rate": self.hit_count / total if total > 0 else 0.0,
            "active_chunks": len(self.active_chunks),
            "max_chunks": self.max_chunks,
            "utilization": len(self.active_chunks) / self.max_chunks,
            "arena_size_mb": self.arena_kv.numel() * self.arena_kv.element_size() / (1024 ** 2),
            "apw_enabled": self.apw_enabled_flag,
        }

    def reset(self):
        self.chunk_to_offset.clear()
        self.active_chunks.clear()
        self.free_offsets = list(range(self.max_chunks))
        self.arena_kv.zero_()

    def compact(self):
        """Active chunks to slots ``0..n-1`` in active order (``chunk_arena.py:298-321``)."""
        if not self.active_chunks:
            return
        cs = self.chunk_size
        new = torch.zeros_like(self.arena_kv)
        old_rows = torch.cat([torch.arange(self.chunk_to_offset[c] * cs, (self.chunk_to_offset[c] + 1) * cs)
                              for c in self.active_chunks]).to(self.arena_kv.device)
        n = len(self.active_chunks) * cs
        new[:, :, :, :, :n] = self.arena_kv.index_select(4, old_rows)
        self.arena_kv = new
        self.chunk_to_offset = {c: i for i, c in enumerate(self.active_chunks)}
        self.free_offsets = list(range(len(self.active_chunks), self.max_chunks))


class ChunkArenaWithAPW(ChunkArena):
    """Variant reserved for an L2 access-policy-window extension (``chunk_arena.py:324-365``)."""

    def __init__(self, config: ChunkArenaConfig):
        super().__init__(config)
        self.apw_stream = None

    def set_l2_cache_policy(self, hit_ratio: float = 0.5, persisting_size_mb: Optional[float] = None):
        if not self.enable_apw:
            return
        self.apw_hit_ratio = hit_ratio


def arena_page_table(page_table: torch.Tensor, chunk_ids: torch.Tensor, pages_per_chunk: int) -> torch.Tensor:
    """Zero-copy working set: ``out[i*ppc + j] = page_table[chunk_ids[i]*ppc + j]``.

    page_table int32 [pages] of one sequence; chunk_ids int32 [n] (device).
    The result is that sequence's arena as a page table for
    :func:`specverify.runtime.tree_attention.attention`.
    """
    _lib.require_cuda(page_table, chunk_ids)
    pt = page_table.to(torch.int32).contiguous()
    ids = chunk_ids.to(torch.int32).contiguous()
    out = torch.empty(ids.numel() * pages_per_chunk, dtype=torch.int32, device=pt.device)
    st = _lib.load().tv_gather_page_table(pt.data_ptr(), pt.numel(), ids.data_ptr(), ids.numel(), pages_per_chunk,
                                          out.data_ptr(), _lib.stream_ptr(pt.device))
    _lib.check(st, "tv_gather_page_table")
    return out
