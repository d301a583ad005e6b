"""Oracle: chunk-arena differential update (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``ChunkArena.update_arena`` and ``ChunkArena.compact`` from
``diffspec/core/kv_cache/chunk_arena.py``:

* arena layout ``[L, 2, 1, H, max_chunks * chunk_size, D]`` (``:51-62``);
* ``update`` (``:86-178``): truncate the request to ``max_chunks``; evict
  ``old - new`` (iterating the Python set), returning offsets to the end of the
  free list; add ``new - old`` (iterating the Python set), taking
  ``free.pop(0)`` (evicting the oldest active chunk when no slot is free),
  and copying each added chunk's rows ``[c * cs, min((c + 1) * cs, S))`` from
  every layer's K and V; return the first ``len(active) * cs`` arena rows;
* ``compact`` (``:298-321``): move active chunks, in active order, to slots
  ``0..n-1`` (untouched slots become zero).
"""

from __future__ import annotations

import numpy as np


class ArenaOracle:
    def __init__(self, max_chunks, chunk_size, num_layers, num_heads, head_dim, dtype=np.float32):
        self.max_chunks, self.cs = max_chunks, chunk_size
        self.L, self.H, self.D = num_layers, num_heads, head_dim
        self.arena = np.zeros((num_layers, 2, 1, num_heads, max_chunks * chunk_size, head_dim), dtype=dtype)
        self.chunk_to_offset = {}
        self.active = []
        self.free = list(range(max_chunks))
        self.copies = []  # (chunk_id, offset) in the order rows were copied

    def update(self, new_top_k, full_kv=None):
        new_top_k = list(new_top_k)[: self.max_chunks]
        old_set, new_set = set(self.active), set(new_top_k)
        for c in old_set - new_set:
            if c in self.chunk_to_offset:
                self.free.append(self.chunk_to_offset.pop(c))
                self.active.remove(c)
        self.copies = []
        if full_kv is not None:
            for c in new_set - old_set:
                if not self.free:
                    if not self.active:
                        raise RuntimeError("Arena overflow and no chunks to evict")
                    oldest = self.active.pop(0)
                    self.free.append(self.chunk_to_offset.pop(oldest))
                off = self.free.pop(0)
                self.chunk_to_offset[c] = off
                self.active.append(c)
                self.copies.append((c, off))
                s0, s1 = c * self.cs, (c + 1) * self.cs
                for layer in range(min(self.L, len(full_kv))):
                    k, v = full_kv[layer]           # [1, H, S, D]
                    e = min(s1, k.shape[2])
                    n = e - s0
                    if n > 0:
                        self.arena[layer, 0, :, :, off * self.cs: off * self.cs + n] = k[:, :, s0:e]
                        self.arena[layer, 1, :, :, off * self.cs: off * self.cs + n] = v[:, :, s0:e]
        return self.arena[:, :, :, :, : len(self.active) * self.cs]

    def compact(self):
        if not self.active:
            return
        new = np.zeros_like(self.arena)
        mapping = {}
        for new_off, c in enumerate(self.active):
            old = self.chunk_to_offset[c]
            mapping[c] = new_off
            new[..., new_off * self.cs:(new_off + 1) * self.cs, :] = self.arena[..., old * self.cs:(old + 1) * self.cs, :]
        self.arena = new
        self.chunk_to_offset = mapping
        self.free = list(range(len(self.active), self.max_chunks))
