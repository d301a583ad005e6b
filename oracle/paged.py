"""Oracle: paged KV page tables, copy-on-write and paged compaction (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates the bookkeeping of ``PagedKVCache`` in
``diffspec/core/kv_cache/paged_kv.py``:

* pool layout ``[L, 2, P, H, page, D]`` (``:53-65``), free pages kept in a
  Python ``set`` and handed out by ``set.pop()`` (``:68``, ``:101``, ``:200``,
  ``:211``), page reference counts (``:71``);
* ``allocate`` (``:81-108``), ``fork`` (``:110-142``, prefix pages shared,
  ref count incremented), ``free`` (``:310-323``);
* ``write_row`` (``:168-223``): a missing logical page gets a fresh page; a
  shared page (ref count > 1) is copied whole -- every layer, K and V -- into
  a fresh page before the write (copy-on-write);
* ``read_row`` (``:225-253``): a missing logical page reads as zeros;
* ``physical_blocks`` (``:325-340``).

``compact_path`` applies verification compaction through that API: the rows
at logical positions ``start + path[j]`` are gathered first, then written to
``start + j`` one by one with ``write_row`` (so copy-on-write fires on the
first write into each shared destination page, in row order).
"""

from __future__ import annotations

import numpy as np


class PagedOracle:
    def __init__(self, num_layers, num_heads, head_dim, page_size, max_pages, dtype=np.float32,
                 enable_cow=True):
        self.L, self.H, self.D = num_layers, num_heads, head_dim
        self.page_size = page_size
        self.max_pages = max_pages
        self.enable_cow = enable_cow
        self.pool = np.zeros((num_layers, 2, max_pages, num_heads, page_size, head_dim), dtype=dtype)
        self.free_pages = set(range(max_pages))
        self.ref = np.zeros(max_pages, dtype=np.int32)
        self.tables = {}

    def allocate(self, seq, num_tokens):
        n = (num_tokens + self.page_size - 1) // self.page_size
        if len(self.free_pages) < n:
            raise RuntimeError("Out of memory")
        t = {}
        for i in range(n):
            p = self.free_pages.pop()
            t[i] = p
            self.ref[p] = 1
        self.tables[seq] = t
        return t

    def fork(self, parent, child, shared_prefix_len):
        pt = self.tables[parent]
        ct = {}
        for i in range(shared_prefix_len // self.page_size):
            if i in pt:
                ct[i] = pt[i]
                self.ref[pt[i]] += 1
        self.tables[child] = ct

    def free(self, seq):
        if seq not in self.tables:
            return
        for p in self.tables[seq].values():
            self.ref[p] -= 1
            if self.ref[p] == 0:
                self.free_pages.add(p)
        del self.tables[seq]

    def _page_for_write(self, seq, lp):
        t = self.tables[seq]
        if lp not in t:
            if not self.free_pages:
                raise RuntimeError("Out of memory")
            p = self.free_pages.pop()
            t[lp] = p
            self.ref[p] = 1
            return p
        p = t[lp]
        if self.enable_cow and self.ref[p] > 1:
            if not self.free_pages:
                raise RuntimeError("Out of memory")
            q = self.free_pages.pop()
            self.pool[:, :, q] = self.pool[:, :, p]
            self.ref[p] -= 1
            self.ref[q] = 1
            t[lp] = q
            return q
        return p

    def write_row(self, seq, layer, token, k, v):
        p = self._page_for_write(seq, token // self.page_size)
        off = token % self.page_size
        self.pool[layer, 0, p, :, off, :] = k
        self.pool[layer, 1, p, :, off, :] = v

    def read_row(self, seq, layer, token):
        t = self.tables[seq]
        lp, off = token // self.page_size, token % self.page_size
        if lp not in t:
            z = np.zeros((self.H, self.D), dtype=self.pool.dtype)
            return z, z.copy()
        p = t[lp]
        return self.pool[layer, 0, p, :, off, :].copy(), self.pool[layer, 1, p, :, off, :].copy()

    def physical_blocks(self, seq):
        t = self.tables.get(seq, {})
        if not t:
            return []
        return [t.get(i, -1) for i in range(max(t) + 1)]

    def compact_path(self, seq, start, path):
        rows = [[self.read_row(seq, layer, start + int(s)) for layer in range(self.L)] for s in path]
        for j, per_layer in enumerate(rows):
            for layer, (k, v) in enumerate(per_layer):
                self.write_row(seq, layer, start + j, k, v)
        return start + len(path)
