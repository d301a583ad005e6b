"""Paged KV cache with copy-on-write: the drop-in for
``diffspec.core.kv_cache.paged_kv``.

Same configuration, pool layout ``[L, 2, P, H, page, D]`` and public methods
as the reference (``paged_kv.py:15-402``).  The page allocator keeps the
reference's exact policy -- free pages in a Python ``set`` handed out by
``set.pop()``, reference counts, copy-on-write on the first write to a shared
page -- so page tables come out identical for the same operation sequence.
What changes is where the bytes move:

* whole-page copies (copy-on-write, ``copy_sequence``) run as one
  ``tv_copy_pages`` launch over every layer and K/V plane;
* :meth:`compact_path` (new) moves the accepted path of a verified tree to its
  final positions -- copy-on-write planned on the host, then one
  ``tv_copy_pages`` + one ``tv_compact_paged`` launch for all layers and
  heads, instead of a per-token, per-layer Python loop;
* :meth:`page_table_tensor` (new) hands the verify-attention kernels a device
  page table, so attention reads the pool directly (the reference's paged
  verifier raises NotImplementedError, ``bundle_verifier.py:341-366``).

Per-token ``write_kv`` / ``read_kv`` stay as tensor indexing (caller glue).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from ... import _lib


@dataclass
class PagedKVConfig:
    """Configuration for :class:`PagedKVCache` (``paged_kv.py:15-25``)."""
    page_size: int = 16
    max_pages: int = 1024
    num_layers: int = 32
    num_heads: int = 32
    head_dim: int = 128
    dtype: torch.dtype = torch.float16
    device: str = "cuda"
    enable_cow: bool = True


class PagedKVCache:
    """Paged KV cache manager with copy-on-write sharing."""

    def __init__(self, config: PagedKVConfig):
        self.config = config
        self.page_size = config.page_size
        self.max_pages = config.max_pages
        self.num_layers = config.num_layers
        self.num_heads = config.num_heads
        self.head_dim = config.head_dim
        self.device = config.device
        self.dtype = config.dtype
        if str(self.device).startswith("cpu") and self.dtype == torch.float16:
            self.dtype = torch.float32
            self.config.dtype = self.dtype
        self.enable_cow = config.enable_cow
        self.page_pool = torch.zeros(config.num_layers, 2, config.max_pages, config.num_heads, config.page_size,
                                     config.head_dim, dtype=self.dtype, device=config.device)
        self.free_pages = set(range(config.max_pages))
        self.page_ref_count = torch.zeros(config.max_pages, dtype=torch.int32, device="cpu")
        self.page_tables: Dict[int, Dict[int, int]] = {}
        self.total_allocated = 0
        self.total_freed = 0
        self.cow_saves = 0

    # ---- allocator (reference policy) ------------------------------------
    def _pop_free(self) -> int:
        if not self.free_pages:
            raise RuntimeError("Out of memory")
        return self.free_pages.pop()

    def allocate_sequence(self, seq_id: int, num_tokens: int) -> Dict[int, int]:
        n = (num_tokens + self.page_size - 1) // self.page_size
        if len(self.free_pages) < n:
            raise RuntimeError(f"Out of memory: need {n} pages, only {len(self.free_pages)} available")
        table = {}
        for lp in range(n):
            p = self.free_pages.pop()
            table[lp] = p
            self.page_ref_count[p] = 1
            self.total_allocated += 1
        self.page_tables[seq_id] = table
        return table

    def fork_sequence(self, parent_seq_id: int, child_seq_id: int, shared_prefix_len: int):
        if not self.enable_cow:
            self.copy_sequence(parent_seq_id, child_seq_id)
            return
        if parent_seq_id not in self.page_tables:
            raise ValueError(f"Parent sequence {parent_seq_id} not found")
        pt = self.page_tables[parent_seq_id]
        ct = {}
        for lp in range(shared_prefix_len // self.page_size):
            if lp in pt:
                ct[lp] = pt[lp]
                self.page_ref_count[pt[lp]] += 1
                self.cow_saves += 1
        self.page_tables[child_seq_id] = ct

    def copy_sequence(self, src_seq_id: int, dst_seq_id: int):
        if src_seq_id not in self.page_tables:
            raise ValueError(f"Source sequence {src_seq_id} not found")
        pairs = []
        dst = {}
        for lp, sp in self.page_tables[src_seq_id].items():
            if not self.free_pages:
                raise RuntimeError("Out of memory")
            dp = self.free_pages.pop()
            dst[lp] = dp
            self.page_ref_count[dp] = 1
            pairs.append((sp, dp))
            self.total_allocated += 1
        self.copy_pages(pairs)
        self.page_tables[dst_seq_id] = dst

    def _page_for_write(self, table: Dict[int, int], lp: int, cow_pairs: List[Tuple[int, int]]) -> int:
        """Reference ``write_kv`` page policy (``paged_kv.py:197-220``); a
        needed copy is appended to ``cow_pairs`` instead of done inline."""
        if lp not in table:
            p = self._pop_free()
            table[lp] = p
            self.page_ref_count[p] = 1
            self.total_allocated += 1
            return p
        p = table[lp]
        if self.enable_cow and self.page_ref_count[p] > 1:
            q = self._pop_free()
            cow_pairs.append((p, q))
            self.page_ref_count[p] -= 1
            self.page_ref_count[q] = 1
            table[lp] = q
            self.total_allocated += 1
            return q
        return p

    # ---- device copies ----------------------------------------------------
    def copy_pages(self, pairs: List[Tuple[int, int]]) -> None:
        """Copy whole pages (every layer, K and V, head) src -> dst.

        A CUDA pool copies with one ``tv_copy_pages`` launch.  A CPU pool
        (the reference also allows ``device="cpu"`` for bookkeeping-only use)
        copies with tensor indexing.
        """
        if not pairs:
            return
        pool = self.page_pool
        if not pool.is_cuda:
            for s, d in pairs:
                pool[:, :, d] = pool[:, :, s]
            return
        es = pool.element_size()
        pt = torch.tensor(pairs, dtype=torch.int32).to(pool.device, non_blocking=True)
        planes = self.num_layers * 2
        plane_stride = pool.stride(1) * es
        page_stride = pool.stride(2) * es
        page_bytes = pool.stride(2) * es
        st = _lib.load().tv_copy_pages(pool.data_ptr(), planes, plane_stride, page_stride, page_bytes,
                                       pt.data_ptr(), len(pairs), self.max_pages, _lib.stream_ptr(pool.device))
        _lib.check(st, "tv_copy_pages")

    # ---- per-token access (reference API) ----------------------------------
    def write_kv(self, seq_id: int, layer_idx: int, token_idx: int, k: torch.Tensor, v: torch.Tensor):
        if seq_id not in self.page_tables:
            raise ValueError(f"Sequence {seq_id} not allocated")
        if k.shape[0] != self.num_heads or k.shape[1] != self.head_dim:
            raise RuntimeError(f"PagedKV k/v shape mismatch: expected ({self.num_heads}, {self.head_dim}), "
                               f"got {tuple(k.shape)}")
        cow: List[Tuple[int, int]] = []
        p = self._page_for_write(self.page_tables[seq_id], token_idx // self.page_size, cow)
        self.copy_pages(cow)
        off = token_idx % self.page_size
        self.page_pool[layer_idx, 0, p, :, off, :] = k
        self.page_pool[layer_idx, 1, p, :, off, :] = v

    def write_tokens(self, seq_id: int, layer_idx: int, token_start: int, k: torch.Tensor, v: torch.Tensor):
        """Write ``n`` consecutive tokens ``k/v [H, n, D]`` starting at ``token_start``."""
        n = k.shape[1]
        t = token_start
        while t < token_start + n:
            lp, off = t // self.page_size, t % self.page_size
            take = min(self.page_size - off, token_start + n - t)
            cow: List[Tuple[int, int]] = []
            p = self._page_for_write(self.page_tables[seq_id], lp, cow)
            if cow:
                self.copy_pages(cow)
            a = t - token_start
            self.page_pool[layer_idx, 0, p, :, off:off + take, :] = k[:, a:a + take]
            self.page_pool[layer_idx, 1, p, :, off:off + take, :] = v[:, a:a + take]
            t += take

    def read_kv(self, seq_id: int, layer_idx: int, token_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if seq_id not in self.page_tables:
            raise ValueError(f"Sequence {seq_id} not allocated")
        table = self.page_tables[seq_id]
        lp, off = token_idx // self.page_size, token_idx % self.page_size
        if lp not in table:
            z = torch.zeros(self.num_heads, self.head_dim, device=self.device, dtype=self.dtype)
            return z, z.clone()
        p = table[lp]
        return self.page_pool[layer_idx, 0, p, :, off, :], self.page_pool[layer_idx, 1, p, :, off, :]

    def get_contiguous_kv(self, seq_id: int, layer_idx: int, start_token: int = 0,
                          end_token: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """``[H, end - start, D]`` copies of a token window (missing pages read as 0)."""
        if seq_id not in self.page_tables:
            raise ValueError(f"Sequence {seq_id} not allocated")
        table = self.page_tables[seq_id]
        if end_token is None:
            end_token = (max(table.keys()) + 1) * self.page_size
        tok = torch.arange(start_token, end_token)
        lp = tok // self.page_size
        phys = torch.tensor([table.get(int(x), -1) for x in range(int(lp.min()) if len(lp) else 0,
                                                                  int(lp.max()) + 1 if len(lp) else 0)],
                            dtype=torch.long)
        k_out = torch.zeros(self.num_heads, len(tok), self.head_dim, device=self.device, dtype=self.dtype)
        v_out = torch.zeros_like(k_out)
        if len(tok):
            pp = phys[lp - lp.min()]
            ok = pp >= 0
            if bool(ok.any()):
                sel_p = pp[ok].to(self.page_pool.device)
                sel_o = (tok % self.page_size)[ok].to(self.page_pool.device)
                idx = torch.nonzero(ok).view(-1).to(self.page_pool.device)
                k_out[:, idx] = self.page_pool[layer_idx, 0, sel_p, :, sel_o, :].transpose(0, 1)
                v_out[:, idx] = self.page_pool[layer_idx, 1, sel_p, :, sel_o, :].transpose(0, 1)
        return k_out, v_out

    def free_sequence(self, seq_id: int):
        if seq_id not in self.page_tables:
            return
        for p in self.page_tables[seq_id].values():
            self.page_ref_count[p] -= 1
            if self.page_ref_count[p] == 0:
                self.free_pages.add(p)
                self.total_freed += 1
        del self.page_tables[seq_id]

    def get_physical_blocks(self, seq_id: int) -> List[int]:
        if seq_id not in self.page_tables:
            return []
        table = self.page_tables[seq_id]
        top = max(table.keys()) if table else -1
        return [table.get(i, -1) for i in range(top + 1)]

    def page_table_tensor(self, seq_id: int, length: Optional[int] = None, device=None) -> torch.Tensor:
        """Device int32 page table ``[length]`` (missing pages = -1)."""
        blocks = self.get_physical_blocks(seq_id)
        if length is not None:
            blocks = (blocks + [-1] * length)[:length]
        return torch.tensor(blocks, dtype=torch.int32).to(device or self.page_pool.device, non_blocking=True)

    def layer_kv(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Paged K / V pool views ``[P, H, page, D]`` of one layer for the kernels."""
        return self.page_pool[layer_idx, 0], self.page_pool[layer_idx, 1]

    def get_statistics(self) -> Dict:
        used = self.max_pages - len(self.free_pages)
        return {
            "total_pages": self.max_pages,
            "used_pages": used,
            "free_pages": len(self.free_pages),
            "utilization": used / self.max_pages,
            "total_allocated": self.total_allocated,
            "total_freed": self.total_freed,
            "cow_saves": self.cow_saves,
            "shared_pages": int((self.page_ref_count > 1).sum().item()),
            "num_sequences": len(self.page_tables),
            "memory_mb": self.page_pool.numel() * self.page_pool.element_size() / (1024 ** 2),
        }

    def defragment(self):
        """Move live pages to the low end of the pool (``paged_kv.py:364-402``)."""
        used = sorted({p for t in self.page_tables.values() for p in t.values()})
        if not used or used[-1] - used[0] + 1 == len(used):
            return
        remap = {old: new for new, old in enumerate(used) if new != old}
        if not remap:
            return
        old_idx = torch.tensor(list(remap.keys()), device=self.page_pool.device)
        new_idx = torch.tensor(list(remap.values()), device=self.page_pool.device)
        self.page_pool[:, :, new_idx] = self.page_pool[:, :, old_idx]   # gather first, then scatter
        for t in self.page_tables.values():
            for lp, p in t.items():
                if p in remap:
                    t[lp] = remap[p]
        ref = torch.zeros_like(self.page_ref_count)
        for old, new in remap.items():
            ref[new] = self.page_ref_count[old]
        for p in used:
            if p not in remap:
                ref[p] = self.page_ref_count[p]
        self.page_ref_count = ref
        self.free_pages = set(range(self.max_pages)) - {p for t in self.page_tables.values() for p in t.values()}

    # ---- verification compaction ------------------------------------------
    def compact_path(self, seq_id: int, start: int, acc, path: Optional[List[int]] = None) -> int:
        """Move logical rows ``start + path[j]`` to ``start + j`` for every layer.

        ``acc`` is the :class:`~specverify.draft.tree_verification.AcceptResult`
        of the verified tree (its device buffer drives the row moves); ``path``
        is its host copy (read back once if not given).  Copy-on-write follows
        the reference's ``write_kv`` order: the first written row of a shared
        destination page copies that page into a fresh one.  Returns the new
        sequence length ``start + n``.
        """
        if seq_id not in self.page_tables:
            raise ValueError(f"Sequence {seq_id} not allocated")
        if path is None:
            path = acc.to_host()["path"]
        table = self.page_tables[seq_id]
        length = max(max(table.keys()) + 1 if table else 0, (start + len(path)) // self.page_size + 1,
                     (start + max(path)) // self.page_size + 1 if path else 0)
        src = self.page_table_tensor(seq_id, length)
        cow: List[Tuple[int, int]] = []
        for j in range(len(path)):
            self._page_for_write(table, (start + j) // self.page_size, cow)
        self.copy_pages(cow)
        dst = self.page_table_tensor(seq_id, length)
        pool = self.page_pool
        es = pool.element_size()
        st = _lib.load().tv_compact_paged(
            pool.data_ptr(), self.num_layers * 2, self.num_heads, pool.stride(1) * es, pool.stride(2) * es,
            pool.stride(3) * es, pool.stride(4) * es, self.head_dim * es, self.page_size, src.data_ptr(),
            dst.data_ptr(), length, self.max_pages, int(start), acc.result.data_ptr(), max(len(path), 1),
            _lib.stream_ptr(pool.device))
        _lib.check(st, "tv_compact_paged")
        return start + len(path)
