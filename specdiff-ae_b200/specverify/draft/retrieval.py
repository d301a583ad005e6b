"""Draft-side chunk retrieval on the device: the drop-in for the retrieval
branch of ``DraftNetwork._select_working_cache_from_chunks``
(``draft/draft_network.py:1514-1612``).

The reference scores the chunks from the last verify's per-token attention
(prefix sums), keeps the ``top_k`` chunks, forms the union of their token
intervals (difference array + cumsum + ``nonzero``) and gathers those token
rows of every layer's full draft K / V into the working cache -- with host
round trips for ``.any()``, ``.tolist()`` and ``nonzero``.  Here
``tv_chunk_select`` does the selection and the union in one launch and
``tv_gather_rows`` copies the rows of all layers' K and V in one more; the
only host read is the number of retrieved tokens (the working cache's
length).  The optional semantic penalty (``gamma_sem``) is not applied.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from .. import _lib


def select_chunks(attn: torch.Tensor, starts: torch.Tensor, ends: torch.Tensor, top_k: int, length: int,
                  *, validate: bool = True) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (selected chunk ids [k] ascending, token indices buffer
    [length] of which the first ``count`` are the union's tokens, count [1]
    int64) -- all on the device, nothing read back."""
    dev = _lib.require_cuda(attn, starts, ends)
    a = attn.reshape(-1).to(torch.float32).contiguous()
    s = starts.to(torch.int64).contiguous().view(-1)
    e = ends.to(torch.int64).contiguous().view(-1)
    n = s.numel()
    if e.numel() != n:
        raise _lib.SpecVerifyError(-1, "starts and ends differ in length")
    k = min(int(top_k), n)
    sel = torch.empty(k, dtype=torch.int64, device=dev)
    idx = torch.empty(max(int(length), 1), dtype=torch.int64, device=dev)
    count = torch.zeros(1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.tv_chunk_select_workspace_size(n, a.numel(), ctypes.byref(need)), "tv_chunk_select_workspace_size")
    ws = torch.empty(max(int(need.value), 16), dtype=torch.uint8, device=dev)
    rc = lib.tv_chunk_select(a.data_ptr(), a.numel(), s.data_ptr(), e.data_ptr(), n, k, int(length), sel.data_ptr(),
                             idx.data_ptr(), idx.numel(), count.data_ptr(), ws.data_ptr(), ws.numel(),
                             _lib.ptr(status), ctypes.c_void_p(_lib.stream_ptr(dev)))
    _lib.check(rc, "tv_chunk_select")
    if status is not None and int(status.item()) != 0:
        raise _lib.SpecVerifyError(int(status.item()), "tv_chunk_select: negative chunk bound")
    return sel, idx, count


class GatherPlan:
    """Outputs and device pointer tables for :func:`gather_rows`, made once per
    (full cache, working length); a plan's gather allocates nothing and can
    be captured in a CUDA graph."""

    def __init__(self, full_kv: Sequence[Tuple[torch.Tensor, torch.Tensor]], rows: int):
        k0 = full_kv[0][0]
        dev = _lib.require_cuda(k0)
        b, h, _, d = k0.shape
        for (fk, fv) in full_kv:
            for t in (fk, fv):
                if t.shape[:2] != (b, h) or t.shape[3] != d or t.dtype != k0.dtype:
                    raise _lib.SpecVerifyError(-1, "all layers' K / V must share [B, H, *, D] and dtype")
                if not t.is_contiguous():
                    raise _lib.SpecVerifyError(-3, "full K / V must be contiguous [B, H, L, D]")
        self.full_kv = list(full_kv)
        self.rows = int(rows)
        self.outputs = [(torch.empty(b, h, rows, d, dtype=k0.dtype, device=dev),
                         torch.empty(b, h, rows, d, dtype=k0.dtype, device=dev)) for _ in full_kv]
        self.src = torch.tensor([t.data_ptr() for pair in full_kv for t in pair], dtype=torch.int64, device=dev)
        self.dst = torch.tensor([t.data_ptr() for pair in self.outputs for t in pair], dtype=torch.int64, device=dev)
        es = k0.element_size()
        self.args = (2 * len(full_kv), b * h, k0.stride(1) * es, k0.stride(2) * es, rows * d * es, d * es, d * es)
        self.device = dev


def gather_rows(plan: GatherPlan, indices: torch.Tensor, count: torch.Tensor) -> List[Tuple[torch.Tensor, torch.Tensor]]:
    """Working cache: for every layer, K[:, :, indices[:rows], :] and the same
    for V into the plan's [B, H, rows, D] outputs (one launch); returns them."""
    planes, heads, shs, srs, dhs, drs, row_bytes = plan.args
    _lib.require_cuda(indices, count)
    lib = _lib.load()
    rc = lib.tv_gather_rows(planes, heads, plan.src.data_ptr(), plan.dst.data_ptr(), shs, srs, dhs, drs, row_bytes,
                            indices.data_ptr(), count.data_ptr(), plan.rows,
                            ctypes.c_void_p(_lib.stream_ptr(plan.device)))
    _lib.check(rc, "tv_gather_rows")
    return plan.outputs


def select_working_cache(full_kv: Sequence[Tuple[torch.Tensor, torch.Tensor]], attn: torch.Tensor,
                         starts: torch.Tensor, ends: torch.Tensor, top_k: int, total_seq_len: int):
    """The retrieval branch end to end: returns (working_kv, selected chunk
    ids as a list, evicted token count), as the reference leaves them in
    ``draft_stable_kv``, ``prev_selected_chunk_ids`` and ``evicted``."""
    sel, idx, count = select_chunks(attn, starts, ends, top_k, total_seq_len)
    n = int(count.item())                       # the working cache's length: the one host read
    working = gather_rows(GatherPlan(full_kv, n), idx, count) if full_kv and n > 0 else []
    return working, sel.tolist(), int(total_seq_len) - n
