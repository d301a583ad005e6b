"""Draft-side chunk retrieval, CPU restatement (numpy).

TEST INFRASTRUCTURE ONLY: the checker for ``tv_chunk_select`` and
``tv_gather_rows``; nothing in the product imports it.

Follows ``DraftNetwork._select_working_cache_from_chunks`` in retrieval mode
(``draft/draft_network.py:1514-1612``) with no semantic penalty
(``gamma_sem`` = 0):

* chunk score = (prefix sum of the per-token attention up to ``end - 1``
  minus the prefix sum up to ``start - 1``) / max(end - start, 1), prefix
  indices clamped to the scored length;
* the ``top_k`` best scores (``torch.topk``: larger first, NaN counts as the
  largest; among equal scores the smaller chunk id here), then sorted by id;
* the union of the selected ``[start, end)`` token intervals (clamped to
  [0, L]), as ascending token indices;
* the working K / V of every layer: ``index_select`` of those token rows.

Sums are taken in float64 and rounded to float32: for the exact (dyadic)
scores of the golden fixtures this equals the reference's float32 prefix
sums bit for bit.
"""

from __future__ import annotations

import numpy as np


def chunk_scores(attn, starts, ends):
    a = np.asarray(attn, dtype=np.float64)
    la = a.size
    s = np.asarray(starts, dtype=np.int64)
    e = np.asarray(ends, dtype=np.int64)
    cum = np.cumsum(a)
    lower = np.where(s > 0, cum[np.clip(s - 1, 0, la - 1)], 0.0)
    upper = cum[np.clip(e - 1, 0, la - 1)]
    sums = (upper - lower).astype(np.float32)
    lengths = np.maximum(e - s, 1).astype(np.float32)
    return sums / lengths


def top_k_sorted(scores, k):
    x = np.asarray(scores, dtype=np.float32)
    n = x.size
    k = min(int(k), n)
    key = np.where(np.isnan(x), np.inf, x)
    nan = np.isnan(x)
    # larger first; NaN before everything; ties: smaller id first
    order = sorted(range(n), key=lambda i: (0 if nan[i] else 1, -key[i] if not nan[i] else 0.0, i))
    return np.sort(np.array(order[:k], dtype=np.int64))


def union_indices(starts, ends, selected, length):
    s = np.clip(np.asarray(starts, dtype=np.int64)[selected], 0, length)
    e = np.clip(np.asarray(ends, dtype=np.int64)[selected], 0, length)
    diff = np.zeros(length + 1, dtype=np.int64)
    np.add.at(diff, s, 1)
    np.add.at(diff, e, -1)
    return np.flatnonzero(np.cumsum(diff[:length]) > 0).astype(np.int64)


def select(attn, starts, ends, top_k, length):
    scores = chunk_scores(attn, starts, ends)
    sel = top_k_sorted(scores, top_k)
    return sel, union_indices(starts, ends, sel, length)


def gather(full, idx):
    """``index_select`` along the token axis (2) of [B, H, L, D]."""
    return np.asarray(full)[:, :, np.asarray(idx, dtype=np.int64), :]
