"""Oracle: tree acceptance, path trace and contiguous KV compaction (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``verify_new`` from ``diffspec/draft/tree_verification.py``:

* step 1, ``:100-106``  -- one target token per node: ``argmax`` over the
  vocabulary (greedy), or one multinomial draw per node from
  ``softmax(processed logits)`` (sample-and-match; the draw itself is an
  input here so both sides see the same samples);
* step 2, ``:110-162``  -- ``ok[i] = draft[i] == next[parent(i)]``,
  ``ok[0] = True``, the synchronous closure ``ok &= ok[parent]`` for at most
  ``min(max_depth + 2, M)`` rounds (stopping early at a fixpoint), then
  ``max_id = argmax(where(ok, pos, 0))`` (first maximum);
* ``:164-182``          -- root-to-``max_id`` path, ``next_token``,
  ``accept_length``;
* step 3, ``:197-217``  -- gather the path's KV rows and write them to
  ``[start, start + n)`` in every per-device buffer, ``start =
  current_length - M``; ``current_length = start + n``.

Integer results here are the bit-exact bar for the GPU acceptance and
compaction kernels.
"""

from __future__ import annotations

import numpy as np


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """First-maximum argmax per row; a NaN counts as the maximum (first NaN wins).

    Matches ``torch.argmax`` on the reference's bf16/fp16 logits (pinned by
    the golden vectors), ``tree_verification.py:102``.
    """
    x = np.asarray(logits, dtype=np.float32)
    out = np.empty(x.shape[0], dtype=np.int64)
    for i in range(x.shape[0]):
        row = x[i]
        nan = np.flatnonzero(np.isnan(row))
        out[i] = int(nan[0]) if nan.size else int(np.argmax(row))
    return out


def parent_ext(parent: np.ndarray, m: int) -> np.ndarray:
    """[M-1] draft parents (-1 = child of the root) -> [M] parents over all rows.

    ``tree_verification.py:120-125``: a parent equal to its own row index is
    treated as -1, then the root is prepended and every index shifted by one;
    row 0 (the root) points at itself.
    """
    p = np.asarray(parent, dtype=np.int64).reshape(-1)
    if p.size != m - 1:
        raise ValueError(f"parent has {p.size} entries, expected {m - 1}")
    rows = np.arange(p.size, dtype=np.int64)
    p = np.where(p == rows, -1, p)
    ext = np.concatenate([np.zeros(1, dtype=np.int64), p + 1])
    if ext.size and (ext.min() < 0 or ext.max() >= m):
        raise IndexError("parent index out of range")
    return ext


def accept_from_next(next_tokens, draft, parent, pos, max_depth):
    """Acceptance given the per-node target tokens (greedy or sampled).

    Returns a dict with ``ok`` (bool [M]), ``max_id``, ``path`` (list of node
    ids root..max_id), ``best_candidate`` (draft tokens on the path),
    ``accept_length`` and ``next_token``.
    ``tree_verification.py:110-182``.
    """
    nxt = np.asarray(next_tokens, dtype=np.int64).reshape(-1)
    d = np.asarray(draft, dtype=np.int64).reshape(-1)
    ps = np.asarray(pos, dtype=np.int64).reshape(-1)
    m = d.size
    ext = parent_ext(parent, m)
    ok = d == nxt[ext]
    ok[0] = True
    for _ in range(min(int(max_depth) + 2, m)):
        new_ok = ok & ok[ext]
        if np.array_equal(new_ok, ok):
            break
        ok = new_ok
    masked = np.where(ok, ps, 0)
    max_id = int(np.argmax(masked))
    back = ext.copy()
    back[0] = -1
    path = []
    cur = max_id
    while cur != -1:
        path.append(cur)
        if len(path) > m:
            raise RuntimeError("parent pointers form a cycle")
        cur = int(back[cur])
    path.reverse()
    return {
        "ok": ok,
        "max_id": max_id,
        "path": path,
        "best_candidate": [int(d[i]) for i in path],
        "accept_length": len(path) - 1,
        "next_token": int(nxt[max_id]),
    }


def accept_greedy(logits, draft, parent, pos, max_depth):
    """Greedy acceptance: ``next = argmax(logits)`` then :func:`accept_from_next`."""
    nxt = argmax_rows(logits)
    res = accept_from_next(nxt, draft, parent, pos, max_depth)
    res["next_tokens"] = nxt
    return res


def compact_contiguous(buffers, current_length: int, m: int, path):
    """Compact the accepted path's KV rows in every buffer (in place).

    buffers: list of numpy arrays ``[..., S_budget, D]``; row ``start +
    path[j]`` moves to ``start + j`` with gather-then-write semantics.
    Returns the new cache length.  ``tree_verification.py:197-217``.
    """
    start = int(current_length) - int(m)
    sel = np.asarray(path, dtype=np.int64) + start
    for data in buffers:
        tgt = data[..., sel, :].copy()
        data[..., start:start + tgt.shape[-2], :] = tgt
    return start + len(path)
