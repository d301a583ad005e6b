"""Final draft-tree build, CPU restatement (numpy).

TEST INFRASTRUCTURE ONLY: the checker for ``tv_tree_finalize``; nothing in the
product imports it.

Follows ``DraftTree.update``'s final branch and ``generate_attention_mask``
(``runtime/draft_tree.py:188-260``), then the root row / column the verify
step prepends (``draft/diffspec_model.py:620-624``,
``draft/tree_verification.py:244-255``):

* the running top-k linear indices ``depth * nnodes + col`` are ordered by
  depth (``torch.argsort``; the order among equal depths is whatever that
  sort returned -- ``order`` reproduces a given one, the default keeps the
  top-k order, which is what the device build does);
* a node's final position goes into a [depth, nnodes] table, and its parent
  position is the table entry of (depth - 1, parents_matrix[depth, col]), or
  -1 for depth 0, a missing parent or a parent that did not make the top-k;
* the mask row of a node holds itself and its ancestors along the parent
  positions (at most depth - 1 hops);
* the verify mask prepends a root row that sees only itself and a root
  column every node sees.
"""

from __future__ import annotations

import numpy as np


def finalize(top_index, parents_matrix, input_ids_matrix, depth: int, nnodes: int, order=None):
    top = np.asarray(top_index, dtype=np.int64).reshape(-1)
    k = top.size
    rows = top // nnodes
    cols = top % nnodes
    if order is None:
        order = np.argsort(rows, kind="stable")
    rows, cols = rows[order], cols[order]
    pos_table = np.full((depth, nnodes), -1, dtype=np.int64)
    pos_table[rows, cols] = np.arange(k)
    pm = np.asarray(parents_matrix, dtype=np.int64)
    parent_pos = np.full(k, -1, dtype=np.int64)
    par_cols = pm[rows, cols]
    has = (rows > 0) & (par_cols >= 0)
    parent_pos[has] = pos_table[rows[has] - 1, par_cols[has]]
    mask = np.zeros((k, k), dtype=np.int8)
    mask[np.arange(k), np.arange(k)] = 1
    for i in range(k):
        cur = parent_pos[i]
        for _ in range(max(depth - 1, 0)):
            if cur < 0 or cur >= k:
                break
            mask[i, cur] = 1
            cur = parent_pos[cur]
    ids = np.asarray(input_ids_matrix, dtype=np.int64)[rows, cols]
    return {"input_ids": ids, "position_ids": rows + 1, "attention_mask": mask, "parent_last": parent_pos,
            "rows": rows, "cols": cols}


def verify_mask(mask: np.ndarray) -> np.ndarray:
    """Root row and column prepended: [K + 1, K + 1] int8."""
    k = mask.shape[0]
    out = np.zeros((k + 1, k + 1), dtype=np.int8)
    out[1:, 1:] = mask
    out[:, 0] = 1
    return out


def pack_bits(mask: np.ndarray) -> np.ndarray:
    """[M, M] 0/1 -> [M, ceil(M / 64)] uint64, bit j of row m = mask[m, j]."""
    m = mask.shape[0]
    words = (m + 63) // 64
    out = np.zeros((m, words), dtype=np.uint64)
    for j in range(m):
        out[:, j // 64] |= (mask[:, j].astype(np.uint64) & np.uint64(1)) << np.uint64(j % 64)
    return out
