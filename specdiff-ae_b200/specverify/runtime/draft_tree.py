"""Final draft-tree build on the device: the drop-in for the end of
``diffspec.runtime.draft_tree.DraftTree.update``.

``DraftTree.update``'s final branch (``runtime/draft_tree.py:217-260``) turns
the running top-k of the draft search into the verify inputs: node order,
tokens, positions, parent positions and the ancestor mask
(``generate_attention_mask``, ``:188-215``, one host sync per ancestor hop);
the caller then prepends the root row / column (``diffspec_model.py:620-624``)
and the verify path converts the mask.  :func:`finalize_tree` does all of it
in one launch (``tv_tree_finalize``) and also returns the root-prepended mask
already packed into the bits the verify kernels read, so no host round trip
is needed between the draft search and verification.

Equal-depth nodes keep their top-k order (``torch.argsort`` in the reference
leaves that order to the sort implementation; it changes node numbering
only, not the tree or what acceptance decides).
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch

from .. import _lib


def finalize_tree(top_index: torch.Tensor, parents_matrix: torch.Tensor, input_ids_matrix: torch.Tensor,
                  depth: int, nnodes: int, *, d2t: Optional[torch.Tensor] = None, with_mask: bool = True,
                  with_bits: bool = True, validate: bool = True) -> Dict[str, torch.Tensor]:
    """Returns ``input_ids``, ``position_ids`` (depth + 1), ``parent_last``,
    ``attention_mask`` ([K, K] int8, as ``update`` returns it) and
    ``mask_bits`` ([K + 1, ceil((K + 1) / 64)] int64 words of the root-prepended
    verify mask, the layout :func:`~specverify.runtime.tree_attention.pack_tree_mask`
    produces)."""
    dev = _lib.require_cuda(top_index, parents_matrix, input_ids_matrix, d2t)
    top = top_index.to(torch.int64).contiguous().view(-1)
    pm = parents_matrix.to(torch.int64)
    im = input_ids_matrix.to(torch.int64)
    if pm.stride(-1) != 1:
        pm = pm.contiguous()
    if im.stride(-1) != 1:
        im = im.contiguous()
    if pm.shape[0] < depth or im.shape[0] < depth or pm.shape[1] != nnodes or im.shape[1] != nnodes:
        raise _lib.SpecVerifyError(-1, f"parents/input_ids matrices must be [>= {depth}, {nnodes}]")
    k = top.numel()
    out = {
        "input_ids": torch.empty(k, dtype=torch.int64, device=dev),
        "position_ids": torch.empty(k, dtype=torch.int64, device=dev),
        "parent_last": torch.empty(k, dtype=torch.int64, device=dev),
    }
    mask = torch.empty(k, k, dtype=torch.int8, device=dev) if with_mask else None
    words = (k + 1 + 63) // 64
    bits = torch.empty(k + 1, words, dtype=torch.int64, device=dev) if with_bits else None
    dd = None
    if d2t is not None:
        dd = d2t.to(torch.int64).contiguous()
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    lib = _lib.load()
    rc = lib.tv_tree_finalize(int(nnodes), int(depth), int(k), top.data_ptr(), pm.data_ptr(), pm.stride(0),
                              im.data_ptr(), im.stride(0), _lib.ptr(dd), 0 if dd is None else dd.numel(),
                              out["input_ids"].data_ptr(), out["position_ids"].data_ptr(),
                              out["parent_last"].data_ptr(), _lib.ptr(mask), _lib.ptr(bits), _lib.ptr(status),
                              ctypes.c_void_p(_lib.stream_ptr(dev)))
    _lib.check(rc, "tv_tree_finalize")
    if status is not None and int(status.item()) != 0:
        raise _lib.SpecVerifyError(int(status.item()), "tv_tree_finalize: top index out of range or repeated, "
                                                        "or a token outside d2t")
    if mask is not None:
        out["attention_mask"] = mask
    if bits is not None:
        out["mask_bits"] = bits
    return out


def finalize_from(tree, **kw) -> Dict[str, torch.Tensor]:
    """:func:`finalize_tree` on a ``DraftTree`` whose search has stopped (its
    ``_run_top_idx``, ``parents_matrix``, ``input_ids_matrix``, ``depth`` and
    ``nnodes``)."""
    return finalize_tree(tree._run_top_idx, tree.parents_matrix, tree.input_ids_matrix, int(tree.depth),
                         int(tree.nnodes), **kw)
