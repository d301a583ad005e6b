"""Bundle verification on B200: the drop-in for
``diffspec.runtime.bundle_verifier``.

:class:`FusedBundleVerifier` keeps the reference's constructor, statistics
keys and ``verify_bundle`` contract (``bundle_verifier.py:142-331``): the
bundle's mask is ``masks[0]`` broadcast over the batch (``:196-205``),
attention runs over all N keys under it, and the result is
``(out [B, M, H, D], lse [B, M, H] fp32)``.  The mask is packed to one bit
per key and the verify-attention kernel scores every node of a KV head in
one CTA, so each KV tile -- the shared prefix included -- is read from
memory once per head for all of the bundle's rows.  The mask covers every
key, as the reference's does; a per-word summary (all rows see all 64 keys)
lets the kernel skip masking the tiles of a shared prefix every row sees,
with the same result for any mask.

:class:`PagedBundleVerifier.verify_bundle_paged` is implemented (the
reference raises ``NotImplementedError``, ``:341-366``): it reads K/V through
the page table straight out of a ``[L, 2, P, H, page, D]`` pool.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch

from .. import _lib
from .tree_attention import attention, mask_word_summary, pack_tree_mask


class FusedBundleVerifier:
    """Verify a bundle of tree nodes with the B200 verify-attention kernels."""

    def __init__(self, bundle_size: int = 3, enable_triton: bool = True, device: str = "cuda"):
        self.bundle_size = bundle_size
        # The flag name is the reference's; it reports whether the B200 kernels run.
        self.enable_triton = bool(enable_triton) and _lib.available()
        self.device = device
        self.total_verifications = 0
        self.total_bundles = 0
        self.prefix_reuse_count = 0

    def _bundle_mask(self, masks: List[torch.Tensor], b: int) -> torch.Tensor:
        """masks[0] for every sequence of the batch (``bundle_verifier.py:196-205``):
        a [M, N] mask stays one [1, M, N] mask (packed once, read with batch
        stride 0 by the kernel); a per-sequence [B, M, N] mask is kept."""
        mask = masks[0]
        if mask.dim() == 2:
            mask = mask.unsqueeze(0)
        return mask if mask.shape[0] in (1, b) else mask.expand(b, -1, -1)

    def verify_bundle(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, masks: List[torch.Tensor],
                      shared_prefix_len: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        """q [B, M, H, D]; k/v [B, N, Hk, D]; masks: list of [M, N] (1 = attend)."""
        self.total_verifications += len(masks)
        self.total_bundles += 1
        if shared_prefix_len > 0:
            self.prefix_reuse_count += 1
        b, m, h, _ = q.shape
        n = k.size(1)
        bits = pack_tree_mask(self._bundle_mask(masks, b).to(q.device), cols=n)
        lse = torch.empty((b, m, h), dtype=torch.float32, device=q.device)
        out = attention(q, k, v, num_keys=n, mask_bits=bits, mask_len=n, lse=lse,
                        mask_full=mask_word_summary(bits))
        return out, lse

    def get_statistics(self) -> Dict:
        return {
            "total_verifications": self.total_verifications,
            "total_bundles": self.total_bundles,
            "avg_bundle_size": self.total_verifications / self.total_bundles if self.total_bundles > 0 else 0,
            "prefix_reuse_rate": self.prefix_reuse_count / self.total_bundles if self.total_bundles > 0 else 0,
            "triton_enabled": self.enable_triton,
        }


class PagedBundleVerifier(FusedBundleVerifier):
    """Bundle verifier reading KV straight from a paged pool."""

    def verify_bundle_paged(self, q: torch.Tensor, kv_pages: torch.Tensor, page_table: torch.Tensor,
                            masks: List[torch.Tensor], shared_prefix_len: int = 0, layer_idx: int = 0,
                            num_keys: int = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """q [B, M, H, D]; kv_pages [L, 2, P, Hk, page, D]; page_table int [n_logical]
        (or [B, n_logical]); masks[0] is [M, N] over the N = num_keys logical
        tokens (default: all pages of the table).  Returns (out, lse [B, M, H])."""
        self.total_verifications += len(masks)
        self.total_bundles += 1
        if shared_prefix_len > 0:
            self.prefix_reuse_count += 1
        b, m, h, _ = q.shape
        pt = page_table.to(device=q.device, dtype=torch.int32)
        if pt.dim() == 1:
            pt = pt.unsqueeze(0).expand(b, -1)
        page = kv_pages.shape[4]
        n = pt.shape[1] * page if num_keys is None else int(num_keys)
        mask = self._bundle_mask(masks, b).to(q.device)
        bits = pack_tree_mask(mask, cols=n)
        lse = torch.empty((b, m, h), dtype=torch.float32, device=q.device)
        out = attention(q, kv_pages[layer_idx, 0], kv_pages[layer_idx, 1], num_keys=n, page_table=pt,
                        mask_bits=bits, mask_len=n, lse=lse, mask_full=mask_word_summary(bits))
        return out, lse
