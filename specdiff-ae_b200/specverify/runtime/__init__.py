"""Verify-attention backends (drop-in for ``diffspec.runtime``'s hot path)."""

from .bundle_verifier import FusedBundleVerifier, PagedBundleVerifier
from .cache_state import KVCache, initialize_past_key_values
from .tree_attention import (KERNELS_AVAILABLE, TRITON_AVAILABLE, attention, pack_tree_mask,
                             prefix_attention_forward, tree_attention_forward, verify_attention)

__all__ = [
    "FusedBundleVerifier",
    "PagedBundleVerifier",
    "KVCache",
    "initialize_past_key_values",
    "KERNELS_AVAILABLE",
    "TRITON_AVAILABLE",
    "attention",
    "pack_tree_mask",
    "prefix_attention_forward",
    "tree_attention_forward",
    "verify_attention",
]
