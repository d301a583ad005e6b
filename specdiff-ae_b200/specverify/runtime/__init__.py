"""Verify-attention backends (drop-in for ``diffspec.runtime``'s hot path)."""

from .bundle_verifier import FusedBundleVerifier, PagedBundleVerifier
from .cache_state import KVCache, initialize_past_key_values
from .rotary import apply_rotary_pos_emb, apply_rotary_pos_emb_L31, rope_append
from .tree_attention import (KERNELS_AVAILABLE, TRITON_AVAILABLE, attention, describe_attention,
                             mask_word_summary, pack_tree_mask, prefix_attention_forward, tree_attention_forward,
                             verify_attention)

__all__ = [
    "FusedBundleVerifier",
    "PagedBundleVerifier",
    "KVCache",
    "initialize_past_key_values",
    "apply_rotary_pos_emb",
    "apply_rotary_pos_emb_L31",
    "rope_append",
    "KERNELS_AVAILABLE",
    "TRITON_AVAILABLE",
    "attention",
    "describe_attention",
    "mask_word_summary",
    "pack_tree_mask",
    "prefix_attention_forward",
    "tree_attention_forward",
    "verify_attention",
]
