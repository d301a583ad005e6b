"""Tree acceptance and KV compaction (drop-in for ``diffspec.draft.tree_verification``)."""

from .tree_verification import AcceptResult, accept, compact_kv, prepare_logits_processor, verify, verify_new

__all__ = ["AcceptResult", "accept", "compact_kv", "prepare_logits_processor", "verify", "verify_new"]
