"""specverify: DiffSpec's target-side tree verification, B200-native (sm_100a).

Module layout mirrors the reference package ``diffspec`` for the hot path:

* ``specverify.runtime.tree_attention``  -- prefix / tree / fused verify attention
* ``specverify.runtime.bundle_verifier`` -- FusedBundleVerifier, PagedBundleVerifier
* ``specverify.runtime.cache_state``     -- KVCache, initialize_past_key_values
* ``specverify.runtime.sharded``         -- sequence-sharded verify over NCCL
* ``specverify.draft.tree_verification`` -- verify / verify_new, acceptance, compaction
* ``specverify.core.kv_cache``           -- PagedKVCache (COW), ChunkArena
* ``specverify.core.bundle_scheduler``   -- BundleScheduler, TreeDescriptorBuilder

All compute runs in ``libspecverify.so`` (C ABI: include/specverify.h).
"""

from ._lib import SpecVerifyError, available, load

__version__ = "0.1.0"

__all__ = ["SpecVerifyError", "available", "load", "__version__"]
