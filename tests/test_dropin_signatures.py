"""The drop-ins keep the reference's call signatures (CPU, no GPU needed).

``tests/golden/signatures.json`` holds the parameter lists of the reference
functions this package replaces, read from the reference source by
``make_golden.py``.  Each drop-in must take the same parameters in the same
order, of the same kind and with the same defaults; it may add parameters
only after them, each with a default (so every existing call still binds).
"""
from __future__ import annotations

import ast
import importlib
import inspect
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))

# reference file (under diffspec/) -> module of this package
MODULES = {
    "runtime/tree_attention.py": "specverify.runtime.tree_attention",
    "runtime/cache_state.py": "specverify.runtime.cache_state",
    "runtime/bundle_verifier.py": "specverify.runtime.bundle_verifier",
    "runtime/llama_target_model.py": "specverify.runtime.rotary",
    "draft/tree_verification.py": "specverify.draft.tree_verification",
    "core/bundle_scheduler.py": "specverify.core.bundle_scheduler",
    "core/kv_cache/paged_kv.py": "specverify.core.kv_cache.paged_kv",
    "core/kv_cache/chunk_arena.py": "specverify.core.kv_cache.chunk_arena",
}
KIND = {"positional": inspect.Parameter.POSITIONAL_OR_KEYWORD, "keyword_only": inspect.Parameter.KEYWORD_ONLY,
        "var_positional": inspect.Parameter.VAR_POSITIONAL, "var_keyword": inspect.Parameter.VAR_KEYWORD}
SNAPSHOT = json.loads((ROOT / "tests" / "golden" / "signatures.json").read_text())


def _resolve(module, qualname):
    obj = importlib.import_module(module)
    for part in qualname.split("."):
        obj = getattr(obj, part)
    return obj


def _same_default(ours, ref_src):
    if ref_src is None:
        return ours is inspect.Parameter.empty
    if ours is inspect.Parameter.empty:
        return False
    try:
        return ours == ast.literal_eval(ref_src)
    except ValueError:            # an expression (a dtype, a name): compare its source text
        return repr(ours).endswith(ref_src.split(".")[-1]) or str(ours) == ref_src


@pytest.mark.parametrize("key", sorted(SNAPSHOT))
def test_dropin_signature_matches_reference(key):
    rel, qualname = key.split(":")
    fn = _resolve(MODULES[rel], qualname)
    params = list(inspect.signature(fn).parameters.values())
    ref = SNAPSHOT[key]
    assert len(params) >= len(ref), (key, [p.name for p in params])
    for p, (name, kind, dflt) in zip(params, ref):
        assert p.name == name, (key, p.name, name)
        assert p.kind == KIND[kind], (key, name, p.kind)
        assert _same_default(p.default, dflt), (key, name, p.default, dflt)
    for p in params[len(ref):]:
        assert p.default is not inspect.Parameter.empty or p.kind in (inspect.Parameter.VAR_POSITIONAL,
                                                                        inspect.Parameter.VAR_KEYWORD), (key, p.name)


def test_snapshot_covers_the_path_entry_points():
    keys = set(SNAPSHOT)
    for k in ("runtime/tree_attention.py:prefix_attention_forward", "runtime/tree_attention.py:tree_attention_forward",
              "draft/tree_verification.py:verify_new", "runtime/bundle_verifier.py:FusedBundleVerifier.verify_bundle",
              "core/kv_cache/paged_kv.py:PagedKVCache.write_kv", "core/kv_cache/chunk_arena.py:ChunkArena.update_arena"):
        assert k in keys
