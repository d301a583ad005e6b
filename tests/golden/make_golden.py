"""Generate the golden fixtures in this directory by running the REFERENCE.

Run once, in a container where the reference tree (package ``diffspec``) is
available:

    python tests/golden/make_golden.py [--reference PATH]

It imports the reference read-only (a one-line ``termcolor`` stub is put on
``sys.path`` because the reference imports it and it is not installed), runs
the reference's own CPU code paths on small seeded inputs and stores inputs +
outputs as ``.npz`` / ``.json``.  The fixtures travel with the repository; the
tests never need the reference at run time.

Fixtures
--------
attn_fp32.npz / attn_bf16.npz
    ``prefix_attention_forward`` + ``tree_attention_forward`` (CPU torch
    path) + the merge of ``llama_target_model.py:862-864`` on GQA-expanded
    inputs built with the reference's ``repeat_kv``.
accept_greedy.npz
    ``verify_new`` (greedy) with a stub model: acceptance, path, compaction of
    a contiguous KV buffer, several cases (random, planted path, ties, NaN).
accept_sample.npz
    ``verify_new`` (sample-and-match, temperature 1.0) with ``torch.multinomial``
    replaced by a seeded draw recorded in the fixture.
paged.npz
    ``PagedKVCache`` operation sequence: allocate, writes, fork, copy-on-write
    writes, path compaction through ``read_kv``/``write_kv``, free.
arena.npz
    ``ChunkArena.update_arena`` sequence + ``compact``.
bundles.json
    ``BundleScheduler.schedule_bundles`` on seeded trees.
bundle_verify.npz
    ``FusedBundleVerifier`` torch path.
tree_final.npz
    ``DraftTree`` (``runtime/draft_tree.py``) driven with seeded draft
    distributions to its depth limit: the final state (running top-k
    indices, per-depth parents and tokens) and ``update``'s final outputs
    (tokens, positions, ancestor mask, parent positions), several sizes.
retrieval.npz
    ``DraftNetwork._select_working_cache_from_chunks`` (retrieval mode) on a
    stand-in object holding its inputs: per-token attention scores (dyadic
    values, so every prefix sum is exact), chunk bounds, top-k; the selected
    chunk ids, the interval-union token indices and the gathered working K/V.
rope_bf16.npz / rope_f16.npz / rope_f32.npz
    ``LlamaRotaryEmbedding`` (theta 500000) cached cos/sin tables,
    ``apply_rotary_pos_emb`` with tree position ids, ``apply_rotary_pos_emb_L31``
    on the gathered per-token tables, and ``KVCache.cat`` of the rotated k and
    of v into a pre-filled cache at ``current_length``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference(ref_root: str):
    stub = Path(tempfile.mkdtemp()) / "termcolor.py"
    stub.write_text("def colored(text, *args, **kwargs):\n    return text\n")
    sys.path.insert(0, str(stub.parent))
    sys.path.insert(0, ref_root)
    from diffspec.runtime import tree_attention as ta           # noqa: E402
    from diffspec.runtime import llama_target_model as ltm      # noqa: E402
    from diffspec.draft import tree_verification as tv          # noqa: E402
    from diffspec.core.kv_cache import paged_kv as pkv          # noqa: E402
    from diffspec.core.kv_cache import chunk_arena as ca        # noqa: E402
    from diffspec.core import bundle_scheduler as bs            # noqa: E402
    from diffspec.runtime import bundle_verifier as bv          # noqa: E402
    return ta, ltm, tv, pkv, ca, bs, bv


def make_tree(gen: torch.Generator, n_nodes: int, per_depth: int):
    """Draft tree: ``per_depth`` nodes per depth; a node at depth d > 0 takes a
    parent drawn uniformly from the nodes at depth d - 1; depth-0 nodes hang
    off the root (parent -1).  Returns (parent [n_nodes] in verify_new's
    convention, depth [n_nodes], keep [n_nodes + 1, n_nodes + 1] int8 with
    the root row/column prepended as in ``diffspec_model.py:620-624``)."""
    depth = np.repeat(np.arange((n_nodes + per_depth - 1) // per_depth), per_depth)[:n_nodes]
    parent = np.full(n_nodes, -1, dtype=np.int64)
    for i in range(n_nodes):
        d = depth[i]
        if d > 0:
            lo = (d - 1) * per_depth
            parent[i] = lo + int(torch.randint(0, per_depth, (1,), generator=gen))
    m = n_nodes + 1
    keep = np.zeros((m, m), dtype=np.int8)
    keep[:, 0] = 1
    for i in range(n_nodes):
        r = i + 1
        keep[r, r] = 1
        p = parent[i]
        while p >= 0:
            keep[r, p + 1] = 1
            p = parent[p]
    keep[0, 0] = 1
    return parent, depth, keep


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gen_attention(ta, ltm, dtype, path: Path):
    gen = torch.Generator().manual_seed(1234)
    b, n_nodes, per_depth, h, hkv, d, s = 2, 16, 4, 8, 2, 64, 160
    parent, depth, keep = make_tree(gen, n_nodes, per_depth)
    m = n_nodes + 1
    q = (torch.randn(b, m, h, d, generator=gen) / d ** 0.5).to(dtype)
    kp = torch.randn(b, hkv, s, d, generator=gen).to(dtype)
    vp = torch.randn(b, hkv, s, d, generator=gen).to(dtype)
    kt = torch.randn(b, hkv, m, d, generator=gen).to(dtype)
    vt = torch.randn(b, hkv, m, d, generator=gen).to(dtype)
    g = h // hkv
    full_k = ltm.repeat_kv(torch.cat([kp, kt], dim=2), g).transpose(1, 2)   # [B, S+M, H, D]
    full_v = ltm.repeat_kv(torch.cat([vp, vt], dim=2), g).transpose(1, 2)
    # Additive float mask exactly as LlamaModel.forward builds it (:1319-1330).
    tm = torch.from_numpy(keep).float()
    am = torch.zeros((m, s + m)).float()
    tmask = torch.where(tm == 0, torch.finfo(torch.float32).min, tm)
    tmask = torch.where(tmask == 1, torch.tensor(0, dtype=torch.float32), tmask)
    am[-m:, -m:] = tmask
    am = am[None, None].expand(b, 1, m, s + m)
    with torch.no_grad():
        p_out, p_lse = ta.prefix_attention_forward(q, full_k[:, :s], full_v[:, :s], b, m, h, d)
        t_out, w = ta.tree_attention_forward(q, full_k[:, s:], full_v[:, s:], am, s, p_lse, b, m, h, d)
        # The merge's ``prefix.to(dtype).mul_(w)`` is in place when the dtypes
        # already match, so keep an untouched copy of the prefix output.
        p_out_saved = p_out.clone()
        merged = t_out.clone()
        merged.mul_(1.0 - w)
        merged.add_(p_out.to(merged.dtype).mul_(w))
    enc = (lambda t: t.numpy()) if dtype == torch.float32 else _bf16_bits
    np.savez_compressed(
        path, dtype=str(dtype), parent=parent, depth=depth, keep=keep,
        q=enc(q), k_prefix=enc(kp), v_prefix=enc(vp), k_tree=enc(kt), v_tree=enc(vt),
        prefix_out=enc(p_out_saved), prefix_lse=p_lse.numpy(), tree_out=enc(t_out), weight=enc(w),
        merged=enc(merged))


class _StubDraft:
    use_retrieval_cache = False
    enable_bundle_scheduling = False

    def build_speculative_tree(self, hidden, input_ids, head, nodes, threshold, max_depth):
        k = 4
        return (torch.zeros(1, k, dtype=torch.long), torch.arange(k, dtype=torch.long),
                torch.eye(k, dtype=torch.int8), torch.full((k,), -1, dtype=torch.long))


class _StubModel:
    def __init__(self):
        self.draft_model = _StubDraft()

        class _B:
            lm_head = None
        self.base_model = _B()


def _run_verify(tv, logits, draft, pos, parent, kv, cur_len, max_depth, processor):
    model = _StubModel()
    input_ids = torch.zeros(1, 5, dtype=torch.long)
    hidden = torch.zeros(1, draft.shape[1], 8)
    cl = torch.full((4,), cur_len, dtype=torch.long)
    out = tv.verify_new(input_ids, logits, draft, pos, hidden, None, [kv], cl, parent, model,
                        4, 1.0, max_depth, processor, None)
    return out, cl


def gen_accept(tv, path_greedy: Path, path_sample: Path):
    gen = torch.Generator().manual_seed(7)
    vocab, n_nodes, per_depth, max_depth = 1000, 32, 4, 8
    cases = {}
    sample_cases = {}
    for case in range(6):
        parent, depth, _ = make_tree(gen, n_nodes, per_depth)
        m = n_nodes + 1
        s_prefix = 40
        logits = (torch.randn(1, m, vocab, generator=gen) * 2.0).to(torch.bfloat16)
        draft = torch.randint(0, vocab, (1, m), generator=gen)
        if case >= 1:
            # Plant a path: make the draft token of every node on a random
            # root-to-leaf chain equal to its parent's argmax.
            leaf = n_nodes - 1 - int(torch.randint(0, per_depth, (1,), generator=gen))
            chain = []
            p = leaf
            while p >= 0:
                chain.append(p)
                p = parent[p]
            chain = chain[::-1]
            am = torch.argmax(logits[0].float(), dim=-1)
            stop = len(chain) if case != 2 else len(chain) // 2
            prev_row = 0
            for i in chain[:stop]:
                draft[0, i + 1] = am[prev_row]
                prev_row = i + 1
        if case == 3:
            # Ties: duplicate the max value at a later index in every row.
            lf = logits[0]
            am = torch.argmax(lf.float(), dim=-1)
            for r in range(m):
                j = (int(am[r]) + 17) % vocab
                lf[r, j] = lf[r, am[r]]
        if case == 4:
            # A NaN in a couple of rows.
            logits[0, 3, 11] = float("nan")
            logits[0, 5, 400] = float("nan")
            logits[0, 5, 401] = float("nan")
        if case == 5:
            # Sibling draft tokens equal: several children of the root match.
            am0 = int(torch.argmax(logits[0, 0].float()))
            for i in range(per_depth):
                draft[0, i + 1] = am0
        pos = torch.cat([torch.tensor([s_prefix]), s_prefix + 1 + torch.from_numpy(depth)])
        kv = torch.randn(4, 1, 2, s_prefix + m + 8, 16, generator=gen)
        kv_in = kv.clone()
        (ids, best, acc, nd, npos, nmask, npar), cl = _run_verify(
            tv, logits, draft, pos, torch.from_numpy(parent), kv, s_prefix + m, max_depth, None)
        cases[f"c{case}"] = dict(
            logits=_bf16_bits(logits[0]), draft=draft[0].numpy(), pos=pos.numpy(), parent=parent,
            kv_in=kv_in.numpy(), kv_out=kv.numpy(), cur_len=np.int64(s_prefix + m),
            best_candidate=np.array(best, dtype=np.int64), accept_length=np.int64(acc),
            next_token=np.int64(nd[0, 0]), new_len=np.int64(cl[0]), root_pos=np.int64(npos[0]))
        # Sample-and-match with a recorded draw (temperature 1.0 -> empty
        # processor list, tree_verification.py:22-31).  Skipped for the NaN
        # case: torch.multinomial rejects NaN probabilities.
        if case == 4:
            continue
        proc = tv.prepare_logits_processor(temperature=1.0)
        drawn = {}
        real = torch.multinomial

        def fake_multinomial(probs, num, _gen=torch.Generator().manual_seed(100 + case)):
            t = real(probs.float(), num, generator=_gen)
            drawn["t"] = t.clone()
            return t

        torch.multinomial = fake_multinomial
        try:
            kv2 = kv_in.clone()
            (ids, best, acc, nd, npos, nmask, npar), cl = _run_verify(
                tv, logits, draft, pos, torch.from_numpy(parent), kv2, s_prefix + m, max_depth, proc)
        finally:
            torch.multinomial = real
        sample_cases[f"c{case}"] = dict(
            sampled=drawn["t"].view(-1).numpy(), draft=draft[0].numpy(), pos=pos.numpy(), parent=parent,
            kv_in=kv_in.numpy(), kv_out=kv2.numpy(), cur_len=np.int64(s_prefix + m),
            best_candidate=np.array(best, dtype=np.int64), accept_length=np.int64(acc),
            next_token=np.int64(nd[0, 0]), new_len=np.int64(cl[0]))
    flat = {f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()}
    np.savez_compressed(path_greedy, max_depth=max_depth, **flat)
    flat = {f"{c}__{k}": v for c, d in sample_cases.items() for k, v in d.items()}
    np.savez_compressed(path_sample, max_depth=max_depth, **flat)


def gen_paged(pkv, path: Path):
    gen = torch.Generator().manual_seed(3)
    cfg = pkv.PagedKVConfig(page_size=4, max_pages=24, num_layers=2, num_heads=2, head_dim=8,
                            dtype=torch.float32, device="cpu", enable_cow=True)
    cache = pkv.PagedKVCache(cfg)
    log = []
    cache.allocate_sequence(0, 22)
    for t in range(22):
        for layer in range(2):
            cache.write_kv(0, layer, t, torch.randn(2, 8, generator=gen), torch.randn(2, 8, generator=gen))
    log.append(("alloc+write seq0", cache.get_physical_blocks(0)))
    cache.fork_sequence(0, 1, shared_prefix_len=22)
    log.append(("fork seq1", cache.get_physical_blocks(1)))
    # Compaction of an accepted path on the child through the public API:
    # rows start+path[j] -> start+j, read first, then written in row order.
    start, path_ids = 9, [0, 2, 5, 6, 11]
    rows = [[tuple(x.clone() for x in cache.read_kv(1, layer, start + s)) for layer in range(2)]
            for s in path_ids]
    for j, per_layer in enumerate(rows):
        for layer, (k, v) in enumerate(per_layer):
            cache.write_kv(1, layer, start + j, k, v)
    log.append(("compact seq1", cache.get_physical_blocks(1)))
    # Writes past the allocation on the parent, then free the child.
    for layer in range(2):
        cache.write_kv(0, layer, 25, torch.randn(2, 8, generator=gen), torch.randn(2, 8, generator=gen))
    log.append(("write past end seq0", cache.get_physical_blocks(0)))
    cache.free_sequence(1)
    cache.allocate_sequence(2, 7)
    log.append(("alloc seq2 after free", cache.get_physical_blocks(2)))
    np.savez_compressed(
        path, pool=cache.page_pool.numpy(), ref=cache.page_ref_count.numpy(),
        free=np.array(sorted(cache.free_pages)), compact_start=start, compact_path=np.array(path_ids),
        log=json.dumps(log))


def gen_arena(ca, path: Path):
    gen = torch.Generator().manual_seed(5)
    cfg = ca.ChunkArenaConfig(max_chunks=6, chunk_size=8, num_layers=2, num_heads=2, head_dim=4,
                              dtype=torch.float32, device="cpu")
    arena = ca.ChunkArena(cfg)
    s = 8 * 12 - 3   # last chunk is ragged
    full = [(torch.randn(1, 2, s, 4, generator=gen), torch.randn(1, 2, s, 4, generator=gen)) for _ in range(2)]
    requests = [[3, 1, 7], [7, 11, 2, 5], [0, 1, 2, 3, 4, 5, 6], [11, 9, 8], [4, 11]]
    states = []
    for req in requests:
        view = arena.update_arena(req, full)
        states.append(dict(req=req, mapping={str(k): v for k, v in arena.get_chunk_mapping().items()},
                           active=list(arena.active_chunks), free=list(arena.free_offsets),
                           view_len=int(view.shape[4])))
    arena_before_compact = arena.arena_kv.clone()
    arena.compact()
    states.append(dict(req="compact", mapping={str(k): v for k, v in arena.get_chunk_mapping().items()},
                       active=list(arena.active_chunks), free=list(arena.free_offsets)))
    np.savez_compressed(path, full_k=np.stack([f[0].numpy() for f in full]),
                        full_v=np.stack([f[1].numpy() for f in full]),
                        arena_pre=arena_before_compact.numpy(), arena_post=arena.arena_kv.numpy(),
                        states=json.dumps(states))


def gen_bundles(bs, path: Path):
    gen = torch.Generator().manual_seed(11)
    out = []
    for case in range(6):
        n = 10 + 7 * case
        parent = [-1]
        for i in range(1, n):
            parent.append(int(torch.randint(0, i, (1,), generator=gen)))
        parent_map = {i: parent[i] for i in range(n)}
        children = set(p for p in parent if p >= 0)
        leaves = [i for i in range(n) if i not in children]
        depth = {}
        for i in range(n):
            d, c = 0, i
            while parent[c] >= 0:
                c = parent[c]
                d += 1
            depth[i] = d
        size = 2 + case % 3
        sched = bs.BundleScheduler(bundle_size=size, max_bundles=100 if case != 4 else 3, device="cpu")
        res = sched.schedule_bundles({"leaf_ids": leaves, "parent_map": parent_map, "depth_map": depth},
                                     return_tensors=False)
        out.append(dict(parent=parent, leaves=leaves, depth={str(k): v for k, v in depth.items()},
                        bundle_size=size, max_bundles=sched.max_bundles, bundles=res,
                        stats=sched.get_statistics()))
    path.write_text(json.dumps(out, indent=1))


def gen_bundle_verify(bv, path: Path):
    gen = torch.Generator().manual_seed(21)
    b, m, h, d, n = 2, 12, 4, 32, 40
    q = torch.randn(b, m, h, d, generator=gen)
    k = torch.randn(b, n, h, d, generator=gen)
    v = torch.randn(b, n, h, d, generator=gen)
    masks = [(torch.rand(m, n, generator=gen) > 0.3).to(torch.int8) for _ in range(3)]
    for mk in masks:
        mk[:, 0] = 1
    ver = bv.FusedBundleVerifier(bundle_size=3, enable_triton=False, device="cpu")
    o, lse = ver.verify_bundle(q, k, v, masks, shared_prefix_len=10)
    np.savez_compressed(path, q=q.numpy(), k=k.numpy(), v=v.numpy(), masks=np.stack([x.numpy() for x in masks]),
                        out=o.numpy(), lse=lse.numpy(), stats=json.dumps(ver.get_statistics()))


def _enc16(t: torch.Tensor) -> np.ndarray:
    """bf16 as uint16 bit patterns, fp16 / fp32 as numpy arrays."""
    if t.dtype == torch.bfloat16:
        return _bf16_bits(t)
    return t.contiguous().numpy()


def gen_rope(ltm, dtype, path: Path):
    from diffspec.runtime import cache_state as cs                # noqa: E402
    gen = torch.Generator().manual_seed(4321)
    b, h, hkv, t, d, max_pos, prefix, budget = 2, 8, 2, 17, 64, 512, 300, 64
    # the module builds its cache in the default dtype and casts on use (:152-211)
    rot = ltm.LlamaRotaryEmbedding(d, max_position_embeddings=max_pos, base=500000)
    q = torch.randn(b, h, t, d, generator=gen).to(dtype)
    k = torch.randn(b, hkv, t, d, generator=gen).to(dtype)
    v = torch.randn(b, hkv, t, d, generator=gen).to(dtype)
    depth = torch.arange(t) // 3                                   # tree-like: several tokens per depth
    position_ids = torch.stack([prefix + depth, prefix + 7 + depth])   # [B, T]
    cos, sin = rot(v, seq_len=max_pos)                             # [1, 1, max_pos, D] in dtype
    q_embed, k_embed = ltm.apply_rotary_pos_emb(q, k, cos, sin, position_ids)
    cos_tok = cos.squeeze(1).squeeze(0)[position_ids]              # [B, T, D]
    sin_tok = sin.squeeze(1).squeeze(0)[position_ids]
    q_l31, k_l31 = ltm.apply_rotary_pos_emb_L31(q, k, cos_tok, sin_tok)
    kdata = torch.randn(b, hkv, budget, d, generator=gen).to(dtype)
    vdata = torch.randn(b, hkv, budget, d, generator=gen).to(dtype)
    k_before, v_before = kdata.clone(), vdata.clone()
    start = 40                                                     # cache index (positions are separate)
    kc = cs.KVCache(kdata, torch.tensor(start, dtype=torch.long))
    vc = cs.KVCache(vdata, torch.tensor(start, dtype=torch.long))
    k_states = kc.cat(k_embed, dim=2)
    v_states = vc.cat(v, dim=2)
    np.savez_compressed(
        path, dtype=str(dtype), position_ids=position_ids.numpy(), start=start,
        q=_enc16(q), k=_enc16(k), v=_enc16(v),
        cos=_enc16(cos.squeeze(1).squeeze(0)), sin=_enc16(sin.squeeze(1).squeeze(0)),
        q_embed=_enc16(q_embed), k_embed=_enc16(k_embed), q_l31=_enc16(q_l31), k_l31=_enc16(k_l31),
        k_cache_before=_enc16(k_before), v_cache_before=_enc16(v_before),
        k_cache_after=_enc16(kdata), v_cache_after=_enc16(vdata),
        k_states_len=k_states.shape[2], v_states_len=v_states.shape[2])


def gen_tree(path: Path):
    from diffspec.runtime import draft_tree as dt                 # noqa: E402
    out = {}
    cases = [(16, 5, 4, 500), (64, 8, 8, 1000), (64, 10, 3, 300), (8, 3, 2, 50)]
    for ci, (nnodes, max_depth, seed, vocab) in enumerate(cases):
        gen = torch.Generator().manual_seed(seed)
        tree = dt.DraftTree(nnodes, "cpu", threshold=-1e30, max_depth=max_depth)
        res = tree.update(torch.softmax(torch.randn(1, 3, vocab, generator=gen), -1))
        while not res["is_final"]:
            res = tree.update(torch.softmax(torch.randn(1, nnodes, vocab, generator=gen), -1))
        top = tree._run_top_idx.clone()
        rows = (top // nnodes).numpy()
        # the final ordering is torch.argsort(rows); record whether it kept the
        # top-k order among equal depths (the GPU sort the reference runs does)
        ref_order = torch.argsort(top // nnodes).numpy()            # the same call update() made
        stable = np.array_equal(np.argsort(rows, kind="stable"), ref_order)
        p = f"c{ci}_"
        out.update({p + "nnodes": nnodes, p + "depth": tree.depth, p + "top_index": top.numpy(),
                    p + "parents_matrix": tree.parents_matrix.numpy(),
                    p + "input_ids_matrix": tree.input_ids_matrix.numpy(),
                    p + "input_ids": res["input_ids"].numpy(), p + "position_ids": res["position_ids"].numpy(),
                    p + "attention_mask": res["attention_mask"].numpy(), p + "parent_last": res["parent_last"].numpy(),
                    p + "argsort_stable": stable, p + "ref_order": ref_order})
    out["cases"] = len(cases)
    np.savez_compressed(path, **out)


def gen_retrieval(path: Path):
    import types
    from diffspec.draft import draft_network as dn                 # noqa: E402
    out = {}
    # (L, chunk size, top-k, layers, heads, head_dim, overlapping chunks)
    cases = [(1000, 32, 7, 2, 2, 16, False), (4096, 256, 5, 1, 2, 8, False), (300, 64, 9, 1, 1, 8, False),
             (777, 50, 4, 2, 2, 8, True)]
    for ci, (L, cs, topk, layers, heads, d, overlap) in enumerate(cases):
        gen = torch.Generator().manual_seed(100 + ci)
        starts = list(range(0, L, cs))
        ends = [min(s0 + cs, L) for s0 in starts]
        if overlap:                                # chunks reaching into the next one
            ends = [min(e + cs // 3, L) for e in ends]
        chunks = [(i, s0, e) for i, (s0, e) in enumerate(zip(starts, ends))]
        # multiples of 2^-12 below 1: every partial sum is exact in fp32
        attn = torch.randint(0, 4096, (L,), generator=gen).float() / 4096.0
        # K/V values k / 16 with |k| < 256: exact in fp16, stored as fp16
        full_kv = [(torch.randint(-255, 256, (1, heads, L, d), generator=gen).float() / 16,
                    torch.randint(-255, 256, (1, heads, L, d), generator=gen).float() / 16) for _ in range(layers)]
        st = types.SimpleNamespace(
            full_draft_kv=full_kv, total_seq_len=L, chunks=chunks, selected_chunks=chunks[:1],
            retrieve_top_k=topk, attn_scores_final=attn.clone(), attn_scores=None, retrieval_condition=True,
            _chunks_starts=torch.tensor(starts), _chunks_ends=torch.tensor(ends), _diff_buf=None, _ones_buf=None,
            gamma_sem=0.0, prev_selected_chunk_ids=[], chunk_arena=None,
            past_key_position_ids=torch.arange(L).unsqueeze(0), evicted=0, retrieval_verbose=False)
        st._record_chunk_overlap_ratio = lambda a, b: None
        st.update_working_cache_from_full = lambda: None
        working = dn.DraftNetwork._select_working_cache_from_chunks(st, top_k_chunks=topk, do_retrieval=True)
        n_ret = working[0][0].shape[2]
        p = f"c{ci}_"
        out.update({p + "L": L, p + "top_k": topk, p + "attn": attn.numpy(), p + "starts": np.array(starts),
                    p + "ends": np.array(ends), p + "selected": np.array(st.prev_selected_chunk_ids),
                    p + "n_ret": n_ret, p + "evicted": st.evicted})
        for li, ((fk, fv), (wk, wv)) in enumerate(zip(full_kv, working)):
            out.update({p + f"full_k{li}": fk.numpy().astype(np.float16), p + f"full_v{li}": fv.numpy().astype(np.float16),
                        p + f"work_k{li}": wk.numpy().astype(np.float16), p + f"work_v{li}": wv.numpy().astype(np.float16)})
        out[p + "layers"] = layers
    out["cases"] = len(cases)
    np.savez_compressed(path, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DIFFSPEC_REFERENCE", "/root/reference"))
    ap.add_argument("--only", default="", help="comma-separated subset: attention, accept, paged, arena, "
                                               "bundles, bundle_verify, rope, tree, retrieval")
    args = ap.parse_args()
    only = set(filter(None, args.only.split(",")))
    want = (lambda name: not only or name in only)
    torch.manual_seed(0)
    ta, ltm, tv, pkv, ca, bs, bv = _import_reference(args.reference)
    if want("attention"):
        gen_attention(ta, ltm, torch.float32, HERE / "attn_fp32.npz")
        gen_attention(ta, ltm, torch.bfloat16, HERE / "attn_bf16.npz")
    if want("accept"):
        gen_accept(tv, HERE / "accept_greedy.npz", HERE / "accept_sample.npz")
    if want("paged"):
        gen_paged(pkv, HERE / "paged.npz")
    if want("arena"):
        gen_arena(ca, HERE / "arena.npz")
    if want("bundles"):
        gen_bundles(bs, HERE / "bundles.json")
    if want("bundle_verify"):
        gen_bundle_verify(bv, HERE / "bundle_verify.npz")
    if want("retrieval"):
        gen_retrieval(HERE / "retrieval.npz")
    if want("tree"):
        gen_tree(HERE / "tree_final.npz")
    if want("rope"):
        gen_rope(ltm, torch.bfloat16, HERE / "rope_bf16.npz")
        gen_rope(ltm, torch.float16, HERE / "rope_f16.npz")
        gen_rope(ltm, torch.float32, HERE / "rope_f32.npz")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
