"""GPU parity: paged copy-on-write compaction, chunk-arena gather, bundle verify.

Page tables, slot mappings and every pool byte must equal the reference's
(golden vectors) and the numpy oracle's, bit for bit.
"""

from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from conftest import cuda_ok, load_golden
from oracle import arena as oarena
from oracle import attention as oatt
from oracle import paged as opaged

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def test_paged_cache_sequence_matches_reference_golden():
    from specverify.core.kv_cache import PagedKVCache, PagedKVConfig
    from specverify.draft.tree_verification import AcceptResult
    z = load_golden("paged.npz")
    log = json.loads(str(z["log"]))
    cfg = PagedKVConfig(page_size=4, max_pages=24, num_layers=2, num_heads=2, head_dim=8, dtype=torch.float32,
                        device="cuda", enable_cow=True)
    cache = PagedKVCache(cfg)
    gen = torch.Generator().manual_seed(3)
    cache.allocate_sequence(0, 22)
    for t in range(22):
        for layer in range(2):
            cache.write_kv(0, layer, t, torch.randn(2, 8, generator=gen).cuda(), torch.randn(2, 8, generator=gen).cuda())
    assert cache.get_physical_blocks(0) == log[0][1]
    cache.fork_sequence(0, 1, shared_prefix_len=22)
    assert cache.get_physical_blocks(1) == log[1][1]
    path = [int(x) for x in z["compact_path"]]
    acc = AcceptResult.from_path(path, rows=16, device="cuda")
    cache.compact_path(1, int(z["compact_start"]), acc, path=path)
    assert cache.get_physical_blocks(1) == log[2][1]
    for layer in range(2):
        cache.write_kv(0, layer, 25, torch.randn(2, 8, generator=gen).cuda(), torch.randn(2, 8, generator=gen).cuda())
    assert cache.get_physical_blocks(0) == log[3][1]
    cache.free_sequence(1)
    cache.allocate_sequence(2, 7)
    assert cache.get_physical_blocks(2) == log[4][1]
    assert np.array_equal(cache.page_pool.cpu().numpy(), z["pool"])
    assert np.array_equal(cache.page_ref_count.numpy(), z["ref"])


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_paged_compaction_random_vs_oracle(seed):
    """Random forks and accepted paths, bf16 pool, vs the numpy oracle."""
    from specverify.core.kv_cache import PagedKVCache, PagedKVConfig
    from specverify.draft.tree_verification import AcceptResult
    rng = np.random.default_rng(seed)
    L, H, D, ps, P = 3, 2, 64, 16, 64
    cache = PagedKVCache(PagedKVConfig(page_size=ps, max_pages=P, num_layers=L, num_heads=H, head_dim=D,
                                       dtype=torch.bfloat16, device="cuda"))
    orc = opaged.PagedOracle(L, H, D, ps, P, dtype=np.float32)
    n_tok = 150
    cache.allocate_sequence(0, n_tok)
    orc.allocate(0, n_tok)
    data = torch.randn(L, 2, n_tok, H, D).bfloat16()
    for t in range(n_tok):
        for layer in range(L):
            cache.write_kv(0, layer, t, data[layer, 0, t].cuda(), data[layer, 1, t].cuda())
            orc.write_row(0, layer, t, data[layer, 0, t].float().numpy(), data[layer, 1, t].float().numpy())
    shared = int(rng.integers(40, 140))
    cache.fork_sequence(0, 1, shared_prefix_len=shared)
    orc.fork(0, 1, shared)
    # the child continues from the parent's prefix; its tree tokens were written at [start, start + m)
    start = 100
    m = 30
    for t in range(start, start + m):
        for layer in range(L):
            k = torch.randn(H, D).bfloat16()
            v = torch.randn(H, D).bfloat16()
            cache.write_kv(1, layer, t, k.cuda(), v.cuda())
            orc.write_row(1, layer, t, k.float().numpy(), v.float().numpy())
    ids = sorted(rng.choice(np.arange(1, m), size=int(rng.integers(1, 9)), replace=False).tolist())
    path = [0] + ids
    acc = AcceptResult.from_path(path, rows=m, device="cuda")
    cache.compact_path(1, start, acc, path=path)
    orc.compact_path(1, start, path)
    assert cache.get_physical_blocks(1) == orc.physical_blocks(1)
    assert cache.get_physical_blocks(0) == orc.physical_blocks(0)
    assert np.array_equal(cache.page_pool.float().cpu().numpy(), orc.pool)


def test_chunk_arena_matches_reference_golden():
    from specverify.core.kv_cache import ChunkArena, ChunkArenaConfig
    z = load_golden("arena.npz")
    states = json.loads(str(z["states"]))
    arena = ChunkArena(ChunkArenaConfig(max_chunks=6, chunk_size=8, num_layers=2, num_heads=2, head_dim=4,
                                        dtype=torch.float32, device="cuda"))
    full = [(torch.from_numpy(z["full_k"][i]).cuda(), torch.from_numpy(z["full_v"][i]).cuda()) for i in range(2)]
    for st in states[:-1]:
        view = arena.update_arena(st["req"], full)
        assert {str(k): v for k, v in arena.get_chunk_mapping().items()} == st["mapping"]
        assert arena.active_chunks == st["active"] and arena.free_offsets == st["free"]
        assert view.shape[4] == st["view_len"]
    assert np.array_equal(arena.arena_kv.cpu().numpy(), z["arena_pre"])
    arena.compact()
    assert {str(k): v for k, v in arena.get_chunk_mapping().items()} == states[-1]["mapping"]
    assert np.array_equal(arena.arena_kv.cpu().numpy(), z["arena_post"])


def test_arena_bf16_random_vs_oracle():
    from specverify.core.kv_cache import ChunkArena, ChunkArenaConfig
    L, H, D, cs, C, S = 4, 8, 128, 64, 16, 64 * 40 - 17
    arena = ChunkArena(ChunkArenaConfig(max_chunks=C, chunk_size=cs, num_layers=L, num_heads=H, head_dim=D,
                                        dtype=torch.bfloat16, device="cuda"))
    orc = oarena.ArenaOracle(C, cs, L, H, D)
    full = [(torch.randn(1, H, S, D).bfloat16(), torch.randn(1, H, S, D).bfloat16()) for _ in range(L)]
    full_np = [(k.float().numpy(), v.float().numpy()) for k, v in full]
    full_gpu = [(k.cuda(), v.cuda()) for k, v in full]
    rng = np.random.default_rng(0)
    for _ in range(4):
        req = rng.choice(40, size=int(rng.integers(3, C + 4)), replace=False).tolist()
        arena.update_arena(req, full_gpu)
        orc.update(req, full_np)
        assert arena.chunk_to_offset == orc.chunk_to_offset
    assert np.array_equal(arena.arena_kv.float().cpu().numpy(), orc.arena)


def test_arena_page_table_zero_copy():
    from specverify.core.kv_cache import arena_page_table
    pt = torch.randperm(512, dtype=torch.int32).cuda()
    ids = torch.tensor([5, 0, 31, 7], dtype=torch.int32).cuda()
    out = arena_page_table(pt, ids, 16)
    ref = torch.cat([pt[i * 16:(i + 1) * 16] for i in ids.tolist()])
    assert torch.equal(out, ref)


def test_bundle_verifier_vs_golden_and_oracle():
    from specverify.runtime import FusedBundleVerifier
    z = load_golden("bundle_verify.npz")
    q, k, v = (torch.from_numpy(z[x]).bfloat16() for x in ("q", "k", "v"))
    masks = [torch.from_numpy(m) for m in z["masks"]]
    ver = FusedBundleVerifier(bundle_size=3, device="cuda")
    out, lse = ver.verify_bundle(q.cuda(), k.cuda(), v.cuda(), [m.cuda() for m in masks], shared_prefix_len=10)
    mask = masks[0][None].expand(q.shape[0], -1, -1)
    ref, ref_lse = oatt.bundle_attention(q.float(), k.float(), v.float(), mask)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-2, rtol=2e-2)
    assert torch.allclose(lse.cpu(), ref_lse, atol=1e-3)
    # The reference's own fp32 outputs agree within bf16 input rounding.
    assert torch.allclose(out.float().cpu(), torch.from_numpy(z["out"]), atol=5e-2, rtol=5e-2)
    stats = ver.get_statistics()
    assert stats["total_verifications"] == 3 and stats["prefix_reuse_rate"] == 1.0


def test_paged_bundle_verifier_reads_pool_directly():
    from specverify.runtime import PagedBundleVerifier
    L, P, H, ps, D = 2, 40, 4, 16, 128
    pool = torch.randn(L, 2, P, H, ps, D).bfloat16().cuda()
    table = torch.randperm(P)[:10].to(torch.int32)
    n = 10 * ps - 5
    b, m = 1, 6
    q = (torch.randn(b, m, 8, D) / math.sqrt(D)).bfloat16().cuda()
    mask = (torch.rand(m, n) > 0.2).to(torch.int8)
    mask[:, 0] = 1
    out, lse = PagedBundleVerifier(device="cuda").verify_bundle_paged(q, pool, table.cuda(), [mask.cuda()],
                                                                      layer_idx=1, num_keys=n)
    kk = pool[1, 0][table.long()].permute(1, 0, 2, 3).reshape(H, -1, D)[:, :n]
    vv = pool[1, 1][table.long()].permute(1, 0, 2, 3).reshape(H, -1, D)[:, :n]
    ref, ref_lse = oatt.full_masked_attention(q.cpu(), kk[None].cpu(), vv[None].cpu(), mask, 0)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-3, rtol=2e-2)
    assert torch.allclose(lse.cpu(), ref_lse, atol=1e-3)


def test_kvcache_length_reads_do_not_synchronise_the_device():
    """KVCache keeps the reference's CPU length tensor: .shape (read once per
    layer by the target model) and .cat run with torch's sync debug mode set
    to error, i.e. without one device synchronisation."""
    from specverify.runtime import KVCache, initialize_past_key_values

    class _Cfg:
        num_hidden_layers, num_key_value_heads, hidden_size, num_attention_heads, head_dim = 2, 8, 4096, 32, 128

    class _Attn:
        def __init__(self):
            self.q_proj = torch.nn.Linear(1, 1, device="cuda")

    class _Layer:
        def __init__(self):
            self.self_attn = _Attn()

    class _Model:
        config = _Cfg()
        dtype = torch.bfloat16

        def __init__(self):
            self.layers = [_Layer(), _Layer()]

    past, data, lengths = initialize_past_key_values(_Model(), 1024)
    assert lengths.device.type == "cpu" and data[0].is_cuda
    new = torch.randn(1, 8, 65, 128, device="cuda").bfloat16()
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for layer in past:
            k, v = layer
            assert k.shape[2] == 0
            ks = k.cat(new)
            vs = v.cat(new)
            assert k.shape[2] == 65 and ks.shape[2] == 65 and vs.shape[2] == 65
    finally:
        torch.cuda.set_sync_debug_mode(0)
    assert isinstance(past[0][0], KVCache)
    assert torch.equal(data[0][0][:, :, :65].cpu(), new.cpu())


@pytest.mark.parametrize("holes", [False, True])
def test_bundle_mask_summary_skips_only_fully_visible_tiles(holes):
    """Bundle verification masks every key (the reference's contract).  With a
    16K-token shared prefix every row sees, the tcgen05 kernel skips masking
    those tiles through the per-word summary -- bit-identical to masking them.
    With a few hidden prefix keys in some rows (holes), the summary marks
    those words and the kernel masks them: the result still matches the
    oracle over the full mask."""
    from specverify.runtime import PagedBundleVerifier, attention, mask_word_summary, pack_tree_mask
    from specverify import workloads as wl
    b, nodes, spl, page = 2, 96, 16384, 16
    gen = torch.Generator().manual_seed(21)
    tree = wl.make_tree(gen, nodes, 12, root=False)
    m = tree.rows
    n = spl + m
    mask = torch.ones(m, n, dtype=torch.int8)
    mask[:, spl:] = tree.keep
    if holes:
        mask[3, 5000] = 0
        mask[40, 129:140] = 0
        mask[95, 16380] = 0
    pages = -(-n // page)
    pool = torch.randn(1, 2, b * pages + 4, 8, page, 128, generator=gen).bfloat16().cuda()
    table = torch.randperm(b * pages, generator=gen).to(torch.int32).view(b, pages).cuda()
    q = (torch.randn(b, m, 32, 128, generator=gen) / math.sqrt(128)).bfloat16().cuda()
    ver = PagedBundleVerifier(device="cuda")
    out, lse = ver.verify_bundle_paged(q, pool, table, [mask.cuda()], shared_prefix_len=spl, num_keys=n)
    bits = pack_tree_mask(mask.cuda(), batch=b, cols=n)
    summary = mask_word_summary(bits)
    words = summary.cpu()
    assert bool(words[:, : spl // 64].all()) != holes
    plain = torch.empty_like(q)
    attention(q, pool[0, 0], pool[0, 1], num_keys=n, page_table=table, mask_bits=bits, mask_len=n, out=plain,
              kernel=2)
    assert torch.equal(out, plain)                     # skipping the mask never changes a bit
    for s in range(b):
        kk = pool[0, 0][table[s].long()].permute(1, 0, 2, 3).reshape(8, -1, 128)[:, :n]
        vv = pool[0, 1][table[s].long()].permute(1, 0, 2, 3).reshape(8, -1, 128)[:, :n]
        ref, ref_lse = oatt.full_masked_attention(q[s:s + 1].cpu(), kk[None].cpu(), vv[None].cpu(), mask, 0)
        assert torch.allclose(out[s:s + 1].float().cpu(), ref, atol=1e-3, rtol=2e-2)
        assert torch.allclose(lse[s:s + 1].cpu(), ref_lse, atol=1e-3)
