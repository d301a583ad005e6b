"""GPU parity of the tensor-memory (tcgen05) verify-attention kernel.

The planner sends long, uniform-length key ranges with >= 64 query rows per KV
head and head_dim 128 to the tcgen05 kernel.  These cases cover its layouts
(paged at several page sizes, contiguous token-major and head-major caches),
one and two 128-row halves, several row blocks, tails that start mid-tile,
both 16-bit types, and the bounded-wait status word.  Tolerance: 2e-2 rel /
1e-3 abs against the fp32 oracle.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import cuda_ok
from oracle import attention as oatt

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _close(got, ref, atol=1e-3, rtol=2e-2):
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bad = err > atol + rtol * ref.abs()
    assert not bool(bad.any()), f"max abs err {err.max().item():.3e}, {int(bad.sum())} elements out of tolerance"


def _paged_case(prefix, nodes, per_depth, page, heads=32, kv_heads=8, batch=1, dtype=torch.bfloat16, seed=0):
    from specverify import workloads as wl
    from specverify.runtime import verify_attention
    w = wl.paged_verify(prefix_len=prefix, nodes=nodes, per_depth=per_depth, root=False, batch=batch,
                        heads=heads, kv_heads=kv_heads, page_size=page, spare_pages=2, dtype=dtype, seed=seed)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    from specverify.runtime import attention, pack_tree_mask
    lse = torch.empty(w.q.shape[:3], device="cuda")
    out = attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table,
                    mask_bits=pack_tree_mask(w.tree.keep.cuda(), batch=batch), mask_len=w.tree.rows, lse=lse,
                    status=status)
    ref_out = attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table,
                        mask_bits=pack_tree_mask(w.tree.keep.cuda(), batch=batch), mask_len=w.tree.rows,
                        kernel=1)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for bb in range(batch):
        k, v = w.contiguous_kv(bb)
        ref, ref_lse = oatt.full_masked_attention(w.q[bb:bb + 1].cpu(), k.permute(1, 0, 2)[None].cpu(),
                                                  v.permute(1, 0, 2)[None].cpu(), w.tree.keep, w.prefix_len)
        _close(out[bb:bb + 1], ref)
        _close(lse[bb:bb + 1], ref_lse, atol=1e-3, rtol=1e-4)
    # the warp-MMA path agrees too
    assert (out.float() - ref_out.float()).abs().max().item() < 4e-3
    return w


@pytest.mark.parametrize("prefix,nodes,per_depth,page", [
    (8192, 64, 8, 16),      # config-2 shape at 8K: 256 rows, two halves
    (6000, 64, 8, 16),      # tail starts mid-tile
    (5000, 24, 6, 8),       # 96 rows: one half, 8-token pages
    (5056, 64, 8, 256),     # pages larger than a tile
    (4864, 96, 12, 16),     # 384 rows: two row blocks
])
def test_tc_paged_matches_oracle(prefix, nodes, per_depth, page):
    _paged_case(prefix, nodes, per_depth, page)


def test_tc_paged_fp16_and_batch():
    _paged_case(8192, 32, 8, 16, dtype=torch.float16, batch=2, seed=5)


def test_tc_config4_tree_shape():
    # 128 nodes over 10 depths (config 4's tree): 512 rows per KV head, four CTAs
    _paged_case(16384, 128, 13, 16, seed=7)


def test_tc_config5_batch_of_96_node_trees():
    # batch of 4 sequences with 96-node trees (config 5's per-sequence shape)
    _paged_case(6144, 96, 12, 16, batch=4, seed=8)


def test_tc_gqa_group_of_one():
    _paged_case(8192, 64, 8, 16, heads=8, kv_heads=8, seed=6)


@pytest.mark.parametrize("token_major", [False, True])
def test_tc_contiguous_cache_layouts(token_major):
    """The reference's cache buffer [B, Hkv, S_budget, D] (head-major) and a
    token-major [B, S, Hkv, D] buffer, with unused budget past the end."""
    from specverify import workloads as wl
    from specverify.runtime import verify_attention
    b, h, hkv, d, s, budget = 2, 32, 8, 128, 5000, 5200
    gen = torch.Generator().manual_seed(9)
    tree = wl.make_tree(gen, 64, 8, root=True)
    m = tree.rows
    q = (torch.randn(b, m, h, d, generator=gen) / math.sqrt(d)).bfloat16()
    kbuf = torch.randn(b, hkv, budget, d, generator=gen).bfloat16()
    vbuf = torch.randn(b, hkv, budget, d, generator=gen).bfloat16()
    kbuf[:, :, s + m:] = float("nan")     # stale budget past the live keys must never be read
    vbuf[:, :, s + m:] = float("nan")
    if token_major:
        kc = kbuf.transpose(1, 2).contiguous().cuda()
        vc = vbuf.transpose(1, 2).contiguous().cuda()
    else:
        kc = kbuf.cuda().transpose(1, 2)
        vc = vbuf.cuda().transpose(1, 2)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = verify_attention(q.cuda(), kc, vc, s, tree.keep.cuda(), return_lse=True)
    ref, ref_lse = oatt.full_masked_attention(q, kbuf[:, :, : s + m], vbuf[:, :, : s + m], tree.keep, s)
    _close(out, ref)
    _close(lse, ref_lse, atol=1e-3, rtol=1e-4)
    assert int(status.item()) == 0


def test_tc_split_counts_agree():
    from specverify import workloads as wl
    from specverify.runtime import verify_attention
    w = wl.paged_verify(prefix_len=16384, seed=4)
    outs = [verify_attention(w.q, w.k_pool, w.v_pool, w.prefix_len, w.tree.keep.cuda(), page_table=w.page_table,
                             num_splits=ns) for ns in (1, 3, 0)]
    for o in outs[1:]:
        assert (o.float() - outs[0].float()).abs().max().item() < 2e-3
