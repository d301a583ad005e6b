"""Sequence-sharded verify: the host-side exchange on two CPU ``gloo`` ranks.

Each rank attends its contiguous, page-aligned shard of the prefix (the last
rank also holds the tree keys and applies the tree mask), the packed partials
go through ONE all_gather, and every rank merges them in rank order.  The
per-rank partial and the merge are the oracle's here (no GPU on this host);
the result must equal one softmax over all keys, on every rank, bit-identical
across ranks.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(0)
    b, m, h, hkv, d, prefix = 1, 12, 8, 2, 32, 200
    q = torch.randn(b, m, h, d, generator=g) / d ** 0.5
    k = torch.randn(b, hkv, prefix + m, d, generator=g)
    v = torch.randn(b, hkv, prefix + m, d, generator=g)
    keep = (torch.rand(m, m, generator=g) < 0.5).to(torch.int8)
    keep |= torch.eye(m, dtype=torch.int8)
    return q, k, v, keep, prefix


def _rank_main(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.attention import full_masked_attention, lse_merge
        from specverify.runtime.sharded import SequenceShardedVerify, shard_bounds
        q, k, v, keep, prefix = _inputs()
        m = q.shape[1]
        lo, hi = shard_bounds(prefix, world, rank, align=16)
        last = rank == world - 1
        if last:   # the last rank's keys: its prefix shard followed by the M tree keys
            ks = torch.cat([k[:, :, lo:hi], k[:, :, prefix:]], dim=2)
            vs = torch.cat([v[:, :, lo:hi], v[:, :, prefix:]], dim=2)
        else:
            ks, vs = k[:, :, lo:hi], v[:, :, lo:hi]

        def partial_fn(part, q_, k_, v_, n, bits, mlen, page_table, num_splits):
            tail = k_.shape[2] - mlen
            o, l = full_masked_attention(q_, k_, v_, keep if mlen else None, tail)
            part.o().copy_(o)
            part.lse().copy_(l)

        def merge_fn(gathered, part, world_, out_dtype, out=None, out_lse=None):
            parts_o = torch.stack([part.o(gathered[r * part.numel:(r + 1) * part.numel]) for r in range(world_)])
            parts_l = torch.stack([part.lse(gathered[r * part.numel:(r + 1) * part.numel]) for r in range(world_)])
            o, l = lse_merge(parts_o, parts_l)
            if out_lse is not None:
                out_lse.copy_(l)
            return o.to(out_dtype)

        sv = SequenceShardedVerify(partial_fn=partial_fn, merge_fn=merge_fn)
        # An int64 mask is taken as already packed (no device packing on this
        # host); the oracle partial reads the keep mask itself.
        tree = keep.to(torch.int64) if last else None
        out, lse = sv(q, ks, vs, ks.shape[2], tree, out_dtype=torch.float32, return_lse=True)
        torch.save({"out": out, "lse": lse}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_gloo_ranks_merge_to_the_full_softmax(tmp_path):
    sys.path.insert(0, str(ROOT))
    from oracle.attention import full_masked_attention
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    q, k, v, keep, prefix = _inputs()
    ref_o, ref_l = full_masked_attention(q, k, v, keep, prefix)
    r0 = torch.load(tmp_path / "rank0.pt")
    r1 = torch.load(tmp_path / "rank1.pt")
    assert torch.equal(r0["out"], r1["out"]) and torch.equal(r0["lse"], r1["lse"])
    torch.testing.assert_close(r0["out"], ref_o, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(r0["lse"], ref_l, rtol=1e-5, atol=1e-5)


def test_shard_bounds_cover_and_align():
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    from specverify.runtime.sharded import shard_bounds
    for total in (0, 1, 15, 16, 200, 65536, 131072 + 5):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r, align=16) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b_), (c, _) in zip(spans, spans[1:]):
                assert b_ == c
            for lo, hi in spans:
                if hi > lo:   # non-empty shards start on a page and end on one (or at the end)
                    assert lo % 16 == 0 and (hi % 16 == 0 or hi == total)
