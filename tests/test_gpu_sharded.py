"""Sequence-sharded verify attention on two GPUs (skipped with fewer).

Each rank attends its page-aligned shard of a paged prefix (the last rank
also the tree keys under the bitmask) and the partials are exchanged -- over
NVLink peer memory (the default) or one NCCL all_gather -- and merged on
every rank.  The merged output must meet the 2e-2 / 1e-3 bar against the
fp32 oracle on the whole cache, match the single-GPU kernel within bf16
rounding, be identical on every rank and stable over repeated steps (the
peer path alternates its two buffer slots).
"""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from conftest import cuda_ok

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from specverify import workloads as wl
        from specverify.runtime import attention, pack_tree_mask
        from specverify.runtime import sharded as sh
        w = wl.paged_verify(prefix_len=8192, nodes=64, per_depth=8, seed=3, device=dev)
        bits = pack_tree_mask(w.tree.keep.to(dev))
        m, page = w.tree.rows, w.page_size
        npp = w.prefix_len // page
        lo, hi = sh.shard_bounds(npp, world, rank)
        last = rank == world - 1
        tbl = w.page_table[:, lo:hi]
        if last:
            tbl = torch.cat([tbl, w.page_table[:, npp:]], dim=1)
        tbl = tbl.contiguous()
        shard_len = (hi - lo) * page + (m if last else 0)
        ref = torch.empty_like(w.q)
        ref_lse = torch.empty(w.q.shape[:3], device=dev)
        attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
                  mask_len=m, out=ref, lse=ref_lse)
        res = {"ref": ref.cpu(), "ref_lse": ref_lse.cpu()}
        if rank == 0:
            k, v = w.contiguous_kv(0)
            res.update(q=w.q.cpu(), k=k.cpu(), v=v.cpu(), keep=w.tree.keep, prefix_len=w.prefix_len)
        for mode in ("peer", "owner", "nccl"):
            ver = sh.SequenceShardedVerify(exchange="nccl" if mode == "nccl" else "peer",
                                           peer_mode="owner" if mode == "owner" else "push")
            outs = [ver(w.q, w.k_pool, w.v_pool, shard_len, bits if last else None, page_table=tbl, return_lse=True)
                    for _ in range(5)]
            torch.cuda.synchronize()
            res[mode] = [(o.cpu(), l.cpu()) for o, l in outs]
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two CUDA devices")
@pytest.mark.timeout(600)
def test_sharded_exchanges_match_single_gpu(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(world)]
    ref, ref_lse = r[0]["ref"].float(), r[0]["ref_lse"]
    from oracle import attention as oatt
    q, k, v = r[0]["q"], r[0]["k"], r[0]["v"]
    anchor, anchor_lse = oatt.full_masked_attention(q, k.permute(1, 0, 2)[None], v.permute(1, 0, 2)[None],
                                                    r[0]["keep"], r[0]["prefix_len"])
    for mode in ("peer", "owner", "nccl"):
        first_o, first_l = r[0][mode][0]
        for rank in range(world):
            for o, l in r[rank][mode]:
                assert torch.equal(o, first_o) and torch.equal(l, first_l), (mode, rank)
        assert torch.isfinite(first_o.float()).all()
        # the north star's bar against the fp32 oracle: 2e-2 relative / 1e-3 absolute
        err = (first_o.float() - anchor).abs()
        assert bool((err <= 1e-3 + 2e-2 * anchor.abs()).all()), (mode, err.max().item())
        assert (first_l - anchor_lse).abs().max().item() < 1e-3, mode
        # and the single-GPU kernel on the whole cache: the same partial algebra
        torch.testing.assert_close(first_l, ref_lse, rtol=1e-5, atol=1e-5)
        assert (first_o.float() - ref).abs().max().item() < 2e-3
    # both NVLink modes run the same merge in rank order: identical bits
    assert torch.equal(r[0]["peer"][0][0], r[0]["owner"][0][0]) and torch.equal(r[0]["peer"][0][1], r[0]["owner"][0][1])
    # both exchanges merge the same partials with the same algebra
    torch.testing.assert_close(r[0]["peer"][0][0].float(), r[0]["nccl"][0][0].float(), rtol=0, atol=2e-3)


def _one_gpu_request(prefix_len, seed):
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    from specverify import workloads as wl
    from specverify.runtime import pack_tree_mask
    w = wl.paged_verify(prefix_len=prefix_len, nodes=64, per_depth=8, seed=seed, device=torch.device("cuda", 0))
    return w, pack_tree_mask(w.tree.keep.cuda())


def _sharded_call(w, bits, bases, world, rank, status=None, num_splits=0, kernel=0, exchange_bytes=None):
    import ctypes
    from specverify import _lib
    from specverify.runtime.tree_attention import attn_args
    out = torch.empty_like(w.q)
    lse = torch.empty(w.q.shape[:3], device="cuda")
    a, _ = attn_args(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
                     mask_len=w.tree.rows, out=out, lse=lse, status=status, num_splits=num_splits, kernel=kernel)
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.tv_verify_attn_sharded_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace")
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), need.value
    arr = (ctypes.c_void_p * world)(*bases)
    if exchange_bytes is None:
        n = ctypes.c_int64(0)
        _lib.check(lib.tv_sharded_exchange_bytes(world, w.q.shape[0] * w.q.shape[1] * w.q.shape[2], w.q.shape[3],
                                                 ctypes.byref(n)), "exchange bytes")
        exchange_bytes = n.value
    _lib.check(lib.tv_verify_attn_sharded(ctypes.byref(a), world, rank, arr, exchange_bytes,
                                          _lib.stream_ptr(out.device)), "tv_verify_attn_sharded")
    torch.cuda.synchronize()
    return out, lse


def _exchange_buffer(world, rows, d):
    import ctypes
    from specverify import _lib
    n = ctypes.c_int64(0)
    _lib.check(_lib.load().tv_sharded_exchange_bytes(world, rows, d, ctypes.byref(n)), "exchange bytes")
    return torch.zeros(n.value, dtype=torch.uint8, device="cuda")


@pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")
@pytest.mark.parametrize("num_splits", [0, 1])             # planned splits; one split (partial, not final)
@pytest.mark.parametrize("prefix_len", [1024, 8192])       # warp-MMA kernel, tensor-memory kernel
def test_sharded_entry_one_rank_equals_verify_attn(prefix_len, num_splits):
    """world = 1: the fused combine + exchange + merge kernel reduces to the
    split combine; five steps walk both slots and the step counter."""
    from specverify.runtime import attention
    w, bits = _one_gpu_request(prefix_len, seed=5)
    b, m, h, d = w.q.shape
    ref = torch.empty_like(w.q)
    ref_lse = torch.empty(w.q.shape[:3], device="cuda")
    attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
              mask_len=m, out=ref, lse=ref_lse, num_splits=num_splits)
    buf = _exchange_buffer(1, b * m * h, d)
    for step in range(5):
        out, lse = _sharded_call(w, bits, [buf.data_ptr()], 1, 0, num_splits=num_splits)
        assert torch.equal(out, ref) and torch.equal(lse, ref_lse), step


@pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")
@pytest.mark.parametrize("mode", [32, 64])                  # owner exchange, push to all
def test_sharded_entry_gives_up_on_a_silent_peer(mode):
    """Two ranks, but the 'peer' buffer is local memory that no rank ever
    writes: every wait runs out (2 s), the status word reads 8 and the
    outputs are NaN instead of a silent one-rank result.  In owner mode
    rank 0 owns half the row blocks (waits for the peer's partials) and
    waits for the peer's final rows on the other half."""
    w, bits = _one_gpu_request(1024, seed=6)
    b, m, h, d = w.q.shape
    mine = _exchange_buffer(2, b * m * h, d)
    silent = _exchange_buffer(2, b * m * h, d)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = _sharded_call(w, bits, [mine.data_ptr(), silent.data_ptr()], 2, 0, status=status, kernel=mode)
    assert int(status.item()) == 8
    assert torch.isnan(out.float()).all() and torch.isnan(lse).all()


def _slot_layout(world, rows, d):
    """Byte offsets of one exchange-buffer slot: [world][rows][d] partial O
    words, [world][rows] partial LSE words, then the final rows (8-byte words:
    fp32 bits low, step number high)."""
    a = lambda x: (x + 255) & ~255
    lse = a(world * rows * d * 8)
    fin = lse + a(world * rows * 8)
    fin_lse = fin + a(rows * d * 8)
    return {"slot": fin_lse + a(rows * 8), "lse": lse}


@pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")
def test_sharded_entry_exchanges_step_tagged_words():
    """Push mode, rank 0 of 2 on one GPU.  The 'peer' has already posted its
    partial for step 1 (words tagged 1 in slot 1, LSE -inf: nothing to add),
    so the merge must give the one-rank result bit for bit; and rank 0's own
    partial must have landed in the peer's buffer as words of step 1 (slot 1)
    whose LSE halves equal the one-rank LSE."""
    from specverify.runtime import attention
    w, bits = _one_gpu_request(1024, seed=7)
    b, m, h, d = w.q.shape
    hkv = w.k_pool.shape[1]
    rows = b * m * h
    ref = torch.empty_like(w.q)
    ref_lse = torch.empty(w.q.shape[:3], device="cuda")
    attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
              mask_len=m, out=ref, lse=ref_lse)
    L = _slot_layout(2, rows, d)
    mine = _exchange_buffer(2, rows, d)
    peer = _exchange_buffer(2, rows, d)
    tag = 1 << 32                                                          # step 1
    words = mine.view(torch.int64)
    o0 = L["slot"] // 8                                                    # step 1 uses slot 1
    words[o0 + rows * d:o0 + 2 * rows * d] = tag                           # rank 1's O: 0.0
    l0 = (L["slot"] + L["lse"]) // 8
    words[l0 + rows:l0 + 2 * rows] = tag | 0xFF800000                      # rank 1's LSE: -inf
    out, lse = _sharded_call(w, bits, [mine.data_ptr(), peer.data_ptr()], 2, 0, kernel=64)
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
    pw = peer.view(torch.int64)
    o1 = L["slot"] // 8                                                    # slot 1, rank 0's region
    assert torch.equal(pw[o1:o1 + rows * d] >> 32, torch.ones(rows * d, dtype=torch.int64, device="cuda"))
    l1 = (L["slot"] + L["lse"]) // 8
    assert torch.equal(pw[l1:l1 + rows] >> 32, torch.ones(rows, dtype=torch.int64, device="cuda"))
    lo = peer.view(torch.int32)[2 * l1:2 * (l1 + rows)].view(rows, 2)[:, 0].contiguous().view(torch.float32)
    # the kernel's row order: (b, kv head, node, group member)
    want = ref_lse.view(b, m, hkv, h // hkv).permute(0, 2, 1, 3).reshape(-1)
    assert torch.equal(lo, want)


@pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")
def test_sharded_entry_lagging_rank_flags_overwritten_words():
    """Push mode, two ranks emulated on one GPU with two local buffers, run
    one after the other.  Rank 0 runs three steps while rank 1 runs none:
    every wait of rank 0 times out (status 8, NaN), and its step-3 partial
    overwrites slot 1 in rank 1's buffer.  When rank 1 then runs its step 1
    (slot 1), the words carry step 3: it must flag its rows (status 8, NaN)
    at once instead of merging step 3's values as step 1's."""
    w, bits = _one_gpu_request(1024, seed=8)
    b, m, h, d = w.q.shape
    rows = b * m * h
    buf0 = _exchange_buffer(2, rows, d)
    buf1 = _exchange_buffer(2, rows, d)
    bases = [buf0.data_ptr(), buf1.data_ptr()]
    for step in range(3):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out, _ = _sharded_call(w, bits, bases, 2, 0, status=status, kernel=64)
        assert int(status.item()) == 8 and torch.isnan(out.float()).all(), step
    L = _slot_layout(2, rows, d)
    tags = buf1.view(torch.int64)[L["slot"] // 8:L["slot"] // 8 + rows * d] >> 32
    assert bool((tags == 3).all())                     # rank 0's step-3 words sit in slot 1
    import time
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    out, lse = _sharded_call(w, bits, bases, 2, 1, status=status, kernel=64)
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 8
    assert torch.isnan(out.float()).all() and torch.isnan(lse).all()
    assert elapsed < 1.5, f"the later step should be seen at once, not after the 2 s deadline ({elapsed:.2f} s)"


@pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")
def test_sharded_entry_owner_mode_hands_back_16bit_final_rows():
    """Owner mode, rank 0 of 2 on one GPU.  The 'peer' has posted, for step 1,
    its partial of the row blocks rank 0 owns (LSE -inf: nothing to add) and
    the final rows of the blocks it owns itself (two bf16 values + the step
    per word, as the reference result's rows).  Rank 0 must then write the
    one-rank result bit for bit on every row, and hand its own blocks' final
    rows to the peer in the same 16-bit word format."""
    from specverify.runtime import attention
    w, bits = _one_gpu_request(1024, seed=9)
    b, m, h, d = w.q.shape
    hkv = w.k_pool.shape[1]
    g = h // hkv
    rows = b * m * h
    ref = torch.empty_like(w.q)
    ref_lse = torch.empty(w.q.shape[:3], device="cuda")
    attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
              mask_len=m, out=ref, lse=ref_lse)
    # the kernel's row order (b, kv head, node, group member)
    ref_rows = ref.view(b, m, hkv, g, d).permute(0, 2, 1, 3, 4).reshape(rows, d)
    lse_rows = ref_lse.view(b, m, hkv, g).permute(0, 2, 1, 3).reshape(rows)
    rpb = 128 // (d // 4)                                   # rows per row block of the exchange kernel
    nrb = -(-rows // rpb)
    own = torch.tensor([(r // rpb) * 2 // nrb == 0 for r in range(rows)], device="cuda")
    a = lambda x: (x + 255) & ~255
    L = _slot_layout(2, rows, d)
    slot = L["slot"]                                         # step 1 uses slot 1
    fin = slot + a(2 * rows * d * 8) + a(2 * rows * 8)
    fin_lse = fin + a(rows * d * 8)
    mine = _exchange_buffer(2, rows, d)
    peer = _exchange_buffer(2, rows, d)
    tag = 1 << 32
    words = mine.view(torch.int64)
    o1 = slot // 8 + rows * d                                # rank 1's partial region
    words[o1:o1 + rows * d] = tag
    l1 = (slot + L["lse"]) // 8 + rows
    words[l1:l1 + rows] = tag | 0xFF800000
    pairs = ref_rows.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF   # [rows, d / 2]
    fw = words[fin // 8:fin // 8 + rows * d // 2].view(rows, d // 2)
    fw[~own] = (pairs | tag)[~own]
    lw = words[fin_lse // 8:fin_lse // 8 + rows]
    lse_bits = lse_rows.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    lw[~own] = (lse_bits | tag)[~own]
    out, lse = _sharded_call(w, bits, [mine.data_ptr(), peer.data_ptr()], 2, 0, kernel=32)
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
    pw = peer.view(torch.int64)
    got = pw[fin // 8:fin // 8 + rows * d // 2].view(rows, d // 2)
    assert torch.equal(got[own], (pairs | tag)[own])
    got_l = pw[fin_lse // 8:fin_lse // 8 + rows]
    assert torch.equal(got_l[own], (lse_bits | tag)[own])
