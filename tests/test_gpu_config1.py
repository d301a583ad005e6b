"""GPU parity at BASELINE config 1, end to end: verify attention, greedy
acceptance over the 128256-word vocabulary and compaction of the accepted
path, on the config's exact shapes (S = 4096 contiguous prefix, 65 tree rows
with the root, 32 / 8 heads, head_dim 128, seed 0).

The fixture ``tests/golden/config1.npz`` holds what the reference itself
computed on these inputs (``make_golden.py``: its RoPE, prefix + tree
attention + merge in fp32, and ``verify_new``); the inputs are regenerated
from the seed (``specverify.workloads.config1``) and checked against the
fixture's checksums first.  Attention runs in bf16 and is held to 2e-2
relative / 1e-3 absolute against both the reference's fp32 output and the
oracle on the bf16-rounded inputs; acceptance and the compacted rows must be
bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cuda_ok, load_golden
from oracle import acceptance as oacc
from oracle import attention as oatt

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

ATOL, RTOL = 1e-3, 2e-2


def _close(got, ref, atol=ATOL, rtol=RTOL):
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bad = err > atol + rtol * ref.abs()
    assert not bool(bad.any()), f"max abs err {err.max().item():.3e}, {int(bad.sum())} elements out of tolerance"


@pytest.fixture(scope="module")
def case():
    from specverify import workloads as wl
    z = load_golden("config1.npz")
    c = wl.config1(seed=0)
    for k in ("q_raw", "k_prefix", "v_prefix", "k_tree_raw", "v_tree", "logits"):
        assert abs(getattr(c, k).double().sum().item() - float(z[f"sum_{k}"])) < 1e-6, k
    assert int(c.draft.sum()) == int(z["sum_draft"])
    return c, z


@pytest.mark.parametrize("kernel", [0, 2, 1 | 16])   # auto (tcgen05 here), tcgen05 only, warp-MMA split-P
def test_config1_verify_accept_compact(case, kernel):
    from specverify.draft import accept, compact_kv
    from specverify.runtime import verify_attention
    c, z = case
    s, m = c.prefix_len, c.tree.rows
    hkv, d = c.k_prefix.shape[1], c.k_prefix.shape[3]
    q = torch.from_numpy(z["q"]).to(torch.bfloat16)                    # rotated by the reference
    k_tree = torch.from_numpy(z["k_tree"])
    # one layer's buffer in the reference layout [2L, B, Hkv, S_budget, D]
    buf = torch.zeros(2, 1, hkv, s + m + 8, d, dtype=torch.bfloat16)
    buf[0, :, :, :s] = c.k_prefix.to(torch.bfloat16)[0]
    buf[1, :, :, :s] = c.v_prefix.to(torch.bfloat16)[0]
    buf[0, :, :, s:s + m] = k_tree.to(torch.bfloat16)[0]
    buf[1, :, :, s:s + m] = c.v_tree.to(torch.bfloat16)[0]
    keys = buf[:, :, :, :s + m].clone()
    dbuf = buf.cuda()
    out, lse = verify_attention(q.cuda(), dbuf[0].transpose(1, 2), dbuf[1].transpose(1, 2), s,
                                c.tree.keep.cuda(), return_lse=True, kernel=kernel)
    torch.cuda.synchronize()
    # (a) the reference's own fp32 result on the unrounded inputs
    _close(out, torch.from_numpy(z["merged"]))
    # (b) the oracle on exactly the bf16 inputs the kernel read
    ref, ref_lse = oatt.full_masked_attention(q, keys[0], keys[1], c.tree.keep, s)
    _close(out, ref)
    _close(lse, ref_lse, atol=1e-3, rtol=1e-4)

    acc = accept(c.logits.cuda(), c.draft.cuda(), c.tree.parent.cuda(), c.positions.cuda(), 8)
    compact_kv([dbuf], s, acc)
    h = acc.to_host()
    assert h["best_candidate"] == list(z["best_candidate"])
    assert h["accept_length"] == int(z["accept_length"])
    assert h["next_token"] == int(z["next_token"])
    n = h["accept_length"] + 1
    want = torch.from_numpy(z["kv_rows"]).to(torch.bfloat16)
    assert torch.equal(dbuf[:, :, :, s:s + n].cpu(), want)
    # rows before the start and past the tree are untouched
    assert torch.equal(dbuf[:, :, :, :s].cpu(), buf[:, :, :, :s])
    assert torch.equal(dbuf[:, :, :, s + m:].cpu(), buf[:, :, :, s + m:])
    # the oracle's acceptance agrees
    ref_acc = oacc.accept_greedy(c.logits.numpy(), c.draft.numpy(), c.tree.parent.numpy(), c.positions.numpy(), 8)
    assert ref_acc["path"] == h["path"] and ref_acc["accept_length"] == h["accept_length"]
    assert int(z["new_len"]) == s + n
    assert np.array_equal(np.asarray(h["path"])[1:] - 1, np.asarray(z["planted"]))
