"""GPU parity: acceptance and contiguous compaction, bit-exact.

Against (a) the golden vectors the reference's own ``verify_new`` produced
and (b) the numpy oracle at the full vocabulary (128256) on seeded inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, cuda_ok, load_golden
from oracle import acceptance as oacc

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _logits_from_bits(bits):
    return torch.from_numpy(bf16_from_bits(bits)).to(torch.bfloat16)


def test_greedy_accept_and_compaction_match_reference_golden():
    from specverify.draft import accept, compact_kv
    z = load_golden("accept_greedy.npz")
    md = int(z["max_depth"])
    for c in range(6):
        g = lambda k: z[f"c{c}__{k}"]
        logits = _logits_from_bits(g("logits")).cuda()
        draft = torch.from_numpy(g("draft")).cuda()
        parent = torch.from_numpy(g("parent")).cuda()
        pos = torch.from_numpy(g("pos")).cuda()
        acc = accept(logits, draft, parent, pos, md)
        kv = torch.from_numpy(g("kv_in")).cuda()
        m = draft.numel()
        compact_kv([kv], int(g("cur_len")) - m, acc)
        h = acc.to_host()
        assert h["best_candidate"] == list(g("best_candidate")), c
        assert h["accept_length"] == int(g("accept_length")), c
        assert h["next_token"] == int(g("next_token")), c
        assert torch.equal(kv.cpu(), torch.from_numpy(g("kv_out"))), c


def test_sample_and_match_with_given_tokens_matches_golden():
    from specverify.draft import accept, compact_kv
    z = load_golden("accept_sample.npz")
    md = int(z["max_depth"])
    for c in sorted({k.split("__")[0] for k in z.files if "__" in k}):
        g = lambda k: z[f"{c}__{k}"]
        draft = torch.from_numpy(g("draft")).cuda()
        acc = accept(None, draft, torch.from_numpy(g("parent")).cuda(), torch.from_numpy(g("pos")).cuda(), md,
                     mode="given", sampled=torch.from_numpy(g("sampled")).cuda())
        kv = torch.from_numpy(g("kv_in")).cuda()
        compact_kv([kv], int(g("cur_len")) - draft.numel(), acc)
        h = acc.to_host()
        assert h["best_candidate"] == list(g("best_candidate")), c
        assert h["accept_length"] == int(g("accept_length")), c
        assert torch.equal(kv.cpu(), torch.from_numpy(g("kv_out"))), c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_full_vocab_greedy_matches_oracle(dtype):
    from specverify import workloads as wl
    from specverify.draft import accept
    for seed in range(3):
        w = wl.acceptance(seed=seed, dtype=dtype)
        acc = accept(w.logits, w.draft, w.parent, w.pos, max_depth=8)
        h = acc.to_host()
        ref = oacc.accept_greedy(w.logits.float().cpu().numpy(), w.draft.cpu().numpy(), w.parent.cpu().numpy(),
                                 w.pos.cpu().numpy(), 8)
        assert np.array_equal(acc.next_tokens.cpu().numpy(), ref["next_tokens"])
        assert h["path"] == ref["path"] and h["best_candidate"] == ref["best_candidate"]
        assert h["next_token"] == ref["next_token"]
        assert h["accept_length"] == len(w.planted)


def test_ties_nan_and_inf_follow_torch_argmax():
    from specverify.draft import accept
    v = 5000
    x = torch.randn(6, v) * 3
    x[0, 10] = x[0, 4000] = 50.0          # tie -> first
    x[1, 77] = float("nan")
    x[1, 10] = float("nan")               # first NaN wins
    x[2, :] = -float("inf")               # all -inf -> index 0
    x[3, 4999] = float("inf")
    x = x.bfloat16()
    ref = torch.argmax(x, dim=-1)
    acc = accept(x.cuda(), torch.zeros(6, dtype=torch.long, device="cuda"),
                 torch.full((5,), -1, dtype=torch.long, device="cuda"), torch.arange(6, device="cuda"), 4)
    assert torch.equal(acc.next_tokens.cpu(), ref)


def test_bad_parent_is_reported_not_trapped():
    from specverify import SpecVerifyError
    from specverify.draft import accept
    logits = torch.randn(4, 100, device="cuda").bfloat16()
    acc = accept(logits, torch.zeros(4, dtype=torch.long, device="cuda"),
                 torch.tensor([-1, 7, 0], device="cuda"), torch.arange(4, device="cuda"), 4)
    with pytest.raises(SpecVerifyError):
        acc.to_host()
    # A cycle (1 -> 2 -> 1 among draft nodes) is caught by the bounded walk.
    pr = torch.tensor([2, 0, 1], device="cuda")   # node0 parent 2, node1 parent 0, node2 parent 1
    x = torch.zeros(4, 100, device="cuda").bfloat16()
    acc = accept(x, torch.zeros(4, dtype=torch.long, device="cuda"), pr, torch.tensor([0, 9, 9, 9], device="cuda"),
                 8)
    with pytest.raises(SpecVerifyError):
        acc.to_host()


def test_gumbel_sampler_distribution():
    """Gumbel-max draws follow softmax(logits / T): chi-square over 4000 draws."""
    from specverify.draft import accept
    v, rows = 8, 400
    base = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 0.3, 1.5, -0.5])
    logits = base.repeat(rows, 1).cuda()
    counts = torch.zeros(v)
    draft = torch.zeros(rows, dtype=torch.long, device="cuda")
    parent = torch.full((rows - 1,), -1, dtype=torch.long, device="cuda")
    pos = torch.arange(rows, device="cuda")
    for t, temp in ((0, 1.0), (1, 0.7)):
        counts.zero_()
        for off in range(10):
            acc = accept(logits, draft, parent, pos, 4, mode="sample", temperature=temp, seed=1234 + t, offset=off)
            counts += torch.bincount(acc.next_tokens.cpu(), minlength=v).float()
        p = torch.softmax(base / temp, -1)
        exp = p * counts.sum()
        chi2 = float(((counts - exp) ** 2 / exp).sum())
        assert chi2 < 24.3, chi2   # 7 dof, p = 0.001
    # Same seed and offset -> same draws.
    a1 = accept(logits, draft, parent, pos, 4, mode="sample", seed=5, offset=3)
    a2 = accept(logits, draft, parent, pos, 4, mode="sample", seed=5, offset=3)
    assert torch.equal(a1.next_tokens, a2.next_tokens)


def test_verify_new_dropin_end_to_end():
    """verify_new with a stub model: same 7-tuple as the reference golden case."""
    from specverify.draft import verify_new
    z = load_golden("accept_greedy.npz")
    md = int(z["max_depth"])

    class Draft:
        use_retrieval_cache = False
        enable_bundle_scheduling = True

        def build_speculative_tree(self, hidden, input_ids, head, nodes, threshold, max_depth):
            k = 4
            return (torch.zeros(1, k, dtype=torch.long, device="cuda"), torch.arange(k, device="cuda"),
                    torch.eye(k, dtype=torch.int8, device="cuda"), torch.full((k,), -1, device="cuda"))

    class Model:
        draft_model = Draft()

        class base_model:
            lm_head = None

    for c in (1, 3):
        g = lambda k: z[f"c{c}__{k}"]
        logits = _logits_from_bits(g("logits"))[None].cuda()
        draft = torch.from_numpy(g("draft"))[None].cuda()
        kv = torch.from_numpy(g("kv_in")).cuda()
        cl = torch.full((4,), int(g("cur_len")), dtype=torch.long)
        ids, best, acc_len, nd, npos, nmask, npar = verify_new(
            torch.zeros(1, 5, dtype=torch.long, device="cuda"), logits, draft, torch.from_numpy(g("pos")).cuda(),
            torch.zeros(1, draft.shape[1], 8, device="cuda"), None, [kv], cl, torch.from_numpy(g("parent")).cuda(),
            Model(), 4, 1.0, md, None, None)
        assert best == list(g("best_candidate"))
        assert acc_len == int(g("accept_length"))
        assert int(nd[0, 0]) == int(g("next_token"))
        assert int(cl[0]) == int(g("new_len"))
        assert int(npos[0]) == int(g("root_pos"))
        assert nmask.shape == (5, 5) and ids.shape[1] == 5 + len(best)
        assert torch.equal(kv.cpu(), torch.from_numpy(g("kv_out")))
        assert Model.draft_model.last_bundle_stats["num_bundles"] > 0
