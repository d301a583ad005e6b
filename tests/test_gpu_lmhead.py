"""lm_head + acceptance in one pass (``tv_lmhead_accept``) against the numpy
oracle and the unfused path (logits -> ``tv_accept``).

Integer-valued hidden states and weights make every fp32 dot product exact,
whatever the accumulation order, so the logits the reference would form
(rounded to bf16 / fp16) are known exactly and the picks -- ties included --
must match bit for bit.  Gaussian inputs at the Llama-3.1-8B shapes are
checked against an fp32 GEMM up to rounding-level near-ties."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cuda_ok
from oracle import acceptance as oacc
from oracle import rope as orope

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")]

KIND = {torch.bfloat16: "bf16", torch.float16: "f16"}


def _int_problem(rows, hidden, vocab, dtype, seed=0, lo=-3, hi=3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(lo, hi + 1, (rows, hidden), generator=g).to(dtype)
    w = torch.randint(lo, hi + 1, (vocab, hidden), generator=g).to(dtype)
    exact = x.double() @ w.double().T                       # integers, exact
    logits = orope.round_to(exact.numpy().astype(np.float32), KIND[dtype])
    return x.cuda(), w.cuda(), logits


def _tree(rows, seed=1):
    """Draft tree: 8 nodes per depth below the root, parents uniform in the
    previous depth (the shape of the verify trees)."""
    rng = np.random.default_rng(seed)
    depth = np.concatenate([[0], 1 + np.arange(rows - 1) // 8])
    parent = np.empty(rows - 1, dtype=np.int64)
    for i in range(1, rows):
        d = depth[i]
        if d == 1:
            parent[i - 1] = -1
        else:
            cands = np.flatnonzero(depth == d - 1)
            parent[i - 1] = int(rng.choice(cands)) - 1      # verify_new's convention: node ids without the root
    pos = 1000 + depth
    return parent, pos, int(depth.max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hidden,vocab", [(65, 512, 5000), (1, 64, 100), (128, 128, 448), (33, 256, 225)])
def test_greedy_picks_match_oracle_exactly(dtype, rows, hidden, vocab):
    from specverify.draft.tree_verification import accept_from_hidden
    x, w, logits = _int_problem(rows, hidden, vocab, dtype)
    res = accept_from_hidden(x, w, None, None, None, 0)
    np.testing.assert_array_equal(res.next_tokens.cpu().numpy(), oacc.argmax_rows(logits))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_acceptance_on_a_planted_path_matches_oracle(dtype):
    from specverify.draft.tree_verification import accept_from_hidden
    rows, hidden, vocab = 65, 512, 3000
    x, w, logits = _int_problem(rows, hidden, vocab, dtype, seed=3)
    nxt = oacc.argmax_rows(logits)
    parent, pos, depth = _tree(rows)
    ext = oacc.parent_ext(parent, rows)
    rng = np.random.default_rng(5)
    draft = rng.integers(0, vocab, rows).astype(np.int64)
    # plant: along one root-to-leaf path each draft token equals its parent's pick
    node = rows - 1
    while node != 0:
        draft[node] = nxt[ext[node]]
        node = int(ext[node])
    ref = oacc.accept_from_next(nxt, draft, parent, pos, depth)
    assert ref["accept_length"] >= 3
    res = accept_from_hidden(x, w, torch.from_numpy(draft).cuda(), torch.from_numpy(parent).cuda(),
                             torch.from_numpy(pos).cuda(), depth)
    got = res.to_host()
    assert got["path"] == ref["path"]
    assert got["best_candidate"] == ref["best_candidate"]
    assert got["accept_length"] == ref["accept_length"]
    assert got["next_token"] == ref["next_token"]


def test_nan_logit_wins_like_torch_argmax():
    from specverify.draft.tree_verification import accept_from_hidden
    x, w, logits = _int_problem(9, 128, 700, torch.bfloat16, seed=7)
    w[500, 3] = float("nan")
    w[610, 0] = float("nan")
    res = accept_from_hidden(x, w, None, None, None, 0)
    assert res.next_tokens.cpu().tolist() == [500] * 9            # the first NaN column wins


@pytest.mark.parametrize("temperature", [1.0, 0.7])
def test_sampling_equals_unfused_path_on_the_same_logits(temperature):
    """Same seed / offset and identical rounded logits: the fused Gumbel-max
    picks equal tv_accept's sampled picks token for token."""
    from specverify.draft.tree_verification import accept, accept_from_hidden
    rows, hidden, vocab = 65, 256, 4000
    x, w, logits = _int_problem(rows, hidden, vocab, torch.bfloat16, seed=11, lo=-1, hi=1)
    lg = torch.from_numpy(logits).to(torch.bfloat16).cuda()
    parent, pos, depth = _tree(rows)
    draft = torch.zeros(rows, dtype=torch.int64)
    args = (torch.from_numpy(parent).cuda(), torch.from_numpy(pos).cuda(), depth)
    for seed, offset in [(1, 0), (12345, 7), (2 ** 40 + 3, 2 ** 33)]:
        fused = accept_from_hidden(x, w, draft.cuda(), *args, mode="sample", temperature=temperature, seed=seed,
                                   offset=offset)
        unfused = accept(lg, draft.cuda(), *args, mode="sample", temperature=temperature, seed=seed, offset=offset)
        assert torch.equal(fused.next_tokens, unfused.next_tokens)
    # different seeds draw differently
    a = accept_from_hidden(x, w, None, None, None, 0, mode="sample", seed=1)
    b = accept_from_hidden(x, w, None, None, None, 0, mode="sample", seed=2)
    assert not torch.equal(a.next_tokens, b.next_tokens)


def test_llama_shapes_match_fp32_gemm_up_to_near_ties():
    """Llama-3.1-8B lm_head: 65 rows, hidden 4096, vocab 128256, bf16."""
    from specverify.draft.tree_verification import accept_from_hidden
    g = torch.Generator(device="cuda").manual_seed(0)
    rows, hidden, vocab = 65, 4096, 128256
    x = torch.randn(rows, hidden, generator=g, device="cuda").bfloat16()
    w = (0.02 * torch.randn(vocab, hidden, generator=g, device="cuda")).bfloat16()
    res = accept_from_hidden(x, w, None, None, None, 0)
    ours = res.next_tokens
    ref32 = x.float() @ w.float().T                                 # fp32 GEMM (TF32 off by default)
    ref = ref32.bfloat16().float()
    best = ref.argmax(dim=1)
    exact = (ours == best).float().mean().item()
    # a different pick is only allowed where it is a rounding-level tie
    top = ref32.gather(1, best[:, None]).squeeze(1)
    mine = ref32.gather(1, ours[:, None]).squeeze(1)
    tol = top.abs() * 2.0 ** -7
    assert bool(((mine >= top - tol)).all()), (ours, best)
    assert exact >= 0.95


def test_errors_are_reported():
    from specverify import SpecVerifyError
    from specverify.draft.tree_verification import accept_from_hidden
    x = torch.zeros(129, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(300, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(SpecVerifyError):                 # more than 128 rows
        accept_from_hidden(x, w, None, None, None, 0)
    with pytest.raises(SpecVerifyError):                 # hidden not a multiple of 64
        accept_from_hidden(x[:4, :48].contiguous(), w[:, :48].contiguous(), None, None, None, 0)
    with pytest.raises(SpecVerifyError):                 # dtypes differ
        accept_from_hidden(x[:4], w.half(), None, None, None, 0)
    with pytest.raises(SpecVerifyError):                 # CPU tensors: no CPU path
        accept_from_hidden(x[:4].cpu(), w.cpu(), None, None, None, 0)
