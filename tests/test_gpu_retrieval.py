"""Draft-side chunk retrieval on the GPU (``tv_chunk_select`` +
``tv_gather_rows``) against the reference's
``DraftNetwork._select_working_cache_from_chunks`` (golden fixtures) and the
numpy oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cuda_ok, load_golden
from oracle import retrieval as oret

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")]


def _cases():
    z = load_golden("retrieval.npz")
    for c in range(int(z["cases"])):
        p = f"c{c}_"
        yield {k[len(p):]: z[k] for k in z.files if k.startswith(p)}


@pytest.mark.parametrize("ci", range(4))
def test_selection_and_union_match_reference(ci):
    from specverify.draft.retrieval import select_chunks
    case = list(_cases())[ci]
    sel, idx, count = select_chunks(torch.from_numpy(case["attn"]).cuda(), torch.from_numpy(case["starts"]).cuda(),
                                    torch.from_numpy(case["ends"]).cuda(), int(case["top_k"]), int(case["L"]))
    np.testing.assert_array_equal(sel.cpu().numpy(), case["selected"])
    n = int(count.item())
    assert n == int(case["n_ret"])
    ref = oret.union_indices(case["starts"], case["ends"], case["selected"], int(case["L"]))
    np.testing.assert_array_equal(idx[:n].cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci", range(4))
def test_working_cache_matches_reference(ci, dtype):
    from specverify.draft.retrieval import select_working_cache
    case = list(_cases())[ci]
    layers = int(case["layers"])
    full = [(torch.from_numpy(case[f"full_k{li}"].astype(np.float32)).to(dtype).cuda(),
             torch.from_numpy(case[f"full_v{li}"].astype(np.float32)).to(dtype).cuda()) for li in range(layers)]
    working, ids, evicted = select_working_cache(full, torch.from_numpy(case["attn"]).cuda(),
                                                 torch.from_numpy(case["starts"]).cuda(),
                                                 torch.from_numpy(case["ends"]).cuda(), int(case["top_k"]),
                                                 int(case["L"]))
    assert ids == case["selected"].tolist()
    assert evicted == int(case["evicted"])
    for li, (wk, wv) in enumerate(working):
        # values are k / 16 with |k| < 256: exact in every dtype
        np.testing.assert_array_equal(wk.float().cpu().numpy(), case[f"work_k{li}"].astype(np.float32))
        np.testing.assert_array_equal(wv.float().cpu().numpy(), case[f"work_v{li}"].astype(np.float32))


def test_random_scores_nan_ties_and_unsorted_overlapping_chunks():
    from specverify.draft.retrieval import select_chunks
    rng = np.random.default_rng(0)
    length = 5000
    starts = rng.integers(0, length - 10, 300)
    ends = np.minimum(starts + rng.integers(1, 120, 300), length)
    attn = rng.random(length).astype(np.float32)
    # a NaN: under the reference's prefix sums every chunk ending after it
    # scores NaN, and NaN scores are taken first (smallest id first)
    attn[starts[17]:ends[17]] = np.nan
    nan_chunks = np.flatnonzero(np.isnan(oret.chunk_scores(attn, starts, ends)))
    assert nan_chunks.size > 1
    for k in (1, 9, 40, 300):
        sel, idx, count = select_chunks(torch.from_numpy(attn).cuda(), torch.from_numpy(starts).cuda(),
                                        torch.from_numpy(ends).cuda(), k, length)
        ref_sel, ref_idx = oret.select(attn, starts, ends, k, length)
        np.testing.assert_array_equal(sel.cpu().numpy(), ref_sel)
        np.testing.assert_array_equal(idx[:int(count.item())].cpu().numpy(), ref_idx)
        assert set(nan_chunks[:k].tolist()) <= set(sel.cpu().tolist())
    # an infinity: chunks ending after it score +inf, chunks starting after it NaN (inf - inf), as the
    # reference's prefix sums give
    inf = rng.random(length).astype(np.float32)
    inf[2500] = np.inf
    st2 = np.arange(0, length, 250)
    en2 = np.minimum(st2 + 250, length)
    for k in (3, 12):
        sel, idx, count = select_chunks(torch.from_numpy(inf).cuda(), torch.from_numpy(st2).cuda(),
                                        torch.from_numpy(en2).cuda(), k, length)
        ref_sel, ref_idx = oret.select(inf, st2, en2, k, length)
        np.testing.assert_array_equal(sel.cpu().numpy(), ref_sel)
    # equal scores: the smaller ids win
    flat = np.full(length, 0.25, dtype=np.float32)
    st = np.arange(0, length, 100)
    sel, _, _ = select_chunks(torch.from_numpy(flat).cuda(), torch.from_numpy(st).cuda(),
                              torch.from_numpy(np.minimum(st + 100, length)).cuda(), 5, length)
    assert sel.cpu().tolist() == [0, 1, 2, 3, 4]


def test_errors():
    from specverify import SpecVerifyError
    from specverify.draft.retrieval import select_chunks
    a = torch.rand(100, device="cuda")
    with pytest.raises(SpecVerifyError):                 # negative bound
        select_chunks(a, torch.tensor([-5, 10], device="cuda"), torch.tensor([10, 20], device="cuda"), 2, 100)
    with pytest.raises(SpecVerifyError):                 # more chunks than one CTA takes
        select_chunks(a, torch.zeros(3000, dtype=torch.long, device="cuda"),
                      torch.ones(3000, dtype=torch.long, device="cuda"), 2, 100)


def test_config5_sizes_match_index_select():
    """262144 draft tokens in 2048-token chunks, top 32 chunks (65536
    tokens) gathered from one draft layer's K / V (8 heads, head_dim 128)."""
    from specverify.draft.retrieval import select_working_cache
    g = torch.Generator(device="cuda").manual_seed(0)
    length, cs, k = 262144, 2048, 32
    attn = torch.rand(length, generator=g, device="cuda")
    starts = torch.arange(0, length, cs, device="cuda")
    ends = starts + cs
    fk = torch.randn(1, 8, length, 128, generator=g, device="cuda").bfloat16()
    fv = torch.randn(1, 8, length, 128, generator=g, device="cuda").bfloat16()
    working, ids, evicted = select_working_cache([(fk, fv)], attn, starts, ends, k, length)
    ref_sel, ref_idx = oret.select(attn.cpu().numpy(), starts.cpu().numpy(), ends.cpu().numpy(), k, length)
    assert ids == ref_sel.tolist() and evicted == length - ref_idx.size == length - k * cs
    ridx = torch.from_numpy(ref_idx).cuda()
    assert torch.equal(working[0][0], fk.index_select(2, ridx))
    assert torch.equal(working[0][1], fv.index_select(2, ridx))
