"""Final draft-tree build on the GPU (``tv_tree_finalize``) against the
reference's ``DraftTree.update`` outputs (golden fixtures) and the numpy
oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cuda_ok, load_golden
from oracle import tree as otree

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")]


def _np(t):
    return t.detach().cpu().numpy()


def _cases():
    z = load_golden("tree_final.npz")
    for c in range(int(z["cases"])):
        p = f"c{c}_"
        yield {k[len(p):]: z[k] for k in z.files if k.startswith(p)}


def _run(case, **kw):
    from specverify.runtime.draft_tree import finalize_tree
    return finalize_tree(torch.from_numpy(case["top_index"]).cuda(), torch.from_numpy(case["parents_matrix"]).cuda(),
                         torch.from_numpy(case["input_ids_matrix"]).cuda(), int(case["depth"]), int(case["nnodes"]),
                         **kw)


@pytest.mark.parametrize("ci", range(4))
def test_matches_oracle_in_top_k_order(ci):
    case = list(_cases())[ci]
    out = _run(case)
    ref = otree.finalize(case["top_index"], case["parents_matrix"], case["input_ids_matrix"], int(case["depth"]),
                         int(case["nnodes"]))
    for key in ("input_ids", "position_ids", "parent_last", "attention_mask"):
        np.testing.assert_array_equal(_np(out[key]), ref[key], err_msg=key)
    bits = otree.pack_bits(otree.verify_mask(ref["attention_mask"]))
    np.testing.assert_array_equal(_np(out["mask_bits"]).view(np.uint64), bits)


@pytest.mark.parametrize("ci", range(4))
def test_matches_reference_up_to_equal_depth_order(ci):
    """The reference's order among equal depths came from its sort; relabel
    our nodes through their (depth, column) identity and compare everything."""
    case = list(_cases())[ci]
    out = _run(case)
    d, n = int(case["depth"]), int(case["nnodes"])
    ours = otree.finalize(case["top_index"], case["parents_matrix"], case["input_ids_matrix"], d, n)
    theirs = otree.finalize(case["top_index"], case["parents_matrix"], case["input_ids_matrix"], d, n,
                            order=case["ref_order"])
    where = {(int(r), int(c)): i for i, (r, c) in enumerate(zip(theirs["rows"], theirs["cols"]))}
    perm = np.array([where[(int(r), int(c))] for r, c in zip(ours["rows"], ours["cols"])])   # ours -> theirs
    k = perm.size
    ids, pos, par, mask = (_np(out[x]) for x in ("input_ids", "position_ids", "parent_last", "attention_mask"))
    np.testing.assert_array_equal(ids, case["input_ids"][perm])
    np.testing.assert_array_equal(pos, case["position_ids"][perm])
    mapped_par = np.where(par >= 0, perm[np.clip(par, 0, k - 1)], -1)
    np.testing.assert_array_equal(mapped_par, case["parent_last"][perm])
    np.testing.assert_array_equal(mask, case["attention_mask"][np.ix_(perm, perm)])


def test_bits_equal_pack_tree_mask_of_the_prepended_mask():
    from specverify.runtime import pack_tree_mask
    case = list(_cases())[1]
    out = _run(case)
    vm = otree.verify_mask(_np(out["attention_mask"]))
    packed = pack_tree_mask(torch.from_numpy(vm).cuda())
    np.testing.assert_array_equal(_np(packed).reshape(out["mask_bits"].shape), _np(out["mask_bits"]))


def _random_state(nnodes, depth, seed):
    rng = np.random.default_rng(seed)
    pm = np.full((depth + 2, nnodes), -1, dtype=np.int64)
    pm[0] = np.arange(nnodes)
    for r in range(1, depth):
        pm[r] = rng.integers(0, nnodes, nnodes)
    im = rng.integers(0, 32000, (depth + 2, nnodes)).astype(np.int64)
    top = rng.choice(depth * nnodes, size=nnodes, replace=False).astype(np.int64)
    return top, pm, im


@pytest.mark.parametrize("nnodes,depth", [(128, 10), (64, 16), (1, 1), (200, 3)])
def test_random_states_match_oracle(nnodes, depth):
    from specverify.runtime.draft_tree import finalize_tree
    top, pm, im = _random_state(nnodes, depth, seed=nnodes * 31 + depth)
    out = finalize_tree(torch.from_numpy(top).cuda(), torch.from_numpy(pm).cuda(), torch.from_numpy(im).cuda(),
                        depth, nnodes)
    ref = otree.finalize(top, pm[:depth], im[:depth], depth, nnodes)
    for key in ("input_ids", "position_ids", "parent_last", "attention_mask"):
        np.testing.assert_array_equal(_np(out[key]), ref[key], err_msg=key)
    np.testing.assert_array_equal(_np(out["mask_bits"]).view(np.uint64),
                                  otree.pack_bits(otree.verify_mask(ref["attention_mask"])))


def test_d2t_mapping_and_errors():
    from specverify import SpecVerifyError
    from specverify.runtime.draft_tree import finalize_tree
    top, pm, im = _random_state(16, 4, seed=3)
    im = im % 100
    d2t = torch.arange(100, dtype=torch.int64).cuda() * 7
    out = finalize_tree(torch.from_numpy(top).cuda(), torch.from_numpy(pm).cuda(), torch.from_numpy(im).cuda(), 4,
                        16, d2t=d2t)
    ref = otree.finalize(top, pm[:4], im[:4], 4, 16)
    np.testing.assert_array_equal(_np(out["input_ids"]), ref["input_ids"] * 8)      # id + 7 * id
    bad = top.copy()
    bad[3] = 4 * 16                                                                 # past the last depth
    with pytest.raises(SpecVerifyError):
        finalize_tree(torch.from_numpy(bad).cuda(), torch.from_numpy(pm).cuda(), torch.from_numpy(im).cuda(), 4, 16)
    dup = top.copy()
    dup[5] = dup[2]
    with pytest.raises(SpecVerifyError):
        finalize_tree(torch.from_numpy(dup).cuda(), torch.from_numpy(pm).cuda(), torch.from_numpy(im).cuda(), 4, 16)
