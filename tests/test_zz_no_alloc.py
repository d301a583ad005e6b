"""tv_verify_attn_static: the same verify attention with its split partials in
a fixed device array of the library instead of a caller workspace.

Collected last on purpose (file name), so it also runs after every other GPU
test in one session; it passes on its own as well.
"""
import contextlib

import pytest
import torch

from conftest import cuda_ok

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def _static_entry():
    """Route the runtime's attention call through the static-scratch entry."""
    from specverify import _lib
    lib = _lib.load()
    orig = lib.tv_verify_attn
    lib.tv_verify_attn = lib.tv_verify_attn_static
    try:
        yield
    finally:
        lib.tv_verify_attn = orig


def _case(seed=0, device=0):
    from specverify import workloads as wl
    from specverify.runtime import pack_tree_mask
    dev = torch.device("cuda", device)
    w = wl.paged_verify(prefix_len=8192, nodes=64, per_depth=8, seed=seed, device=dev)
    bits = pack_tree_mask(w.tree.keep.to(dev))
    return w, bits


def _run(w, bits, **kw):
    from specverify.runtime import attention
    out = torch.empty_like(w.q)
    lse = torch.empty(w.q.shape[:3], device=w.q.device)
    attention(w.q, w.k_pool, w.v_pool, num_keys=w.num_keys, page_table=w.page_table, mask_bits=bits,
              mask_len=w.tree.rows, out=out, lse=lse, **kw)
    return out, lse


@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_static_scratch_matches_workspace_entry_twice():
    w, bits = _case()
    ref_out, ref_lse = _run(w, bits)
    with _static_entry():
        out1, lse1 = _run(w, bits)
        out2, lse2 = _run(w, bits)
    torch.cuda.synchronize()
    # Same kernels, same split plan: bit-identical to the workspace entry.
    assert torch.equal(out1, ref_out) and torch.equal(lse1, ref_lse)
    assert torch.equal(out2, ref_out) and torch.equal(lse2, ref_lse)
    assert torch.isfinite(ref_out.float()).all()


@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_static_scratch_uses_splits_and_rejects_oversize():
    from specverify import _lib
    w, bits = _case(seed=1)
    # The default plan for this case splits the keys, so the scratch is used.
    ref_out, _ = _run(w, bits)
    with _static_entry():
        out, _ = _run(w, bits)
        # One split per 128-key tile (65) over 8 x 256 rows: 68 MB of partials.
        with pytest.raises(_lib.SpecVerifyError) as e:
            _run(w, bits, num_splits=256)
    assert e.value.status == -5   # TV_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)


@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two CUDA devices")
def test_static_scratch_on_a_second_device():
    """The array's address is resolved per device, with that device current:
    on device 1 the static entry must use device 1's copy of the array and
    match the workspace entry there, twice in a row."""
    with torch.cuda.device(1):
        w, bits = _case(seed=2, device=1)
        ref_out, ref_lse = _run(w, bits)
        with _static_entry():
            out1, lse1 = _run(w, bits)
            out2, lse2 = _run(w, bits)
        torch.cuda.synchronize(1)
    assert torch.equal(out1, ref_out) and torch.equal(lse1, ref_lse)
    assert torch.equal(out2, ref_out) and torch.equal(lse2, ref_lse)
