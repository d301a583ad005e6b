"""Rotary embedding + KV append on the GPU (``tv_rope_append``) against the
reference's outputs (golden fixtures) and the numpy oracle: bit-identical in
bf16, fp16 and fp32."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cuda_ok, load_golden
from oracle import rope as orope

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs CUDA")]

DT = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16, "torch.float32": torch.float32}
KIND = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}


def _dev(z, key, dtype):
    a = z[key]
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.asarray(a, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.asarray(a)).to(dtype).cuda()


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.view(torch.int32).numpy().view(np.uint32)


def _fixture_bits(z, key, dtype):
    a = np.asarray(z[key])
    if dtype == torch.bfloat16:
        return a.view(np.uint16)
    if dtype == torch.float16:
        return a.astype(np.float16).view(np.uint16)
    return a.astype(np.float32).view(np.uint32)


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


@pytest.fixture(params=["rope_bf16.npz", "rope_f16.npz", "rope_f32.npz"])
def case(request):
    z = load_golden(request.param)
    return z, DT[str(z["dtype"])]


def test_apply_rotary_pos_emb_bitwise(case):
    from specverify.runtime import apply_rotary_pos_emb
    z, dt = case
    q, k = _dev(z, "q", dt), _dev(z, "k", dt)
    cos, sin = _dev(z, "cos", dt)[None, None], _dev(z, "sin", dt)[None, None]   # the cached [1, 1, S, D] form
    pos = torch.from_numpy(z["position_ids"]).cuda()
    qe, ke = apply_rotary_pos_emb(q, k, cos, sin, pos)
    np.testing.assert_array_equal(_bits(qe), _fixture_bits(z, "q_embed", dt))
    np.testing.assert_array_equal(_bits(ke), _fixture_bits(z, "k_embed", dt))


def test_apply_rotary_pos_emb_l31_bitwise(case):
    from specverify.runtime import apply_rotary_pos_emb_L31
    z, dt = case
    q, k = _dev(z, "q", dt), _dev(z, "k", dt)
    pos = torch.from_numpy(z["position_ids"]).cuda()
    cos, sin = _dev(z, "cos", dt)[pos], _dev(z, "sin", dt)[pos]               # [B, T, D]
    q31, k31 = apply_rotary_pos_emb_L31(q, k, cos, sin)
    np.testing.assert_array_equal(_bits(q31), _fixture_bits(z, "q_l31", dt))
    np.testing.assert_array_equal(_bits(k31), _fixture_bits(z, "k_l31", dt))
    # the [B, T, heads, D] form (unsqueeze_dim=2)
    q2, k2 = apply_rotary_pos_emb_L31(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(), cos, sin,
                                      unsqueeze_dim=2)
    np.testing.assert_array_equal(_bits(q2.transpose(1, 2)), _fixture_bits(z, "q_l31", dt))


def test_rope_append_contiguous_cache_bitwise(case):
    from specverify.runtime import KVCache, rope_append
    z, dt = case
    q, k, v = _dev(z, "q", dt), _dev(z, "k", dt), _dev(z, "v", dt)
    cos, sin = _dev(z, "cos", dt)[None, None], _dev(z, "sin", dt)[None, None]
    pos = torch.from_numpy(z["position_ids"]).cuda()
    kc = KVCache(_dev(z, "k_cache_before", dt), torch.tensor(int(z["start"]), dtype=torch.long))
    vc = KVCache(_dev(z, "v_cache_before", dt), torch.tensor(int(z["start"]), dtype=torch.long))
    qe, ks, vs = rope_append(q, k, v, cos, sin, pos, kc, vc)
    np.testing.assert_array_equal(_bits(qe), _fixture_bits(z, "q_embed", dt))
    np.testing.assert_array_equal(_bits(kc.data), _fixture_bits(z, "k_cache_after", dt))
    np.testing.assert_array_equal(_bits(vc.data), _fixture_bits(z, "v_cache_after", dt))
    assert ks.shape[2] == int(z["k_states_len"]) and vs.shape[2] == int(z["v_states_len"])
    assert int(kc.current_length) == int(z["k_states_len"])


def test_rope_append_in_place_and_strided_views(case):
    """q rotated in place inside a [B, T, H * D] projection output viewed as
    [B, H, T, D] (the reference's view + transpose); k / v strided too."""
    from specverify.runtime import KVCache, rope_append
    z, dt = case
    q0, k0, v0 = _dev(z, "q", dt), _dev(z, "k", dt), _dev(z, "v", dt)
    b, h, t, d = q0.shape
    hkv = k0.shape[1]
    proj_q = q0.transpose(1, 2).reshape(b, t, h * d).clone()          # [B, T, H*D]
    proj_kv = torch.cat([k0.transpose(1, 2).reshape(b, t, hkv * d), v0.transpose(1, 2).reshape(b, t, hkv * d)], -1)
    q = proj_q.view(b, t, h, d).transpose(1, 2)
    k = proj_kv[..., :hkv * d].reshape(b, t, hkv, d).transpose(1, 2)
    v = proj_kv[..., hkv * d:].reshape(b, t, hkv, d).transpose(1, 2)
    cos, sin = _dev(z, "cos", dt)[None, None], _dev(z, "sin", dt)[None, None]
    pos = torch.from_numpy(z["position_ids"]).cuda()
    kc = KVCache(_dev(z, "k_cache_before", dt), torch.tensor(int(z["start"]), dtype=torch.long))
    vc = KVCache(_dev(z, "v_cache_before", dt), torch.tensor(int(z["start"]), dtype=torch.long))
    qe, _, _ = rope_append(q, k, v, cos, sin, pos, kc, vc, out=q)
    assert qe.data_ptr() == q.data_ptr()
    np.testing.assert_array_equal(_bits(q), _fixture_bits(z, "q_embed", dt))
    np.testing.assert_array_equal(_bits(kc.data), _fixture_bits(z, "k_cache_after", dt))
    np.testing.assert_array_equal(_bits(vc.data), _fixture_bits(z, "v_cache_after", dt))


@pytest.mark.parametrize("page_size", [16, 8])
def test_rope_append_paged_matches_oracle(case, page_size):
    from specverify.runtime import rope_append
    z, dt = case
    q, k, v = _dev(z, "q", dt), _dev(z, "k", dt), _dev(z, "v", dt)
    b, h, t, d = q.shape
    hkv = k.shape[1]
    cos, sin = _dev(z, "cos", dt)[None, None], _dev(z, "sin", dt)[None, None]
    pos = torch.from_numpy(z["position_ids"]).cuda()
    start = 37                                                        # not page aligned
    n_pages_row = (start + t + page_size - 1) // page_size
    g = torch.Generator().manual_seed(7)
    pool_pages = b * n_pages_row + 5
    perm = torch.randperm(pool_pages, generator=g)[: b * n_pages_row].view(b, n_pages_row).to(torch.int32)
    kpool = torch.randn(pool_pages, hkv, page_size, d, generator=g).to(dt).cuda()
    vpool = torch.randn(pool_pages, hkv, page_size, d, generator=g).to(dt).cuda()
    k_before, v_before = _f32(kpool), _f32(vpool)
    qe, _, _ = rope_append(q, k, v, cos, sin, pos, kpool, vpool, start=start, page_table=perm.cuda(),
                           page_size=page_size)
    kind = KIND[dt]
    qe_o, ke_o = orope.apply_rotary_pos_emb(_f32(q), _f32(k), _f32(cos[0, 0]), _f32(sin[0, 0]), z["position_ids"],
                                            kind)
    np.testing.assert_array_equal(_f32(qe), qe_o)
    np.testing.assert_array_equal(_f32(kpool), orope.paged_append(k_before, perm.numpy(), start, ke_o))
    np.testing.assert_array_equal(_f32(vpool), orope.paged_append(v_before, perm.numpy(), start, _f32(v)))


def test_rope_append_config2_shapes():
    """Llama-3.1-8B verify shapes: 32 / 8 heads, D = 128, 65 rows (root + 64
    nodes) at positions prefix + depth, appended into 16-token pages."""
    from specverify.runtime import rope_append
    g = torch.Generator().manual_seed(11)
    b, h, hkv, t, d, prefix, page = 1, 32, 8, 65, 128, 65536, 16
    q = torch.randn(b, h, t, d, generator=g).bfloat16().cuda()
    k = torch.randn(b, hkv, t, d, generator=g).bfloat16().cuda()
    v = torch.randn(b, hkv, t, d, generator=g).bfloat16().cuda()
    cos_t, sin_t = orope.rope_table(d, prefix + 16, 500000.0)
    cos = torch.from_numpy(cos_t).bfloat16().cuda()
    sin = torch.from_numpy(sin_t).bfloat16().cuda()
    depth = np.concatenate([[0], np.repeat(np.arange(1, 9), 8)])       # root, then 8 nodes per depth
    pos = torch.from_numpy(prefix - 1 + depth).view(1, t).cuda()
    # only the logical pages the new rows land in need physical pages
    n_pages = (prefix + t + page - 1) // page
    first = prefix // page
    table = torch.full((1, n_pages), -1, dtype=torch.int32)
    table[0, first:] = torch.randperm(8, generator=g)[: n_pages - first].to(torch.int32)
    kpool = torch.zeros(8, hkv, page, d, dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    qe, _, _ = rope_append(q, k, v, cos, sin, pos, kpool, vpool, start=prefix, page_table=table.cuda(),
                           page_size=page)
    qe_o, ke_o = orope.apply_rotary_pos_emb(_f32(q), _f32(k), _f32(cos), _f32(sin), pos.cpu().numpy(), "bf16")
    np.testing.assert_array_equal(_f32(qe), qe_o)
    kp = orope.paged_append(np.zeros(kpool.shape, np.float32), table.numpy(), prefix, ke_o)
    np.testing.assert_array_equal(_f32(kpool), kp)


def test_rope_append_errors():
    from specverify import SpecVerifyError
    from specverify.runtime import KVCache, apply_rotary_pos_emb, rope_append
    q = torch.randn(1, 4, 3, 64, device="cuda").bfloat16()
    k = torch.randn(1, 2, 3, 64, device="cuda").bfloat16()
    v = torch.randn(1, 2, 3, 64, device="cuda").bfloat16()
    cos = torch.randn(10, 64, device="cuda").bfloat16()
    sin = torch.randn(10, 64, device="cuda").bfloat16()
    with pytest.raises(SpecVerifyError):                               # position past the table
        apply_rotary_pos_emb(q, k, cos, sin, torch.tensor([[1, 2, 10]], device="cuda"))
    with pytest.raises(SpecVerifyError):                               # negative position
        apply_rotary_pos_emb(q, k, cos, sin, torch.tensor([[-1, 2, 3]], device="cuda"))
    kc = KVCache(torch.zeros(1, 2, 4, 64, device="cuda", dtype=torch.bfloat16), torch.tensor(2))
    vc = KVCache(torch.zeros(1, 2, 4, 64, device="cuda", dtype=torch.bfloat16), torch.tensor(2))
    with pytest.raises(SpecVerifyError):                               # cache full
        rope_append(q, k, v, cos, sin, torch.tensor([[1, 2, 3]], device="cuda"), kc, vc)
    assert int(kc.current_length) == 2
    pool = torch.zeros(4, 2, 16, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SpecVerifyError):                               # page id out of range
        rope_append(q, k, v, cos, sin, torch.tensor([[1, 2, 3]], device="cuda"), pool, pool.clone(), start=0,
                    page_table=torch.tensor([[9]], dtype=torch.int32, device="cuda"))
    with pytest.raises(SpecVerifyError):                               # mixed dtypes
        apply_rotary_pos_emb(q, k.float(), cos, sin, torch.tensor([[1, 2, 3]], device="cuda"))
    with pytest.raises(SpecVerifyError):                               # CPU tensors: no CPU path
        apply_rotary_pos_emb(q.cpu(), k.cpu(), cos.cpu(), sin.cpu(), torch.tensor([[1, 2, 3]]))
    # empty token count is a no-op
    qe, ke = apply_rotary_pos_emb(q[:, :, :0], k[:, :, :0], cos, sin, torch.zeros(1, 0, dtype=torch.long,
                                                                                    device="cuda"))
    assert qe.shape[2] == 0 and ke.shape[2] == 0


def test_rope_pair_path_on_unaligned_views(case):
    """Views that start two elements into a row are not 16-byte aligned: the
    kernel falls back to element pairs and must give the same bits."""
    from specverify.runtime import apply_rotary_pos_emb
    z, dt = case
    q0, k0 = _dev(z, "q", dt), _dev(z, "k", dt)
    b, h, t, d = q0.shape
    qb = torch.zeros(b, h, t, d + 2, dtype=dt, device="cuda")
    kb = torch.zeros(b, k0.shape[1], t, d + 2, dtype=dt, device="cuda")
    qb[..., 2:] = q0
    kb[..., 2:] = k0
    q, k = qb[..., 2:], kb[..., 2:]
    assert q.data_ptr() % 16 != 0
    cos, sin = _dev(z, "cos", dt)[None, None], _dev(z, "sin", dt)[None, None]
    pos = torch.from_numpy(z["position_ids"]).cuda()
    qe, ke = apply_rotary_pos_emb(q, k, cos, sin, pos)
    np.testing.assert_array_equal(_bits(qe), _fixture_bits(z, "q_embed", dt))
    np.testing.assert_array_equal(_bits(ke), _fixture_bits(z, "k_embed", dt))
