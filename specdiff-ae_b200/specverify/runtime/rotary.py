"""Rotary embedding and KV-cache append: the step right before verify attention.

Drop-ins for ``diffspec/runtime/llama_target_model.py``:

* ``apply_rotary_pos_emb(q, k, cos, sin, position_ids)`` (:429-449) -- the
  cached ``[1, 1, S, D]`` cos/sin tables gathered by ``position_ids``;
* ``apply_rotary_pos_emb_L31(q, k, cos, sin, position_ids=None,
  unsqueeze_dim=1)`` (:452-474) -- per-token ``[B, T, D]`` tables as
  ``LlamaRotaryEmbedding_L31`` returns them;

and the fused form of what ``LlamaAttention.forward`` does with them on the
verify branch (:765-783): rotate q and k, then ``past_key_value[0].cat(k)``
and ``past_key_value[1].cat(v)`` (``cache_state.py:52-66``) --
:func:`rope_append`, one launch that writes the rotated k and v straight into
the contiguous cache or into the pages of a paged pool.

The kernel (``tv_rope_append``) rounds every product and the sum to the
element type, as torch's element-wise ops do in the reference, so q_embed,
k_embed and the cache contents are bit-identical to the reference's given the
same cos / sin tensors.  CUDA tensors only; there is no CPU path.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from .. import _lib


def _bhtd(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.dim() != 4:
        raise _lib.SpecVerifyError(-1, f"{name} must be [B, heads, T, D], got {tuple(x.shape)}")
    return x if x.stride(3) == 1 else x.contiguous()


def _table(cos: torch.Tensor, sin: torch.Tensor, position_ids: Optional[torch.Tensor], batch: int, tokens: int):
    """(cos, sin, cs_sb, cs_sr, cs_rows, pos, pos_sb) for the kernel."""
    if cos.shape != sin.shape or cos.dtype != sin.dtype or cos.stride() != sin.stride():
        raise _lib.SpecVerifyError(-1, "cos and sin must have the same shape, dtype and strides")
    if position_ids is not None:
        # cached table [1, 1, S, D] / [S, D], gathered by position ids [B|1, T] / [T]
        tab = cos.reshape(-1, cos.shape[-1]) if cos.dim() != 2 else cos
        stab = sin.reshape(-1, sin.shape[-1]) if sin.dim() != 2 else sin
        if tab.stride(-1) != 1:
            tab, stab = tab.contiguous(), stab.contiguous()
        pos = position_ids
        if pos.dim() == 1:
            pos = pos.unsqueeze(0)
        if pos.dim() != 2 or pos.shape[-1] != tokens or pos.shape[0] not in (1, batch):
            raise _lib.SpecVerifyError(-1, f"position_ids {tuple(position_ids.shape)} vs [B={batch}, T={tokens}]")
        pos = pos.to(torch.int64)
        if pos.stride(-1) != 1:
            pos = pos.contiguous()
        pos_sb = pos.stride(0) if pos.shape[0] == batch and batch > 1 else 0
        return tab, stab, 0, tab.stride(0), tab.shape[0], pos, pos_sb
    # per-token tables [B|1, T, D]
    c, s = cos, sin
    if c.dim() == 2:
        c, s = c.unsqueeze(0), s.unsqueeze(0)
    if c.dim() != 3 or c.shape[1] != tokens or c.shape[0] not in (1, batch):
        raise _lib.SpecVerifyError(-1, f"cos {tuple(cos.shape)} vs [B={batch}, T={tokens}, D]")
    if c.stride(-1) != 1:
        c, s = c.contiguous(), s.contiguous()
    cs_sb = c.stride(0) if c.shape[0] == batch and batch > 1 else 0
    return c, s, cs_sb, c.stride(1), tokens, None, 0


def _launch(q, k, v, cos, sin, position_ids, q_out, k_out, k_cache, v_cache, start, capacity,
            page_table, page_size, validate: bool):
    dev = _lib.require_cuda(q, k, v, cos, sin, q_out, k_out, k_cache, v_cache, page_table)
    if position_ids is not None:
        position_ids = position_ids.to(device=dev, dtype=torch.int64)
    for name, x in (("out", q_out), ("k_out", k_out), ("k_cache", k_cache), ("v_cache", v_cache)):
        if x is not None and x.stride(-1) != 1:
            raise _lib.SpecVerifyError(-3, f"{name} needs unit stride on head_dim")
    b, h, t, d = q.shape
    hkv = k.shape[1]
    if k.shape != (b, hkv, t, d) or (v is not None and v.shape != k.shape):
        raise _lib.SpecVerifyError(-1, f"k/v must be [B, kv_heads, T, D] matching q {tuple(q.shape)}")
    for x in (k, v, cos, sin, q_out, k_out, k_cache, v_cache):
        if x is not None and x.dtype != q.dtype:
            raise _lib.SpecVerifyError(-2, f"all tensors must be {q.dtype}, got {x.dtype}")
    if cos.shape[-1] != d:
        raise _lib.SpecVerifyError(-1, f"cos/sin last dim {cos.shape[-1]} != head_dim {d}")
    tab, stab, cs_sb, cs_sr, cs_rows, pos, pos_sb = _table(cos, sin, position_ids, b, t)
    a = _lib.RopeArgs()
    a.dtype = _lib.dtype_code(q.dtype)
    a.batch, a.tokens, a.heads, a.kv_heads, a.head_dim = b, t, h, hkv, d
    a.q = q.data_ptr(); a.q_sb, a.q_sh, a.q_st = q.stride(0), q.stride(1), q.stride(2)
    a.k = k.data_ptr(); a.k_sb, a.k_sh, a.k_st = k.stride(0), k.stride(1), k.stride(2)
    if v is not None:
        a.v = v.data_ptr(); a.v_sb, a.v_sh, a.v_st = v.stride(0), v.stride(1), v.stride(2)
    a.cos, a.sin = tab.data_ptr(), stab.data_ptr()
    a.cs_sb, a.cs_sr, a.cs_rows = cs_sb, cs_sr, cs_rows
    if pos is not None:
        a.pos, a.pos_sb = pos.data_ptr(), pos_sb
    a.q_out = q_out.data_ptr(); a.qo_sb, a.qo_sh, a.qo_st = q_out.stride(0), q_out.stride(1), q_out.stride(2)
    if k_out is not None:
        a.k_out = k_out.data_ptr(); a.ko_sb, a.ko_sh, a.ko_st = k_out.stride(0), k_out.stride(1), k_out.stride(2)
    if k_cache is not None:
        a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        a.kc_sb, a.kc_sh, a.kc_st = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
        a.vc_sb, a.vc_sh, a.vc_st = v_cache.stride(0), v_cache.stride(1), v_cache.stride(2)
        a.start, a.capacity = int(start), int(capacity)
        if page_table is not None:
            pt = page_table if page_table.dim() == 2 else page_table.unsqueeze(0)
            if pt.dtype != torch.int32:
                pt = pt.to(torch.int32)
            if pt.stride(-1) != 1:
                pt = pt.contiguous()
            a.page_table, a.pt_sb = pt.data_ptr(), (pt.stride(0) if pt.shape[0] > 1 else 0)
            a.page_size, a.num_pages = int(page_size), k_cache.shape[0]
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    a.status = _lib.ptr(status)
    lib = _lib.load()
    _lib.check(lib.tv_rope_append(ctypes.byref(a), ctypes.c_void_p(_lib.stream_ptr(dev))), "tv_rope_append")
    if status is not None:
        code = int(status.item())
        if code != 0:
            raise _lib.SpecVerifyError(code, "tv_rope_append: position id, cache index or page out of range")


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         position_ids: torch.Tensor, *, validate: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """``llama_target_model.py:429-449``: q [B, H, T, D], k [B, H_kv, T, D];
    cos / sin the cached ``[1, 1, S, D]`` tables; position_ids [B|1, T].
    Returns new (q_embed, k_embed)."""
    q, k = _bhtd(q, "q"), _bhtd(k, "k")
    q_out, k_out = torch.empty(q.shape, dtype=q.dtype, device=q.device), torch.empty(k.shape, dtype=k.dtype,
                                                                                       device=k.device)
    _launch(q, k, None, cos, sin, position_ids, q_out, k_out, None, None, 0, 0, None, 0, validate)
    return q_out, k_out


def apply_rotary_pos_emb_L31(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                             position_ids=None, unsqueeze_dim: int = 1, *, validate: bool = True
                             ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``llama_target_model.py:452-474``: cos / sin [B, T, D] per token.
    ``unsqueeze_dim=1`` takes q/k as [B, heads, T, D], ``2`` as [B, T, heads, D]."""
    if unsqueeze_dim not in (1, 2):
        raise _lib.SpecVerifyError(-1, f"unsqueeze_dim must be 1 or 2, got {unsqueeze_dim}")
    qv = q.transpose(1, 2) if unsqueeze_dim == 2 else q
    kv = k.transpose(1, 2) if unsqueeze_dim == 2 else k
    qv, kv = _bhtd(qv, "q"), _bhtd(kv, "k")
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    k_out = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    qo = q_out.transpose(1, 2) if unsqueeze_dim == 2 else q_out
    ko = k_out.transpose(1, 2) if unsqueeze_dim == 2 else k_out
    _launch(qv, kv, None, cos, sin, None, qo, ko, None, None, 0, 0, None, 0, validate)
    return q_out, k_out


def rope_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                position_ids: Optional[torch.Tensor], k_cache, v_cache, *, start: Optional[int] = None,
                page_table: Optional[torch.Tensor] = None, page_size: int = 16, out: Optional[torch.Tensor] = None,
                validate: bool = True):
    """Rotate q and k and append the rotated k and v to the cache, in one launch.

    Contiguous cache: ``k_cache`` / ``v_cache`` are the layer's
    :class:`~specverify.runtime.cache_state.KVCache` objects (``data``
    ``[B, H_kv, S_budget, D]``); the tokens go to ``current_length ..``, the
    lengths advance and the return value is ``(q_embed, key_states,
    value_states)`` with the cache views ``data[:, :, :current_length]`` --
    what ``LlamaAttention.forward`` holds after its two ``cat`` calls.
    Paged cache: ``k_cache`` / ``v_cache`` are pool tensors
    ``[P, H_kv, page_size, D]``, ``page_table`` ``[B|1, pages]`` int32 maps
    token index ``start + t`` to its page; returns ``(q_embed, None, None)``.
    ``position_ids=None`` takes per-token ``[B, T, D]`` cos / sin.
    ``out`` (optional, may be ``q``) receives q_embed.
    """
    q, k, v = _bhtd(q, "q"), _bhtd(k, "k"), _bhtd(v, "v")
    q_out = out if out is not None else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if page_table is None:
        kd, vd = k_cache.data, v_cache.data
        st = int(k_cache.current_length) if start is None else int(start)
        cap = kd.shape[2]
        t = q.shape[2]
        if st < 0 or st + t > cap:
            raise _lib.SpecVerifyError(-1, f"cache of {cap} tokens cannot take {t} more at {st}")
        _launch(q, k, v, cos, sin, position_ids, q_out, None, kd, vd, st, cap, None, 0, validate)
        k_cache.current_length.add_(t)
        v_cache.current_length.add_(t)
        return (q_out, torch.narrow(kd, 2, 0, int(k_cache.current_length)),
                torch.narrow(vd, 2, 0, int(v_cache.current_length)))
    if start is None:
        raise _lib.SpecVerifyError(-1, "start is required with a page table")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or k_cache.shape[2] != page_size:
        raise _lib.SpecVerifyError(-1, f"paged pools must be [P, H_kv, {page_size}, D], got {tuple(k_cache.shape)}")
    _launch(q, k, v, cos, sin, position_ids, q_out, None, k_cache, v_cache, start, 0, page_table, page_size,
            validate)
    return q_out, None, None
