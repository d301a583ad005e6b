"""Verify attention on B200: the drop-in for ``diffspec.runtime.tree_attention``.

Public functions keep the reference's names, argument meaning and return
contract (``diffspec/runtime/tree_attention.py``):

* :func:`prefix_attention_forward` -- ``:414-446``: unmasked attention over the
  cached prefix, returns ``(out [B,M,H,D], lse [B,H,M] fp32)``;
* :func:`tree_attention_forward` -- ``:462-539``: attention of the M tree rows
  over the M tree keys under the tree mask, returns
  ``(out [B,M,H,D], weight [B,M,H,1])`` with
  ``weight = sigmoid(prefix_lse - tree_lse)`` in the query dtype;
* :data:`TRITON_AVAILABLE` -- the flag callers test before taking the
  accelerated branch (``tree_attention.py:493``); here it reports whether the
  B200 library is loaded.

New entry points the B200 design adds:

* :func:`verify_attention` -- the whole verify step of one layer in one call:
  prefix and tree keys of an unexpanded GQA cache (contiguous or paged, the
  tree's K/V already appended after the prefix) under an ancestor bitmask,
  producing the merged output the reference builds from three kernels and an
  in-place merge (``llama_target_model.py:795-864``);
* :func:`attention` -- the general form every other function calls;
* :func:`pack_tree_mask` -- any reference mask form to the bitmask the kernels
  read (one bit per node and key).

Unlike the reference there is no silent fallback (``tree_attention.py:
497-511``): errors raise :class:`specverify.SpecVerifyError`, and CPU tensors
are rejected.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from .. import _lib

__all__ = [
    "TRITON_AVAILABLE",
    "KERNELS_AVAILABLE",
    "prefix_attention_forward",
    "tree_attention_forward",
    "verify_attention",
    "attention",
    "describe_attention",
    "mask_word_summary",
    "pack_tree_mask",
]

KERNELS_AVAILABLE = _lib.available()
# Name kept for callers that gate the accelerated branch on it.
TRITON_AVAILABLE = KERNELS_AVAILABLE

_KIND = {torch.int8: 0, torch.uint8: 0, torch.bool: 0, torch.float32: 1, torch.float16: 2, torch.bfloat16: 3}


def pack_tree_mask(mask: torch.Tensor, q_len: Optional[int] = None, batch: Optional[int] = None,
                   cols: Optional[int] = None) -> torch.Tensor:
    """Pack a tree mask into uint64 bits ``[B, M, ceil(N/64)]`` on the device.

    Accepted forms (the reference's, ``tree_attention.py:449-460``):

    * additive float mask ``[B, 1, T, T]`` / ``[B, T, T]`` (fp32/fp16/bf16):
      the lower-right ``q_len x q_len`` block, keep where the value is 0;
    * int8 / uint8 / bool ``[M, N]`` or ``[B, M, N]``: keep where non-zero
      (``DraftTree.generate_attention_mask`` output, bundle masks).

    ``cols`` limits the packed columns for int masks (default: all).
    """
    dev = _lib.require_cuda(mask)
    kind = _KIND.get(mask.dtype)
    if kind is None:
        raise _lib.SpecVerifyError(-2, f"mask dtype {mask.dtype}")
    if kind == 0:
        m3 = mask if mask.dim() == 3 else mask.unsqueeze(0)
        if m3.dim() != 3:
            raise _lib.SpecVerifyError(-1, f"int mask must be [M, N] or [B, M, N], got {tuple(mask.shape)}")
        if m3.dtype == torch.bool:
            m3 = m3.view(torch.uint8)
        b, m, n = m3.shape
        if cols is not None:
            n = cols
    else:
        if q_len is None:
            raise _lib.SpecVerifyError(-1, "q_len is required for a float mask")
        blk = mask[:, -q_len:, -q_len:] if mask.dim() == 3 else mask[:, :, -q_len:, -q_len:]
        if blk.dim() == 4:
            blk = blk[:, 0]
        m3 = blk
        b, m, n = m3.shape
    if batch is not None and b == 1 and batch > 1:
        m3 = m3.expand(batch, m3.shape[1], m3.shape[2])
        b = batch
    words = (n + 63) // 64
    out = torch.empty((b, m, max(words, 1)), dtype=torch.int64, device=dev)
    s = m3.stride()
    lib = _lib.load()
    st = lib.tv_pack_mask(kind, m3.data_ptr(), s[0], s[1], s[2], b, m, n, out.data_ptr(),
                          out.stride(0), out.stride(1), _lib.stream_ptr(dev))
    _lib.check(st, "tv_pack_mask")
    return out


def mask_word_summary(bits: torch.Tensor) -> torch.Tensor:
    """uint8 ``[B, words]``: 1 where a 64-key word of the packed mask
    ``[B, M, words]`` is all ones in every row (``tv_mask_word_summary``)."""
    dev = _lib.require_cuda(bits)
    if bits.dim() != 3 or bits.dtype != torch.int64 or bits.stride(2) != 1:
        raise _lib.SpecVerifyError(-1, "bits must be packed int64 [B, M, words] with unit word stride")
    b, m, words = bits.shape
    out = torch.empty((b, words), dtype=torch.uint8, device=dev)
    st = _lib.load().tv_mask_word_summary(bits.data_ptr(), b, m, words, bits.stride(0), bits.stride(1),
                                          out.data_ptr(), out.stride(0), _lib.stream_ptr(dev))
    _lib.check(st, "tv_mask_word_summary")
    return out


def _kv_strides(t: torch.Tensor, paged: bool):
    """(sb, sn, sh): contiguous [B, N, Hkv, D] or a paged pool [P, Hkv, page, D]."""
    if t.dim() != 4 or t.stride(3) != 1:
        raise _lib.SpecVerifyError(-3, f"KV tensor must be 4-D with unit stride on head_dim, got "
                                       f"shape {tuple(t.shape)} strides {t.stride()}")
    if paged:
        return t.stride(0), t.stride(2), t.stride(1)
    return t.stride(0), t.stride(1), t.stride(2)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
              num_keys: Optional[int] = None,
              kv_lens: Optional[torch.Tensor] = None,
              page_table: Optional[torch.Tensor] = None,
              mask_bits: Optional[torch.Tensor] = None,
              mask_len: int = 0,
              out: Optional[torch.Tensor] = None,
              out_f32: bool = False,
              lse: Optional[torch.Tensor] = None,
              lse_strides: Optional[Tuple[int, int, int]] = None,
              aux_lse: Optional[torch.Tensor] = None,
              aux_strides: Optional[Tuple[int, int, int]] = None,
              weight: Optional[torch.Tensor] = None,
              weight_strides: Optional[Tuple[int, int, int]] = None,
              scale: Optional[float] = None,
              num_splits: int = 0,
              kernel: int = 0,
              status: Optional[torch.Tensor] = None,
              mask_full: Optional[torch.Tensor] = None) -> torch.Tensor:
    """General verify attention (see ``tv_verify_attn`` in include/specverify.h).

    q: [B, M, H, D]; k/v: contiguous ``[B, N, Hkv, D]`` views, or a paged pool
    ``[P, Hkv, page, D]`` with ``page_table`` int32 ``[B, pages]``.  The last
    ``mask_len`` keys of each sequence are gated by ``mask_bits``
    (``[B, M, words]`` uint64 as int64).  ``lse``/``aux_lse``/``weight`` are
    addressed as ``[b, m, h]`` through the given strides (default: their
    own ``[B, M, H]`` strides).  ``status`` (int32 [1], zeroed by the caller)
    receives a nonzero code if a kernel had to abandon a bounded wait.
    ``mask_full`` (uint8 ``[B, words]`` from :func:`mask_word_summary`) lets
    the tcgen05 kernel skip masking key tiles every row fully sees.
    Returns ``out``.
    """
    lib = _lib.load()
    # Fast path: a request whose shapes, strides, dtypes, devices and options
    # were validated before reuses that call's argument block and workspace
    # size; only the data pointers change.  A decode loop calls this once per
    # layer with the same geometry every step.
    key = _request_key(q, k, v, num_keys, kv_lens, page_table, mask_bits, mask_len, out, out_f32, lse,
                       lse_strides, aux_lse, aux_strides, weight, weight_strides, scale, num_splits, kernel, status,
                       mask_full)
    hit = _PLANS.get(key)
    if hit is None:
        a, out = attn_args(q, k, v, num_keys=num_keys, kv_lens=kv_lens, page_table=page_table,
                           mask_bits=mask_bits, mask_len=mask_len, out=out, out_f32=out_f32, lse=lse,
                           lse_strides=lse_strides, aux_lse=aux_lse, aux_strides=aux_strides, weight=weight,
                           weight_strides=weight_strides, scale=scale, num_splits=num_splits, kernel=kernel,
                           status=status, mask_full=mask_full)
        need = ctypes.c_size_t(0)
        _lib.check(lib.tv_attn_workspace_size(ctypes.byref(a), ctypes.byref(need)), "tv_attn_workspace_size")
        if len(_PLANS) >= 512:
            _PLANS.clear()
        _PLANS[key] = (bytes(a), need.value)
        need = need.value
    else:
        a = _lib.AttnArgs.from_buffer_copy(hit[0])
        need = hit[1]
        if out is None:
            b, m, h, d = q.shape
            out = torch.empty((b, m, h, d), dtype=torch.float32 if out_f32 else q.dtype, device=q.device)
        a.q, a.k, a.v, a.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
        a.page_table = page_table.data_ptr() if page_table is not None else None
        a.kv_lens = kv_lens.data_ptr() if kv_lens is not None else None
        a.mask = mask_bits.data_ptr() if mask_len else None
        a.lse = lse.data_ptr() if lse is not None else None
        a.aux_lse = aux_lse.data_ptr() if aux_lse is not None else None
        a.weight = weight.data_ptr() if aux_lse is not None else None
        a.status = status.data_ptr() if status is not None else None
        a.mask_words_full = mask_full.data_ptr() if (mask_len and mask_full is not None) else None
    ws = None
    if need:
        ws = torch.empty(need, dtype=torch.uint8, device=out.device)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = need
    _lib.check(lib.tv_verify_attn(ctypes.byref(a), _lib.stream_ptr(out.device)), "tv_verify_attn")
    return out


_PLANS: dict = {}


def _geom(t):
    """Everything of a tensor argument but its data pointer (None stays None)."""
    return None if t is None else (t.shape, t.stride(), t.dtype, t.device)


def _request_key(q, k, v, num_keys, kv_lens, page_table, mask_bits, mask_len, out, out_f32, lse, lse_strides,
                 aux_lse, aux_strides, weight, weight_strides, scale, num_splits, kernel, status, mask_full):
    return (_geom(q), _geom(k), _geom(v), num_keys, _geom(kv_lens), _geom(page_table), _geom(mask_bits),
            int(mask_len), _geom(out), bool(out_f32), _geom(lse), lse_strides, _geom(aux_lse), aux_strides,
            _geom(weight), weight_strides, scale, int(num_splits), int(kernel), _geom(status), _geom(mask_full))


def describe_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, **kw) -> dict:
    """The plan :func:`attention` would run for the same arguments (host only):
    ``kernel`` ("tcgen05" or "warp-mma"), ``splits`` (key splits), ``wide``
    (tcgen05 loads whole-head TMA boxes) and ``split_p`` (warp-MMA hi+lo P)."""
    a, _ = attn_args(q, k, v, **kw)
    info = (ctypes.c_int32 * 4)()
    _lib.check(_lib.load().tv_attn_describe(ctypes.byref(a), info), "tv_attn_describe")
    return {"kernel": {2: "tcgen05", 1: "warp-mma"}.get(info[0], "none"), "splits": info[1],
            "wide": bool(info[2]), "split_p": bool(info[3])}


def attn_args(q, k, v, *, num_keys=None, kv_lens=None, page_table=None, mask_bits=None, mask_len=0, out=None,
              out_f32=False, lse=None, lse_strides=None, aux_lse=None, aux_strides=None, weight=None,
              weight_strides=None, scale=None, num_splits=0, kernel=0, status=None, mask_full=None):
    """The checked ``tv_attn_args`` of an :func:`attention` request (no
    workspace set) and its output tensor (allocated when ``out`` is None).
    The tensors must stay alive while the struct is used."""
    dev = _lib.require_cuda(q, k, v, page_table, kv_lens, mask_bits, out, lse, aux_lse, weight, mask_full)
    if q.dim() != 4 or q.stride(3) != 1:
        raise _lib.SpecVerifyError(-3, f"q must be [B, M, H, D] with unit stride on D, got {tuple(q.shape)}")
    b, m, h, d = q.shape
    paged = page_table is not None
    hkv = k.shape[1]
    if k.shape[3] != d or v.shape[3] != d or v.shape[1] != hkv:
        raise _lib.SpecVerifyError(-1, f"q {tuple(q.shape)} / k {tuple(k.shape)} / v {tuple(v.shape)}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise _lib.SpecVerifyError(-2, f"q/k/v dtypes differ: {q.dtype} {k.dtype} {v.dtype}")
    if not paged:
        hkv = k.shape[2]
        if v.shape[2] != hkv or k.shape[0] != b or v.shape[0] != b:
            raise _lib.SpecVerifyError(-1, f"q {tuple(q.shape)} / k {tuple(k.shape)} / v {tuple(v.shape)}")
        n_default = min(k.shape[1], v.shape[1])
    else:
        if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != b:
            raise _lib.SpecVerifyError(-1, "page_table must be int32 [B, pages]")
        n_default = page_table.shape[1] * k.shape[2]
    if h % hkv != 0:
        raise _lib.SpecVerifyError(-1, f"heads {h} not a multiple of kv heads {hkv}")
    n = n_default if num_keys is None else int(num_keys)
    if out is None:
        out = torch.empty((b, m, h, d), dtype=torch.float32 if out_f32 else q.dtype, device=dev)
    a = _lib.AttnArgs()
    a.dtype = _lib.dtype_code(q.dtype)
    a.batch, a.rows, a.heads, a.kv_heads, a.head_dim = b, m, h, hkv, d
    a.scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    a.q = q.data_ptr()
    a.q_sb, a.q_sm, a.q_sh = q.stride(0), q.stride(1), q.stride(2)
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.k_sb, a.k_sn, a.k_sh = _kv_strides(k, paged)
    a.v_sb, a.v_sn, a.v_sh = _kv_strides(v, paged)
    if paged:
        a.page_table = page_table.data_ptr()
        a.pt_sb = page_table.stride(0)
        a.page_size = k.shape[2]
        a.num_pages = min(k.shape[0], v.shape[0])
    if kv_lens is not None:
        if kv_lens.dtype != torch.int32:
            raise _lib.SpecVerifyError(-2, "kv_lens must be int32")
        a.kv_lens = kv_lens.data_ptr()
    a.num_keys = n
    a.mask_len = int(mask_len)
    if mask_len:
        if mask_bits is None:
            raise _lib.SpecVerifyError(-8, "mask_len > 0 needs mask_bits")
        if mask_bits.shape[-1] * 64 < mask_len:
            raise _lib.SpecVerifyError(-1, "mask_bits has fewer words than mask_len needs")
        a.mask = mask_bits.data_ptr()
        a.mask_sb = mask_bits.stride(0) if mask_bits.shape[0] > 1 else 0
        a.mask_sm = mask_bits.stride(1)
        if mask_full is not None:
            if mask_full.dtype != torch.uint8 or mask_full.dim() != 2 or mask_full.shape[1] < -(-mask_len // 64):
                raise _lib.SpecVerifyError(-1, "mask_full must be uint8 [B, words] covering mask_len")
            a.mask_words_full = mask_full.data_ptr()
            a.mask_words_full_sb = mask_full.stride(0) if mask_full.shape[0] > 1 else 0
    a.out = out.data_ptr()
    a.o_sb, a.o_sm, a.o_sh = out.stride(0), out.stride(1), out.stride(2)
    if out.stride(3) != 1:
        raise _lib.SpecVerifyError(-3, "out must have unit stride on D")
    a.out_f32 = 1 if out.dtype == torch.float32 else 0
    if not a.out_f32 and out.dtype != q.dtype:
        raise _lib.SpecVerifyError(-2, f"out dtype {out.dtype} must be {q.dtype} or float32")
    if lse is not None:
        if lse.dtype != torch.float32:
            raise _lib.SpecVerifyError(-2, "lse must be float32")
        a.lse = lse.data_ptr()
        a.lse_sb, a.lse_sm, a.lse_sh = lse_strides or lse.stride()[:3]
    if aux_lse is not None:
        if aux_lse.dtype != torch.float32 or weight is None:
            raise _lib.SpecVerifyError(-2, "aux_lse must be float32 and needs a weight output")
        a.aux_lse = aux_lse.data_ptr()
        a.aux_sb, a.aux_sm, a.aux_sh = aux_strides or aux_lse.stride()[:3]
        if weight.dtype != q.dtype:
            raise _lib.SpecVerifyError(-2, "weight dtype must match q")
        a.weight = weight.data_ptr()
        a.w_sb, a.w_sm, a.w_sh = weight_strides or weight.stride()[:3]
    a.num_splits = int(num_splits)
    a.kernel = int(kernel)
    if status is not None:
        if status.dtype != torch.int32 or not status.is_cuda:
            raise _lib.SpecVerifyError(-2, "status must be a CUDA int32 tensor")
        a.status = status.data_ptr()
    return a, out


def prefix_attention_forward(query_states, key_states, value_states, bsz, q_len, num_heads, hidden_dim):
    """Prefix attention with LSE.  Reference: ``tree_attention.py:414-446``.

    query_states [B, M, H, D]; key/value_states [B, N, Hk, D] (Hk may also be
    the KV-head count: GQA is handled without expansion).
    Returns ``(out [B, M, H, D] in the query dtype, lse [B, H, M] fp32)``.
    """
    b, m, h, d = bsz, q_len, num_heads, hidden_dim
    if tuple(query_states.shape) != (b, m, h, d):
        raise _lib.SpecVerifyError(-1, f"query_states shape {tuple(query_states.shape)} != {(b, m, h, d)}")
    lse = torch.empty((b, h, m), dtype=torch.float32, device=query_states.device)
    out = attention(query_states, key_states, value_states, lse=lse,
                    lse_strides=(lse.stride(0), lse.stride(2), lse.stride(1)))
    return out, lse


def tree_attention_forward(query_states, key_states, value_states, tree_mask,
                           cache_lens, prefix_lse, bsz, q_len, num_heads, hidden_dim):
    """Tree-block attention + merge weight.  Reference: ``tree_attention.py:462-539``.

    query/key/value_states [B, M, H, D] (K/V may carry the KV-head count);
    tree_mask: additive float ``[B, 1, T, T]`` (lower-right M x M block used)
    or an int8/bool keep mask; cache_lens is unused (signature compatibility);
    prefix_lse laid out ``[B, H, M]`` (any shape with that element order).
    Returns ``(current_out [B, M, H, D], weight [B, M, H, 1])`` in the query dtype.
    """
    b, m, h, d = bsz, q_len, num_heads, hidden_dim
    if tuple(query_states.shape[:3]) != (b, m, h) or query_states.shape[3] != d:
        raise _lib.SpecVerifyError(-1, f"query_states shape {tuple(query_states.shape)} != {(b, m, h, d)}")
    if key_states.shape[0] != b or key_states.shape[1] != m or value_states.shape[1] != m:
        raise _lib.SpecVerifyError(-1, "key/value must be the post-cache [B, M, Hk, D] block")
    bits = pack_tree_mask(tree_mask, q_len=m, batch=b, cols=m)
    plse = prefix_lse.reshape(b, h, m).to(torch.float32)
    weight = torch.empty((b, m, h, 1), dtype=query_states.dtype, device=query_states.device)
    out = attention(query_states, key_states, value_states, num_keys=m, mask_bits=bits, mask_len=m,
                    aux_lse=plse, aux_strides=(plse.stride(0), plse.stride(2), plse.stride(1)),
                    weight=weight, weight_strides=(weight.stride(0), weight.stride(1), weight.stride(2)))
    return out, weight


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_len: int,
                     tree_mask: torch.Tensor, *, page_table: Optional[torch.Tensor] = None,
                     kv_lens: Optional[torch.Tensor] = None, return_lse: bool = False,
                     out: Optional[torch.Tensor] = None, out_f32: bool = False, num_splits: int = 0,
                     kernel: int = 0):
    """One layer's verify attention, prefix + tree in one pass.

    q [B, M, H, D] (post-RoPE); ``k_cache``/``v_cache`` hold the prefix followed
    by the M tree keys, either contiguous ``[B, N, Hkv, D]`` views (e.g.
    ``past_key_values_data[2l].transpose(1, 2)`` of the reference's cache) or a
    paged pool ``[P, Hkv, page, D]`` with ``page_table``.  ``cache_len`` is the
    prefix length (keys ``[cache_len, cache_len + M)`` are the tree).
    ``tree_mask`` is the M x M keep mask (int8/bool, 1 = visible) or its packed
    bits ``[B, M, words]`` (int64).
    Returns the merged attention output ``[B, M, H, D]`` (and the LSE
    ``[B, M, H]`` fp32 when ``return_lse``).
    """
    b, m = q.shape[0], q.shape[1]
    bits = tree_mask if tree_mask.dtype == torch.int64 else pack_tree_mask(tree_mask, batch=b)
    lse = torch.empty((b, m, q.shape[2]), dtype=torch.float32, device=q.device) if return_lse else None
    o = attention(q, k_cache, v_cache, num_keys=None if kv_lens is not None else cache_len + m, kv_lens=kv_lens,
                  page_table=page_table, mask_bits=bits, mask_len=m, out=out, out_f32=out_f32, lse=lse,
                  num_splits=num_splits, kernel=kernel)
    return (o, lse) if return_lse else o
