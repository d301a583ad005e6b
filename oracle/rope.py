"""Rotary embedding and KV-cache append, CPU restatement (numpy).

TEST INFRASTRUCTURE ONLY: the checker for ``tv_rope_append``; nothing in the
product imports it.

Follows the reference (package ``diffspec``):

* ``rotate_half`` -- ``runtime/llama_target_model.py:414-427``:
  ``cat(-x[..., D/2:], x[..., :D/2])``;
* ``apply_rotary_pos_emb`` -- ``:429-449``: the cached ``[1, 1, S, D]``
  tables gathered by ``position_ids`` and broadcast over heads, then
  ``q * cos + rotate_half(q) * sin`` (same for k);
* ``apply_rotary_pos_emb_L31`` -- ``:452-474``: the same with per-token
  ``[B, T, D]`` tables;
* ``LlamaRotaryEmbedding`` -- ``:152-211``: ``inv_freq = 1 / base **
  (arange(0, D, 2) / D)``, table rows ``t * inv_freq`` repeated twice, cos /
  sin built in float32 and cast to the activation dtype on use;
* ``KVCache.cat`` -- ``runtime/cache_state.py:52-66``: the new rows go to
  ``data[:, :, current_length : current_length + T]``, the length advances.

torch evaluates each bf16 / fp16 element-wise op in float32 and rounds the
result once, so every product and the sum are rounded to the element type
here too ("kind": "bf16", "f16" or "f32"; values are carried as float32
arrays holding exactly representable numbers).
"""

from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16, nearest-even; NaN stays a quiet NaN."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)


def round_to(x: np.ndarray, kind: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if kind == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if kind == "f16":
        return x.astype(np.float16).astype(np.float32)
    if kind == "f32":
        return x
    raise ValueError(kind)


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, kind: str) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` with the reference's roundings."""
    x = np.asarray(x, dtype=np.float32)
    a = round_to(x * np.asarray(cos, dtype=np.float32), kind)
    b = round_to(rotate_half(x) * np.asarray(sin, dtype=np.float32), kind)
    return round_to(a + b, kind)


def apply_rotary_pos_emb(q, k, cos_table, sin_table, position_ids, kind):
    """q [B, H, T, D], k [B, H_kv, T, D]; tables [S, D]; position_ids [B, T]."""
    pos = np.asarray(position_ids, dtype=np.int64)
    cos = np.asarray(cos_table, dtype=np.float32)[pos][:, None]     # [B, 1, T, D]
    sin = np.asarray(sin_table, dtype=np.float32)[pos][:, None]
    return rope(q, cos, sin, kind), rope(k, cos, sin, kind)


def apply_rotary_pos_emb_l31(q, k, cos, sin, kind):
    """Per-token tables cos / sin [B, T, D], broadcast over heads."""
    c = np.asarray(cos, dtype=np.float32)[:, None]
    s = np.asarray(sin, dtype=np.float32)[:, None]
    return rope(q, c, s, kind), rope(k, c, s, kind)


def rope_table(dim: int, max_pos: int, base: float):
    """cos / sin tables [max_pos, dim] in float32 (before the dtype cast)."""
    inv_freq = (1.0 / (np.float32(base) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))).astype(
        np.float32)
    t = np.arange(max_pos, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def kv_cat(data: np.ndarray, start: int, x: np.ndarray):
    """``KVCache.cat`` along dim 2: returns (new data, new length)."""
    out = np.array(data, copy=True)
    t = x.shape[2]
    out[:, :, start:start + t] = x
    return out, start + t


def paged_append(pool: np.ndarray, page_table: np.ndarray, start: int, x: np.ndarray):
    """Paged form of the append: token t of batch row b lands in page
    ``page_table[b, (start + t) // page]``, slot ``(start + t) % page`` of
    the pool ``[P, H_kv, page, D]``."""
    out = np.array(pool, copy=True)
    page = pool.shape[2]
    b, _, t, _ = x.shape
    for bi in range(b):
        for ti in range(t):
            idx = start + ti
            out[page_table[bi, idx // page], :, idx % page] = x[bi, :, ti]
    return out
