"""Oracle: tree-verify attention on the CPU (torch, fp32 unless told otherwise).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates, from the reference package ``diffspec``:

* ``prefix_attention``  -- ``diffspec/runtime/tree_attention.py:439-446``
  (the torch path of ``prefix_attention_forward``): unmasked attention over the
  cached prefix, LSE laid out ``[B, H, M]``.
* ``tree_attention``    -- ``diffspec/runtime/tree_attention.py:40-63``
  (``tree_attention_forward_naive``): attention of the M tree queries over the
  M tree keys under the keep-mask, plus
  ``weight = sigmoid(prefix_lse - tree_lse)`` cast to the query dtype.
* ``merge``             -- ``diffspec/runtime/llama_target_model.py:862-864``:
  ``out = tree * (1 - w) + prefix * w`` in the query dtype.
* ``repeat_kv``         -- ``diffspec/runtime/llama_target_model.py:543-560``.
* ``keep_from_float_mask`` -- ``tree_attention.py:449-460`` /
  ``llama_target_model.py:1324-1330``: the additive float mask the target
  model builds, and the ``== 0`` keep rule the kernels apply to it.

``full_masked_attention`` is the precision anchor: one softmax over
``prefix ++ tree`` keys in fp32, which the prefix/tree/merge decomposition
equals mathematically.  It is what the bf16 GPU kernels are compared with
(2e-2 relative / 1e-3 absolute).
"""

from __future__ import annotations

import math

import torch


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[B, Hkv, S, D] -> [B, Hkv * n_rep, S, D]; head h reads kv head h // n_rep.

    Reference: ``llama_target_model.py:543-560``.
    """
    if n_rep == 1:
        return x
    b, hkv, s, d = x.shape
    return x[:, :, None, :, :].expand(b, hkv, n_rep, s, d).reshape(b, hkv * n_rep, s, d)


def prefix_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """q [B,M,H,D], k/v [B,N,H,D] -> (out [B,M,H,D] in v.dtype, lse [B,H,M] fp32).

    Reference: ``tree_attention.py:439-446`` (scores and LSE in fp32, the
    softmax weights cast back to the value dtype before the PV product).
    """
    scale = 1.0 / math.sqrt(q.shape[-1])
    qh = q.transpose(1, 2).float()
    kh = k.transpose(1, 2).float()
    vh = v.transpose(1, 2)
    scores = torch.matmul(qh, kh.transpose(-2, -1)) * scale
    probs = torch.softmax(scores, dim=-1).to(v.dtype)
    out = torch.matmul(probs, vh).transpose(1, 2)
    lse = torch.logsumexp(scores, dim=-1)
    return out, lse


def keep_from_float_mask(float_mask: torch.Tensor, m: int) -> torch.Tensor:
    """Lower-right MxM block of an additive float mask -> int8 keep (1 = attend).

    Reference: ``tree_attention.py:42-43`` and ``:449-460`` (``mask == 0``
    means keep for float masks; bool/int masks are taken as keep directly).
    """
    if float_mask.dim() == 3:
        block = float_mask[:, -m:, -m:]
    else:
        block = float_mask[:, :, -m:, -m:]
    if block.dtype in (torch.bool, torch.int8, torch.uint8):
        keep = block.to(torch.int8)
    else:
        keep = (block == 0).to(torch.int8)
    return keep.reshape(block.shape[0], m, m)


def float_mask_from_keep(keep_mm: torch.Tensor, prefix_len: int) -> torch.Tensor:
    """int8 [M,M] tree mask (1 = visible) -> additive float mask [1,1,M,P+M].

    Reference: ``llama_target_model.py:1319-1330`` (zeros over the prefix,
    ``finfo(float32).min`` where the tree mask is 0, 0 where it is 1).
    """
    m = keep_mm.shape[-1]
    out = torch.zeros((m, prefix_len + m), dtype=torch.float32)
    blk = torch.where(keep_mm == 0, torch.tensor(torch.finfo(torch.float32).min), torch.tensor(0.0))
    out[:, prefix_len:] = blk
    return out[None, None]


def tree_attention(q, k, v, keep, prefix_lse):
    """Tree-block attention + merge weight.

    q/k/v [B,M,H,D]; keep int8 [B,M,M] (1 = attend); prefix_lse [B,H,M].
    Returns (out [B,M,H,D] in q.dtype, weight [B,M,H,1] in q.dtype).

    Reference: ``tree_attention.py:40-63``.
    """
    b, m, h, d = q.shape
    scale = 1.0 / math.sqrt(d)
    qh = q.transpose(1, 2)
    kt = k.permute(0, 2, 3, 1)
    vh = v.transpose(1, 2)
    score = (torch.matmul(qh, kt) * scale).float()
    blocked = keep.reshape(b, 1, m, m).expand(-1, h, -1, -1) == 0
    score = score.masked_fill(blocked, -float("inf"))
    probs = torch.softmax(score, dim=-1).to(q.dtype)
    out = torch.matmul(probs, vh).permute(0, 2, 1, 3)
    lse = score.logsumexp(dim=-1, keepdim=True).transpose(1, 2)
    plse = prefix_lse.reshape(b, h, m, -1).transpose(1, 2)
    weight = torch.sigmoid(plse - lse).to(q.dtype)
    return out, weight


def merge(tree_out, prefix_out, weight):
    """``out = tree * (1 - w) + prefix * w`` in the tree-output dtype.

    Reference: ``llama_target_model.py:862-864`` (in-place mul_/add_).
    """
    out = tree_out.clone()
    out.mul_(1.0 - weight)
    out.add_(prefix_out.to(out.dtype).mul_(weight))
    return out


def reference_verify_layer(q, k_prefix, v_prefix, k_tree, v_tree, keep):
    """The reference's verify-attention pipeline for one layer, unexpanded KV.

    q [B,M,H,D]; k_prefix/v_prefix [B,Hkv,S,D]; k_tree/v_tree [B,Hkv,M,D];
    keep int8 [M,M] or [B,M,M].  Mirrors ``llama_target_model.py:795-864``:
    GQA expansion by ``repeat_kv``, prefix attention, tree attention, merge.
    Returns the merged output [B,M,H,D] in q.dtype.
    """
    b, m, h, d = q.shape
    g = h // k_prefix.shape[1]
    kp = repeat_kv(k_prefix, g).transpose(1, 2)
    vp = repeat_kv(v_prefix, g).transpose(1, 2)
    kt = repeat_kv(k_tree, g).transpose(1, 2)
    vt = repeat_kv(v_tree, g).transpose(1, 2)
    if keep.dim() == 2:
        keep = keep.unsqueeze(0).expand(b, -1, -1)
    p_out, p_lse = prefix_attention(q, kp, vp)
    t_out, w = tree_attention(q, kt, vt, keep, p_lse)
    return merge(t_out, p_out, w)


def full_masked_attention(q, k, v, keep_tail, tail_start):
    """Precision anchor: one fp32 softmax over all N keys.

    q [B,M,H,D]; k/v [B,Hkv,N,D] (unexpanded, GQA by head // G);
    keys ``[tail_start, N)`` are gated per query row by ``keep_tail``
    ([B,M,N-tail_start] or [M,N-tail_start], 1 = attend); keys before
    ``tail_start`` are visible to every row.
    Returns (out [B,M,H,D] fp32, lse [B,M,H] fp32, natural log).
    Rows that see no key return out = 0 and lse = -inf.
    """
    b, m, h, d = q.shape
    hkv, n = k.shape[1], k.shape[2]
    g = h // hkv
    scale = 1.0 / math.sqrt(d)
    kf = repeat_kv(k.float(), g)                       # [B,H,N,D]
    vf = repeat_kv(v.float(), g)
    qf = q.float().transpose(1, 2)                     # [B,H,M,D]
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale  # [B,H,M,N]
    if tail_start < n:
        kt = keep_tail
        if kt.dim() == 2:
            kt = kt.unsqueeze(0).expand(b, -1, -1)
        blocked = torch.zeros((b, m, n), dtype=torch.bool)
        blocked[:, :, tail_start:] = kt[:, :, : n - tail_start] == 0
        s = s.masked_fill(blocked[:, None], -float("inf"))
    lse = torch.logsumexp(s, dim=-1)                   # [B,H,M]
    finite = torch.isfinite(lse)
    p = torch.exp(s - torch.where(finite, lse, torch.zeros_like(lse))[..., None])
    p = torch.where(finite[..., None], p, torch.zeros_like(p))
    out = torch.matmul(p, vf).transpose(1, 2)          # [B,M,H,D]
    return out, lse.transpose(1, 2)


def bundle_attention(q, k, v, mask):
    """``FusedBundleVerifier._verify_pytorch``: masked attention over N keys.

    q [B,M,H,D]; k/v [B,N,H,D]; mask [B,M,N] (1 = attend).
    Returns (out [B,M,H,D], lse [B,M,H]).  Reference:
    ``diffspec/runtime/bundle_verifier.py:259-297``.
    """
    b, m, h, d = q.shape
    scale = 1.0 / math.sqrt(d)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    s = torch.matmul(qh, kh.transpose(-2, -1)) * scale
    s = s.masked_fill(mask.unsqueeze(1).expand(-1, h, -1, -1) == 0, float("-inf"))
    p = torch.softmax(s, dim=-1)
    out = torch.matmul(p, vh)
    lse = torch.logsumexp(s, dim=-1)
    return out.transpose(1, 2).contiguous(), lse.transpose(1, 2).contiguous()


def lse_merge(parts_o, parts_lse):
    """Merge R partial attentions over disjoint key sets.

    parts_o [R, ..., D] (each normalised over its own keys), parts_lse [R, ...]
    natural-log LSE.  ``O = sum_r e^{lse_r - L} O_r / sum_r e^{lse_r - L}``.
    This is the algebra the split-KV combine and the sequence-sharded
    multi-GPU merge implement; the reference applies it pairwise in
    ``tree_attention.py:535-539`` (``sigmoid(a - b) = e^a / (e^a + e^b)``).
    """
    po = parts_o.double()
    pl = parts_lse.double()
    mx = pl.max(dim=0).values
    safe = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    w = torch.exp(pl - safe)
    w = torch.where(torch.isfinite(pl), w, torch.zeros_like(w))
    tot = w.sum(dim=0)
    out = (w[..., None] * po).sum(dim=0) / torch.where(tot > 0, tot, torch.ones_like(tot))[..., None]
    lse = torch.where(tot > 0, safe + torch.log(torch.where(tot > 0, tot, torch.ones_like(tot))),
                      torch.full_like(tot, -float("inf")))
    return out.float(), lse.float()
