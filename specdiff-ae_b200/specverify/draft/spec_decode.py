"""Speculative decode loop on the B200 path: draft tree -> target verify ->
acceptance -> compaction, every step of it on the device.

This is the loop of ``DiffSpecModel.diffspec_generate``
(``diffspec/draft/diffspec_model.py:268-754``) reduced to what one verify
step costs, built from this package's kernels:

* the target (a Llama-3.1-8B-architecture decoder, ``runtime/llama_target_model.py``)
  runs its 32 layers over the M = nodes + 1 tree rows (root first,
  ``diffspec_model.py:620-624``): RMSNorm, the q / k / v projection, RoPE and
  the KV append into the paged cache in one launch (``tv_rope_append``),
  verify attention over the cached prefix and the tree under the ancestor
  bitmask (``tv_verify_attn``), the output projection and the SwiGLU MLP;
  the projections and the MLP are plain torch GEMMs (cuBLAS);
* lm_head and acceptance in one pass (``tv_lmhead_accept``: greedy argmax or
  the Gumbel-max sample at ``temperature``, ``tree_verification.py:100-162``),
  then the accepted path's K / V of all layers moved into place
  (``tv_compact_paged``, ``:197-217``);
* the draft is a one-layer EAGLE3-shaped head (``draft/draft_network.py``):
  ``fc`` fuses the target's hidden states of three layers, one decoder
  layer whose attention reads a working cache (the retrieval working set:
  the reference drafts over retrieved chunks, ``draft_network.py:1514-1612``)
  plus the tree so far, and a reduced draft vocabulary mapped to target ids
  by ``d2t``.  The tree grows depth by depth: each frontier node's top
  ``width`` continuations, the best ``width`` by cumulative log-probability
  become the next frontier (``runtime/draft_tree.py``); ``tv_tree_finalize``
  turns the result into the verify inputs.

:meth:`SpecDecodeModel.from_config` is the tokenizer-free constructor:
random-init weights, N(0, 0.02) as the reference's ``_init_weights``
(``llama_target_model.py:1077-1086``), no tokenizer or checkpoint files
(``diffspec_model.py:100`` loads a tokenizer the decode loop never needs).
With random weights acceptance is close to zero, so a step verifies about
one token; the loop is a cost model of the real one, not a quality claim.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from .. import _lib
from ..runtime.rotary import rope_append
from ..runtime.tree_attention import attention, pack_tree_mask
from ..runtime.draft_tree import finalize_tree
from .tree_verification import RESULT_HEADER, accept_from_hidden


@dataclass
class LlamaShape:
    """Llama-3.1-8B shapes."""
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    draft_vocab: int = 32000
    feature_layers: tuple = (2, 16, 29)      # llama_target_model.py:1356


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``LlamaRMSNorm`` (``llama_target_model.py:124-138``) of the rows of a 2-D
    ``x``: fp32 statistics, the normalised row rounded to the input dtype
    before the weight multiply; one launch (``tv_rms_norm``)."""
    if x.dim() != 2 or x.stride(1) != 1 or w.dim() != 1 or w.stride(0) != 1:
        raise _lib.SpecVerifyError(-3, "rms_norm needs x [rows, cols] with unit column stride and a 1-D weight")
    y = torch.empty((x.shape[0], x.shape[1]), dtype=x.dtype, device=x.device)
    st = _lib.load().tv_rms_norm(x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), x.shape[0],
                                 x.shape[1], float(eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
    _lib.check(st, "tv_rms_norm")
    return y


def silu_mul(gu: torch.Tensor, ffn: int) -> torch.Tensor:
    """``act_fn(gate) * up`` of ``LlamaMLP`` (SiLU, ``llama_target_model.py:506-538``)
    for the fused ``[rows, 2 ffn]`` gate/up projection; one launch (``tv_silu_mul``)."""
    if gu.dim() != 2 or gu.stride(1) != 1 or gu.shape[1] != 2 * ffn:
        raise _lib.SpecVerifyError(-3, "silu_mul needs gu [rows, 2 * ffn] with unit column stride")
    y = torch.empty((gu.shape[0], ffn), dtype=gu.dtype, device=gu.device)
    g, u = gu[:, :ffn], gu[:, ffn:]
    st = _lib.load().tv_silu_mul(g.data_ptr(), u.data_ptr(), gu.stride(0), y.data_ptr(), y.stride(0), gu.shape[0],
                                 ffn, _lib.dtype_code(gu.dtype), _lib.stream_ptr(gu.device))
    _lib.check(st, "tv_silu_mul")
    return y


def rope_tables(head_dim: int, max_pos: int, theta: float, device, dtype=torch.bfloat16):
    """The cached cos / sin of ``LlamaRotaryEmbedding`` ([1, 1, max_pos, D])."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    t = torch.arange(max_pos, dtype=torch.float32)
    emb = torch.cat([torch.outer(t, inv)] * 2, dim=-1)
    return emb.cos().to(dtype).to(device)[None, None], emb.sin().to(dtype).to(device)[None, None]


class _Layer:
    """One decoder layer's weights (fused q/k/v and gate/up projections)."""

    def __init__(self, s: LlamaShape, in_dim: int, gen: torch.Generator, device, dtype):
        qkv = s.heads * s.head_dim + 2 * s.kv_heads * s.head_dim

        def w(o, i):
            t = torch.empty(o, i, device=device, dtype=dtype)
            t.normal_(0.0, 0.02, generator=gen)
            return t
        self.ln1 = torch.ones(in_dim, device=device, dtype=dtype)
        self.wqkv = w(qkv, in_dim)
        self.wo = w(s.hidden, s.heads * s.head_dim)
        self.ln2 = torch.ones(s.hidden, device=device, dtype=dtype)
        self.wgu = w(2 * s.ffn, s.hidden)
        self.wdown = w(s.hidden, s.ffn)


def _layer_forward(s: LlamaShape, L: _Layer, x_in: torch.Tensor, resid: torch.Tensor, pool_k, pool_v, page_table,
                   start: int, pos: torch.Tensor, bits: torch.Tensor, mask_len: int, cos, sin):
    """x_in [T, in_dim] normalised input, resid [T, H] residual stream ->
    new residual.  K / V of the T tokens go to rows ``start ..`` of the paged
    cache; attention covers ``start + T`` keys, the last ``mask_len`` gated
    by ``bits``."""
    t = x_in.shape[0]
    hq, hk, d = s.heads, s.kv_heads, s.head_dim
    qkv = x_in @ L.wqkv.t()
    q = qkv[:, : hq * d].view(1, t, hq, d).transpose(1, 2)
    k = qkv[:, hq * d: (hq + hk) * d].view(1, t, hk, d).transpose(1, 2)
    v = qkv[:, (hq + hk) * d:].view(1, t, hk, d).transpose(1, 2)
    qr, _, _ = rope_append(q, k, v, cos, sin, pos.view(1, t), pool_k, pool_v, start=start, page_table=page_table,
                           page_size=pool_k.shape[2], validate=False)
    o = attention(qr.transpose(1, 2), pool_k, pool_v, num_keys=start + t, page_table=page_table, mask_bits=bits,
                  mask_len=mask_len)
    h = torch.addmm(resid, o.view(t, hq * d), L.wo.t())
    gu = rms_norm(h, L.ln2, s.rms_eps) @ L.wgu.t()
    return torch.addmm(h, silu_mul(gu, s.ffn), L.wdown.t())


class SpecDecodeModel:
    """Target + EAGLE3-shaped draft head + paged caches, all on one GPU."""

    def __init__(self, shape: LlamaShape, device, dtype, gen: torch.Generator, max_tokens: int, draft_ctx: int,
                 page_size: int = 16):
        s = self.shape = shape
        self.device, self.dtype, self.page = device, dtype, page_size
        d = s.head_dim

        def w(o, i):
            t = torch.empty(o, i, device=device, dtype=dtype)
            t.normal_(0.0, 0.02, generator=gen)
            return t
        self.embed = w(s.vocab, s.hidden)
        self.layers = [_Layer(s, s.hidden, gen, device, dtype) for _ in range(s.layers)]
        self.norm = torch.ones(s.hidden, device=device, dtype=dtype)
        self.lm_head = w(s.vocab, s.hidden)
        # draft head: fc over three target layers' hidden states, one layer
        # taking [embedding ; fused hidden] (2 H), its own norm and vocabulary
        self.d_fc = w(s.hidden, 3 * s.hidden)
        self.d_layer = _Layer(s, 2 * s.hidden, gen, device, dtype)
        self.d_norm = torch.ones(s.hidden, device=device, dtype=dtype)
        self.d_head = w(s.draft_vocab, s.hidden)
        # draft ids -> target ids; tv_tree_finalize takes EAGLE3's offset form
        # (target = draft + d2t[draft])
        if s.draft_vocab == s.vocab:
            self.d2t_map, self.d2t = torch.arange(s.vocab, device=device), None
        else:
            self.d2t_map = torch.sort(torch.randperm(s.vocab, generator=torch.Generator().manual_seed(3))[
                : s.draft_vocab])[0].to(device)
            self.d2t = self.d2t_map - torch.arange(s.draft_vocab, device=device)
        # target paged cache: one pool [L, 2, P, Hkv, page, D], identity page table
        self.max_tokens = max_tokens
        pages = -(-max_tokens // page_size)
        self.pool = torch.empty((s.layers, 2, pages, s.kv_heads, page_size, d), device=device, dtype=dtype)
        self.page_table = torch.arange(pages, dtype=torch.int32, device=device).view(1, pages)
        # draft working cache (the retrieval working set) + room for the tree
        dpages = -(-(draft_ctx + 128) // page_size)
        self.d_pool = torch.empty((2, dpages, s.kv_heads, page_size, d), device=device, dtype=dtype)
        self.d_table = torch.arange(dpages, dtype=torch.int32, device=device).view(1, dpages)
        self.draft_ctx = draft_ctx
        self.cos, self.sin = rope_tables(d, max_tokens + 64, s.rope_theta, device, dtype)
        # the draft reads the step's start position from the device, so its
        # whole tree growth can be replayed as one CUDA graph per step
        self._start = torch.zeros((), dtype=torch.int64, device=device)
        self._graphs: Dict[tuple, object] = {}
        # verify through per-layer-boundary CUDA graphs (verify_graphed)
        self.graph_verify = True

    @classmethod
    def from_config(cls, shape: Optional[LlamaShape] = None, *, device="cuda", dtype=torch.bfloat16, seed: int = 0,
                    max_tokens: int = 65536 + 1024, draft_ctx: int = 2048) -> "SpecDecodeModel":
        """Tokenizer-free constructor: random-init weights from ``seed``."""
        gen = torch.Generator(device=device).manual_seed(seed)
        return cls(shape or LlamaShape(), torch.device(device), dtype, gen, max_tokens, draft_ctx)

    def fill_context(self, length: int, seed: int = 0):
        """Stand-in for the prefill of a ``length``-token prompt: the cache rows
        ``[0, length)`` of every layer (and the draft's working cache) get
        N(0, 1) keys / values.  Returns the root token for the first step."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        pages = -(-length // self.page)
        self.pool[:, :, :pages].normal_(generator=g)
        self.d_pool.normal_(generator=g)
        return int(torch.randint(0, self.shape.vocab, (1,), generator=torch.Generator().manual_seed(seed)))

    # ---- target -------------------------------------------------------------
    def verify(self, ids: torch.Tensor, pos: torch.Tensor, bits: torch.Tensor, start: int):
        """Target forward over the M tree rows (ids [M], positions [M], packed
        root-prepended mask bits [M, words]); returns the final normalised
        hidden [M, H] and the feature layers' hidden states [M, 3 H]."""
        s = self.shape
        x = self.embed[ids]
        feats = []
        for li, L in enumerate(self.layers):
            x = _layer_forward(s, L, rms_norm(x, L.ln1, s.rms_eps), x, self.pool[li, 0], self.pool[li, 1],
                               self.page_table, start, pos, bits[None], ids.numel(), self.cos, self.sin)
            if li in s.feature_layers:
                feats.append(x)
        return rms_norm(x, self.norm, s.rms_eps), torch.cat(feats, dim=-1)

    def verify_graphed(self, ids: torch.Tensor, pos: torch.Tensor, bits: torch.Tensor, start: int):
        """:meth:`verify` with the torch work between two attention calls (the
        output projection, the MLP, the next layer's norm and q / k / v
        projection) replayed from CUDA graphs, one per layer boundary,
        captured on first use per row count.  RoPE + KV append and the
        attention, whose arguments change every step (the cache length), are
        launched between the replays.  Returns static buffers, overwritten by
        the next call: the final normalised hidden [M, H] and the feature
        layers' hidden states [M, 3 H]."""
        t = ids.numel()
        key = ("verify", t, bits.shape[-1])
        if key not in self._graphs:
            self._graphs[key] = self._capture_verify(t, bits.shape[-1])
        vs = self._graphs[key]
        vs["ids"].copy_(ids)
        vs["pos"].copy_(pos)
        vs["bits"].copy_(bits)
        vs["graphs"][0].replay()
        for li in range(self.shape.layers):
            self._verify_attend(vs, li, start, t)
            vs["graphs"][li + 1].replay()
        return vs["hidden"], vs["feats"]

    def _verify_segment(self, vs, li: int):
        """The torch work after layer li's attention (li = -1: the embedding)
        up to layer li + 1's q / k / v projection (or the final norm)."""
        s = self.shape
        x = vs["x"]
        if li < 0:
            torch.index_select(self.embed, 0, vs["ids"], out=x)
        else:
            L = self.layers[li]
            x.addmm_(vs["o"].view(x.shape[0], -1), L.wo.t())
            gu = rms_norm(x, L.ln2, s.rms_eps) @ L.wgu.t()
            x.addmm_(silu_mul(gu, s.ffn), L.wdown.t())
            if li in s.feature_layers:
                j = s.feature_layers.index(li)
                vs["feats"][:, j * s.hidden:(j + 1) * s.hidden].copy_(x)
        if li + 1 < s.layers:
            L = self.layers[li + 1]
            torch.matmul(rms_norm(x, L.ln1, s.rms_eps), L.wqkv.t(), out=vs["qkv"])
        else:
            vs["hidden"].copy_(rms_norm(x, self.norm, s.rms_eps))

    def _verify_attend(self, vs, li: int, start: int, t: int):
        """Layer li's RoPE + KV append and verify attention on the static buffers."""
        s = self.shape
        hq, hk, d = s.heads, s.kv_heads, s.head_dim
        qkv = vs["qkv"]
        q = qkv[:, : hq * d].view(1, t, hq, d).transpose(1, 2)
        k = qkv[:, hq * d: (hq + hk) * d].view(1, t, hk, d).transpose(1, 2)
        v = qkv[:, (hq + hk) * d:].view(1, t, hk, d).transpose(1, 2)
        pk, pv = self.pool[li, 0], self.pool[li, 1]
        rope_append(q, k, v, self.cos, self.sin, vs["pos"].view(1, t), pk, pv, start=start,
                    page_table=self.page_table, page_size=self.page, out=vs["qr"], validate=False)
        attention(vs["qr"].transpose(1, 2), pk, pv, num_keys=start + t, page_table=self.page_table,
                  mask_bits=vs["bits"][None], mask_len=t, out=vs["o"])

    def _capture_verify(self, t: int, words: int):
        s = self.shape
        dev, dt = self.device, self.dtype
        qkv_dim = (s.heads + 2 * s.kv_heads) * s.head_dim
        vs = {"ids": torch.zeros(t, dtype=torch.int64, device=dev),
              "pos": torch.zeros(t, dtype=torch.int64, device=dev),
              "bits": torch.zeros((t, words), dtype=torch.int64, device=dev),
              "x": torch.zeros((t, s.hidden), dtype=dt, device=dev),
              "qkv": torch.zeros((t, qkv_dim), dtype=dt, device=dev),
              "qr": torch.zeros((1, s.heads, t, s.head_dim), dtype=dt, device=dev),
              "o": torch.zeros((1, t, s.heads, s.head_dim), dtype=dt, device=dev),
              "hidden": torch.zeros((t, s.hidden), dtype=dt, device=dev),
              "feats": torch.zeros((t, len(s.feature_layers) * s.hidden), dtype=dt, device=dev)}
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for li in range(-1, s.layers):
                self._verify_segment(vs, li)           # warm-up outside the capture
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graphs = []
        for li in range(-1, s.layers):
            g = torch.cuda.CUDAGraph()
            # replayed in capture order, never concurrently: one memory pool
            with torch.cuda.graph(g, pool=graphs[0].pool() if graphs else None):
                self._verify_segment(vs, li)
            graphs.append(g)
        vs["graphs"] = graphs
        return vs

    # ---- draft --------------------------------------------------------------
    def draft_tree(self, root: torch.Tensor, root_feat: torch.Tensor, width: int, depth: int):
        """Grow a ``width`` x ``depth`` tree from the root.  root [1] target id,
        root_feat [1, 3 H] target features; the root's position is the device
        scalar ``self._start``.  Nothing is read back to the host.  Returns the
        finalize_tree dict."""
        s = self.shape
        dev = self.device
        ctx = self.draft_ctx
        fused = root_feat @ self.d_fc.t()                                   # [1, H]
        tok = root.view(1)
        feat = fused
        # (no Python scalars written into device tensors: the growth is
        # captured as a CUDA graph, where a host-to-device copy is not allowed)
        one = torch.ones(width, dtype=torch.int8, device=dev)
        anc = torch.zeros((1 + width * depth, 1 + width * depth), dtype=torch.int8, device=dev)
        anc[0, 0:1].fill_(1)
        rows_now = torch.zeros(1, dtype=torch.long, device=dev)               # tree rows of the inputs
        parents_matrix = torch.zeros((depth, width), dtype=torch.int64, device=dev)
        ids_matrix = torch.zeros((depth, width), dtype=torch.int64, device=dev)
        score = torch.zeros(1, device=dev)
        written = 0
        for dd in range(depth):
            t = tok.numel()
            emb = self.embed[tok]
            x_in = torch.cat([rms_norm(emb, self.d_layer.ln1[: s.hidden], s.rms_eps),
                              rms_norm(feat, self.d_layer.ln1[s.hidden:], s.rms_eps)], dim=-1)
            pos = (self._start + dd).expand(t).contiguous()
            keep = anc[rows_now][:, : written + t]
            bits = pack_tree_mask(keep)
            h = _layer_forward(s, self.d_layer, x_in, feat, self.d_pool[0], self.d_pool[1], self.d_table,
                               ctx + written, pos, bits, written + t, self.cos, self.sin)
            written += t
            logp = torch.log_softmax((rms_norm(h, self.d_norm, s.rms_eps) @ self.d_head.t()).float(), dim=-1)
            top_lp, top_tok = logp.topk(width, dim=-1)                         # [t, width]
            cand = (score[:, None] + top_lp).view(-1)
            best_score, best = cand.topk(width)
            par = best // width                                               # index among the inputs
            new_tok = top_tok.view(-1)[best]
            parents_matrix[dd] = par
            ids_matrix[dd] = new_tok
            new_rows = 1 + dd * width + torch.arange(width, device=dev)
            anc[new_rows] = anc[rows_now[par]]
            anc.index_put_((new_rows, new_rows), one)
            rows_now = new_rows
            score = best_score
            tok = self.d2t_map[new_tok]
            feat = h[par]
        top = torch.arange(depth * width, device=dev)
        return finalize_tree(top, parents_matrix, ids_matrix, depth, width, d2t=self.d2t, validate=False)

    # ---- one speculative step ------------------------------------------------
    def step(self, root: torch.Tensor, root_feat: torch.Tensor, start: int, width: int, depth: int,
             temperature: float, seed: int, offset: int, tree: Optional[Dict[str, torch.Tensor]] = None):
        """Draft (unless ``tree`` is given: a :func:`finalize_tree` result),
        verify, accept, compact.  Returns (accept result, features of the tree
        rows [M, 3 H], CUDA events around the phases)."""
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        if tree is None:
            tree = self._draft_graphed(root, root_feat, start, width, depth)
        ev[1].record()
        ids = torch.cat([root.view(1), tree["input_ids"]])
        pos = torch.cat([torch.full((1,), start, dtype=torch.int64, device=self.device),
                         start + tree["position_ids"]])
        parent = tree["parent_last"]
        if self.graph_verify:
            hidden, feats = self.verify_graphed(ids, pos, tree["mask_bits"], start)
        else:
            hidden, feats = self.verify(ids, pos, tree["mask_bits"], start)
        ev[2].record()
        acc = accept_from_hidden(hidden, self.lm_head, ids, parent, pos,
                                 depth, mode="sample" if temperature > 0 else "greedy", temperature=temperature,
                                 seed=seed, offset=offset)
        self._compact(start, acc, ids.numel())
        ev[3].record()
        return acc, feats, ev

    def _draft_graphed(self, root, root_feat, start: int, width: int, depth: int):
        """draft_tree replayed from a CUDA graph captured on first use (static
        input and output buffers per tree shape)."""
        self._start.fill_(start)
        key = (width, depth)
        if key not in self._graphs:
            s_root = torch.zeros(1, dtype=torch.int64, device=self.device)
            s_feat = torch.zeros((1, 3 * self.shape.hidden), dtype=self.dtype, device=self.device)
            s_root.copy_(root.view(1))
            s_feat.copy_(root_feat)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self.draft_tree(s_root, s_feat, width, depth)           # warm-up outside the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self.draft_tree(s_root, s_feat, width, depth)
            self._graphs[key] = (g, s_root, s_feat, out)
        g, s_root, s_feat, out = self._graphs[key]
        s_root.copy_(root.view(1))
        s_feat.copy_(root_feat)
        g.replay()
        return out

    def _compact(self, start: int, acc, rows: int):
        """Accepted path rows ``start + path[j]`` -> ``start + j`` in every layer's K and V."""
        pool = self.pool
        es = pool.element_size()
        length = -(-(start + rows) // self.page)
        st = _lib.load().tv_compact_paged(
            pool.data_ptr(), pool.shape[0] * 2, pool.shape[3], pool.stride(1) * es, pool.stride(2) * es,
            pool.stride(3) * es, pool.stride(4) * es, pool.shape[5] * es, self.page, self.page_table.data_ptr(),
            self.page_table.data_ptr(), length, pool.shape[2], int(start), acc.result.data_ptr(), rows,
            _lib.stream_ptr(pool.device))
        _lib.check(st, "tv_compact_paged")

    def diffspec_generate(self, prompt_len: int = 65536, max_new_tokens: int = 512, nodes: int = 64,
                          max_depth: int = 8, temperature: float = 1.0, seed: int = 0,
                          max_steps: Optional[int] = None) -> Dict:
        """Decode ``max_new_tokens`` after a ``prompt_len``-token context (filled
        by :meth:`fill_context`).  ``nodes`` = width x ``max_depth``.  One host
        read per step (the accepted length, as the reference's loop reads it).
        Returns the tokens and per-phase device times."""
        width = nodes // max_depth
        if width * max_depth != nodes:
            raise ValueError("nodes must be a multiple of max_depth")
        if prompt_len + max_new_tokens + nodes + 2 > self.max_tokens:
            raise ValueError("cache too small for the request")
        root_tok = self.fill_context(prompt_len, seed)
        root = torch.tensor([root_tok], device=self.device)
        root_feat = torch.zeros((1, 3 * self.shape.hidden), device=self.device, dtype=self.dtype)
        start = prompt_len
        out: List[int] = []
        phases = {"draft_ms": 0.0, "verify_ms": 0.0, "accept_compact_ms": 0.0}
        accepted = []
        steps = 0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        evs = []
        while len(out) < max_new_tokens and (max_steps is None or steps < max_steps):
            acc, feats, ev = self.step(root, root_feat, start, width, max_depth, temperature, seed, offset=steps)
            evs.append(ev)
            res = acc.result
            n = int(res[2].item())                       # the one host read per step
            toks = res[RESULT_HEADER + acc.rows:RESULT_HEADER + acc.rows + n].tolist()
            nxt = res[3:4]
            out.extend(toks[1:] + [None])                # accepted nodes, then the bonus token
            accepted.append(n - 1)
            last_row = res[RESULT_HEADER + n - 1]
            root_feat = feats[last_row].view(1, -1)
            root = nxt
            start += n
            steps += 1
            out[-1] = int(nxt.item())
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        for ev in evs:
            phases["draft_ms"] += ev[0].elapsed_time(ev[1])
            phases["verify_ms"] += ev[1].elapsed_time(ev[2])
            phases["accept_compact_ms"] += ev[2].elapsed_time(ev[3])
        out = out[:max_new_tokens]
        return {"tokens": out, "steps": steps, "wall_s": wall, "accepted_per_step": accepted,
                "phases_ms": phases, "final_length": start}
