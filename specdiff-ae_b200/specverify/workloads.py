"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No checkpoints or datasets are involved: Llama-3.1-8B attention shapes
(32 query heads, 8 KV heads, head_dim 128, RoPE theta 500000), N(0, 1)
keys/values, tree queries N(0, 1)/sqrt(128) rotated at their absolute
positions, and draft trees with a fixed number of nodes per depth whose
parents are drawn uniformly from the previous depth.

Tree convention (the reference's, ``diffspec_model.py:620-624`` and
``tree_verification.py:120-125``): when ``root`` is set, row 0 is the root
(the last accepted token), its row sees only itself and every row sees it;
``parent`` lists, for each drafted node, the index of its parent among the
drafted nodes or -1 for children of the root.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

HEADS, KV_HEADS, HEAD_DIM, ROPE_THETA, VOCAB = 32, 8, 128, 500000.0, 128256


@dataclass
class Tree:
    parent: torch.Tensor      # [n] int64, -1 = child of the root (or of the prefix)
    depth: torch.Tensor       # [n] int64
    keep: torch.Tensor        # [M, M] int8, 1 = visible (M = n + root)
    root: bool

    @property
    def rows(self) -> int:
        return self.keep.shape[0]

    def parent_ext(self) -> torch.Tensor:
        """[M] parent row of every row (root and depth-0 nodes -> the root / -1)."""
        off = 1 if self.root else 0
        p = torch.where(self.parent >= 0, self.parent + off, torch.full_like(self.parent, 0 if self.root else -1))
        return torch.cat([torch.zeros(1, dtype=torch.int64), p]) if self.root else p


def make_tree(gen: torch.Generator, nodes: int, per_depth: int, root: bool = True) -> Tree:
    depth = torch.arange(nodes) // per_depth
    parent = torch.full((nodes,), -1, dtype=torch.int64)
    for i in range(nodes):
        d = int(depth[i])
        if d > 0:
            parent[i] = (d - 1) * per_depth + int(torch.randint(0, per_depth, (1,), generator=gen))
    off = 1 if root else 0
    m = nodes + off
    keep = torch.zeros((m, m), dtype=torch.int8)
    if root:
        keep[:, 0] = 1
    for i in range(nodes):
        r = i + off
        keep[r, r] = 1
        p = int(parent[i])
        while p >= 0:
            keep[r, p + off] = 1
            p = int(parent[p])
    return Tree(parent, depth.to(torch.int64), keep, root)


def rope(x: torch.Tensor, pos: torch.Tensor, theta: float = ROPE_THETA) -> torch.Tensor:
    """Rotary embedding (rotate-half form) of x [..., M, H, D] at positions pos [M]."""
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=x.device) / d))
    ang = pos.to(x.device, torch.float64)[:, None] * inv[None]
    cos = torch.cat([ang.cos(), ang.cos()], -1).float()[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1).float()[:, None, :]
    xf = x.float()
    rot = torch.cat([-xf[..., d // 2:], xf[..., : d // 2]], dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


@dataclass
class PagedVerify:
    """Config-2-style single-layer paged verify problem (batch B)."""
    q: torch.Tensor             # [B, M, H, D]
    k_pool: torch.Tensor        # [P, Hkv, page, D]
    v_pool: torch.Tensor
    page_table: torch.Tensor    # [B, pages] int32 (prefix pages then tree pages)
    tree: Tree
    prefix_len: int
    page_size: int
    extra: dict = field(default_factory=dict)

    @property
    def num_keys(self) -> int:
        return self.prefix_len + self.tree.rows

    def algorithmic_bytes(self) -> int:
        """Bytes one verify call must move at minimum: every visible K/V row once,
        Q and O once, the LSE, page table and bitmask."""
        b, m, h, d = self.q.shape
        hkv = self.k_pool.shape[1]
        es = self.q.element_size()
        kv = b * (self.prefix_len + m) * hkv * d * 2 * es
        qo = 2 * b * m * h * d * es
        lse = b * m * h * 4
        pt = self.page_table.numel() * 4
        bits = b * m * ((m + 63) // 64) * 8
        return kv + qo + lse + pt + bits

    def flops(self) -> int:
        b, m, h, d = self.q.shape
        vis = int(self.tree.keep.sum())
        return b * (4 * m * h * d * self.prefix_len + 4 * h * d * vis)

    def contiguous_kv(self, b: int = 0):
        """[S+M, Hkv, D] K and V of sequence b gathered through the page table."""
        pages = self.page_table[b].long()
        k = self.k_pool[pages].permute(0, 2, 1, 3).reshape(-1, self.k_pool.shape[1], self.k_pool.shape[3])
        v = self.v_pool[pages].permute(0, 2, 1, 3).reshape(-1, self.v_pool.shape[1], self.v_pool.shape[3])
        return k[: self.num_keys], v[: self.num_keys]


def paged_verify(*, prefix_len: int = 65536, nodes: int = 64, per_depth: int = 8, root: bool = False,
                 batch: int = 1, heads: int = HEADS, kv_heads: int = KV_HEADS, head_dim: int = HEAD_DIM,
                 page_size: int = 16, spare_pages: int = 64, dtype=torch.bfloat16, device="cuda",
                 seed: int = 0) -> PagedVerify:
    """Paged verify workload (BASELINE config 2 at the defaults).

    The prefix's logical pages map to a seeded random permutation of the
    first ``batch * prefix_len / page_size`` physical pages; the tree's
    tokens follow in fresh pages; ``spare_pages`` more stay free for
    copy-on-write.  K/V are drawn on ``device`` from a seeded generator.
    """
    gen = torch.Generator().manual_seed(seed)
    tree = make_tree(gen, nodes, per_depth, root=root)
    m = tree.rows
    ctx_pages = -(-prefix_len // page_size)
    tree_pages = -(-(prefix_len + m) // page_size) - prefix_len // page_size
    n_pages = batch * (ctx_pages + tree_pages) + spare_pages
    perm = torch.randperm(batch * ctx_pages, generator=gen).to(torch.int32).view(batch, ctx_pages)
    tree_ids = (batch * ctx_pages + torch.arange(batch * tree_pages, dtype=torch.int32)).view(batch, tree_pages)
    first_tree_lp = prefix_len // page_size
    table = torch.full((batch, first_tree_lp + tree_pages), -1, dtype=torch.int32)
    table[:, :first_tree_lp] = perm[:, :first_tree_lp]
    table[:, first_tree_lp:] = tree_ids
    if prefix_len % page_size:
        # The partially filled last prefix page is shared with the tree tokens.
        table[:, first_tree_lp] = perm[:, first_tree_lp]
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (n_pages, kv_heads, page_size, head_dim)
    k_pool = torch.randn(shape, generator=dgen, device=device, dtype=torch.float32).to(dtype)
    v_pool = torch.randn(shape, generator=dgen, device=device, dtype=torch.float32).to(dtype)
    pos = prefix_len + tree.depth + (1 if root else 0)
    if root:
        pos = torch.cat([torch.tensor([prefix_len]), pos])
    q = torch.randn((batch, m, heads, head_dim), generator=gen) / math.sqrt(head_dim)
    q = rope(q, pos).to(dtype).to(device)
    return PagedVerify(q, k_pool, v_pool, table.to(device), tree, prefix_len, page_size,
                       extra={"positions": pos})


@dataclass
class Acceptance:
    logits: torch.Tensor     # [M, V]
    draft: torch.Tensor      # [M] int64 (row 0 = root token)
    parent: torch.Tensor     # [M-1] int64
    pos: torch.Tensor        # [M] int64
    tree: Tree
    planted: list


def acceptance(*, nodes: int = 64, per_depth: int = 8, vocab: int = VOCAB, prefix_len: int = 65536,
               plant: bool = True, dtype=torch.bfloat16, device="cuda", seed: int = 0) -> Acceptance:
    """Greedy-acceptance workload: logits ~ N(0, 4) (sigma 2) over the vocabulary,
    random draft ids, and (``plant``) one root-to-leaf chain whose draft ids
    equal their parent's argmax so the accepted length is non-trivial."""
    gen = torch.Generator().manual_seed(seed)
    tree = make_tree(gen, nodes, per_depth, root=True)
    m = tree.rows
    dgen = torch.Generator(device=device).manual_seed(seed + 7)
    logits = (torch.randn((m, vocab), generator=dgen, device=device) * 2.0).to(dtype)
    draft = torch.randint(0, vocab, (m,), generator=gen)
    chain = []
    if plant:
        leaf = nodes - 1 - int(torch.randint(0, per_depth, (1,), generator=gen))
        p = leaf
        while p >= 0:
            chain.append(p)
            p = int(tree.parent[p])
        chain.reverse()
        am = torch.argmax(logits.float(), dim=-1).cpu()
        prev = 0
        for i in chain:
            draft[i + 1] = am[prev]
            prev = i + 1
    pos = torch.cat([torch.tensor([prefix_len]), prefix_len + 1 + tree.depth])
    return Acceptance(logits, draft.to(device), tree.parent.to(device), pos.to(device), tree, chain)


@dataclass
class Config1:
    """BASELINE config 1 (the CPU-runnable single-layer verify), fp32 on the CPU.

    Prefix keys/values in the reference cache layout ``[B, Hkv, S, D]``; the
    M = 65 tree rows are the root (the last accepted token, position S: the
    reference's loop keeps ``past_key_values[0][0].shape[2] == draft_position_ids[0]``,
    ``diffspec_model.py:637``) and 64 drafted nodes at positions S + 1 + depth
    (``diffspec_model.py:620-624``).  ``q_raw`` / ``k_tree_raw`` are the
    projections before RoPE; the tree's values need none."""
    q_raw: torch.Tensor          # [1, M, H, D]
    k_prefix: torch.Tensor       # [1, Hkv, S, D]
    v_prefix: torch.Tensor
    k_tree_raw: torch.Tensor     # [1, Hkv, M, D]
    v_tree: torch.Tensor
    positions: torch.Tensor      # [M] int64
    tree: Tree
    logits: torch.Tensor         # [M, V] fp32, N(0, 4) (sigma 2)
    draft: torch.Tensor          # [M] int64 (row 0 = root token)
    planted: list                # drafted nodes of the planted root-to-leaf chain

    @property
    def prefix_len(self) -> int:
        return self.k_prefix.shape[2]


def config1(*, seed: int = 0, prefix_len: int = 4096, nodes: int = 64, per_depth: int = 8,
            heads: int = HEADS, kv_heads: int = KV_HEADS, head_dim: int = HEAD_DIM, vocab: int = VOCAB) -> Config1:
    """Seeded config-1 inputs (one CPU generator, draws in a fixed order):
    tree parents, q ~ N(0,1)/sqrt(D), prefix K, V ~ N(0,1), tree K, V ~ N(0,1),
    logits ~ N(0, 4) over the vocabulary, draft ids ~ U[0, V), then the planted
    chain (draft id of each chain node = its parent row's argmax)."""
    gen = torch.Generator().manual_seed(seed)
    tree = make_tree(gen, nodes, per_depth, root=True)
    m = tree.rows
    q = torch.randn((1, m, heads, head_dim), generator=gen) / math.sqrt(head_dim)
    kp = torch.randn((1, kv_heads, prefix_len, head_dim), generator=gen)
    vp = torch.randn((1, kv_heads, prefix_len, head_dim), generator=gen)
    kt = torch.randn((1, kv_heads, m, head_dim), generator=gen)
    vt = torch.randn((1, kv_heads, m, head_dim), generator=gen)
    logits = torch.randn((m, vocab), generator=gen) * 2.0
    draft = torch.randint(0, vocab, (m,), generator=gen)
    leaf = nodes - 1 - int(torch.randint(0, per_depth, (1,), generator=gen))
    chain = []
    p = leaf
    while p >= 0:
        chain.append(p)
        p = int(tree.parent[p])
    chain.reverse()
    am = torch.argmax(logits, dim=-1)
    prev = 0
    for i in chain:
        draft[i + 1] = am[prev]
        prev = i + 1
    pos = torch.cat([torch.tensor([prefix_len]), prefix_len + 1 + tree.depth])
    return Config1(q, kp, vp, kt, vt, pos, tree, logits, draft, chain)
