"""Sequence-sharded verify attention across the GPUs of one node.

The reference attends the whole prefix on one device
(``llama_target_model.py:839-845``) and has no distributed code.  For long
contexts the prefix KV is split into contiguous, page-aligned shards, one per
rank.  Each rank runs the verify-attention kernel over its shard -- the rank
that owns the tree tail also applies the tree bitmask to the M tree keys --
and produces its partial ``(O_r fp32 [B, M, H, D], lse_r [B, M, H])``.  The
partials are exchanged and every rank merges them in rank order:

    O = sum_r e^{lse_r - L} O_r / sum_r e^{lse_r - L},   L = max_r lse_r

Default exchange: NVLink peer memory, one C call per rank
(``tv_verify_attn_sharded``).  After the attention kernel one kernel combines
this rank's split partials and stores the result straight into the peers'
exchange buffers (mapped into every rank through torch symmetric memory) as
8-byte words carrying the value and the step number, waits on its own
buffer until the peers' words of its rows carry the step, and merges -- no
collective launch, no remote reads, no flags or fences, and no step-wide
barrier.  Fallback (and the host-testable form): ONE NCCL
``all_gather`` of the packed partials and ``tv_merge_partials``.  Both are
order-fixed, so every rank gets bit-identical results (the next layer's
replicated projections need that).  An all-reduce formulation would need a
max-reduce first: two collectives.
"""

from __future__ import annotations

import ctypes
import warnings
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from .. import _lib
from .tree_attention import attention, attn_args, pack_tree_mask


def shard_bounds(total: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Contiguous shard ``[lo, hi)`` of ``total`` tokens for ``rank``.

    Shards are multiples of ``align`` tokens (a page) except the last; all
    ranks but the last get ``ceil(total / world)`` rounded up to ``align``.
    """
    per = -(-total // world)
    per = -(-per // align) * align
    lo = min(total, rank * per)
    hi = min(total, lo + per)
    return lo, hi


class PackedPartial:
    """One rank's partial in a flat fp32 buffer: ``[O (B*M*H*D) | lse (B*M*H)]``."""

    def __init__(self, b, m, h, d, device, dtype=torch.float32):
        self.shape = (b, m, h, d)
        self.n_o = b * m * h * d
        self.n_l = b * m * h
        self.buf = torch.empty(self.n_o + self.n_l, dtype=dtype, device=device)

    @property
    def numel(self):
        return self.n_o + self.n_l

    def o(self, buf=None):
        return (self.buf if buf is None else buf)[: self.n_o].view(*self.shape)

    def lse(self, buf=None):
        b, m, h, _ = self.shape
        return (self.buf if buf is None else buf)[self.n_o:].view(b, m, h)


def merge_packed(gathered: torch.Tensor, part: PackedPartial, world: int, out_dtype: torch.dtype,
                 out: Optional[torch.Tensor] = None, out_lse: Optional[torch.Tensor] = None):
    """``tv_merge_partials`` over ``world`` packed partials laid end to end."""
    b, m, h, d = part.shape
    dev = _lib.require_cuda(gathered)
    if out is None:
        out = torch.empty((b, m, h, d), dtype=out_dtype, device=dev)
    stride = part.numel
    st = _lib.load().tv_merge_partials(world, b * m * h, d, gathered.data_ptr(), stride,
                                       gathered.data_ptr() + part.n_o * gathered.element_size(), stride,
                                       _lib.dtype_code(out_dtype), out.data_ptr(),
                                       _lib.ptr(out_lse), _lib.stream_ptr(dev))
    _lib.check(st, "tv_merge_partials")
    return out


class PeerExchange:
    """This rank's exchange buffer for ``tv_verify_attn_sharded``, mapped into
    every rank of ``group`` (torch symmetric memory): two slots of all ranks'
    partials (8-byte words: value and step number), owner mode's final rows
    and the per-block step counts, zeroed once.
    Successive steps alternate the slots inside the kernel, so the calls can
    be captured into CUDA graphs and replayed any number of times."""

    def __init__(self, group, rows, d, device):
        import torch.distributed._symmetric_memory as symm
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = _lib.load()
        nbytes = ctypes.c_int64(0)
        _lib.check(lib.tv_sharded_exchange_bytes(self.world, rows, d, ctypes.byref(nbytes)),
                   "tv_sharded_exchange_bytes")
        self.nbytes = nbytes.value
        self.buf = symm.empty(-(-nbytes.value // 4), dtype=torch.int32, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm.rendezvous(self.buf, group if group is not None else dist.group.WORLD)
        self.bases = (ctypes.c_void_p * self.world)(*list(self.handle.buffer_ptrs))
        self._ws = None
        dist.barrier(group)    # every rank's buffer is zeroed before any peer writes into it

    def run(self, a, device):
        """``tv_verify_attn_sharded`` of the request ``a`` (see ``attn_args``)."""
        lib = _lib.load()
        need = ctypes.c_size_t(0)
        _lib.check(lib.tv_verify_attn_sharded_workspace_size(ctypes.byref(a), ctypes.byref(need)),
                   "tv_verify_attn_sharded_workspace_size")
        if self._ws is None or self._ws.numel() < need.value:
            self._ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device=device)
        a.workspace = self._ws.data_ptr()
        a.workspace_bytes = self._ws.numel()
        _lib.check(lib.tv_verify_attn_sharded(ctypes.byref(a), self.world, self.rank, self.bases, self.nbytes,
                                              _lib.stream_ptr(device)), "tv_verify_attn_sharded")


class SequenceShardedVerify:
    """Verify attention over a prefix sharded across the ranks of ``group``.

    ``partial_fn`` computes this rank's partial into a :class:`PackedPartial`
    (default: the CUDA kernel); ``merge_fn`` merges the gathered buffer
    (default: ``tv_merge_partials``).  Both are replaceable so the host-side
    exchange can be exercised with CPU ``gloo`` ranks.
    """

    _PEER_MODES = {"auto": 0, "owner": 32, "push": 64}

    def __init__(self, group=None, partial_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None,
                 exchange: str = "auto", peer_mode: str = "auto"):
        """``exchange``: ``"peer"`` (NVLink peer memory, kernels only),
        ``"nccl"`` (one all_gather), or ``"auto"`` (peer when the default
        CUDA partial and merge are used and peer mapping succeeds; a failed
        mapping warns, records ``fallback_reason`` and uses the all_gather).
        ``peer_mode`` (peer exchange): ``"push"`` (every rank's partial to
        every peer, one hop), ``"owner"`` (each row block's partials to the
        rank owning it, which hands the final rows back: two hops, less
        NVLink traffic from four ranks on) or ``"auto"`` (push below four
        ranks, owner from four on)."""
        if peer_mode not in self._PEER_MODES:
            raise ValueError(f"peer_mode must be one of {sorted(self._PEER_MODES)}")
        self.peer_bits = self._PEER_MODES[peer_mode]
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.partial_fn = partial_fn or self._cuda_partial
        self.merge_fn = merge_fn or merge_packed
        self.exchange = exchange
        self._bufs = {}
        self._peer = {}
        self.fallback_reason = None    # set when exchange="auto" fell back to NCCL

    def _peer_exchange(self, b, m, h, d, device):
        if self.exchange == "nccl" or (self.exchange == "auto" and (self.partial_fn != self._cuda_partial
                                                                     or self.merge_fn is not merge_packed)):
            return None
        key = (b, m, h, d, str(device))
        if key not in self._peer:
            try:
                self._peer[key] = PeerExchange(self.group, b * m * h, d, device)
            except Exception as exc:
                if self.exchange == "peer":
                    raise
                # exchange="auto": the NCCL all_gather path takes over, and says so
                warnings.warn(f"SequenceShardedVerify: NVLink peer mapping failed ({type(exc).__name__}: {exc}); "
                              f"using the NCCL all_gather exchange", RuntimeWarning, stacklevel=3)
                self.fallback_reason = f"{type(exc).__name__}: {exc}"
                self._peer[key] = None
        return self._peer[key]

    def buffers(self, b, m, h, d, device):
        key = (b, m, h, d, str(device))
        if key not in self._bufs:
            part = PackedPartial(b, m, h, d, device)
            gathered = torch.empty(self.world * part.numel, dtype=part.buf.dtype, device=device)
            self._bufs[key] = (part, gathered)
        return self._bufs[key]

    @staticmethod
    def _cuda_partial(part: PackedPartial, q, k, v, num_keys, mask_bits, mask_len, page_table, num_splits):
        attention(q, k, v, num_keys=num_keys, page_table=page_table, mask_bits=mask_bits, mask_len=mask_len,
                  out=part.o(), lse=part.lse(), num_splits=num_splits)

    def __call__(self, q, k_shard, v_shard, shard_len: int, tree_mask=None, *, page_table=None,
                 out_dtype=None, num_splits: int = 0, return_lse: bool = False):
        """q [B, M, H, D] (replicated); k_shard/v_shard: this rank's keys (contiguous
        ``[B, n, Hkv, D]`` or a paged pool with ``page_table``), ``shard_len``
        keys in all.  The rank holding the tree passes ``tree_mask`` (M x M keep
        mask or packed bits) and has the M tree keys as its last ``M`` keys.
        Returns the merged output on every rank."""
        b, m, h, d = q.shape
        bits, mlen = None, 0
        if tree_mask is not None:
            bits = tree_mask if tree_mask.dtype == torch.int64 else pack_tree_mask(tree_mask, batch=b)
            mlen = m
        peer = self._peer_exchange(b, m, h, d, q.device)
        if peer is not None:
            out = torch.empty((b, m, h, d), dtype=out_dtype or q.dtype, device=q.device)
            lse = torch.empty((b, m, h), dtype=torch.float32, device=q.device) if return_lse else None
            a, out = attn_args(q, k_shard, v_shard, num_keys=shard_len, page_table=page_table, mask_bits=bits,
                               mask_len=mlen, out=out, lse=lse, num_splits=num_splits, kernel=self.peer_bits)
            peer.run(a, q.device)
            return (out, lse) if return_lse else out
        part, gathered = self.buffers(b, m, h, d, q.device)
        self.partial_fn(part, q, k_shard, v_shard, shard_len, bits, mlen, page_table, num_splits)
        dist.all_gather_into_tensor(gathered, part.buf, group=self.group)
        lse = torch.empty((b, m, h), dtype=torch.float32, device=q.device) if return_lse else None
        out = self.merge_fn(gathered, part, self.world, out_dtype or q.dtype, out_lse=lse)
        return (out, lse) if return_lse else out
