"""Contiguous target KV cache: the drop-in for ``diffspec.runtime.cache_state``.

``KVCache`` and ``initialize_past_key_values`` keep the reference's layout and
return contract (``cache_state.py:4-151``): one pre-allocated buffer
``[2 * layers_on_device, B, H_kv, S_budget, D]`` per device that hosts layers,
``KVCache`` views of K and V per layer, and a CPU int64 length per K/V.  The
verify kernels read these buffers in place (``buffer[2l].transpose(1, 2)`` is
the ``[B, S, H_kv, D]`` view :func:`specverify.runtime.tree_attention.verify_attention`
takes) -- no GQA expansion -- and :func:`specverify.draft.tree_verification.compact_kv`
compacts them after acceptance.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch


class KVCache:
    """One layer's K or V view of a device buffer plus its CPU length."""

    def __init__(self, data, current_length):
        self.data = data
        self.current_length = current_length

    @property
    def shape(self):
        # current_length is one element of the CPU int64 length tensor that
        # initialize_past_key_values makes (cache_state.py:124-125): reading
        # it is a host memory load, not a device synchronisation.  It is read
        # at every use rather than mirrored, because callers update the shared
        # length tensor directly (verify_new's current_length_data.fill_).
        return (self.data.shape[0], self.data.shape[1], int(self.current_length), self.data.shape[3])

    def copy(self, indices: torch.Tensor, prev_length: int, dim: int = 2):
        tgt = self.data.index_select(dim, indices)
        self.data.narrow(dim, prev_length, tgt.shape[dim]).copy_(tgt, non_blocking=True)
        self.current_length.fill_(prev_length + tgt.shape[dim])

    def cat(self, tensor: torch.Tensor, dim: int = 2):
        self.data.narrow(dim, self.current_length, tensor.shape[dim]).copy_(tensor)
        self.current_length.add_(tensor.shape[dim])
        return torch.narrow(self.data, 2, 0, self.current_length)


def initialize_past_key_values(model, full_cache_budget: int, batch_size: int = 1
                               ) -> Tuple[List[List[KVCache]], List[torch.Tensor], torch.Tensor]:
    """Allocate per-device KV buffers (``cache_state.py:69-151``)."""
    if batch_size < 1:
        raise ValueError(f"batch_size must be >=1, got {batch_size}")
    cfg = model.config
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    devices = []
    for i in range(cfg.num_hidden_layers):
        try:
            d = model.model.layers[i].self_attn.q_proj.weight.device
        except AttributeError:
            d = model.layers[i].self_attn.q_proj.weight.device
        devices.append(d)
    counts: Dict[torch.device, int] = {}
    for d in devices:
        counts[d] = counts.get(d, 0) + 1
    buffers = {d: torch.zeros((2 * n), batch_size, cfg.num_key_value_heads, full_cache_budget, head_dim, device=d,
                              dtype=model.dtype) for d, n in counts.items()}
    lengths = torch.zeros((cfg.num_hidden_layers * 2,), dtype=torch.long, device="cpu")
    used = {d: 0 for d in counts}
    past = []
    for i, d in enumerate(devices):
        base = 2 * used[d]
        past.append([KVCache(buffers[d][base], lengths[2 * i]), KVCache(buffers[d][base + 1], lengths[2 * i + 1])])
        used[d] += 1
    return past, list(buffers.values()), lengths
