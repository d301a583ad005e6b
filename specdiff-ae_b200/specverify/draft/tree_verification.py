"""Tree acceptance and KV compaction on B200: the drop-in for
``diffspec.draft.tree_verification``.

:func:`verify_new` / :func:`verify` keep the reference's 15 positional
arguments and 7-tuple return (``diffspec/draft/tree_verification.py:66-257``).
Steps 1-3 of the reference -- per-node target token, acceptance closure,
deepest-node pick, path trace and the KV compaction -- run as device kernels
(``tv_accept``, ``tv_compact_contig``); the host reads back one small result
buffer instead of four tensors plus Python loops
(``tree_verification.py:112-179``), and the compaction is already queued on
the stream when it does.  Step 4 (appending tokens and asking the caller's
draft model for the next tree) is the caller's glue and stays as in the
reference.

Sampling (``logits_processor`` given): the reference draws one token per node
with ``torch.multinomial(softmax(logits))`` (``:104-106``).  Here the draw is
the Gumbel-max rule on the device (an exact sample from the same
distribution) with Philox noise seeded from torch's default generator, so
``torch.manual_seed`` still fixes the result.  The logits processors
themselves are the caller's (transformers) and are applied exactly as the
reference does; at temperature 1.0 the list is empty and nothing runs.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import _lib
from ..core.bundle_scheduler import BundleScheduler

__all__ = ["prepare_logits_processor", "tree_decoding", "verify", "verify_new", "accept", "compact_kv",
           "AcceptResult"]

MODE_GREEDY, MODE_SAMPLE, MODE_GIVEN = 0, 1, 2
RESULT_HEADER = 8


def prepare_logits_processor(temperature: float = 0.0, repetition_penalty: float = 0.0, top_p: float = 0.0,
                             top_k: int = 0):
    """Same rule as ``tree_verification.py:15-32`` (None when greedy)."""
    from transformers.generation.logits_process import (LogitsProcessorList, RepetitionPenaltyLogitsProcessor,
                                                        TemperatureLogitsWarper, TopKLogitsWarper,
                                                        TopPLogitsWarper)
    procs = LogitsProcessorList()
    if temperature > 1e-5:
        if temperature != 1.0:
            procs.append(TemperatureLogitsWarper(temperature))
        if repetition_penalty > 1.0:
            procs.append(RepetitionPenaltyLogitsProcessor(repetition_penalty))
        if 1e-8 <= top_p < 1.0:
            procs.append(TopPLogitsWarper(top_p))
        if top_k > 0:
            procs.append(TopKLogitsWarper(top_k))
        return procs
    return None


def tree_decoding(model, draft_input_ids, past_key_values, draft_position_ids, tree_attention_mask):
    """Target forward over the draft tree (caller glue, ``tree_verification.py:35-64``)."""
    dm = model.draft_model
    if dm.use_retrieval_cache:
        cond = dm.timestep % dm.retrieve_every_n_steps == 0
        dm.retrieval_condition = cond
    else:
        cond = False
    outputs, tree_logits, hidden_state = model(draft_input_ids, tree_attention_mask=tree_attention_mask,
                                               output_orig=True, past_key_values=past_key_values,
                                               position_ids=draft_position_ids, init=False,
                                               retrieve_attn_scores=cond, best=dm.best)
    draft_device = dm.lm_head.weight.device
    if outputs["hidden_states"][0].device != draft_device:
        outputs["hidden_states"] = [x.to(draft_device) for x in outputs["hidden_states"]]
    return tree_logits, torch.cat(outputs["hidden_states"], dim=-1), outputs


@dataclass
class AcceptResult:
    """Device-side acceptance outcome (see ``tv_accept`` in include/specverify.h)."""
    next_tokens: torch.Tensor   # [M] int64, target token per node
    result: torch.Tensor        # [8 + 2M] int64
    rows: int

    @classmethod
    def from_path(cls, path: List[int], rows: int, device, tokens: Optional[List[int]] = None) -> "AcceptResult":
        """Result buffer for an accepted path decided elsewhere (e.g. on the host),
        so the compaction kernels can consume it."""
        res = torch.zeros(RESULT_HEADER + 2 * rows, dtype=torch.int64)
        res[1] = path[-1] if path else 0
        res[2] = len(path)
        res[RESULT_HEADER:RESULT_HEADER + len(path)] = torch.tensor(path, dtype=torch.int64)
        if tokens is not None:
            res[RESULT_HEADER + rows:RESULT_HEADER + rows + len(tokens)] = torch.tensor(tokens, dtype=torch.int64)
        return cls(torch.zeros(rows, dtype=torch.int64, device=device), res.to(device), rows)

    def to_host(self):
        """One D2H copy; returns a dict with python ints / lists."""
        h = self.result.cpu().tolist()
        if h[0] != 0:
            raise _lib.SpecVerifyError(h[0], "tv_accept: parent pointers out of range or cyclic")
        n = h[2]
        return {
            "max_id": h[1],
            "path": h[RESULT_HEADER:RESULT_HEADER + n],
            "best_candidate": h[RESULT_HEADER + self.rows:RESULT_HEADER + self.rows + n],
            "accept_length": n - 1,
            "next_token": h[3],
        }


def _i64(t: torch.Tensor, dev) -> torch.Tensor:
    return t.to(device=dev, dtype=torch.int64).contiguous().view(-1)


def accept(logits: Optional[torch.Tensor], draft: torch.Tensor, parent: torch.Tensor,
           position_ids: torch.Tensor, max_depth: int, *, mode: str = "greedy",
           sampled: Optional[torch.Tensor] = None, temperature: float = 1.0,
           seed: Optional[int] = None, offset: int = 0) -> AcceptResult:
    """Run the acceptance kernels.

    logits [1, M, V] / [M, V] (bf16, fp16 or fp32, unit stride on V);
    draft [1, M] / [M]; parent [M-1]; position_ids [M] / [1, M].
    mode: "greedy" (argmax), "sample" (Gumbel-max at ``temperature``),
    "given" (``sampled`` [M] target tokens supplied by the caller).
    """
    dev = _lib.require_cuda(draft)
    d = _i64(draft, dev)
    m = d.numel()
    par = _i64(parent, dev) if m > 1 else torch.zeros(1, dtype=torch.int64, device=dev)
    pos = _i64(position_ids.reshape(-1)[:m] if position_ids.dim() == 1 else position_ids[0], dev)
    a = _lib.AcceptArgs()
    a.mode = {"greedy": MODE_GREEDY, "sample": MODE_SAMPLE, "given": MODE_GIVEN}[mode]
    a.rows = m
    a.draft, a.parent, a.pos = d.data_ptr(), par.data_ptr(), pos.data_ptr()
    a.max_depth = int(max_depth)
    keep = [d, par, pos]
    if a.mode != MODE_GIVEN:
        lg = logits.reshape(-1, logits.shape[-1])
        _lib.require_cuda(lg)
        if lg.shape[0] != m:
            raise _lib.SpecVerifyError(-1, f"logits rows {lg.shape[0]} != draft nodes {m}")
        if lg.stride(1) != 1:
            lg = lg.contiguous()
        a.logits_dtype = _lib.dtype_code(lg.dtype)
        a.logits = lg.data_ptr()
        a.logits_sm = lg.stride(0)
        a.vocab = lg.shape[1]
        keep.append(lg)
    else:
        s = _i64(sampled, dev)
        a.sampled = s.data_ptr()
        keep.append(s)
    if a.mode == MODE_SAMPLE:
        a.temperature = float(temperature)
        if seed is None:
            seed = int(torch.randint(0, 2 ** 62, (1,)).item())
        a.seed = int(seed) & (2 ** 64 - 1)
        a.offset = int(offset) & (2 ** 64 - 1)
    nxt = torch.empty(m, dtype=torch.int64, device=dev)
    res = torch.empty(RESULT_HEADER + 2 * m, dtype=torch.int64, device=dev)
    a.next_tokens, a.result = nxt.data_ptr(), res.data_ptr()
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.tv_accept_workspace_size(ctypes.byref(a), ctypes.byref(need)), "tv_accept_workspace_size")
    ws = torch.empty(max(int(need.value), 16), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.tv_accept(ctypes.byref(a), _lib.stream_ptr(dev)), "tv_accept")
    return AcceptResult(nxt, res, m)


def accept_from_hidden(hidden: torch.Tensor, lm_head_weight: torch.Tensor, draft: Optional[torch.Tensor],
                       parent: Optional[torch.Tensor], position_ids: Optional[torch.Tensor], max_depth: int, *,
                       mode: str = "greedy", temperature: float = 1.0, seed: Optional[int] = None,
                       offset: int = 0) -> AcceptResult:
    """lm_head and acceptance in one pass: ``logits = hidden @ lm_head_weight.T``
    (``diffspec_model.py:229-231``) is never materialised; each node's
    argmax (or Gumbel-max sample at ``temperature``) over the logits rounded to
    the weight's dtype feeds the acceptance rule of :func:`accept`
    (``tree_verification.py:100-162``).

    hidden [1, M, H] / [M, H] (M <= 128, H a multiple of 64), weight [V, H],
    both bf16 or fp16.  With ``draft=None`` only ``next_tokens`` is filled.
    The same ``seed`` / ``offset`` give the same samples as :func:`accept` on
    the same rounded logits.
    """
    dev = _lib.require_cuda(hidden, lm_head_weight, draft)
    x = hidden.reshape(-1, hidden.shape[-1])
    if x.stride(1) != 1:
        x = x.contiguous()
    w = lm_head_weight if lm_head_weight.stride(1) == 1 else lm_head_weight.contiguous()
    if x.dtype != w.dtype:
        raise _lib.SpecVerifyError(-2, f"hidden {x.dtype} and lm_head weight {w.dtype} differ")
    if w.shape[1] != x.shape[1]:
        raise _lib.SpecVerifyError(-1, f"weight {tuple(w.shape)} does not match hidden size {x.shape[1]}")
    m = x.shape[0]
    a = _lib.LmheadArgs()
    a.dtype = _lib.dtype_code(x.dtype)
    a.rows, a.hidden, a.vocab = m, x.shape[1], w.shape[0]
    a.x, a.x_sm, a.weight, a.w_sv = x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0)
    a.mode = {"greedy": MODE_GREEDY, "sample": MODE_SAMPLE}[mode]
    keep = [x, w]
    if draft is not None:
        d = _i64(draft, dev)
        if d.numel() != m:
            raise _lib.SpecVerifyError(-1, f"hidden rows {m} != draft nodes {d.numel()}")
        par = _i64(parent, dev) if m > 1 else torch.zeros(1, dtype=torch.int64, device=dev)
        pos = _i64(position_ids.reshape(-1)[:m] if position_ids.dim() == 1 else position_ids[0], dev)
        a.draft, a.parent, a.pos = d.data_ptr(), par.data_ptr(), pos.data_ptr()
        a.max_depth = int(max_depth)
        keep += [d, par, pos]
    if a.mode == MODE_SAMPLE:
        a.temperature = float(temperature)
        if seed is None:
            seed = int(torch.randint(0, 2 ** 62, (1,)).item())
        a.seed = int(seed) & (2 ** 64 - 1)
        a.offset = int(offset) & (2 ** 64 - 1)
    nxt = torch.empty(m, dtype=torch.int64, device=dev)
    res = torch.zeros(RESULT_HEADER + 2 * m, dtype=torch.int64, device=dev)
    a.next_tokens, a.result = nxt.data_ptr(), res.data_ptr()
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.tv_lmhead_accept_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "tv_lmhead_accept_workspace_size")
    ws = torch.empty(max(int(need.value), 16), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.tv_lmhead_accept(ctypes.byref(a), _lib.stream_ptr(dev)), "tv_lmhead_accept")
    return AcceptResult(nxt, res, m)


def compact_kv(past_key_values_data: List[torch.Tensor], start: int, acc: AcceptResult,
               max_rows: Optional[int] = None) -> None:
    """Move the accepted path's KV rows to ``[start, start + n)`` in every buffer.

    Each buffer is ``[..., S_budget, D]`` with the last two dims addressable as
    rows (the reference's ``[2L, B, H_kv, S_budget, D]``).  n and the path come
    from ``acc`` on the device.  ``tree_verification.py:197-217``.
    """
    lib = _lib.load()
    max_rows = acc.rows if max_rows is None else max_rows
    for data in past_key_values_data:
        _lib.require_cuda(data)
        if data.stride(-1) != 1:
            raise _lib.SpecVerifyError(-3, "KV buffer must have unit stride on head_dim")
        lead = data.shape[:-2]
        flat = data.reshape(-1, data.shape[-2], data.shape[-1]) if len(lead) != 1 else data
        if flat.data_ptr() != data.data_ptr():
            raise _lib.SpecVerifyError(-3, "KV buffer leading dims must be collapsible")
        es = data.element_size()
        st = lib.tv_compact_contig(flat.data_ptr(), flat.shape[0], flat.stride(0) * es, flat.stride(1) * es,
                                   flat.shape[2] * es, int(start), acc.result.data_ptr(), int(max_rows),
                                   _lib.stream_ptr(data.device))
        _lib.check(st, "tv_compact_contig")


@torch.no_grad()
def verify_new(input_ids, logits, draft, position_ids, hidden_states, tree_attention_mask,
               past_key_values_data, current_length_data, parent, model, nodes, threshold, max_depth,
               logits_processor, hazard_tracker=None):
    """Verify the draft tree and advance the generation state.

    Same arguments and 7-tuple return as ``tree_verification.py:75-257``:
    ``(input_ids, best_candidate, accept_length, next_draft, next_position_ids,
    next_tree_attention_mask, next_parent)``.
    """
    if logits_processor is None:
        acc = accept(logits, draft, parent, position_ids, max_depth, mode="greedy")
    else:
        if len(logits_processor) > 0:
            logits = logits_processor(None, logits)
        acc = accept(logits, draft, parent, position_ids, max_depth, mode="sample", temperature=1.0)

    start = int(current_length_data[0].item()) - int(draft.size(1))
    compact_kv(past_key_values_data, start, acc)
    h = acc.to_host()
    max_id = h["max_id"]
    best_candidate = h["best_candidate"]
    best_candidate_id = h["path"]
    accept_length = h["accept_length"]

    dm = model.draft_model
    if getattr(dm, "enable_bundle_scheduling", False):
        scheduler = getattr(dm, "bundle_scheduler", None)
        if scheduler is None:
            scheduler = BundleScheduler(bundle_size=3, max_bundles=100, device=str(draft.device))
            dm.bundle_scheduler = scheduler
        par = parent.detach().to("cpu").tolist()
        m = int(draft.size(1))
        parent_map = {0: -1}
        for i in range(1, m):
            p = par[i - 1]
            parent_map[i] = 0 if (p == i - 1 or p < 0) else p + 1
        children = set(parent_map.values()) - {-1}
        leaf_ids = [i for i in range(m) if i not in children]
        pos_cpu = (position_ids[0] if position_ids.dim() == 2 else position_ids).detach().to("cpu").tolist()
        bundles = scheduler.schedule_bundles({"leaf_ids": leaf_ids, "parent_map": parent_map,
                                              "depth_map": {i: int(pos_cpu[i]) for i in range(m)}},
                                             return_tensors=False)
        dm.last_bundle_stats = {"num_leaves": len(leaf_ids), "num_bundles": len(bundles),
                                "avg_prefix_length": scheduler.avg_prefix_length}

    next_token = acc.next_tokens[max_id].view(1, 1)

    if hazard_tracker is not None:
        pos_cpu = (position_ids[0] if position_ids.dim() == 2 else position_ids).detach().to("cpu")
        observed = int(max(0, (pos_cpu.max() - pos_cpu[0]).item()))
        hazard_tracker.update(-1 if accept_length >= observed else int(accept_length))

    budget = getattr(model, "tree_budget_controller", None)
    next_nodes = int(nodes) if budget is None else budget.observe(int(accept_length))
    dm.last_tree_node_budget = next_nodes

    if getattr(dm, "use_retrieval_cache", False) and getattr(dm, "retrieval_condition", False):
        prev_len = input_ids.shape[1]
        last_scores = dm.attn_scores[:, :, best_candidate_id[-1], :].mean(dim=1).squeeze()
        ids_abs = torch.tensor(best_candidate_id, device=last_scores.device) + prev_len
        dm.attn_scores_final = torch.cat((last_scores[:prev_len], last_scores[ids_abs]), dim=0)

    current_length_data.fill_(start + len(best_candidate_id))

    input_ids = torch.cat([input_ids, torch.tensor(best_candidate, device=input_ids.device,
                                                   dtype=input_ids.dtype).unsqueeze(0)], dim=-1)
    new_hidden = hidden_states[:, torch.tensor(best_candidate_id, device=hidden_states.device), :]
    next_draft, next_pos, next_mask, next_parent = dm.build_speculative_tree(
        new_hidden, input_ids=torch.cat((input_ids, next_token.to(input_ids.device)), dim=1),
        head=model.base_model.lm_head, nodes=next_nodes, threshold=threshold, max_depth=max_depth)
    next_draft = torch.cat([next_token.to(next_draft.device), next_draft], dim=-1)
    root_pos = (position_ids[0, max_id] if position_ids.dim() == 2 else position_ids[max_id]) + 1
    next_pos = torch.cat([root_pos.to(next_pos.device).view(1), next_pos], dim=-1)
    next_mask = torch.cat([torch.zeros(1, next_mask.size(1), dtype=next_mask.dtype, device=next_mask.device),
                           next_mask], dim=0)
    next_mask = torch.cat([torch.ones(next_mask.size(0), 1, dtype=next_mask.dtype, device=next_mask.device),
                           next_mask], dim=1)
    return input_ids, best_candidate, accept_length, next_draft, next_pos, next_mask, next_parent


def verify(input_ids, logits, draft, position_ids, hidden_states, tree_attention_mask, past_key_values_data,
           current_length_data, parent, model, nodes, threshold, max_depth, logits_processor,
           hazard_tracker=None):
    """Alias of :func:`verify_new` (``tree_verification.py:66-72``)."""
    return verify_new(input_ids, logits, draft, position_ids, hidden_states, tree_attention_mask,
                      past_key_values_data, current_length_data, parent, model, nodes, threshold, max_depth,
                      logits_processor, hazard_tracker)
