#!/usr/bin/env python3
"""Benchmark: tree-verify attention on B200 (BASELINE config 2 and the sharded scaling run).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload verify|config3|config4|config5|rope-append|lmhead-accept|
                                tree-finalize|chunk-retrieve]
                    [--nodes M --per-depth P --root] [--no-e2e --no-extras --no-cpu-baseline --no-graph]

Default (--workload verify): a step is one verify-attention pass of one layer
over the config-2 problem: 64K-token paged KV cache (16-token pages, seeded
random page permutation), a 64-node depth-8 draft tree, Llama-3.1-8B
attention shapes (32 query / 8 KV heads, head_dim 128), bf16.  Steps rotate
over 4 independent layer pools (1 GiB of KV in all) so no step finds the
previous step's KV in the 126 MB L2.

N = 1 runs config 2 on one GPU.  N > 1 (torchrun, one rank per GPU) runs the
same 64K problem sequence-sharded: each rank attends its contiguous share of
the pages; one kernel per rank then exchanges the (O, lse) partials over
NVLink (to every peer below four ranks, to each row block's owner from four
on) and merges them by log-sum-exp, so every rank holds the full result
("scaling": "strong": total work fixed).  Time = max over ranks of CUDA-event
time.

`value` = algorithmic bytes (every visible K/V row once + Q/O/LSE/page
table/bitmask) / step time, in GB/s, whole job.  `e2e` measures the same call
through the public Python API with the per-step inputs (queries, tree mask)
copied from pinned host memory and the result (output + LSE) read back to
the host inside the timed region; the KV cache is device-resident state.
Side measurements on one GPU: the root-row shape (M = 65), the reference's
GPU op sequence for the same step, and the CPU baseline.

--impl reference times the reference's own CPU path (prefix attention + tree
attention + merge on repeat_kv-expanded K/V, fp32, restated in oracle/) on the
host cores over the full config-2 problem, one pass per step.

Other workloads: config3 (the speculative decode loop, verified tok/s),
config4 (32 layers x 131072 tokens, sequence-sharded, 128-node tree), config5
(batch-4 bundle verify over a chunk arena), and the steps on either side of
the path (rope-append, lmhead-accept, tree-finalize, chunk-retrieve); each
function's docstring says what it times.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))

import torch  # noqa: E402

METRIC = "tree-verify attn HBM GB/s (%peak) + verified tok/s @64K ctx, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one attn_tc_kernel launch on
# this workload, from a full ncu capture of the current kernel (the dominant
# kernel: 90 % of the call's device time; profiles/attn_tc_config2_full.md).
NCU_TRAFFIC_BYTES = 274_913_024


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def physical_gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [x.strip() for x in vis.split(",") if x.strip()]
    if local < len(ids) and ids[local].isdigit():
        return int(ids[local])
    return local


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[2:6]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

TREE = {"nodes": 64, "per_depth": 8, "root": False}     # config 2's tree; --nodes / --per-depth / --root change it


def build_problems(rotate: int, dev, seed: int = 0):
    return [wl_paged(seed=seed + 100 * i, dev=dev, root=TREE["root"]) for i in range(rotate)]


def wl_paged(seed: int, dev, root: bool = False):
    from specverify import workloads as wl
    return wl.paged_verify(seed=seed, device=dev, root=root, nodes=TREE["nodes"], per_depth=TREE["per_depth"])


def run_ours(args, rank, world, dev):
    from specverify.runtime import attention, pack_tree_mask, verify_attention
    from specverify.runtime import sharded as sh

    rotate = 4
    probs = build_problems(rotate, dev)
    p0 = probs[0]
    bits = [pack_tree_mask(p.tree.keep.to(dev)) for p in probs]
    alg_bytes = p0.algorithmic_bytes()
    flops = p0.flops()
    m = p0.tree.rows
    page = p0.page_size

    if world == 1:
        outs = [torch.empty_like(p.q) for p in probs]
        lses = [torch.empty(p.q.shape[:3], dtype=torch.float32, device=dev) for p in probs]

        def step(i):
            p = probs[i % rotate]
            attention(p.q, p.k_pool, p.v_pool, num_keys=p.num_keys, page_table=p.page_table,
                      mask_bits=bits[i % rotate], mask_len=m, out=outs[i % rotate], lse=lses[i % rotate])
        from specverify.runtime.tree_attention import describe_attention
        plan0 = describe_attention(p0.q, p0.k_pool, p0.v_pool, num_keys=p0.num_keys, page_table=p0.page_table,
                                   mask_bits=bits[0], mask_len=m)
        # one attention kernel, plus the split combine when the keys are split
        launches_per_step = 1 if plan0["splits"] == 1 else 2
        workload = (f"config2: paged tree verify, S=65536, {TREE['nodes']}-node depth-"
                    f"{-(-TREE['nodes'] // TREE['per_depth'])} tree{' + root row' if TREE['root'] else ''}, 1 layer, "
                    f"bf16, B=1")
    else:
        # Sequence-sharded: this rank's share of the prefix pages; the last rank
        # also holds the tree's pages and applies the tree bitmask.
        verifier = sh.SequenceShardedVerify(peer_mode=args.peer_mode)
        n_pages_prefix = p0.prefix_len // page
        lo, hi = sh.shard_bounds(n_pages_prefix, world, rank)
        shards = []
        for p in probs:
            tbl = p.page_table[:, lo:hi]
            if rank == world - 1:
                tbl = torch.cat([tbl, p.page_table[:, n_pages_prefix:]], dim=1)
            shards.append(tbl.contiguous())
        shard_len = (hi - lo) * page + (m if rank == world - 1 else 0)

        def step(i):
            p = probs[i % rotate]
            verifier(p.q, p.k_pool, p.v_pool, shard_len, bits[i % rotate] if rank == world - 1 else None,
                     page_table=shards[i % rotate])
        launches_per_step = 2
        workload = (f"config2 sequence-sharded over {world} GPUs: S=65536 paged, 64-node depth-8 tree, 1 layer, "
                    f"bf16, partials exchanged over NVLink as step-tagged words "
                    f"({'pushed to every peer' if (args.peer_mode == 'push' or (args.peer_mode == 'auto' and world < 4)) else 'merged by each row block owner'}) "
                    f"and merged by one fused kernel per step")

    for _ in range(args.warmup):
        for i in range(rotate):
            step(i)
    torch.cuda.synchronize()
    # The timed steps replay CUDA graphs of the launch sequence (one per
    # rotated problem; the sharded step's peer exchange included), so the
    # device time is not bounded by Python launch overhead.
    graphs = []
    if not args.no_graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(rotate):
                step(i)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for i in range(rotate):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(i)
            graphs.append(g)
        torch.cuda.synchronize()

        def step(i):  # noqa: F811 -- the timed loop replays the captured steps
            graphs[i % rotate].replay()

        for i in range(rotate):
            step(i)
        torch.cuda.synchronize()

    sampler = ClockSampler(physical_gpu_index(torch.cuda.current_device()))
    if rank == 0:
        sampler.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        step(i)
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop() if rank == 0 else None
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())

    # ---- end to end through the public API with host buffers -------------
    # Every step copies its Q (and, on the tree rank, the keep mask) from
    # pinned host memory, calls the public API, and copies O and the LSE back
    # to pinned host memory.  Successive steps are independent problems, so
    # the copies of neighbouring steps overlap the kernels (a serving loop
    # does the same); the K steps are replayed as one CUDA graph like the
    # device-timed steps, so Python overhead stays out.
    e2e = None
    if not args.no_e2e:
        tree_rank = world == 1 or rank == world - 1
        q_host = [p.q.cpu().pin_memory() for p in probs]
        keep_host = [p.tree.keep.clone().pin_memory() for p in probs]
        out_host = [torch.empty(p.q.shape, dtype=p.q.dtype).pin_memory() for p in probs]
        lse_host = [torch.empty(p.q.shape[:3], dtype=torch.float32).pin_memory() for p in probs]
        # Inputs are double-buffered on the device; results stay referenced
        # until the timed region ends, so no later step reuses their memory
        # while a copy engine still reads them.
        q_dev = [torch.empty_like(p0.q) for _ in range(2)]
        keep_dev = [torch.empty(p0.tree.keep.shape, dtype=p0.tree.keep.dtype, device=dev) for _ in range(2)]
        cin, cout = torch.cuda.Stream(), torch.cuda.Stream()

        def e2e_steps(first, count, held):
            """Steps first .. first+count-1, pipelined over three streams: the
            input copy of step i+1 (stream cin) overlaps step i's kernels,
            the result copy of step i (stream cout) overlaps step i+1's."""
            main = torch.cuda.current_stream()
            cin.wait_stream(main)
            cout.wait_stream(main)
            freed = [None, None]      # kernels that last read input buffer j
            for i in range(first, first + count):
                j = i % 2
                p = probs[i % rotate]
                with torch.cuda.stream(cin):
                    if freed[j] is not None:
                        cin.wait_event(freed[j])
                    q_dev[j].copy_(q_host[i % rotate], non_blocking=True)
                    if tree_rank:
                        keep_dev[j].copy_(keep_host[i % rotate], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(cin)
                main.wait_event(ready)
                if world == 1:
                    o, lse = verify_attention(q_dev[j], p.k_pool, p.v_pool, p.prefix_len, keep_dev[j],
                                              page_table=p.page_table, return_lse=True)
                else:
                    o, lse = verifier(q_dev[j], p.k_pool, p.v_pool, shard_len, keep_dev[j] if tree_rank else None,
                                      page_table=shards[i % rotate], return_lse=True)
                done = torch.cuda.Event()
                done.record(main)
                freed[j] = done
                with torch.cuda.stream(cout):
                    cout.wait_event(done)
                    out_host[i % rotate].copy_(o, non_blocking=True)
                    lse_host[i % rotate].copy_(lse, non_blocking=True)
                held.append((o, lse))
            main.wait_stream(cin)
            main.wait_stream(cout)

        held = []
        e2e_steps(0, args.warmup, held)
        torch.cuda.synchronize()
        held.clear()
        e2e_graph = None
        if not args.no_graph:
            # The K timed steps are captured as ONE graph (the pipeline would
            # drain at every graph boundary), replayed once untimed first.
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                e2e_steps(0, 2, held)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            held.clear()
            e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(e2e_graph):
                e2e_steps(0, args.steps, held)
            torch.cuda.synchronize()
            e2e_graph.replay()
            torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        if e2e_graph is not None:
            e2e_graph.replay()
        else:
            e2e_steps(0, args.steps, held)
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3 / args.steps
        ems = max(e0.elapsed_time(e1) / args.steps, wall)
        if world > 1:
            t = torch.tensor([ems], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ems = float(t.item())
        e2e_graph = None
        held.clear()
        h2d = p0.q.numel() * p0.q.element_size() * world + p0.tree.keep.numel() * p0.tree.keep.element_size()
        d2h = (p0.q.numel() * p0.q.element_size() + p0.q.shape[0] * p0.q.shape[1] * p0.q.shape[2] * 4) * world
        api = ("specverify.runtime.verify_attention" if world == 1 else
               "specverify.runtime.sharded.SequenceShardedVerify")
        e2e = {"value": round(alg_bytes / (ems * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ems, 4),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": api + " (pinned host q/mask in, out/lse back to pinned host every step"
                            + "; step i+1's input copy and step i's result copy overlap the kernels on two "
                            "copy streams" + ("" if args.no_graph else "; the K steps replayed as one CUDA graph")
                            + ")"}

        if not args.no_graph:
            # The same pipeline without the graph: every step pays the public
            # API's host cost (argument packing, checks, tensor-map encoding,
            # launches) the way an eager serving loop does.
            e2e_steps(0, args.warmup, held)      # untimed: the eager path's own warm-up after the graph
            torch.cuda.synchronize()
            held.clear()
            # host-bound, so sensitive to other work on the host's cores: the
            # median of three timed passes
            reps = []
            for _ in range(3):
                if world > 1:
                    torch.distributed.barrier()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                e0.record()
                e2e_steps(0, args.steps, held)
                e1.record()
                torch.cuda.synchronize()
                wall = (time.perf_counter() - t0) * 1e3 / args.steps
                reps.append(max(e0.elapsed_time(e1) / args.steps, wall))
                held.clear()
            ems_eager = statistics.median(reps)
            if world > 1:
                t = torch.tensor([ems_eager], device=dev)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                ems_eager = float(t.item())
            held.clear()
            e2e["eager"] = {"value": round(alg_bytes / (ems_eager * 1e-3) / 1e9, 1), "unit": "GB/s",
                            "ms_per_step": round(ems_eager, 4),
                            "what": "the same pipelined steps issued eagerly (no graph): host cost per call visible"}

    extra = {}
    if world == 1 and not args.no_extras:
        from specverify.runtime.tree_attention import describe_attention
        extra["plan"] = describe_attention(p0.q, p0.k_pool, p0.v_pool, num_keys=p0.num_keys,
                                           page_table=p0.page_table, mask_bits=bits[0], mask_len=m)
        # The reference's own verify shape: the root row prepended (M = 65), so
        # the keys (65536 + 65) end inside a page.
        rprobs = [wl_paged(seed=100 * i, root=True, dev=dev) for i in range(rotate)]
        rbits = [pack_tree_mask(p.tree.keep.to(dev)) for p in rprobs]
        routs = [torch.empty_like(p.q) for p in rprobs]

        def rstep(i):
            p = rprobs[i]
            return lambda: attention(p.q, p.k_pool, p.v_pool, num_keys=p.num_keys, page_table=p.page_table,
                                     mask_bits=rbits[i], mask_len=p.tree.rows, out=routs[i])
        rms = _timed_graph_steps([rstep(i) for i in range(rotate)], args.steps, args.warmup)
        ralg = rprobs[0].algorithmic_bytes()
        extra["with_root_row"] = {
            "rows": rprobs[0].tree.rows, "num_keys": rprobs[0].num_keys, "ms_per_step": round(rms, 4),
            "value": round(ralg / (rms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "plan": describe_attention(rprobs[0].q, rprobs[0].k_pool, rprobs[0].v_pool,
                                       num_keys=rprobs[0].num_keys, page_table=rprobs[0].page_table,
                                       mask_bits=rbits[0], mask_len=rprobs[0].tree.rows)}
        del rprobs, rbits, routs
        torch.cuda.empty_cache()
        # The reference's GPU sequence for the same step on this GPU.
        ref_ms, ref_impl, ref_out = reference_gpu_bar(probs, max(3, args.steps // 2), args.warmup)
        ours_out = verify_attention(p0.q, p0.k_pool, p0.v_pool, p0.prefix_len, p0.tree.keep.to(dev),
                                    page_table=p0.page_table)
        extra["reference_gpu"] = {
            "ms_per_step": round(ref_ms, 4), "value": round(alg_bytes / (ref_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "speedup": round(ref_ms / ms, 2), "prefix": ref_impl, "launch": "eager, as the reference runs it",
            "max_abs_diff_vs_ours": round(float((ref_out.float() - ours_out.float()).abs().max()), 5),
            "what": "repeat_kv of the contiguous cache + prefix attention with LSE + masked tree attention with "
                    "the sigmoid merge weight + in-place merge (llama_target_model.py:793-864) on the same GPU"}
        torch.cuda.empty_cache()
        extra["acceptance"] = acceptance_bar(dev, args.steps, args.warmup)

    graphs.clear()   # graphs holding NCCL work are released before the process group goes
    total_bytes = alg_bytes  # whole job: the full 64K problem once per step (sharded or not)
    value = total_bytes / (ms * 1e-3) / 1e9
    hbm, kind = peaks()
    per_gpu_peak = hbm
    achieved_per_gpu = value / world
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, RoPE'd N(0,1)/sqrt(128) queries, random page permutation)",
        "config": {
            "workload": workload,
            "context": p0.prefix_len, "tree_nodes": m, "heads": p0.q.shape[2], "kv_heads": p0.k_pool.shape[1],
            "head_dim": p0.q.shape[3], "page_size": page, "layers_rotated": rotate,
            "l2": "inputs larger than L2: 4 independent 268 MB KV pools rotated per step",
            "algorithmic_bytes_per_step": alg_bytes, "flops_per_step": flops,
            "launch": "eager" if args.no_graph else "CUDA graph replay of each step's launches",
            "parallelism": "single GPU" if world == 1 else f"sequence-sharded x{world}",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved_per_gpu, 1),
            "peak": per_gpu_peak,
            "unit": "GB/s",
            "frac": round(achieved_per_gpu / per_gpu_peak, 4),
            "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback 6.65 TB/s",
            "traffic": NCU_TRAFFIC_BYTES if world == 1 and TREE == {"nodes": 64, "per_depth": 8, "root": False}
            else None,
            "kernel": "attn_tc_kernel + split_combine_kernel: achieved is timed over the whole verify call "
                      "(both launches, CUDA events); traffic is attn_tc_kernel's per launch (ncu)",
            "tensor_tflops": round(flops / (ms * 1e-3) / 1e12 / world, 1),
        },
        "gpu_launches": launches_per_step * args.steps,
        "e2e": e2e,
        "clocks": clocks,
    }
    result.update(extra)
    return result


def _timed_graph_steps(step_fns, steps, warmup):
    """Device ms per step: each step function captured as a CUDA graph,
    replayed round-robin (the inputs rotate), CUDA events on the stream."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for f in step_fns:
            f()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for f in step_fns:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            f()
        graphs.append(g)
    for i in range(max(warmup, len(graphs))):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        graphs[i % len(graphs)].replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graphs
    return ms


def reference_gpu_bar(probs, steps, warmup):
    """The reference's verify-attention sequence on this GPU, as its own ops
    (``llama_target_model.py:793-864``): ``repeat_kv`` of the layer's
    contiguous cache (the reference has no paged kernel, so the pages are
    gathered once, untimed), prefix attention with LSE through flash-attn's
    ``flash_attn_with_kvcache`` (``:839-845``; torch's own attention kernels
    when flash-attn cannot run here), the tree block as masked softmax
    attention with the ``sigmoid(prefix_lse - tree_lse)`` weight
    (``tree_attention.py:40-63``, the math of its Triton kernel), and the
    in-place merge (``:862-864``).  Eager, as the reference runs it."""
    def repeat_kv(x, n_rep):                               # llama_target_model.py:543-560
        bb, hh, nn, dd = x.shape
        return x[:, :, None].expand(bb, hh, n_rep, nn, dd).reshape(bb, hh * n_rep, nn, dd)

    p0 = probs[0]
    b, m, h, d = p0.q.shape
    hkv = p0.k_pool.shape[1]
    g = h // hkv
    s = p0.prefix_len
    scale = 1.0 / math.sqrt(d)
    caches = []
    for p in probs:
        k, v = p.contiguous_kv(0)                          # [S+M, Hkv, D]
        caches.append((k.permute(1, 0, 2)[None].contiguous(), v.permute(1, 0, 2)[None].contiguous(),
                       p.tree.keep.to(p.q.device).bool()))
    prefix_impl = None
    try:
        from flash_attn import flash_attn_with_kvcache
        kk = repeat_kv(caches[0][0], g).transpose(1, 2)
        vv = repeat_kv(caches[0][1], g).transpose(1, 2)
        o, lse = flash_attn_with_kvcache(p0.q, kk, vv, causal=False, cache_seqlens=s, return_softmax_lse=True)
        torch.cuda.synchronize()
        prefix_impl = "flash_attn.flash_attn_with_kvcache"
    except Exception as exc:                               # flash-attn not built for this GPU
        log(f"reference_gpu: flash-attn unavailable here ({type(exc).__name__}: {exc}); torch attention instead")

    def step(i):
        p = probs[i % len(probs)]
        kc, vc, keep = caches[i % len(caches)]
        kk = repeat_kv(kc, g)                              # [B, H, S+M, D], written and re-read
        vv = repeat_kv(vc, g)
        q_flash = p.q
        if prefix_impl:
            p_out, p_lse = flash_attn_with_kvcache(q_flash, kk.transpose(1, 2), vv.transpose(1, 2), causal=False,
                                                   cache_seqlens=s, return_softmax_lse=True)
        else:
            p_out, p_lse, *_ = torch.ops.aten._scaled_dot_product_efficient_attention(
                q_flash.transpose(1, 2), kk[:, :, :s], vv[:, :, :s], None, True, scale=scale)
            p_out = p_out.transpose(1, 2)
        qt = q_flash.transpose(1, 2).float()               # [B, H, M, D]
        sc = torch.matmul(qt, kk[:, :, s:].float().transpose(-2, -1)) * scale
        sc = sc.masked_fill(~keep[None, None], float("-inf"))
        t_lse = torch.logsumexp(sc, dim=-1)                # [B, H, M]
        t_out = torch.matmul(torch.softmax(sc, dim=-1).to(q_flash.dtype), vv[:, :, s:]).transpose(1, 2)
        w = torch.sigmoid(p_lse - t_lse).transpose(1, 2)[..., None].to(q_flash.dtype)
        out = t_out.contiguous()
        out.mul_(1.0 - w)
        out.add_(p_out.to(out.dtype).mul_(w))
        return out

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    out = step(0)
    return ms, prefix_impl or "torch efficient attention (aten._scaled_dot_product_efficient_attention)", out


# ---------------------------------------------------------------------------
# reference CPU path (oracle restatement)
# ---------------------------------------------------------------------------

def acceptance_bar(dev, steps: int, warmup: int):
    """Greedy acceptance at BASELINE config 1's shape (65 tree rows over the
    128256-word vocabulary, seed 0): the device kernels through the public
    API (``specverify.draft.accept``, CUDA events, logits already on the
    device), and the reference's ``verify_new`` greedy restated on the host
    (the oracle: argmax rows, closure along parents, best path) timed on the
    same logits -- BASELINE's CPU acceptance row."""
    from oracle import acceptance as oacc
    from specverify import workloads as wl
    from specverify.draft import accept
    c = wl.config1(seed=0)
    logits, draft = c.logits.to(dev), c.draft.to(dev)
    parent, pos = c.tree.parent.to(dev), c.positions.to(dev)
    for _ in range(warmup):
        accept(logits, draft, parent, pos, 8)
    torch.cuda.synchronize()
    n = max(steps, 10)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        acc = accept(logits, draft, parent, pos, 8)
    e1.record()
    torch.cuda.synchronize()
    gpu_ms = e0.elapsed_time(e1) / n
    got = acc.to_host()
    ln, dn, pn, qn = c.logits.numpy(), c.draft.numpy(), c.tree.parent.numpy(), c.positions.numpy()
    oacc.accept_greedy(ln, dn, pn, qn, 8)
    best = float("inf")
    for _ in range(3):
        t0 = time.perf_counter()
        ref = oacc.accept_greedy(ln, dn, pn, qn, 8)
        best = min(best, time.perf_counter() - t0)
    # the reference's CPU verify-attention layer at the same config-1 shapes
    # (S = 4096 contiguous, 65 rows, fp32, repeat_kv, all host cores)
    from oracle import attention as oatt
    torch.set_num_threads(os.cpu_count() or 1)
    layer = lambda: oatt.reference_verify_layer(c.q_raw, c.k_prefix, c.v_prefix, c.k_tree_raw, c.v_tree,
                                                c.tree.keep)
    layer()
    att = float("inf")
    for _ in range(3):
        t0 = time.perf_counter()
        layer()
        att = min(att, time.perf_counter() - t0)
    return {"rows": int(c.logits.shape[-2]), "vocab": int(c.logits.shape[-1]),
            "gpu_ms_per_call": round(gpu_ms, 4), "cpu_ms_per_call": round(best * 1e3, 3), "cpu_cores": 1,
            "cpu_config1_attention_ms": round(att * 1e3, 2), "cpu_config1_attention_cores": torch.get_num_threads(),
            "same_path": got["path"] == ref["path"] and got["accept_length"] == ref["accept_length"],
            "what": "greedy acceptance (argmax over the vocabulary, closure along parents, best path): "
                    "device kernels eagerly through specverify.draft.accept vs the reference's verify_new "
                    "greedy restated on the host (numpy, one core)"}


def cpu_reference_setup(prefix: int = 65536, seed: int = 0):
    """The reference's CPU verify pipeline (fp32, repeat_kv-expanded, pages
    gathered by index_select: it has no paged kernel) on the config-2
    problem with a ``prefix``-token context.  Returns (one_pass, algorithmic
    bytes of the problem counted at bf16 like the GPU problem, threads,
    description)."""
    from oracle import attention as oatt
    from specverify import workloads as wl
    torch.set_num_threads(os.cpu_count() or 1)
    w = wl.paged_verify(prefix_len=prefix, device="cpu", dtype=torch.float32, seed=seed, spare_pages=0)
    s = w.prefix_len
    keep = w.tree.keep

    def one_pass():
        pages = w.page_table[0].long()
        k2 = w.k_pool.index_select(0, pages).permute(1, 0, 2, 3).reshape(w.k_pool.shape[1], -1, w.k_pool.shape[3])
        v2 = w.v_pool.index_select(0, pages).permute(1, 0, 2, 3).reshape(w.v_pool.shape[1], -1, w.v_pool.shape[3])
        k2, v2 = k2[None, :, : w.num_keys], v2[None, :, : w.num_keys]
        return oatt.reference_verify_layer(w.q, k2[:, :, :s], v2[:, :, :s], k2[:, :, s:], v2[:, :, s:], keep)

    b, m, h, d = w.q.shape
    alg = (s + m) * w.k_pool.shape[1] * d * 2 * 2 + 2 * m * h * d * 2 + m * h * 4 + w.page_table.numel() * 4
    desc = (f"reference CPU path (prefix_attention_forward + tree_attention_forward + merge, repeat_kv, fp32, "
            f"pages gathered by index_select) on config 2 ({prefix}-token context, 64-node tree)")
    return one_pass, alg, torch.get_num_threads(), desc


def cpu_reference_time(passes: int = 2, prefix: int = 65536):
    """(GB/s, seconds per pass, threads, description): best of ``passes``
    timed passes after one warm-up pass."""
    one_pass, alg, thr, desc = cpu_reference_setup(prefix)
    one_pass()
    best = float("inf")
    for _ in range(passes):
        t0 = time.perf_counter()
        one_pass()
        best = min(best, time.perf_counter() - t0)
    return alg / best / 1e9, best, thr, desc


def run_reference(args, rank, world):
    """The reference arm: its CPU path for the path, on the full config-2
    problem, every step one whole pass (rank 0 only)."""
    if rank != 0:
        return None
    one_pass, alg, thr, desc = cpu_reference_setup(65536)
    for _ in range(args.warmup):
        one_pass()
    secs = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        one_pass()
        secs.append(time.perf_counter() - t0)
    sec = statistics.median(secs)
    value = alg / sec / 1e9
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "config2: paged tree verify, S=65536, 64-node depth-8 tree, 1 layer, B=1 "
                               "(the reference's CPU path, full size)", "sample": desc},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": thr, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def run_config4(args, rank, world, dev):
    """one verify step of all 32 layers over a 131072-token
    paged context with a 128-node depth-10 tree, the context sharded by
    sequence over the ranks (contiguous, page-aligned shards).

    Each rank allocates only its own shard's pages (and, on the last rank,
    the tree's pages) of every layer, so per-rank memory falls as 1/N.  A
    step runs the 32 layers in order -- layer l + 1's queries depend on layer
    l's output in a real forward pass, so nothing is overlapped across
    layers: per layer, the verify kernel on the shard, then one kernel that
    exchanges the partials over NVLink and merges them.  The 32-layer step is
    one CUDA graph; time = max over ranks.  Also timed: the same step with
    attention only (each rank's shard, no exchange), which splits the step
    into attention and exchange + merge, and (N >= 2) both exchange modes."""
    from specverify import workloads as wl
    from specverify.runtime import attention, pack_tree_mask
    from specverify.runtime import sharded as sh
    from specverify.runtime.tree_attention import describe_attention
    layers, ctx, nodes, per_depth, page = 32, 131072, 128, 13, 16
    h, hkv, d = wl.HEADS, wl.KV_HEADS, wl.HEAD_DIM
    gen = torch.Generator().manual_seed(4)
    tree = wl.make_tree(gen, nodes, per_depth, root=False)
    m = tree.rows
    bits = pack_tree_mask(tree.keep.to(dev))
    n_prefix_pages = ctx // page
    tree_pages = -(-m // page)
    lo, hi = sh.shard_bounds(n_prefix_pages, world, rank)
    last = rank == world - 1
    own = (hi - lo) + (tree_pages if last else 0)
    shard_len = (hi - lo) * page + (m if last else 0)
    dgen = torch.Generator(device=dev).manual_seed(1000 + rank)
    pools, tables, qs = [], [], []
    for layer in range(layers):
        kp = torch.randn((own, hkv, page, d), generator=dgen, device=dev, dtype=torch.bfloat16)
        vp = torch.randn((own, hkv, page, d), generator=dgen, device=dev, dtype=torch.bfloat16)
        perm = torch.randperm(own, generator=gen).to(torch.int32)
        pools.append((kp, vp))
        tables.append(perm.view(1, own).to(dev))
        # layer-independent queries (seeded; the same on every rank)
        qg = torch.Generator().manual_seed(7000 + layer)
        qs.append((torch.randn((1, m, h, d), generator=qg) / math.sqrt(d)).to(torch.bfloat16).to(dev))
    outs = [torch.empty((1, m, h, d), dtype=torch.bfloat16, device=dev) for _ in range(layers)]
    torch.cuda.synchronize()

    per_layer_kv = ctx * hkv * d * 2 * 2 + m * hkv * d * 2 * 2
    alg_layer = per_layer_kv + 2 * m * h * d * 2 + m * h * 4 + (n_prefix_pages + tree_pages) * 4 + m * 2 * 8
    alg = layers * alg_layer
    vis = int(tree.keep.sum())
    flops = layers * (4 * m * h * d * ctx + 4 * h * d * vis)
    plan = describe_attention(qs[0], pools[0][0], pools[0][1], num_keys=shard_len, page_table=tables[0],
                              mask_bits=bits if last else None, mask_len=m if last else 0)

    def attn_only():
        for layer in range(layers):
            kp, vp = pools[layer]
            attention(qs[layer], kp, vp, num_keys=shard_len, page_table=tables[layer],
                      mask_bits=bits if last else None, mask_len=m if last else 0, out=outs[layer])

    results = {}
    if world > 1:
        for mode in ("push", "owner"):
            ver = sh.SequenceShardedVerify(exchange="peer", peer_mode=mode)

            def step(ver=ver):
                for layer in range(layers):
                    kp, vp = pools[layer]
                    ver(qs[layer], kp, vp, shard_len, bits if last else None, page_table=tables[layer])
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize()
            torch.distributed.barrier()
            results[mode] = _max_over_ranks(_timed_graph_steps([step], args.steps, args.warmup), world, dev)
    # attention alone on this rank's shard (max over ranks): the exchange's share
    if world > 1:
        torch.distributed.barrier()
    a_ms = _max_over_ranks(_timed_graph_steps([attn_only], args.steps, args.warmup), world, dev)
    if world == 1:
        results["single"] = a_ms
    best_mode = min(results, key=results.get)
    ms = results[best_mode]
    hbm, _ = peaks()
    mp = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tpeak = float(mp.get("bf16_tflops_sustained", 1400.0))
    value = alg / (ms * 1e-3) / 1e9
    tflops = flops / (ms * 1e-3) / 1e12
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V, N(0,1)/sqrt(128) queries)",
        "config": {"workload": f"config4: sequence-sharded verify, {layers} layers x {ctx}-token paged context, "
                               f"{m}-node depth-10 tree, bf16, B=1, over {world} GPU(s)",
                   "parallelism": "single GPU" if world == 1 else f"sequence-sharded x{world}",
                   "exchange": best_mode, "l2": "inputs larger than L2 (537 MB of KV per layer)",
                   "algorithmic_bytes_per_step": alg, "flops_per_step": flops,
                   "per_rank_pages_per_layer": own, "plan_rank0": plan if rank == 0 else None,
                   "launch": "one CUDA graph per 32-layer step"},
        "latency_ms": round(ms, 4), "us_per_layer": round(ms * 1e3 / layers, 2),
        "modes_ms": {k: round(v, 4) for k, v in results.items()},
        "attention_only_ms": round(a_ms, 4),
        "exchange_and_merge_ms": round(ms - a_ms, 4) if world > 1 else 0.0,
        "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": tpeak, "unit": "TFLOP/s",
                     "frac": round(tflops / world / tpeak, 4),
                     "peak_kind": "measured bf16_tflops_sustained (MEASURED_PEAKS.json)" if mp else "fallback",
                     "hbm_frac": round(value / world / hbm, 4), "traffic": None,
                     "kernel": "attn_tc_kernel + " + ("split_combine_kernel" if world == 1 else "sharded_combine_kernel")
                               + " per layer"},
        "gpu_launches": args.steps * layers * 2,
    }


def run_config5(args, rank, world, dev):
    """bundle verify over a chunk-arena working set.

    Batch of 4 sequences, each a 262144-token context (one layer's K / V) in
    2048-token chunks; chunk salience ~ U(0, 1); the top 32 chunks of each
    sequence form its 65536-token arena, followed by the 96 tokens of a
    96-node depth-8 tree whose leaves are grouped into 8 bundles by their
    branching ancestor (``BundleScheduler``).  The verify step is
    ``FusedBundleVerifier`` semantics (one mask over all keys, ones over the
    shared arena) over the arena.  Two arena forms are timed:

    * zero-copy: the arena is a page table (``tv_gather_page_table`` of the
      chunks' pages), verified in place in the paged pool
      (``PagedBundleVerifier.verify_bundle_paged``);
    * physical: the chunks are copied into a contiguous arena
      (``tv_arena_gather``, ``ChunkArena``'s layout) and verified there.

    Also timed: the reference's call pattern -- one ``verify_bundle`` call per
    bundle over that bundle's rows -- against the single call that scores
    every bundle's rows in one pass over the arena.  With N > 1 the batch's
    sequences are split over the ranks (no collective: each rank verifies
    whole sequences; "scaling": strong, total work fixed)."""
    from specverify.core.bundle_scheduler import BundleScheduler
    from specverify.core.kv_cache.chunk_arena import arena_page_table
    from specverify import _lib, workloads as wl
    from specverify.runtime import FusedBundleVerifier, PagedBundleVerifier
    batch, ctx, cs, topk, nodes, per_depth, page = 4, 262144, 2048, 32, 96, 12, 16
    if batch % world:
        raise SystemExit(f"config5 splits {batch} sequences over the ranks: use 1, 2 or 4 GPUs")
    h, hkv, d = wl.HEADS, wl.KV_HEADS, wl.HEAD_DIM
    ppc, nch = cs // page, ctx // cs
    gen = torch.Generator().manual_seed(5)
    tree = wl.make_tree(gen, nodes, per_depth, root=False)
    m = tree.rows
    parent = tree.parent.tolist()
    children = {p for p in parent if p >= 0}
    leaves = [i for i in range(nodes) if i not in children]
    sched = BundleScheduler(bundle_size=3, max_bundles=8, device="cpu")
    bundles = sched.schedule_bundles({"leaf_ids": leaves, "parent_map": {i: parent[i] for i in range(nodes)},
                                      "depth_map": {i: int(tree.depth[i]) for i in range(nodes)}},
                                     return_tensors=False)
    arena = topk * cs
    n = arena + m
    mask = torch.ones(m, n, dtype=torch.int8)
    mask[:, arena:] = tree.keep
    mask = mask.to(dev)
    # bundle rows: every node on the paths from the bundle's leaves to the root
    bundle_rows = []
    for bd in bundles:
        rows = set()
        for leaf in bd["leaves"]:
            c = leaf
            while c >= 0:
                rows.add(c)
                c = parent[c]
        bundle_rows.append(torch.tensor(sorted(rows), dtype=torch.long, device=dev))
    per_rank = batch // world
    seqs = list(range(rank * per_rank, (rank + 1) * per_rank))
    tree_pages = -(-m // page)
    # paged pool: this rank's sequences' full contexts, then their tree pages
    pool_pages = per_rank * (nch * ppc + tree_pages)
    dgen = torch.Generator(device=dev).manual_seed(50 + rank)
    pool = torch.empty((1, 2, pool_pages, hkv, page, d), dtype=torch.bfloat16, device=dev)
    pool.normal_(generator=dgen)
    perm = torch.randperm(per_rank * nch * ppc, generator=gen).to(torch.int32).view(per_rank, nch * ppc).to(dev)
    tree_tbl = (per_rank * nch * ppc + torch.arange(per_rank * tree_pages, dtype=torch.int32)).view(
        per_rank, tree_pages).to(dev)
    chunk_ids = []
    for s_ in seqs:
        sal = torch.rand(nch, generator=torch.Generator().manual_seed(500 + s_))
        chunk_ids.append(torch.sort(torch.topk(sal, topk).indices)[0].to(torch.int32).to(dev))
    qg = torch.Generator().manual_seed(77)
    q_all = (torch.randn((batch, m, h, d), generator=qg) / math.sqrt(d)).to(torch.bfloat16)
    q = q_all[seqs[0]:seqs[-1] + 1].contiguous().to(dev)
    # physical variant: contiguous full caches [B, Hkv, ctx, D] gathered from the pool once (untimed)
    full_k = torch.empty((per_rank, hkv, ctx, d), dtype=torch.bfloat16, device=dev)
    full_v = torch.empty_like(full_k)
    for i in range(per_rank):
        pg = perm[i].long()
        full_k[i] = pool[0, 0][pg].permute(1, 0, 2, 3).reshape(hkv, ctx, d)
        full_v[i] = pool[0, 1][pg].permute(1, 0, 2, 3).reshape(hkv, ctx, d)
    arena_kv = torch.empty((per_rank, 2, hkv, n, d), dtype=torch.bfloat16, device=dev)   # arena + tree rows
    for i in range(per_rank):
        tp = tree_tbl[i].long()
        arena_kv[i, 0, :, arena:] = pool[0, 0][tp].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :m]
        arena_kv[i, 1, :, arena:] = pool[0, 1][tp].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :m]
    copies = [torch.stack([c, torch.arange(topk, dtype=torch.int32, device=dev)], 1).contiguous()
              for c in chunk_ids]
    src_k = torch.tensor([full_k[i].data_ptr() for i in range(per_rank)], dtype=torch.int64, device=dev)
    src_v = torch.tensor([full_v[i].data_ptr() for i in range(per_rank)], dtype=torch.int64, device=dev)
    lib = _lib.load()
    es = 2
    torch.cuda.synchronize()
    pver = PagedBundleVerifier(bundle_size=3, device="cuda")
    fver = FusedBundleVerifier(bundle_size=3, device="cuda")
    k_arena = arena_kv[:, 0].transpose(1, 2)
    v_arena = arena_kv[:, 1].transpose(1, 2)

    def zero_copy():
        tbl = torch.cat([torch.stack([arena_page_table(perm[i], chunk_ids[i], ppc) for i in range(per_rank)]),
                         tree_tbl], dim=1)
        return pver.verify_bundle_paged(q, pool, tbl, [mask], shared_prefix_len=arena, num_keys=n)

    def gather():
        for i in range(per_rank):
            st = lib.tv_arena_gather(1, hkv, src_k[i:i + 1].data_ptr(), src_v[i:i + 1].data_ptr(), ctx * d * es,
                                     d * es, ctx, arena_kv[i].data_ptr(), 0, hkv * n * d * es, n * d * es, d * es,
                                     cs, n, copies[i].data_ptr(), topk, _lib.stream_ptr(dev))
            _lib.check(st, "tv_arena_gather")

    def physical():
        gather()
        return fver.verify_bundle(q, k_arena, v_arena, [mask], shared_prefix_len=arena)

    def per_bundle():
        outs = []
        tbl = torch.cat([torch.stack([arena_page_table(perm[i], chunk_ids[i], ppc) for i in range(per_rank)]),
                         tree_tbl], dim=1)
        for rows in bundle_rows:
            outs.append(pver.verify_bundle_paged(q[:, rows], pool, tbl, [mask[rows]], shared_prefix_len=arena,
                                                 num_keys=n))
        return outs

    # parity of the two arena forms (same keys, same kernel): identical bits
    o1, l1 = zero_copy()
    o2, l2 = physical()
    torch.cuda.synchronize()
    same = bool(torch.equal(o1, o2) and torch.equal(l1, l2))
    pb = per_bundle()
    pb_diff = max(float((o[0].float() - o1[:, rows].float()).abs().max()) for o, rows in zip(pb, bundle_rows))
    times = {}
    for name, fn in (("zero_copy", zero_copy), ("physical", physical), ("gather_only", gather),
                     ("per_bundle_calls", per_bundle)):
        if world > 1:
            torch.distributed.barrier()
        times[name] = _max_over_ranks(_timed_graph_steps([fn], args.steps, args.warmup), world, dev)
    ms = times["zero_copy"]
    kv_bytes = batch * n * hkv * d * 2 * es
    alg = kv_bytes + 2 * batch * m * h * d * es + batch * m * h * 4 + batch * (arena // page + tree_pages) * 4 \
        + m * ((n + 63) // 64) * 8
    vis = int(tree.keep.sum())
    flops = batch * (4 * m * h * d * arena + 4 * h * d * vis)
    hbm, _ = peaks()
    mp = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tpeak = float(mp.get("bf16_tflops_sustained", 1400.0))
    value = alg / (ms * 1e-3) / 1e9
    tflops = flops / (ms * 1e-3) / 1e12
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V, U(0,1) chunk salience)",
        "config": {"workload": f"config5: bundle verify, batch {batch}, {ctx}-token contexts in {cs}-token chunks, "
                               f"top-{topk} arena ({arena} tokens) + {m}-node depth-8 tree in {len(bundles)} "
                               f"bundles, bf16, over {world} GPU(s)",
                   "parallelism": "single GPU" if world == 1 else f"sequences split over {world} GPUs",
                   "bundles": [len(r) for r in bundle_rows], "algorithmic_bytes_per_step": alg,
                   "flops_per_step": flops, "l2": "inputs larger than L2 (1.07 GB of arena KV per step)",
                   "launch": "one CUDA graph per step"},
        "arena_forms_ms": {k: round(v, 4) for k, v in times.items()},
        "zero_copy_equals_physical": same, "per_bundle_vs_single_call_max_abs_diff": round(pb_diff, 6),
        # 96 rows x GQA 4 per sequence: 384 flops per byte, past the ridge -> tensor-bound
        "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": tpeak, "unit": "TFLOP/s",
                     "frac": round(tflops / world / tpeak, 4),
                     "peak_kind": "measured bf16_tflops_sustained (MEASURED_PEAKS.json)" if mp else "fallback",
                     "hbm_achieved_gbs": round(value / world, 1), "hbm_frac": round(value / world / hbm, 4),
                     "traffic": None, "kernel": "attn_tc_kernel + split_combine_kernel (zero-copy arena)"},
        "gpu_launches": args.steps * (per_rank + 4),
    }


def run_config3(args):
    """the speculative decode loop on a random-init
    Llama-3.1-8B-architecture target (32 layers, hidden 4096, 32 / 8 heads,
    SwiGLU 14336, vocabulary 128256, RoPE theta 500000, bf16) with a
    one-layer EAGLE3-shaped draft head, after a 65536-token context, 64-node
    depth-8 trees, stochastic acceptance at temperature 1.0, seed 0
    (``specverify.draft.spec_decode``).  The context's K / V are filled with
    N(0, 1) values in place of a prefill (not part of the decode metric).
    value = verified tokens per second of the decode loop (wall clock, host
    reads included).  Replicas only across GPUs: the loop does not shard."""
    from specverify.draft.spec_decode import SpecDecodeModel
    from specverify.runtime import attention, pack_tree_mask
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --workload config3 needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prompt, new_tokens, nodes, depth = 65536, 512, 64, 8
    model = SpecDecodeModel.from_config(device=dev, seed=0, max_tokens=prompt + new_tokens + 2 * nodes + 64)
    model.diffspec_generate(prompt, max_new_tokens=8 * args.warmup, nodes=nodes, max_depth=depth,
                            temperature=1.0, seed=1, max_steps=args.warmup)           # warm-up
    torch.cuda.synchronize()
    r = model.diffspec_generate(prompt, max_new_tokens=new_tokens, nodes=nodes, max_depth=depth, temperature=1.0,
                                seed=0)
    tok_s = len(r["tokens"]) / r["wall_s"]
    steps = r["steps"]
    ph = r["phases_ms"]
    step_ms = r["wall_s"] * 1e3 / steps
    # the verify step's attention alone: 32 layers of the verify kernel at the
    # loop's shapes (65 rows, ~66K keys), graph-replayed
    s = model.shape
    m = nodes + 1
    start = prompt + new_tokens // 2
    q = (torch.randn(1, m, s.heads, s.head_dim, device=dev) / math.sqrt(s.head_dim)).to(model.dtype)
    keep = torch.tril(torch.ones(m, m, dtype=torch.int8, device=dev))
    bits = pack_tree_mask(keep)

    def layers_attention():
        for li in range(s.layers):
            attention(q, model.pool[li, 0], model.pool[li, 1], num_keys=start + m, page_table=model.page_table,
                      mask_bits=bits, mask_len=m)
    attn_ms = _timed_graph_steps([layers_attention], 10, 3)
    weights = sum(t.numel() * t.element_size() for t in
                  [model.embed, model.lm_head] + [w for L in model.layers for w in (L.wqkv, L.wo, L.wgu, L.wdown)])
    return {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "verified tok/s", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0, 0.02) weights, N(0,1) context K/V, seeded sampling)",
        "config": {"workload": f"config3: speculative decode loop, random-init Llama-3.1-8B target (32 layers) + "
                               f"1-layer EAGLE3-shaped draft (draft vocab {s.draft_vocab}, working set "
                               f"{model.draft_ctx} tokens), {prompt}-token context, {new_tokens} new tokens, "
                               f"{nodes}-node depth-{depth} trees, temperature 1.0, seed 0",
                   "parallelism": "single GPU (replicas only across GPUs)",
                   "launch": "eager loop, one host read per step (the accepted length)"},
        "tokens": len(r["tokens"]), "accepted_per_step_mean": round(sum(r["accepted_per_step"]) / steps, 4),
        "phase_ms_per_step": {k.replace("_ms", ""): round(v / steps, 4) for k, v in ph.items()},
        "verify_attention_ms_per_step": round(attn_ms, 4),
        "attention_share_of_step": round(attn_ms / step_ms, 4),
        "target_weight_bytes": weights,
        "roofline": {"bound": "hbm", "achieved": round((weights + s.layers * start * s.kv_heads * s.head_dim * 4)
                                                      / (step_ms * 1e-3) / 1e9, 1),
                     "peak": peaks()[0], "unit": "GB/s", "frac": None, "traffic": None,
                     "kernel": "whole step: target weights + KV read once per step over the step time",
                     "note": "frac omitted: the step also runs the draft (8 forwards) and host work"},
        # per step, this library's kernels: draft 8 x (mask pack, rope + append, attention, split
        # combine) + tree finalize; target 32 x (rope + append, attention, split combine); lm_head scan +
        # acceptance; paged compaction
        "gpu_launches": steps * (8 * 4 + 1 + 32 * 3 + 2 + 1),
    }


_JSON_OUT = sys.stdout


# ncu (dram__bytes_read.sum + dram__bytes_write.sum) of one tv_rope_append
# launch on the rope-append workload below.
NCU_ROPE_TRAFFIC_BYTES = 762_554_624
# the same for one lmhead_scan_kernel launch on the lmhead-accept workload
NCU_LMHEAD_TRAFFIC_BYTES = 1_056_964_720


def _graph_us(fn, reps: int, steps: int, warmup: int) -> float:
    """Device time per call of `fn`, replayed as a CUDA graph of `reps` calls."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (steps * reps)
    del g
    return us


def run_rope(args):
    """Rotary embedding + KV append (the step before verify attention)."""
    from specverify.runtime import KVCache, rope_append
    from oracle import rope as orope
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --workload rope-append needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(0)
    h, hkv, d, start = 32, 8, 128, 8192

    def problem(b, t):
        # q / k / v as views of the projection outputs, as LlamaAttention holds them
        q = torch.randn(b, t, h * d, generator=g).bfloat16().to(dev).view(b, t, h, d).transpose(1, 2)
        kv = torch.randn(b, t, 2 * hkv * d, generator=g).bfloat16().to(dev)
        k = kv[..., :hkv * d].reshape(b, t, hkv, d).transpose(1, 2)
        v = kv[..., hkv * d:].reshape(b, t, hkv, d).transpose(1, 2)
        cos_t, sin_t = orope.rope_table(d, start + t, 500000.0)
        cos = torch.from_numpy(cos_t).bfloat16().to(dev)[None, None]
        sin = torch.from_numpy(sin_t).bfloat16().to(dev)[None, None]
        pos = (start - 1 + torch.arange(t) // 8).view(1, t).expand(b, t).contiguous().to(dev)
        kd = torch.zeros(b, hkv, start + t, d, dtype=torch.bfloat16, device=dev)
        vd = torch.zeros_like(kd)
        kc, vc = KVCache(kd, torch.tensor(start)), KVCache(vd, torch.tensor(start))
        qo = torch.empty(b, h, t, d, dtype=torch.bfloat16, device=dev)

        def ours():
            kc.current_length.fill_(start)
            vc.current_length.fill_(start)
            rope_append(q, k, v, cos, sin, pos, kc, vc, out=qo, validate=False)

        def rot(x):
            return torch.cat((-x[..., d // 2:], x[..., :d // 2]), dim=-1)

        def reference_ops():      # llama_target_model.py:443-449 and cache_state.py:63-64
            c = cos.squeeze(1).squeeze(0)[pos].unsqueeze(1)
            s_ = sin.squeeze(1).squeeze(0)[pos].unsqueeze(1)
            qe = q * c + rot(q) * s_
            ke = k * c + rot(k) * s_
            kd.narrow(2, start, t).copy_(ke)
            vd.narrow(2, start, t).copy_(v)
            return qe

        alg = 2 * q.numel() * 2 + 2 * k.numel() * 2 + 2 * v.numel() * 2 + 2 * b * t * d * 2
        return ours, reference_ops, alg, (q, k, v, cos, sin, pos)

    b, t = 16, 2048
    ours, ref_ops, alg, _ = problem(b, t)
    us = _graph_us(ours, 4, args.steps, args.warmup)
    ref_us = _graph_us(ref_ops, 4, max(3, args.steps // 4), args.warmup)
    small, small_ref, _, small_in = problem(1, 65)
    small_us = _graph_us(small, 20, args.steps, args.warmup)
    small_ref_us = _graph_us(small_ref, 20, args.steps, args.warmup)
    peak, kind = peaks()
    gbs = alg / (us * 1e-6) / 1e9
    res = {
        "metric": "rope + KV append GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v)",
        "config": {"workload": f"rope-append: B={b} x {t} new tokens, 32/8 heads, head_dim 128, contiguous cache at "
                               f"{start}", "launch": "CUDA graph replays of the public API call",
                   "l2": "inputs larger than L2 (822 MB moved per call)", "algorithmic_bytes_per_step": alg},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": NCU_ROPE_TRAFFIC_BYTES,
                     "peak_kind": kind, "kernel": "rope_append_kernel (one launch per call)"},
        "gpu_launches": args.steps * 4,
        "reference_ops_on_gpu": {"us": round(ref_us, 2), "speedup": round(ref_us / us, 2),
                                 "what": "the reference's torch ops for the step (cos/sin gather, q*cos + "
                                         "rotate_half(q)*sin for q and k, two KVCache.cat copies)"},
        "verify_shape_us": {"ours": round(small_us, 2), "reference_ops": round(small_ref_us, 2),
                            "config": "B=1, 65 rows, 32/8 heads, head_dim 128"},
    }
    if not args.no_cpu_baseline:
        q, k, v, cos, sin, pos = small_in
        qf, kf = q.float().cpu().numpy(), k.float().cpu().numpy()
        cf, sf = cos[0, 0].float().cpu().numpy(), sin[0, 0].float().cpu().numpy()
        pf = pos.cpu().numpy()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 2.0:
            orope.apply_rotary_pos_emb(qf, kf, cf, sf, pf, "bf16")
            n += 1
        sec = (time.perf_counter() - t0) / n
        small_alg = 2 * q.numel() * 2 + 2 * k.numel() * 2 + 2 * v.numel() * 2 + 2 * 65 * d * 2
        res["cpu_baseline"] = {"value": round(small_alg / sec / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                               "sample": f"numpy restatement, B=1 x 65 rows; {sec * 1e6:.0f} us per call"}
    return res


def run_lmhead(args):
    """lm_head + acceptance in one pass (the step after verify attention)."""
    from specverify.draft.tree_verification import accept, accept_from_hidden
    from oracle import acceptance as oacc
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --workload lmhead-accept needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(0)
    rows, hidden, vocab, max_depth = 65, 4096, 128256, 8
    x = torch.randn(rows, hidden, generator=g).bfloat16().to(dev)
    w = (0.02 * torch.randn(vocab, hidden, generator=g)).bfloat16().to(dev)
    depth = torch.cat([torch.zeros(1, dtype=torch.long), 1 + torch.arange(rows - 1) // 8])
    parent = torch.cat([torch.full((8,), -1), torch.arange(rows - 9) // 8 * 8]).to(dev)
    pos = (65535 + depth).to(dev)
    draft = torch.randint(0, vocab, (rows,), generator=g).to(dev)

    def ours():
        accept_from_hidden(x, w, draft, parent, pos, max_depth)

    def reference_ops():     # diffspec_model.py:229-231 then tree_verification.py:102
        return torch.argmax(torch.nn.functional.linear(x, w), dim=-1)

    def unfused_ours():
        accept(torch.nn.functional.linear(x, w), draft, parent, pos, max_depth)

    us = _graph_us(ours, 5, args.steps, args.warmup)
    ref_us = _graph_us(reference_ops, 5, args.steps, args.warmup)
    unf_us = _graph_us(unfused_ours, 5, args.steps, args.warmup)
    alg = vocab * hidden * 2 + rows * hidden * 2 + 2 * rows * 8
    peak, kind = peaks()
    gbs = alg / (us * 1e-6) / 1e9
    res = {
        "metric": "lm_head + acceptance GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) hidden, "
                                                                          "N(0,0.02) weight)",
        "config": {"workload": f"lmhead-accept: {rows} rows x hidden {hidden} x vocab {vocab} (Llama-3.1-8B "
                               f"lm_head), greedy, 64-node depth-8 tree",
                   "launch": "CUDA graph replays of the public API call",
                   "l2": "weight (1.05 GB) larger than L2", "algorithmic_bytes_per_step": alg,
                   "flops_per_step": 2 * 128 * hidden * vocab},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": NCU_LMHEAD_TRAFFIC_BYTES, "peak_kind": kind,
                     "kernel": "lmhead_scan_kernel + acceptance (two launches per call); traffic is "
                               "lmhead_scan_kernel's per launch (ncu)"},
        "gpu_launches": args.steps * 5 * 3,
        "reference_ops_on_gpu": {"us": round(ref_us, 2), "speedup": round(ref_us / us, 3),
                                 "what": "the reference's ops: lm_head (torch linear, cuBLAS) writing bf16 logits "
                                         "[65, 128256], then torch.argmax per node"},
        "unfused_ours_us": round(unf_us, 2),
    }
    if not args.no_cpu_baseline:
        xs, ws = x.float().cpu().numpy(), w[:8192].float().cpu().numpy()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 2.0:
            oacc.argmax_rows(xs @ ws.T)
            n += 1
        sec = (time.perf_counter() - t0) / n
        res["cpu_baseline"] = {"value": round(ws.size * 2 / sec / 1e9, 3), "unit": "GB/s",
                               "cores": torch.get_num_threads(), "kind": "port",
                               "sample": f"numpy lm_head + argmax over the first 8192 vocab rows; "
                                         f"{sec * 1e3:.1f} ms per call"}
    return res


def run_tree(args):
    """Final draft-tree build (the step that produces the verify inputs)."""
    from specverify.runtime.draft_tree import finalize_tree
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --workload tree-finalize needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nnodes, depth = 64, 8
    g = torch.Generator(device="cpu").manual_seed(0)
    pm = torch.randint(0, nnodes, (depth, nnodes), generator=g)
    pm[0] = torch.arange(nnodes)
    im = torch.randint(0, 128256, (depth, nnodes), generator=g)
    top = torch.randperm(depth * nnodes, generator=g)[:nnodes]
    pm, im, top = pm.to(dev), im.to(dev), top.to(dev)

    def ours():
        finalize_tree(top, pm, im, depth, nnodes, validate=False)

    def reference_ops():
        # DraftTree.update's final branch and generate_attention_mask
        # (runtime/draft_tree.py:236-260, 188-215), then the root row / column
        # (diffspec_model.py:620-624), as torch ops on the same GPU
        rows = (top // nnodes).to(torch.long)
        cols = (top % nnodes).to(torch.long)
        order = torch.argsort(rows)
        rows, cols = rows[order], cols[order]
        k = nnodes
        pos_table = torch.full((depth, nnodes), -1, dtype=torch.long, device=dev)
        pos_table[rows, cols] = torch.arange(k, device=dev)
        parent_pos = torch.full((k,), -1, dtype=torch.long, device=dev)
        par_cols = pm[rows, cols]
        has_parent = (rows > 0) & (par_cols >= 0)
        if bool(has_parent.any()):
            parent_pos[has_parent] = pos_table[rows[has_parent] - 1, par_cols[has_parent]]
        attn = torch.zeros((k, k), dtype=torch.int8, device=dev)
        diag = torch.arange(k, device=dev)
        attn[diag, diag] = 1
        cur = parent_pos
        for _ in range(max(depth - 1, 0)):
            valid = (cur >= 0) & (cur < k)
            if not bool(valid.any()):
                break
            attn[diag[valid], cur[valid]] = 1
            nxt = torch.full((k,), -1, dtype=torch.long, device=dev)
            nxt[valid] = parent_pos[cur[valid]]
            cur = nxt.clone()
        ids = im[rows, cols]
        m = torch.cat([torch.zeros(1, k, dtype=attn.dtype, device=dev), attn], dim=0)
        m = torch.cat([torch.ones(k + 1, 1, dtype=attn.dtype, device=dev), m], dim=1)
        return ids, rows + 1, parent_pos, m

    us = _graph_us(ours, 20, args.steps, args.warmup)
    for _ in range(args.warmup):
        reference_ops()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_ops()
    torch.cuda.synchronize()
    ref_us = (time.perf_counter() - t0) * 1e6 / args.steps
    return {
        "metric": "draft-tree finalize latency", "value": round(us, 2), "unit": "us", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic (seeded random tree state)",
        "config": {"workload": f"tree-finalize: {nnodes} nodes kept from {depth} depths, root-prepended verify "
                               f"bitmask", "launch": "CUDA graph replays of the public API call"},
        "roofline": {"bound": "latency", "achieved": round(us, 2), "peak": None, "unit": "us", "frac": None,
                     "traffic": None, "kernel": "tree_finalize_kernel (one CTA, one launch)"},
        "gpu_launches": args.steps * 20,
        "reference_ops_on_gpu": {"us": round(ref_us, 1), "speedup": round(ref_us / us, 1),
                                 "what": "the reference's final-branch torch ops on the same GPU (eager: it reads "
                                         "a flag back to the host on every ancestor hop)"},
    }


def run_retrieve(args):
    """Draft-side chunk retrieval: selection + working-cache gather (config 5 sizes)."""
    from specverify.draft.retrieval import GatherPlan, gather_rows, select_chunks
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --workload chunk-retrieve needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    length, cs, k, heads, d = 262144, 2048, 32, 8, 128
    g = torch.Generator(device="cpu").manual_seed(0)
    attn = torch.rand(length, generator=g).to(dev)
    starts = torch.arange(0, length, cs, device=dev)
    ends = starts + cs
    full = [(torch.randn(1, heads, length, d, generator=g).bfloat16().to(dev),
             torch.randn(1, heads, length, d, generator=g).bfloat16().to(dev))]
    rows = k * cs                                 # the working cache's length for disjoint chunks
    plan = GatherPlan(full, rows)

    def ours():
        sel, idx, count = select_chunks(attn, starts, ends, k, length, validate=False)
        gather_rows(plan, idx, count)

    def reference_ops():
        # draft_network.py:1524-1594 as torch ops on the same GPU (with its host reads)
        cum = torch.cumsum(attn, dim=0)
        lower = torch.zeros_like(starts, dtype=cum.dtype)
        mask_pos = starts > 0
        if bool(mask_pos.any()):
            lower[mask_pos] = cum.index_select(0, (starts[mask_pos] - 1).clamp_(min=0, max=length - 1))
        upper = cum.index_select(0, (ends - 1).clamp_(min=0, max=length - 1))
        score = (upper - lower) / (ends - starts).clamp_min(1).to(cum.dtype)
        selected = torch.sort(torch.topk(score, k=k, dim=0).indices)[0]
        _ = selected.tolist()
        diff = torch.zeros(length + 1, dtype=torch.int32, device=dev)
        diff.index_add_(0, starts.index_select(0, selected).clamp_(0, length),
                        torch.ones(k, dtype=torch.int32, device=dev))
        diff.index_add_(0, ends.index_select(0, selected).clamp_(0, length),
                        -torch.ones(k, dtype=torch.int32, device=dev))
        idx = torch.nonzero(torch.cumsum(diff[:length], dim=0) > 0, as_tuple=False).squeeze(1)
        return [(fk.index_select(2, idx).contiguous(), fv.index_select(2, idx).contiguous()) for fk, fv in full]

    us = _graph_us(ours, 5, args.steps, args.warmup)
    for _ in range(args.warmup):
        reference_ops()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_ops()
    torch.cuda.synchronize()
    ref_us = (time.perf_counter() - t0) * 1e6 / args.steps
    alg = 2 * 2 * heads * rows * d * 2 + length * 4          # K and V rows read + written, the scores read
    peak, kind = peaks()
    gbs = alg / (us * 1e-6) / 1e9
    return {
        "metric": "chunk retrieval GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded uniform scores, N(0,1) K/V)",
        "config": {"workload": f"chunk-retrieve: {length} draft tokens in {cs}-token chunks, top {k} chunks, one "
                               f"draft layer's K/V ({heads} heads, head_dim {d}) gathered",
                   "launch": "CUDA graph replays of the public API calls", "algorithmic_bytes_per_step": alg},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": None, "peak_kind": kind,
                     "kernel": "chunk_select_kernel + gather_rows_kernel (two launches per call)"},
        "gpu_launches": args.steps * 5 * 2,
        "reference_ops_on_gpu": {"us": round(ref_us, 1), "speedup": round(ref_us / us, 2),
                                 "what": "the reference's retrieval ops on the same GPU (eager: it reads the "
                                         "selection back to the host)"},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of CUDA graph replays")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the side measurements (root-row variant, reference GPU ops)")
    ap.add_argument("--nodes", type=int, default=64, help="verify workload: tree nodes (config 2: 64)")
    ap.add_argument("--per-depth", type=int, default=8, help="verify workload: nodes per depth (config 2: 8)")
    ap.add_argument("--root", action="store_true", help="verify workload: prepend the root row (M = nodes + 1)")
    ap.add_argument("--peer-mode", choices=["auto", "push", "owner"], default="auto",
                    help="N > 1 verify workload: NVLink exchange mode (auto: push below 4 ranks, owner from 4)")
    ap.add_argument("--workload", choices=["verify", "config3", "config4", "config5", "rope-append", "lmhead-accept", "tree-finalize",
                                           "chunk-retrieve"], default="verify")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    TREE.update(nodes=args.nodes, per_depth=args.per_depth, root=args.root)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # Exactly one JSON line on stdout: libraries (NCCL's version banner) that
    # print to stdout are sent to stderr instead.
    global _JSON_OUT
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    if args.workload == "rope-append":
        if rank == 0:
            print(json.dumps(run_rope(args)), file=_JSON_OUT, flush=True)
        return
    if args.workload == "lmhead-accept":
        if rank == 0:
            print(json.dumps(run_lmhead(args)), file=_JSON_OUT, flush=True)
        return
    if args.workload == "tree-finalize":
        if rank == 0:
            print(json.dumps(run_tree(args)), file=_JSON_OUT, flush=True)
        return
    if args.workload == "chunk-retrieve":
        if rank == 0:
            print(json.dumps(run_retrieve(args)), file=_JSON_OUT, flush=True)
        return
    if args.workload == "config3":
        if rank == 0:
            print(json.dumps(run_config3(args)), file=_JSON_OUT, flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), file=_JSON_OUT, flush=True)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py (ours) needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    try:
        if args.workload == "config4":
            res = run_config4(args, rank, world, dev)
        elif args.workload == "config5":
            res = run_config5(args, rank, world, dev)
        else:
            res = run_ours(args, rank, world, dev)
        if rank == 0:
            if not args.no_cpu_baseline and world == 1 and args.workload == "verify":
                gbs, sec, thr, desc = cpu_reference_time(passes=2)
                res["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
                                       "sample": desc + f"; best of 2 passes, {sec * 1e3:.0f} ms per pass"}
            print(json.dumps(res), file=_JSON_OUT, flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
