"""Benchmark of the paged-attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|flashinfer]
                    [--workload cfg1|cfg2|cfg3|cfg4|cfg5] [--headline-only]

Metric: paged-decode attention HBM GB/s (fraction of the
measured HBM peak) and decode tok/s, at 1/2/4/8 B200.

Headline workload (default cfg2 = configuration 2): the attention of a
TinyLlama-1.1B decode step — 22 layers, 32 q / 4 kv heads, head_dim 64,
bf16 — for 256 requests per GPU with contexts ~ U[1024, 4096], page size 16,
KV pre-filled N(0,1), page ids a random permutation of the pool. One step =
the device plan + batch indices/positions once, then for each of the 22
layers the KV append of the step's token and the decode attention — one
launch per layer (run_with_append; FlashInfer's arm makes the reference's
two calls, append_paged_kv_cache then run). Requests are sharded
round-robin over GPUs (weak scaling: 256 per GPU), each GPU owning its pool;
no data-path collective (gloo is used only for the barrier and the max over
ranks of the timed region).

value = algorithmic bytes of all ranks (every K/V element read once, q read,
o written, appended rows read + written) / max-over-ranks device time of
the step replayed from a CUDA graph (captured once after warm-up; --eager
times eager launches instead). roofline.avg_launch_ms is one event span
around the 22 decode launches inside that same replayed graph, divided by
22. The same steps are also timed with eager launches (eager_ms_per_step).
e2e = the same bytes / device time of the same step driven through the
public API from pinned host buffers (tables, q, new K/V copied in; outputs
copied out every layer).

Unless --headline-only (or another --workload) is given, the same line also
carries the other configurations, each measured the same way after the
previous one's memory is freed: prefill_cfg3 (the mixed chunked-prefill +
decode step, with the prefill kernel's tensor roofline), long_cfg5 (512
requests of 8-32 k tokens, split across the GPUs: strong scaling),
cascade_cfg4 (64 requests sharing a 2048-token prefix: plain decode and the
two-level cascade, logical and unique bytes) and small_cfg1 (8 requests).
With N > 1 the line adds per-rank figures (per_rank) of every rank's step
time, decode roofline fraction, e2e throughput and host-copy rates.

--impl reference: the reference's attention math on the host cores (the
CPU oracle: fp32 eager attention over gathered pages), rank 0 only, each
step a bounded sample of the same workload.
--impl flashinfer: the same step through FlashInfer itself (the reference's
GPU path, when the flashinfer package is installed), for comparison.
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

PKG = "llm-inference-runtime_b200"
METRIC = "paged-decode attn HBM GB/s (% peak); decode tok/s at 1/2/4/8 B200"


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        # short: ranks that wait for one another end with an error, not a hang
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    return rank, world, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": ["no samples"]}
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# workload name -> (geometry name, requests per GPU (global for strong scaling),
# context lo, hi, layers, description)
WORKLOADS = {
    "cfg1": ("TINYLLAMA", 8, 16, 512, 22, "cfg1 TinyLlama-1.1B decode step, 8 requests"),
    "cfg2": ("TINYLLAMA", 256, 1024, 4096, 22, "cfg2 TinyLlama-1.1B decode step attention"),
    "cfg3": ("LLAMA3_8B", 128, 256, 4096, 1, "cfg3 chunked-prefill mixed batch (decode part)"),
    "cfg4": ("LLAMA3_8B", 64, 32, 256, 1, "cfg4 64 requests sharing a 2048-token prefix"),
    "cfg5": ("LLAMA3_8B", 512, 8192, 32768, 1, "cfg5 long-context split-KV decode"),
}


def _workload(name: str):
    wl = importlib.import_module(PKG + ".workloads")
    gname, per_gpu, lo, hi, layers, desc = WORKLOADS[name]
    return wl, getattr(wl, gname), per_gpu, lo, hi, layers, desc


def _gather(x, world: int) -> list:
    """Every rank's value of x, in rank order (rank 0 alone: [x])."""
    if world == 1:
        return [x]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, x)
    return out


def _global_lengths(batch_total: int, lo: int, hi: int, seed: int = 0) -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (batch_total,), generator=g).numpy().astype(np.int64) + 1


def _backend(args):
    """The attention module a run drives: this package's FlashInfer-compatible
    API, or (--impl flashinfer) FlashInfer itself — the reference's GPU path —
    through the same calls."""
    if args.impl == "flashinfer":
        import flashinfer
        return flashinfer, False
    lir = importlib.import_module(PKG)
    lir.build.build()
    return importlib.import_module(PKG + ".flashinfer_api"), True


def _mark_flashinfer(line: dict) -> None:
    """The --impl flashinfer line: same workload and metric, FlashInfer's kernels."""
    import flashinfer
    line["impl"] = "flashinfer"
    line["flashinfer_version"] = flashinfer.__version__
    line["gpu_launches"] = 0  # none of this package's kernels run
    line["roofline"]["kernel"] = "flashinfer BatchDecodeWithPagedKVCacheWrapper"
    line["roofline"]["traffic"] = None
    if "prefill" in line:
        line["prefill"]["roofline"]["kernel"] = "flashinfer BatchPrefillWithPagedKVCacheWrapper"


def _check(lir, ours: bool, what: str) -> None:
    if ours:
        lir._lib.check_device(what)


# ------------------------------------------------------------------ ours
def run_ours(args, ctx, workload: str, strong: bool = False, cpu_budget_s: float = 15.0):
    """One decode workload (cfg1 / cfg2 / cfg4 / cfg5) on every rank; returns
    rank 0's line (None on the other ranks). strong: the workload's request
    count is the global batch, split round-robin over the ranks (otherwise
    each rank serves that many requests: weak scaling)."""
    rank, world, local = ctx
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lir = importlib.import_module(PKG)
    fi, ours = _backend(args)
    wl, geom, per_gpu, lo, hi, layers, wname = _workload(workload)
    P = geom.page_size

    total_requests = per_gpu if strong else per_gpu * world
    if workload == "cfg4":
        # every GPU serves its own 64 requests over one shared 2048-token prefix
        prob = wl.make_shared_prefix_problem(geom, per_gpu, 2048, lo, hi, seed=1000 + rank,
                                             device=dev, num_layers=layers)
    else:
        # request i on GPU i mod world
        lengths_all = _global_lengths(total_requests, lo, hi)
        mine = wl.round_robin(total_requests, world, rank)
        prob = wl.make_decode_problem(geom, len(mine), 0, 0, seed=1000 + rank, device=dev,
                                      num_layers=layers, lengths=lengths_all[mine])
    B = prob.batch
    indptr, indices, last = prob.device_tables(dev)
    seq = torch.from_numpy(prob.lengths.astype(np.int32)).to(dev)
    append_indptr = torch.arange(B + 1, dtype=torch.int32, device=dev)
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=dev)
    wrap = fi.BatchDecodeWithPagedKVCacheWrapper(ws, "HND")
    q = prob.q
    k_new, v_new = prob.k_new, prob.v_new
    out = torch.empty_like(q)
    pool = prob.pool

    bytes_decode = prob.decode_bytes_per_layer()
    bytes_append = prob.append_bytes_per_layer()
    bytes_step = layers * (bytes_decode + bytes_append)
    # positions + plan, then per layer the decode with the step's KV append
    # fused in (this package) or the reference's append + decode pair
    launches_per_step = 2 + (1 if ours else 2) * layers

    stream = torch.cuda.current_stream()
    dec_events = []

    state = {}

    def prologue():
        state["bi"], state["pos"] = fi.get_batch_indices_positions(append_indptr, seq, B)
        wrap.plan(indptr, indices, last, geom.num_qo_heads, geom.num_kv_heads, geom.head_dim,
                  P, q_data_type=q.dtype)

    def decode_layers():
        for layer in range(layers):
            wrap.run_with_append(q, pool[layer], k_new, v_new, state["pos"], out=out)

    def step(record: bool, span=None):
        prologue()
        bi, pos = state["bi"], state["pos"]
        # Decode-kernel timing: this package's layers are back-to-back decode
        # launches, timed as one span per step (events between them would
        # stop each launch from overlapping its predecessor's tail) and
        # divided by the layer count; FlashInfer's interleave append kernels,
        # so each of its decode launches is bracketed alone.
        if record and ours:
            span = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        if span is not None:
            span[0].record(stream)
        for layer in range(layers):
            if not ours:
                fi.append_paged_kv_cache(k_new, v_new, bi, pos, pool[layer], indices, indptr,
                                         last, kv_layout="HND")
            if record and not ours:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            if ours:
                wrap.run_with_append(q, pool[layer], k_new, v_new, pos, out=out)
            else:
                wrap.run(q, pool[layer], out=out)
            if record and not ours:
                e1.record(stream)
                dec_events.append((e0, e1, 1))
        if span is not None:
            span[1].record(stream)
            if record:
                dec_events.append((span[0], span[1], layers))

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    _check(lir, ours, f"bench {workload} warm-up")

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    # Configurations whose KV fits in L2 (cfg1, cfg4) time each step alone
    # after reading a 256 MiB buffer (clean L2 lines, nothing to write back);
    # the others stream more than L2 per step and run back to back.
    unique_kv = (int(prob.extra["unique_pages"]) * geom.page_size * geom.kv_bytes_per_token
                 if "unique_pages" in prob.extra else bytes_decode)
    small = unique_kv < (100 << 20)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if small else None

    def timed(run_step, after=None) -> float:
        if small:
            total = 0.0
            for _ in range(args.steps):
                flush.view(torch.int64).sum()
                t0.record(stream)
                run_step()
                t1.record(stream)
                torch.cuda.synchronize()
                total += t0.elapsed_time(t1)
                if after is not None:
                    after()
            return total
        t0.record(stream)
        for _ in range(args.steps):
            run_step()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)

    # Eager launches first, then -- this package only -- the same step
    # captured once in a CUDA graph and replayed, which is how a serving loop
    # runs a launch-bound decode step. The decode kernel's duration for the
    # roofline comes from a second graph holding only the step's decode
    # launches (the prologue's plan stays valid in the workspace), replayed
    # back to back with an event between replays (one per replay after an
    # L2 flush for the configurations that fit in L2): the step's launches
    # as the timed step runs them, without its prologue. FlashInfer's plan works on the host
    # and cannot be captured, so its arm stays eager and its decode launches
    # are timed one by one.
    eager_local = timed(lambda: step(True))
    spans = []
    if ours and not args.eager:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(False)
        graph.replay()
        torch.cuda.synchronize()
        _barrier(world)
        ms_local = timed(graph.replay)
        dgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(dgraph):
            decode_layers()
        dgraph.replay()
        torch.cuda.synchronize()
        _barrier(world)
        if small:
            for _ in range(args.steps):
                flush.view(torch.int64).sum()
                t0.record(stream)
                dgraph.replay()
                t1.record(stream)
                torch.cuda.synchronize()
                spans.append(t0.elapsed_time(t1))
        else:
            # back to back, one event between replays, read after one sync
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
            evs[0].record(stream)
            for k in range(args.steps):
                dgraph.replay()
                evs[k + 1].record(stream)
            torch.cuda.synchronize()
            spans = [evs[k].elapsed_time(evs[k + 1]) for k in range(args.steps)]
        del graph, dgraph
    else:
        ms_local = eager_local
    _barrier(world)
    clocks = sampler.stop()
    ms = _max_over_ranks(ms_local, world)
    eager_ms = _max_over_ranks(eager_local, world)
    if spans:
        dec_ms_local = statistics.mean(spans) / layers
        dec_timing = ("one event span around a graph of the step's decode launches, "
                      "replayed back to back as in the step graph")
    else:
        dec_ms_local = (sum(a.elapsed_time(b) for a, b, _ in dec_events)
                        / sum(n for _, _, n in dec_events))
        dec_timing = "event pairs around each eager decode launch"
    # ranks decode different requests: the line's kernel figures are the mean
    # over ranks of the bytes per launch and of the launch duration (the
    # slowest rank's step time is in ms_per_step; per_rank lists each rank)
    dec_ms = _sum_over_ranks(dec_ms_local, world) / world
    total_bytes = _sum_over_ranks(float(bytes_step) * args.steps, world)
    value = total_bytes / (ms * 1e-3) / 1e9
    tok_s = _sum_over_ranks(float(B) * args.steps, world) / (ms * 1e-3)
    _check(lir, ours, f"bench {workload} timed region")

    # ---- end to end through the public API from pinned host memory
    # Every step copies its inputs in (tables once, then each layer's q and new
    # K/V rows) and each layer's attention output out. The copies run on two
    # copy streams, double-buffered per layer, so layer l+1's inputs and layer
    # l-1's output move while layer l computes; the timed region ends only
    # when the last output has landed in host memory.
    h_indptr = torch.from_numpy(prob.kv_indptr).pin_memory()
    h_indices = torch.from_numpy(prob.kv_indices).pin_memory()
    h_last = torch.from_numpy(prob.kv_last_page_len).pin_memory()
    h_seq = seq.cpu().pin_memory()
    h_q = torch.stack([q.cpu()] * layers).pin_memory()
    h_k = torch.stack([k_new.cpu()] * layers).pin_memory()
    h_v = torch.stack([v_new.cpu()] * layers).pin_memory()
    h_out = torch.empty((layers,) + tuple(q.shape), dtype=q.dtype).pin_memory()
    d_q = [torch.empty_like(q) for _ in range(2)]
    d_k = [torch.empty_like(k_new) for _ in range(2)]
    d_v = [torch.empty_like(v_new) for _ in range(2)]
    d_out = [torch.empty_like(q) for _ in range(2)]
    d_indptr, d_indices, d_last = (torch.empty_like(indptr), torch.empty_like(indices),
                                   torch.empty_like(last))
    d_seq = torch.empty_like(seq)
    h2d = (h_indptr.numel() + h_indices.numel() + h_last.numel() + h_seq.numel()) * 4 + \
        layers * (q.numel() + k_new.numel() + v_new.numel()) * 2
    d2h = layers * q.numel() * 2
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731

    def e2e_step():
        tables = ev()
        with torch.cuda.stream(s_in):
            s_in.wait_stream(stream)  # previous step's users of the buffers are done
            d_indptr.copy_(h_indptr, non_blocking=True)
            d_indices.copy_(h_indices, non_blocking=True)
            d_last.copy_(h_last, non_blocking=True)
            d_seq.copy_(h_seq, non_blocking=True)
            tables.record(s_in)
        in_ready = [ev() for _ in range(layers)]
        in_free = [ev() for _ in range(layers)]
        out_ready = [ev() for _ in range(layers)]
        out_free = [ev() for _ in range(layers)]

        def load(layer):
            b = layer % 2
            with torch.cuda.stream(s_in):
                if layer >= 2:
                    s_in.wait_event(in_free[layer - 2])
                d_q[b].copy_(h_q[layer], non_blocking=True)
                d_k[b].copy_(h_k[layer], non_blocking=True)
                d_v[b].copy_(h_v[layer], non_blocking=True)
                in_ready[layer].record(s_in)

        load(0)
        stream.wait_event(tables)
        bi, pos = fi.get_batch_indices_positions(append_indptr, d_seq, B)
        wrap.plan(d_indptr, d_indices, d_last, geom.num_qo_heads, geom.num_kv_heads,
                  geom.head_dim, P, q_data_type=q.dtype)
        for layer in range(layers):
            b = layer % 2
            if layer + 1 < layers:
                load(layer + 1)
            stream.wait_event(in_ready[layer])
            if layer >= 2:
                stream.wait_event(out_free[layer - 2])
            if ours:
                wrap.run_with_append(d_q[b], pool[layer], d_k[b], d_v[b], pos, out=d_out[b])
            else:
                fi.append_paged_kv_cache(d_k[b], d_v[b], bi, pos, pool[layer], d_indices,
                                         d_indptr, d_last, kv_layout="HND")
                wrap.run(d_q[b], pool[layer], out=d_out[b])
            in_free[layer].record(stream)
            out_ready[layer].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(out_ready[layer])
                h_out[layer].copy_(d_out[b], non_blocking=True)
                out_free[layer].record(s_out)
        stream.wait_stream(s_out)  # the step ends when the last output is in host memory

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    t0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    t1.record(stream)
    torch.cuda.synchronize()
    e2e_local = t0.elapsed_time(t1)
    _barrier(world)
    e2e_ms = _max_over_ranks(e2e_local, world)
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    ok = torch.equal(h_out[layers - 1], out.cpu())  # same q, same pool state: same result
    _check(lir, ours, f"bench {workload} e2e")

    # ---- host-copy rates alone: every rank moves one step's input and output
    # bytes at the same time (the contention the e2e steps run under)
    def copy_rate(direction: str) -> float:
        _barrier(world)
        torch.cuda.synchronize()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s_in):
            c0.record(s_in)
            for _ in range(args.steps):
                for layer in range(layers):
                    b = layer % 2
                    if direction == "h2d":
                        d_q[b].copy_(h_q[layer], non_blocking=True)
                        d_k[b].copy_(h_k[layer], non_blocking=True)
                        d_v[b].copy_(h_v[layer], non_blocking=True)
                    else:
                        h_out[layer].copy_(d_out[b], non_blocking=True)
            c1.record(s_in)
        torch.cuda.synchronize()
        n = layers * ((q.numel() + k_new.numel() + v_new.numel()) * 2 if direction == "h2d"
                      else q.numel() * 2)
        return n * args.steps / (c0.elapsed_time(c1) * 1e-3) / 1e9

    h2d_gbs, d2h_gbs = copy_rate("h2d"), copy_rate("d2h")
    _barrier(world)

    # configuration 2 is a full decode step: also time the whole model
    model = (model_step(args, ours, prob, indptr, indices, last, seq, world)
             if workload == "cfg2" and not args.no_model else None)
    if ours:
        _check(lir, ours, "bench model step")
    # configuration 4: the same step with the shared prefix attended once
    cascade = (cascade_step(args, fi, prob, geom, layers, seq, append_indptr, out, small, flush,
                            world, bytes_step)
               if workload == "cfg4" and ours else None)
    if ours:
        _check(lir, ours, "bench cascade step")

    peak, peak_kind = _peaks()
    # the timed launch: decode + the step's fused append (ours), decode alone (FlashInfer)
    bytes_launch_local = bytes_decode + (bytes_append if ours else 0)
    bytes_launch = int(round(_sum_over_ranks(float(bytes_launch_local), world) / world))
    achieved = bytes_launch / (dec_ms * 1e-3) / 1e9
    per_rank = _gather({"ms_per_step": round(ms_local / args.steps, 4),
                        "decode_frac_of_hbm": round(bytes_launch_local / (dec_ms_local * 1e-3)
                                                    / 1e9 / peak, 4),
                        "e2e_gbs": round(bytes_step * args.steps / (e2e_local * 1e-3) / 1e9, 1),
                        "h2d_gbs": round(h2d_gbs, 2), "d2h_gbs": round(d2h_gbs, 2),
                        "requests": B}, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and ours:
        cpu = cpu_baseline(prob_lengths=prob.lengths, geom=geom, layers=layers,
                           budget_s=cpu_budget_s)
    # every collective of this workload before rank 0 alone builds the line
    unique_total = (_sum_over_ranks(float(layers * unique_kv) * args.steps, world)
                    if workload == "cfg4" else 0.0)
    _barrier(world)
    del prob, pool, ws, flush
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/K/V, random page permutation, random-init",
        "step_launch": "CUDA graph replay" if ours and not args.eager else "eager",
        "eager_ms_per_step": round(eager_ms / args.steps, 4),
        "config": _config(workload, geom, layers, total_requests, world, lo, hi,
                          "L2 flushed between timed steps (256 MiB read); distinct KV "
                          f"of one layer {unique_kv / 1e6:.1f} MB" if small else
                          "inputs larger than L2 (KV of one layer "
                          f"{bytes_decode / 1e6:.0f} MB vs 126 MB L2)", strong),
        "decode_tok_s": round(tok_s, 1),
        **({"unique_kv_bytes_per_layer": int(unique_kv),
            "logical_kv_bytes_per_layer": int(bytes_decode),
            "unique_value": round(unique_total / (ms * 1e-3) / 1e9, 2),
            "note": "value counts the shared prefix once per request (logical bytes); its "
                    "pages stay in L2, so logical GB/s can exceed the HBM peak; unique_value "
                    "counts every distinct page once"}
           if workload == "cfg4" else {}),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_kind": peak_kind,
                     "kernel": "decode_kernel (step's KV append fused)" if ours
                     else "decode_kernel",
                     "bytes_per_launch": bytes_launch,
                     "avg_launch_ms": round(dec_ms, 5),
                     "launch_timing": dec_timing,
                     "traffic": _traffic_from_profile(bytes_launch, geom.head_dim) if ours
                     else None},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / args.steps, 4),
                "copies": "pinned host buffers, two copy streams overlapped with compute",
                "last_layer_matches_device_run": ok},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if world > 1:
        line["per_rank"] = per_rank
    if model is not None:
        line["model_step"] = model
    if cascade is not None:
        line["cascade"] = cascade
    if not ours:
        _mark_flashinfer(line)
    return line


def _config(workload, geom, layers, total_requests, world, lo, hi, l2, strong=False) -> dict:
    """The config object every arm reports for a workload (same keys and
    values on this package's, FlashInfer's and the reference's lines)."""
    per_gpu = -(-total_requests // world) if strong else total_requests // world
    return {"workload": WORKLOADS[workload][5], "layers": layers,
            "num_qo_heads": geom.num_qo_heads, "num_kv_heads": geom.num_kv_heads,
            "head_dim": geom.head_dim, "page_size": geom.page_size,
            "requests_per_gpu": per_gpu, "global_batch": total_requests,
            "context": f"U[{lo},{hi}] + 1 appended",
            "parallelism": f"request-sharded x{world}, no collective", "l2": l2}


def cascade_step(args, fi, prob, geom, layers, seq, append_indptr, plain_out, small, flush,
                 world: int, bytes_step: int) -> dict:
    """Configuration 4 through the two-level cascade wrapper: level 0 the
    2048-token prefix every request shares (attended once for all requests),
    level 1 each request's own pages. One step = positions + cascade plan,
    then per layer the cascade run with the step's KV append; replayed from a
    CUDA graph, timed like the plain step (L2 flushed before each step).
    The append is fused into the level-1 decode, as the plain step fuses it.
    Throughput is reported in the same logical bytes as the plain step."""
    dev = prob.pool.device
    B = prob.batch
    sp = int(prob.extra["shared_pages"])
    indptr, indices = prob.kv_indptr, prob.kv_indices
    uniq, uptr = [], [0]
    for b in range(B):
        pages = indices[indptr[b]:indptr[b + 1]]
        uniq.append(pages[sp:])
        uptr.append(uptr[-1] + len(pages) - sp)
    t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    s_indptr, s_indices, s_last = t([0, sp]), t(indices[:sp]), t([geom.page_size])
    u_indptr, u_indices = t(uptr), t(np.concatenate(uniq))
    u_last = t(prob.kv_last_page_len)
    ws = torch.empty(max(fi.cascade_workspace_bytes(B, geom.num_qo_heads, geom.num_kv_heads,
                                                    geom.head_dim), 1 << 20),
                     dtype=torch.uint8, device=dev)
    w = fi.MultiLevelCascadeAttentionWrapper(2, ws, "HND")
    out = torch.empty_like(prob.q)
    qo_levels = [torch.tensor([0, B], dtype=torch.int32),
                 torch.arange(B + 1, dtype=torch.int32)]

    def step():
        _, pos = fi.get_batch_indices_positions(append_indptr, seq, B)
        w.plan(qo_levels, [s_indptr, u_indptr], [s_indices, u_indices], [s_last, u_last],
               geom.num_qo_heads, geom.num_kv_heads, geom.head_dim, geom.page_size)
        for layer in range(layers):
            w.run_with_append(prob.q, prob.pool[layer], prob.k_new, prob.v_new, pos, out=out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _barrier(world)
    total = 0.0
    for _ in range(args.steps):
        if small:
            flush.view(torch.int64).sum()
        t0.record(stream)
        graph.replay()
        t1.record(stream)
        torch.cuda.synchronize()
        total += t0.elapsed_time(t1)
    ms = _max_over_ranks(total / args.steps, world)
    diff = (out.float() - plain_out.float()).abs()
    mx, mean = float(diff.max()), float(diff.mean())
    del graph
    return {"levels": f"level 0: {sp} shared pages, level 1: each request's own pages",
            "ms_per_step": round(ms, 4),
            "value": round(_sum_over_ranks(float(bytes_step), world) / (ms * 1e-3) / 1e9, 2),
            "unit": "GB/s (logical bytes, as the plain step)",
            "step_launch": "CUDA graph replay",
            "matches_plain_step": {"max_abs": round(mx, 5), "mean_abs": round(mean, 6),
                                   "within_tolerance": bool(mx <= 2e-2 and mean <= 2e-3)}}


def model_step(args, ours: bool, prob, indptr, indices, last, seq, world: int) -> dict:
    """Configuration 2's full decode step: a TinyLlama-1.1B-geometry HF LLaMA
    (22 layers, hidden 2048, MLP 5632, 32 q / 4 kv heads, vocab 32000,
    RMSNorm, RoPE theta 1e4; random-init bf16 weights) patched with this
    package's ``llama`` module exactly as the reference engine patches its
    model, decoding one token for each of the step's requests over the same
    paged pool. One step = positions + plan + the model forward (22 x
    qkv GEMM, RoPE + append, paged decode, o_proj, MLP; lm_head).

    FlashInfer's arm runs the same model with the reference's per-layer calls
    (apply_rope_pos_ids_inplace, append_paged_kv_cache, decode forward; its
    plan works on the host, so eager only). This package's step is also
    replayed from a CUDA graph. transformers builds no attention mask for a
    one-token causal query under its "sdpa" setting; the patched attention
    reads none either way."""
    from transformers import LlamaConfig, LlamaForCausalLM
    lm = importlib.import_module(PKG + ".llama")
    saved = (lm.flashinfer, lm.paged_attention)
    B = prob.batch
    dev = prob.pool.device
    if not ours:
        import flashinfer as real_fi
        lm.flashinfer = real_fi

        def fi_paged_attention(attn, q_flat, k_flat, v_flat):
            st = lm.PagedAttnState
            layer_kv_cache = st.kv_pool[attn.layer_idx]
            real_fi.apply_rope_pos_ids_inplace(q_flat, k_flat, st.positions, rotary_dim=None,
                                               interleave=False, rope_scale=attn.rope_scale,
                                               rope_theta=attn.rope_theta)
            real_fi.append_paged_kv_cache(k_flat, v_flat, st.batch_indices, st.positions,
                                          layer_kv_cache, st.kv_indices, st.kv_indptr,
                                          st.kv_last_page_len, kv_layout="HND")
            return st.decode_wrapper.forward(q=q_flat, paged_kv_cache=layer_kv_cache)

        lm.paged_attention = fi_paged_attention
    try:
        g = prob.geom
        cfg = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                          num_hidden_layers=g.num_layers, num_attention_heads=g.num_qo_heads,
                          num_key_value_heads=g.num_kv_heads, max_position_embeddings=8192,
                          rms_norm_eps=1e-5, rope_theta=10000.0)
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(0)
        with torch.device(dev):
            model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
        lm.patch_llama_model(model)
        params = sum(p.numel() for p in model.parameters())
        lm.init_flashinfer_state(kv_pool=prob.pool, page_size=g.page_size, device=dev)
        append_indptr = torch.arange(B + 1, dtype=torch.int32, device=dev)
        ids = torch.randint(0, 32000, (B, 1), device=dev,
                            generator=torch.Generator(dev).manual_seed(1))

        def step():
            lm.build_batch_indices_positions(append_indptr, seq, **({"nnz": B} if ours else {}))
            lm.plan_decode(kv_indptr=indptr, kv_indices=indices, kv_last_page_len=last,
                           num_qo_heads=g.num_qo_heads, num_kv_heads=g.num_kv_heads,
                           head_dim=g.head_dim)
            with torch.no_grad():
                return model(input_ids=ids, use_cache=False).logits

        stream = torch.cuda.current_stream()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)

        def timed(run) -> float:
            _barrier(world)
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(args.steps):
                run()
            t1.record(stream)
            torch.cuda.synchronize()
            return _max_over_ranks(t0.elapsed_time(t1) / args.steps, world)

        for _ in range(max(3, args.warmup)):
            step()
        eager_ms = timed(step)
        res = {"model": "TinyLlama-1.1B geometry, random-init bf16 weights",
               "parameters": params, "requests_per_gpu": B,
               "eager_ms_per_step": round(eager_ms, 4),
               "eager_decode_tok_s": round(_sum_over_ranks(B / (eager_ms * 1e-3), world), 1)}
        if ours and not args.eager:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                logits = step()
            graph.replay()
            torch.cuda.synchronize()
            graph_ms = timed(graph.replay)
            check = step()
            torch.cuda.synchronize()
            res.update({"ms_per_step": round(graph_ms, 4),
                        "decode_tok_s": round(_sum_over_ranks(B / (graph_ms * 1e-3), world), 1),
                        "step_launch": "CUDA graph replay",
                        "graph_logits_equal_eager": bool(torch.equal(logits, check))})
            del graph
        else:
            res.update({"ms_per_step": res["eager_ms_per_step"],
                        "decode_tok_s": res["eager_decode_tok_s"], "step_launch": "eager"})
        del model
        return res
    finally:
        lm.flashinfer, lm.paged_attention = saved


def _traffic_from_profile(bytes_launch: int, head_dim: int, name="decode_kernel_traffic.json"):
    """DRAM bytes per launch of the kernel instance for this head size, from
    the committed ncu summary (None if none was captured): the capture's
    bytes scaled by the algorithmic bytes of this launch over the capture's
    (traffic grows with the K/V bytes processed)."""
    path = os.path.join(REPO, "profiles", name)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)["by_head_dim"].get(str(head_dim))
    if d is None:
        return None
    return int(d["dram_bytes_per_launch"] * bytes_launch / d["algorithmic_bytes_per_launch"])


# --------------------------------------------------------------- cfg3
def run_mixed(args, ctx, cpu_budget_s: float = 8.0):
    """Configuration 3: one Llama-3-8B attention layer serving a mixed step —
    16 prefill chunks of 512 rows over cached prefixes U[0, 2048] (causal,
    tcgen05 prefill kernel) and 128 decode rows with contexts U[256, 4096]
    (decode kernel), both on the same pool. Requests are sharded round-robin
    (weak scaling: the whole mixed batch per GPU). value = decode GB/s of the
    step's decode part; the prefill part is reported as TFLOP/s of visible
    (unmasked) query-key pairs. Returns rank 0's line (None elsewhere)."""
    rank, world, local = ctx
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lir = importlib.import_module(PKG)
    fi, ours = _backend(args)
    wl, geom, n_dec, lo, hi, layers, wname = _workload("cfg3")
    pre = wl.config3_prefill(seed=rank, device=dev)
    dec = wl.make_decode_problem(geom, n_dec, lo, hi, seed=100 + rank, device=dev, num_layers=1,
                                 append=False)
    qo, kvp, kvi, last = pre.device_tables(dev)
    dindptr, dindices, dlast = dec.device_tables(dev)
    ws_p = torch.empty(128 << 20, dtype=torch.uint8, device=dev)
    ws_d = torch.empty(128 << 20, dtype=torch.uint8, device=dev)
    pw = fi.BatchPrefillWithPagedKVCacheWrapper(ws_p, "HND")
    dw = fi.BatchDecodeWithPagedKVCacheWrapper(ws_d, "HND")
    q_pre, q_dec = pre.q, dec.q
    out_pre, out_dec = torch.empty_like(q_pre), torch.empty_like(q_dec)
    flops = pre.flops(causal=True)
    dbytes = dec.decode_bytes_per_layer()
    stream = torch.cuda.current_stream()
    ev = []

    def step(record):
        e = None
        # total_qo (this package's extension) lets the prefill plan run on the
        # device without reading qo_indptr back; FlashInfer plans on the host
        extra = {"total_qo": q_pre.shape[0]} if ours else {}
        pw.plan(qo, kvp, kvi, last, geom.num_qo_heads, geom.num_kv_heads, geom.head_dim, 16,
                causal=True, q_data_type=q_pre.dtype, **extra)
        dw.plan(dindptr, dindices, dlast, geom.num_qo_heads, geom.num_kv_heads, geom.head_dim,
                16, q_data_type=q_dec.dtype)
        if record:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        if e is not None:
            e[0].record(stream)
        pw.run(q_pre, pre.pool[0], out=out_pre)
        if e is not None:
            e[1].record(stream)
        dw.run(q_dec, dec.pool[0], out=out_dec)
        if e is not None:
            e[2].record(stream)
            if record:
                ev.append(e)

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    _check(lir, ours, "bench cfg3 warm-up")
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)

    def timed(run_step) -> float:
        t0.record(stream)
        for _ in range(args.steps):
            run_step()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)

    # eager launches first, then this package's step replayed from a CUDA
    # graph (both plans run on the device). The two kernels' durations come
    # from two more graphs, the step's prefill launch and its decode launch
    # (the plans stay valid in the workspaces), replayed one after the other
    # between events, in the step's order (eager events for FlashInfer).
    eager_local = timed(lambda: step(True))
    graph = None
    spans = []
    if ours and not args.eager:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(False)
        graph.replay()
        torch.cuda.synchronize()
        _barrier(world)
        ms_local = timed(graph.replay)
        gp, gd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gp):
            pw.run(q_pre, pre.pool[0], out=out_pre)
        with torch.cuda.graph(gd):
            dw.run(q_dec, dec.pool[0], out=out_dec)
        gp.replay()
        gd.replay()
        torch.cuda.synchronize()
        # back to back, events between the replays, read after one sync
        ge = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
        ge[0].record(stream)
        for k in range(args.steps):
            gp.replay()
            ge[2 * k + 1].record(stream)
            gd.replay()
            ge[2 * k + 2].record(stream)
        torch.cuda.synchronize()
        spans = [(ge[2 * k].elapsed_time(ge[2 * k + 1]), ge[2 * k + 1].elapsed_time(ge[2 * k + 2]))
                 for k in range(args.steps)]
        del graph, gp, gd
    else:
        ms_local = eager_local
    _barrier(world)
    clocks = sampler.stop()
    ms = _max_over_ranks(ms_local, world)
    eager_ms = _max_over_ranks(eager_local, world)
    if spans:
        pre_ms = statistics.mean(a for a, _ in spans)
        dec_ms = statistics.mean(b for _, b in spans)
        launch_timing = "events around graphs of the step's prefill and decode launches"
    else:
        pre_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
        dec_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
        launch_timing = "event pairs around each eager launch"
    # mean over ranks (each rank serves its own mixed batch), as in run_ours
    pre_ms_local, dec_ms_local = pre_ms, dec_ms
    pre_ms = _sum_over_ranks(pre_ms, world) / world
    dec_ms = _sum_over_ranks(dec_ms, world) / world
    flops_local, dbytes_local = flops, dbytes
    flops = _sum_over_ranks(float(flops), world) / world
    dbytes = int(round(_sum_over_ranks(float(dbytes), world) / world))
    _check(lir, ours, "bench cfg3")
    total_dbytes = _sum_over_ranks(float(dbytes) * args.steps, world)
    value = total_dbytes / (ms * 1e-3) / 1e9

    # ---- end to end: every step copies the tables and both q batches in from
    # pinned host memory and both outputs back, around the same calls. Device
    # buffers are double-buffered across steps: step i+1's inputs go up on
    # one copy stream and step i-1's outputs come down on another while step
    # i computes, so both PCIe directions overlap the kernels; the timed
    # region ends when the last output is in host memory.
    host = {k: v.cpu().pin_memory() for k, v in
            dict(qo=qo, kvp=kvp, kvi=kvi, last=last, di=dindptr, dx=dindices, dl=dlast,
                 qp=q_pre, qd=q_dec).items()}
    dev_in = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in range(2)]
    d_out_pre = [torch.empty_like(out_pre) for _ in range(2)]
    d_out_dec = [torch.empty_like(out_dec) for _ in range(2)]
    h_out_pre = torch.empty(out_pre.shape, dtype=out_pre.dtype).pin_memory()
    h_out_dec = torch.empty(out_dec.shape, dtype=out_dec.dtype).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_pre.numel() * out_pre.element_size() + out_dec.numel() * out_dec.element_size()
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    for e in in_free + out_free:
        e.record(stream)

    def e2e_step(i):
        b = i % 2
        d = dev_in[b]
        ready, done = torch.cuda.Event(), torch.cuda.Event()
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[b])  # step i-2 no longer reads these inputs
            for k, v in host.items():
                d[k].copy_(v, non_blocking=True)
            ready.record(s_in)
        stream.wait_event(ready)
        stream.wait_event(out_free[b])  # step i-2's outputs have left the device
        extra = {"total_qo": q_pre.shape[0]} if ours else {}
        pw.plan(d["qo"], d["kvp"], d["kvi"], d["last"], geom.num_qo_heads,
                geom.num_kv_heads, geom.head_dim, 16, causal=True, q_data_type=q_pre.dtype,
                **extra)
        dw.plan(d["di"], d["dx"], d["dl"], geom.num_qo_heads, geom.num_kv_heads,
                geom.head_dim, 16, q_data_type=q_dec.dtype)
        pw.run(d["qp"], pre.pool[0], out=d_out_pre[b])
        dw.run(d["qd"], dec.pool[0], out=d_out_dec[b])
        done.record(stream)
        in_free[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            h_out_pre.copy_(d_out_pre[b], non_blocking=True)
            h_out_dec.copy_(d_out_dec[b], non_blocking=True)
            out_free[b].record(s_out)

    for i in range(args.warmup):
        e2e_step(i)
    stream.wait_stream(s_out)
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    t1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_ms = _max_over_ranks(t0.elapsed_time(t1), world)
    e2e_value = total_dbytes / (e2e_ms * 1e-3) / 1e9
    _check(lir, ours, "bench cfg3 e2e")
    peak_bw, bw_kind = _peaks()
    with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
        peak_tf = float(json.load(f)["bf16_tflops"])
    pre_tf = flops / (pre_ms * 1e-3) / 1e12
    dec_gbs = dbytes / (dec_ms * 1e-3) / 1e9
    cpu, cpu_pre = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and ours:
        from oracle import cpu_baseline as cb
        cpu = cb.time_decode_sample(dec.lengths, geom, budget_s=cpu_budget_s, sample=16)
        cpu_pre = cb.time_prefill_sample(pre.qo_lens, pre.prefix_lens, geom,
                                         budget_s=cpu_budget_s)
    pre_counters = _prefill_counters()
    per_rank = _gather({"ms_per_step": round(ms_local / args.steps, 4),
                        "prefill_tflops": round(flops_local / (pre_ms_local * 1e-3) / 1e12, 1),
                        "decode_frac_of_hbm": round(dbytes_local / (dec_ms_local * 1e-3) / 1e9
                                                    / peak_bw, 4)}, world)
    _barrier(world)
    del pre, dec, ws_p, ws_d
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) q/K/V, random page permutation",
            "step_launch": "CUDA graph replay" if spans else "eager",
            "eager_ms_per_step": round(eager_ms / args.steps, 4),
            "config": {"workload": wname, "layers": 1, "num_qo_heads": geom.num_qo_heads,
                       "num_kv_heads": geom.num_kv_heads, "head_dim": geom.head_dim,
                       "page_size": 16, "prefill": "16 chunks x 512 rows, prefix U[0,2048]",
                       "decode_rows": n_dec, "context": f"U[{lo},{hi}]",
                       "parallelism": f"request-sharded x{world}, no collective",
                       "l2": "decode KV 1.1 GB per step exceeds L2"},
            "roofline": {"bound": "hbm", "achieved": round(dec_gbs, 1), "peak": peak_bw,
                         "unit": "GB/s", "frac": round(dec_gbs / peak_bw, 4),
                         "peak_kind": bw_kind, "kernel": "decode_kernel",
                         "bytes_per_launch": dbytes, "avg_launch_ms": round(dec_ms, 5),
                         "launch_timing": launch_timing,
                         "traffic": _traffic_from_profile(dbytes, geom.head_dim) if ours
                         else None},
            "prefill": {"tflops": round(pre_tf, 1), "gflop_per_launch": round(flops / 1e9, 2),
                        "avg_launch_ms": round(pre_ms, 5), "launch_timing": launch_timing,
                        "roofline": {"bound": "tensor", "achieved": round(pre_tf, 1),
                                     "peak": peak_tf, "unit": "TFLOP/s",
                                     "frac": round(pre_tf / peak_tf, 4),
                                     "peak_kind": "measured (cuBLAS bf16 burst)",
                                     "kernel": "prefill_kernel",
                                     "traffic": pre_counters.get("dram_bytes_per_launch")},
                        "tensor_pipe_active": pre_counters.get("tensor_pipe_active"),
                        "counters_source": pre_counters.get("source"),
                        "cpu_baseline": cpu_pre},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / args.steps, 4),
                    "copies": "pinned host buffers, double-buffered across steps on two copy streams"},
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if world > 1:
            line["per_rank"] = per_rank
        if not ours:
            _mark_flashinfer(line)
    return line


def _prefill_counters() -> dict:
    """The prefill kernel's ncu counters on configuration 3 (committed
    summary), if captured: tensor-pipe activity and DRAM bytes per launch."""
    path = os.path.join(REPO, "profiles", "prefill_kernel_counters.json")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


# ------------------------------------------------------------- CPU side
def cpu_baseline(prob_lengths: np.ndarray, geom, layers: int, budget_s: float = 15.0,
                 sample: int = 16) -> dict:
    """Times the CPU oracle (fp32 eager attention over gathered pages) on a
    seeded sample of the workload's requests, one layer; reports GB/s of the
    same algorithmic bytes."""
    from oracle import cpu_baseline as cb
    return cb.time_decode_sample(prob_lengths, geom, budget_s=budget_s, sample=sample)


def run_reference(args, ctx):
    rank, world, local = ctx
    if rank != 0:
        return None
    workload = args.workload
    wl, geom, per_gpu, lo, hi, layers, wname = _workload(workload)
    from oracle import cpu_baseline as cb
    lengths_all = _global_lengths(per_gpu * world, lo, hi)
    mine = wl.round_robin(per_gpu * world, world, 0)
    lens = lengths_all[mine]
    res = cb.run_reference_arm(lens, geom, steps=args.steps, warmup=args.warmup)
    # the same config object as this package's line for the workload
    bytes_decode = int(lens.sum()) * geom.kv_bytes_per_token + \
        2 * len(lens) * geom.num_qo_heads * geom.head_dim * 2
    l2 = ("inputs larger than L2 (KV of one layer "
          f"{bytes_decode / 1e6:.0f} MB vs 126 MB L2)")
    line = {
        "metric": METRIC, "value": round(res["value"], 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) q/K/V, random page permutation",
        "config": _config(workload, geom, layers, per_gpu * world, world, lo, hi, l2),
        "impl": "reference",
        "cpu_baseline": {"value": round(res["value"], 3), "unit": "GB/s", "cores": res["cores"],
                         "kind": "port", "sample": res["sample"] + "; host cores of rank 0"},
        "e2e": {"value": round(res["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    return line


# other configurations carried in the headline line: (key, workload, strong scaling)
EXTRA = [("prefill_cfg3", "cfg3", False), ("long_cfg5", "cfg5", True),
         ("cascade_cfg4", "cfg4", False), ("small_cfg1", "cfg1", False)]
# keys of a configuration's own line kept in its sub-object
SUB_KEYS = ("value", "unit", "ms_per_step", "scaling", "step_launch", "eager_ms_per_step",
            "config", "decode_tok_s", "roofline", "prefill", "e2e", "cpu_baseline", "clocks",
            "gpu_launches", "cascade", "unique_value", "unique_kv_bytes_per_layer",
            "logical_kv_bytes_per_layer", "note", "per_rank")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "flashinfer"], default="ours")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"],
                    default="cfg2")
    ap.add_argument("--headline-only", action="store_true",
                    help="measure the headline workload only (no other configurations)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the full-model decode step of configuration 2")
    ap.add_argument("--eager", action="store_true",
                    help="time the decode step with eager launches instead of a CUDA graph")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ctx = _dist()
    try:
        if args.impl == "reference":
            line = run_reference(args, ctx)
        elif args.workload == "cfg3":
            line = run_mixed(args, ctx)
        else:
            line = run_ours(args, ctx, args.workload, strong=args.workload == "cfg5")
        if (args.workload == "cfg2" and args.impl == "ours" and not args.headline_only):
            for key, workload, strong in EXTRA:
                torch.cuda.empty_cache()
                sub = (run_mixed(args, ctx, cpu_budget_s=5.0) if workload == "cfg3" else
                       run_ours(args, ctx, workload, strong=strong, cpu_budget_s=5.0))
                if line is not None:
                    line[key] = {k: sub[k] for k in SUB_KEYS if k in sub}
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if ctx[1] > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
