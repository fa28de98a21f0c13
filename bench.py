"""Benchmark of the windowed-eviction decode path on B200.

Workload (one "step"): one decode step of one attention layer of the
isolated decode-attention geometry at 32k context — batch 16, 32 query heads,
8 KV heads (GQA 4), head_dim 64, fp16, retained cache 0.40 x 32768 = 13100
tokens (4 fp16 sinks + 3280 fp16 local + 9816 int4 tier tokens): append the
new token, decode attention with the fused window-mass accumulation, and on
every 8th step the fused eviction (select, compact, re-rotate, quantise).
Inputs are synthetic N(0,1) (seeded); the working set (~208 MB per step) is
larger than the 126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The timed steps replay one captured CUDA graph per step (the host code of a
step runs once, at capture); `e2e` runs the same steps through the public API
(WindowedCache stepped by DecodeGraphs) with each step's inputs copied in
from pinned host memory and its output copied back.  N > 1 runs as torchrun ranks, one GPU each, the 16 rows
partitioned over the ranks (strong scaling, no collective on the attention
path); the reported value is the 16 rows decoded per second, timed as the max
over ranks.  The default line also carries `model_e2e`: the Llama-3.2-1B
shaped decoder of run_e2e with its global batch of 32 rows partitioned over
the ranks (skip with --no-model), and at N = 1 `evict_first`: the isolated
first eviction of a bf16 16k-token cache of run_evict_first (skip with
--no-evict-first).
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, HQ, HKV, D, CTX = 16, 32, 8, 64, 32768
WS, SINKS, LOCAL, BUDGET = 8, 4, 0.25, 0.40
METRIC = "decode tokens/s (32k ctx, int4 tier, one attention layer)"
UNIT = "tokens/s"


def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


class _no_gc:
    """Collect now, then keep Python's cyclic collector out of a timed region
    (in a process with transformers loaded one full collection takes tens of
    milliseconds, which would land in a host-driven step)."""

    def __enter__(self):
        import gc
        gc.collect()
        self.was = gc.isenabled()
        gc.disable()

    def __exit__(self, *exc):
        import gc
        if self.was:
            gc.enable()
        return False


def max_over_ranks(values, dev, world):
    """Element-wise max of per-rank timings over all ranks (every rank gets
    the result; the job is as slow as its slowest rank)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def rows_per_rank(batch, world):
    """Rows of the global batch each rank decodes: the batch is partitioned
    across the ranks (rows never interact, so no collective is needed on the
    attention path)."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split evenly over {world} ranks")
    return batch // world


def gather_logits(logits, gathered, world):
    """All-gather every rank's last-position logits [rows, vocab] into
    `gathered` [world * rows, vocab] in rank order over NCCL (the end-to-end
    run's one collective)."""
    import torch.distributed as dist
    if world > 1:
        dist.all_gather_into_tensor(gathered, logits)
        return gathered
    return logits


def build_steady_cache(dev, seed, rows=B, tier=True, dtype=None, ctx=None, steps=WS + 1):
    """A layer cache at the workload's context (32k unless --ctx) after
    `steps` decode steps: with the default nine, the ninth (generation step
    8) runs the first eviction and the cache is in its steady state."""
    import torch

    from stickykv_b200 import WindowedCache, WindowedCacheConfig
    from stickykv_b200.hooks import ATTN_IMPLEMENTATION  # noqa: F401

    class MC:
        num_attention_heads, num_key_value_heads, hidden_size, head_dim = HQ, HKV, HQ * D, D

    class RoPE(torch.nn.Module):
        def __init__(self, theta):
            super().__init__()
            self.inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))

        def forward(self, x, pos):
            f = pos[..., None].float() * self.inv.to(x.device)
            emb = torch.cat([f, f], -1)
            return emb.cos().to(x.dtype), emb.sin().to(x.dtype)

    cfg = WindowedCacheConfig(window_size=WS, num_sink_tokens=SINKS, local_window_size=LOCAL,
                              cache_budget=BUDGET, int4_tier=tier)
    dtype = dtype or torch.float16
    ctx = ctx or CTX
    cache = WindowedCache(cfg, ctx, MC(), dtype, RoPE(500000.0), num_layers=1, max_tokens=0)
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(rows, HKV, ctx, D, device=dev, generator=g, dtype=dtype)
    v = torch.randn(rows, HKV, ctx, D, device=dev, generator=g, dtype=dtype)
    cache.update(k, v, 0)
    del k, v
    st = cache._states[0]
    W = math.ceil((ctx - SINKS) / WS)
    st.sides[st.cur].scores[:, :, :W] = torch.rand(rows, HQ, W, device=dev, generator=g)
    st.has_scores, st.W, st.next_window_id = True, W, W
    q = torch.randn(rows, HQ, 1, D, device=dev, generator=g, dtype=dtype)
    for _ in range(steps):
        kn = torch.randn(rows, HKV, 1, D, device=dev, generator=g, dtype=dtype)
        cache.update(kn, kn.clone(), 0)
        cache.decode_attention(0, q, D ** -0.5)
    torch.cuda.synchronize(dev)
    return cache


def algorithmic_bytes(cache):
    """HBM bytes one decode-attention launch must move: every retained token's
    K and V once (fp16 tokens 2*D*2 B; int4 tokens their page share) plus q and
    out.  The window-mass write is not counted."""
    from stickykv_b200 import _lib
    st = cache._states[0]
    n_fp = st.T - st.tier_pages * 8
    per_int4 = _lib.page_bytes(D) / 8
    return st.B * HKV * (n_fp * 2 * D * 2 + st.tier_pages * 8 * per_int4) + st.B * HQ * D * 2 * 2


def evict_algorithmic_bytes(cache):
    """HBM bytes of the eviction the cache's next evicting step runs (with
    the length it will have then): the accumulated scores read and the
    retained ones written, every fp token that stays fp read and written
    (K and V: compaction and re-rotation), the fp windows that may enter the
    tier read (all candidates, an upper bound) and their int4 pages written,
    ids and page tables read and written."""
    from stickykv_b200 import _lib
    st = cache._states[0]
    r = cache.resolved
    n = (WS - cache._generation_step[0] % WS) % WS  # updates before the evicting one
    T = st.T + n + 1                                 # its length after its append
    W = math.ceil((T - 1 - SINKS) / WS)              # windows its scores cover
    plan = _lib.evict_plan(T, W, SINKS, WS, r.top_k_windows, cache.local_windows, cache.tier)
    n_tw_old = st.tier_pages * 8 // WS
    n_cand = plan.evictable_windows - n_tw_old
    fp_kept = plan.seq_len_new - plan.tier_pages_new * 8
    rows = st.B
    kv = rows * HKV * D * 2 * 2                                   # K+V bytes per token, all kv heads
    return (rows * HQ * W * 4 + rows * HQ * plan.retained_windows * 4 + rows * (W + plan.retained_windows) * 8
            + fp_kept * kv * 2 + n_cand * WS * kv + rows * HKV * n_cand * (WS // 8) * _lib.page_bytes(D)
            + 2 * rows * st.page_cap * 4)


class StepGraphs:
    """CUDA graphs of a 16-step cycle (two evictions apart, so the ping-pong
    stores are back where they started): in steady state every step of the
    cycle launches the same kernels with the same lengths, so the graph of
    phase j replays step j of every cycle with no host work but one graph
    launch, and one graph of the whole cycle replays 16 steps at once.
    Capture runs the host code of the steps (advancing its counters by a
    whole number of cycles) without device work; replaying the graphs in
    phase order performs those steps on the device, and replays stay in phase
    with the host's counters modulo the cycle."""

    def __init__(self, step, cycle, stream):
        import torch
        self.graphs = []
        self.cycle = cycle
        self.pos = 0
        for j in range(cycle):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(j)
            self.graphs.append(g)
        self.whole = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.whole, stream=stream):
            for j in range(cycle):
                step(j)

    def replay(self, n):
        while n > 0:
            if self.pos == 0 and n >= self.cycle:
                self.whole.replay()
                n -= self.cycle
                continue
            self.graphs[self.pos].replay()
            self.pos = (self.pos + 1) % self.cycle
            n -= 1

    def finish_cycle(self):
        """Replay up to the end of the current cycle (device and host state
        agree again)."""
        if self.pos:
            self.replay(self.cycle - self.pos)


def run_ours(args, rank, world, dev):
    import numpy as np
    import torch
    import torch.distributed as dist

    rows = args.rows or rows_per_rank(B, world)
    cache = build_steady_cache(dev, seed=1 + rank, rows=rows, tier=not args.no_tier)
    st = cache._states[0]
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    cycle = 2 * WS
    qs = torch.randn(cycle, rows, HQ, 1, D, device=dev, generator=g, dtype=torch.float16)
    ks = torch.randn(cycle, rows, HKV, 1, D, device=dev, generator=g, dtype=torch.float16)
    vs = torch.randn(cycle, rows, HKV, 1, D, device=dev, generator=g, dtype=torch.float16)
    stream = torch.cuda.Stream(dev)
    scale = D ** -0.5
    # below 32k context a step's working set fits in the 126 MB L2: every
    # timed step and decode launch then starts with a 256 MB write that
    # flushes it, timed on its own and subtracted
    flush = CTX < 32768
    fbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush else None

    def step(j):
        if flush:
            fbuf.fill_(j)
        cache.update(ks[j], vs[j], 0)
        return cache.decode_attention(0, qs[j], scale)

    def flush_ms(n):
        """Device time of one flush write, from n of them in one graph."""
        if not flush:
            return 0.0
        gf = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gf, stream=stream):
            for i in range(n):
                fbuf.fill_(i)
        gf.replay()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(5):
            gf.replay()
        f1.record(stream)
        torch.cuda.synchronize(dev)
        return f0.elapsed_time(f1) / (5 * n)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i % cycle)
        # align to the start of a cycle, then one host-driven cycle with
        # events around the evicting updates (and the host time per step)
        while cache._generation_step[0] % cycle:
            step(cache._generation_step[0] % cycle)
        evict_bytes = evict_algorithmic_bytes(cache)
        ev = []
        t_host = time.perf_counter()
        for j in range(cycle):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            gs = cache._generation_step[0]  # update() at generation step gs evicts when gs % WS == 0
            e[0].record(stream)
            cache.update(ks[j], vs[j], 0)
            e[1].record(stream)
            cache.decode_attention(0, qs[j], scale)
            ev.append((e, gs > 0 and gs % WS == 0))
        host_us = (time.perf_counter() - t_host) * 1e6 / cycle
        torch.cuda.synchronize(dev)
        evict_ms = [a[0].elapsed_time(a[1]) for a, is_ev in ev if is_ev]
        # decode launches alone (decode + merge), back to back in one graph: no
        # host gaps, the cache unchanged between calls
        bytes_per_launch = algorithmic_bytes(cache)
        n_dec = 20
        gd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gd, stream=stream):
            for i in range(n_dec):
                if flush:
                    fbuf.fill_(i)
                cache.decode_attention(0, qs[0], scale)
        for _ in range(2):
            gd.replay()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(5):
            gd.replay()
        d1.record(stream)
        torch.cuda.synchronize(dev)
        fl_ms = flush_ms(n_dec)
        attn_ms = d0.elapsed_time(d1) / (5 * n_dec) - fl_ms
        # the timed steps: graph replays (host-launch gaps removed)
        graphs = StepGraphs(step, cycle, stream)
        graphs.replay(2 * cycle)  # the two captured cycles, untimed, on the device
        torch.cuda.synchronize(dev)
        n_evict = sum(1 for i in range(args.steps) if i % WS == 0)  # phases 0 and 8 evict
        sampler = ClockSampler(dev.index if dev.index is not None else 0)
        sampler.start()
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with _no_gc():
            t0.record(stream)
            graphs.replay(args.steps)
            t1.record(stream)
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        clocks = sampler.stop()
        ms = t0.elapsed_time(t1) - args.steps * fl_ms
        graphs.finish_cycle()
        torch.cuda.synchronize(dev)
        del graphs, gd

    # e2e: the same steps through the public API -- WindowedCache driven by
    # DecodeGraphs, which replays a captured graph of each steady-state step
    # (the call a serving loop makes) -- with host buffers inside the timed
    # region.  Each step issues, at its start, one pinned H2D copy of its
    # packed q|k|v on a copy stream into one of two device buffers (after the
    # step that last read that buffer) and, behind it on the same stream, the
    # D2H copy of the previous step's attention output (after that step); its
    # replay waits for its own input copy.  The timed region ends after the
    # last step's output is back.
    from stickykv_b200 import DecodeGraphs
    cstream = torch.cuda.current_stream(dev)
    nq_el, nk_el = rows * HQ * D, rows * HKV * D
    nbuf = cycle
    hin = torch.randn(nbuf, nq_el + 2 * nk_el, generator=torch.Generator().manual_seed(7),
                      dtype=torch.float16).pin_memory()
    hout = torch.empty(nbuf, rows, 1, HQ, D, dtype=torch.float16).pin_memory()
    din = [torch.empty(nq_el + 2 * nk_el, device=dev, dtype=torch.float16) for _ in range(2)]
    dviews = [(x[:nq_el].view(rows, HQ, 1, D), x[nq_el:nq_el + nk_el].view(rows, HKV, 1, D),
               x[nq_el + nk_el:].view(rows, HKV, 1, D)) for x in din]
    outs = {}  # each phase's attention output (the graph's own buffer)

    def graph_step(j):
        dq, dk, dv = dviews[j % 2]  # the period is even: a phase always reads the same buffer
        cache.update(dk, dv, 0)
        outs[j] = cache.decode_attention(0, dq, scale)

    n_pre = 0
    while not DecodeGraphs.ready(cache):  # to a period boundary (untimed)
        graph_step(n_pre % cycle)
        n_pre += 1
    torch.cuda.synchronize(dev)
    dgraphs = DecodeGraphs(cache, graph_step, stream=torch.cuda.Stream(dev), whole_period=False)
    copy_stream = torch.cuda.Stream(dev)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    step_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(cycle)]
    for e in step_done + d2h_done:
        e.record(cstream)
    pending = []  # (phase, buffer, host slot) of the step whose output is not copied back yet

    def copy_back():
        j, k, slot = pending.pop()
        copy_stream.wait_event(step_done[k])
        hout[slot].copy_(outs[j], non_blocking=True)
        d2h_done[j].record(copy_stream)

    def e2e_step(i):
        j = dgraphs.pos
        k = j % 2
        copy_stream.wait_event(step_done[k])  # the step that last read this input buffer
        with torch.cuda.stream(copy_stream):
            din[k].copy_(hin[i % nbuf], non_blocking=True)
            h2d_done[k].record(copy_stream)
            if pending:
                copy_back()
        cstream.wait_event(h2d_done[k])
        cstream.wait_event(d2h_done[j])  # this phase's previous output has been copied back
        dgraphs.replay(1)
        step_done[k].record(cstream)
        pending.append((j, k, i % nbuf))

    def drain():
        if pending:
            with torch.cuda.stream(copy_stream):
                copy_back()
        cstream.wait_stream(copy_stream)

    for i in range(args.warmup):
        e2e_step(i)
    drain()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with _no_gc():  # a full collection in this process takes tens of ms: not in the timed steps
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cstream)
        copy_stream.wait_event(e0)  # the first input copy starts inside the timed region
        for i in range(args.steps):
            e2e_step(i)
        drain()
        e1.record(cstream)
        torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)  # no flush: the copies and host work of a step are part of it
    del dgraphs
    h2d = din[0].numel() * 2
    d2h = hout[0].numel() * 2
    evict_host = float(np.mean(evict_ms)) if evict_ms else 0.0
    ms, e2e_ms, attn_ms, evict_host, host_us = max_over_ranks([ms, e2e_ms, attn_ms, evict_host, host_us], dev,
                                                              world)
    # GPU time of one eviction, from the graph-timed numbers: the steps of a
    # cycle beyond their decode launches, per eviction (WS steps apart)
    evict_avg = max(0.0, (ms / args.steps - attn_ms) * WS)
    del cache
    torch.cuda.empty_cache()
    model = None
    if not args.no_model:
        model = run_e2e(args, rank, world, dev)
    first = None
    if world == 1 and not args.no_evict_first:  # the isolated first eviction, 3 repetitions
        first = run_evict_first(argparse.Namespace(**{**vars(args), "steps": 3}), dev)
    if rank != 0:
        return None
    peak, peak_kind = measured_hbm_peak()
    achieved = bytes_per_launch / (attn_ms * 1e-3) / 1e9
    step_bytes = (bytes_per_launch + evict_bytes / WS) * world
    step_achieved = step_bytes / (ms / args.steps * 1e-3) / 1e9
    # every step: decode with its fused append, then the split merge; an
    # evicting step adds the keys, select and apply kernels (its append rides
    # in the apply)
    gpu_launches = args.steps * 2 + n_evict * 3
    traffic = None
    tp = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tp) and CTX == 32768 and rows == B:  # the captured workload
        try:
            traffic = json.load(open(tp)).get("bytes_per_launch")
        except (OSError, ValueError):
            traffic = None
    line = {
        "metric": METRIC, "value": rows * world * args.steps / (ms * 1e-3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f16 (int4 tier codes, fp32 accumulate)", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "decode-attention + eviction step of one layer, 32k context, "
                               + ("all-fp16 retained cache" if args.no_tier else "int4 tier"),
                   "global_batch": rows * world, "rows_per_gpu": rows, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                   "context": CTX, "cache_budget": BUDGET, "window_size": WS, "sinks": SINKS, "local": LOCAL,
                   "retained_tokens": st.T, "int4_tokens": st.tier_pages * 8,
                   "evictions_in_timed_region": n_evict,
                   "l2": ("a 256 MB write before every graph-timed step and decode launch flushes the "
                          "126 MB L2 (working set below it), its time subtracted; e2e unflushed" if flush else
                          "working set per step > 126 MB L2; no flush"),
                   "launch": "timed steps replay captured CUDA graphs (16-step cycles, single steps "
                             "for the remainder)",
                   "parallelism": f"batch partitioned over {world} GPUs ({rows} rows each), "
                                  "no collective on the attention path"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                     "kernel": "decode attention (split + merge) per layer-step",
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "avg_launch_us": attn_ms * 1e3},
        "step_roofline": {"bound": "hbm", "achieved": step_achieved, "peak": peak * world, "unit": "GB/s",
                          "frac": step_achieved / (peak * world),
                          "algorithmic_bytes_per_step": step_bytes,
                          "note": "decode launch + one eighth of an eviction per step, all GPUs, "
                                  "over ms_per_step"},
        "evict": {"algorithmic_bytes": evict_bytes, "avg_us": evict_avg * 1e3,
                  "achieved_gbs": evict_bytes / (evict_avg * 1e-3) / 1e9 if evict_avg else None,
                  "frac": evict_bytes / (evict_avg * 1e-3) / 1e9 / peak if evict_avg else None,
                  "host_driven_us": evict_host * 1e3,
                  "note": "GPU time per eviction = (ms_per_step - decode launch) x window_size from the graph-timed "
                          "steps (keys + select + apply with the step's append, select overlapped by the apply's moves); "
                          "host_driven_us: events around an evicting update() called from Python"},
        "host_us_per_step": host_us,
        "e2e": {"value": rows * world * args.steps / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": gpu_launches,
        "clocks": clocks,
    }
    if model is not None:
        line["model_e2e"] = model
    if first is not None:
        line["evict_first"] = {k: first[k] for k in ("metric", "value", "unit", "device_us_per_eviction",
                                                    "host_driven_us_per_eviction", "algorithmic_bytes",
                                                    "roofline", "config")}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    return line


# ------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's algorithm restated in numpy (oracle)
# ------------------------------------------------------------------------------------------

def cpu_reference_setup(rows: int):
    """A reference-mode (all fp16) oracle cache for `rows` rows in the same
    32k steady state (the reference has no int4 tier)."""
    import numpy as np

    from oracle import skv_oracle as O
    inv = (1.0 / (500000.0 ** (np.arange(0, D, 2) / D))).astype(np.float32)
    cos, sin = O.rope_tables(inv, CTX + 64)
    r = O.resolve(WS, SINKS, LOCAL, BUDGET, CTX, HKV, D, 2, 0)
    oc = O.OracleCache(r, "f16", cos, sin, tier=False)
    rng = np.random.default_rng(0)
    oc.update(rng.standard_normal((rows, HKV, CTX, D)).astype(np.float32),
              rng.standard_normal((rows, HKV, CTX, D)).astype(np.float32), None)
    W = math.ceil((CTX - SINKS) / WS)
    oc.add_scores(rng.random((rows, HQ, W)).astype(np.float32))
    for _ in range(WS + 1):
        kn = rng.standard_normal((rows, HKV, 1, D)).astype(np.float32)
        oc.update(kn, kn, None)
    return oc, rng


def cpu_step(oc, rng):
    """One reference decode step: append (concatenate), eager attention with
    the window scores of that step, accumulate, evict every 8th step."""
    import numpy as np

    from oracle import skv_oracle as O
    rows = oc.k.shape[0]
    kn = rng.standard_normal((rows, HKV, 1, D)).astype(np.float32)
    scores = None
    if getattr(oc, "_pending", None) is not None:
        scores = oc._pending
    oc.update(kn, kn, scores)
    q = rng.standard_normal((rows, HQ, D)).astype(np.float32)
    _, sc = O.eager_decode_attention(O.round_to(q, "f16"), oc.k, oc.v, D ** -0.5, SINKS, WS, "f16")
    oc._pending = sc


E2E = dict(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192, theta=5e5, vocab=128256,
           batch=32, prompt=8192, decode=256, budget=BUDGET, name="Llama-3.2-1B shape, 8k prompt")
# the 8B-class configuration: 64 rows of 32k-token prompts, 128 greedy steps, budget 0.25
E2E_8B = dict(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=14336, theta=5e5, vocab=128256,
              batch=64, prompt=32768, decode=128, budget=0.25, name="Llama-3.1-8B shape, 32k prompt")


def run_e2e(args, rank, world, dev):
    """End-to-end decode through transformers: a Llama-3.2-1B-shaped decoder
    (random N(0,0.02) weights, bf16) prefills 8192 random tokens per row and
    greedily decodes 256 tokens with the windowed cache (budget 0.40, int4
    tier).  The global batch of 32 rows is split across the ranks.  Decoding
    runs eagerly until the cache reaches its steady state, then the remaining
    steps replay CUDA graphs of the whole forward (DecodeGraphs); decode
    tokens/s = rows x steps / time over those steps (max over ranks).
    At N > 1 the ranks all-gather each step's logits.  Also reported,
    as the reference's perf runner does: time to first token (the prefill
    forward), time per output token and peak device memory; `--e2e-budget`
    sets the cache budget (0.10 / 0.25 / 0.50 in the reference's sweep)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from transformers import LlamaConfig, LlamaForCausalLM

    from stickykv_b200 import DecodeGraphs, WindowedCache, WindowedCacheConfig, install_score_hooks

    c = dict(E2E_8B if args.e2e_8b else E2E)
    if args.e2e_prompt:
        c["prompt"] = args.e2e_prompt
    if args.e2e_decode:
        c["decode"] = args.e2e_decode
    budget = args.e2e_budget or c["budget"]
    rows = args.e2e_rows or rows_per_rank(c["batch"], world)
    cfg = LlamaConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["ffn"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["heads"],
                      num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], rope_theta=c["theta"],
                      max_position_embeddings=131072, tie_word_embeddings=True, initializer_range=0.02)
    torch.manual_seed(1234 + rank)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    if args.e2e_stock:
        return run_stock_e2e(args, rank, world, dev, model, c, rows)
    wcfg = WindowedCacheConfig(window_size=WS, num_sink_tokens=SINKS, local_window_size=LOCAL,
                               cache_budget=budget, int4_tier=True)
    torch.cuda.reset_peak_memory_stats(dev)
    cache = WindowedCache(wcfg, c["prompt"], model.config, torch.bfloat16, model.model.rotary_emb,
                          num_layers=c["layers"], max_tokens=c["decode"])
    handles = install_score_hooks(model, cache, wcfg)
    g = torch.Generator(device=dev).manual_seed(55 + rank)
    ids = torch.randint(0, c["vocab"], (rows, c["prompt"]), device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        p1.record(stream)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        torch.cuda.synchronize(dev)
        sampler = ClockSampler(dev.index if dev.index is not None else 0)
        sampler.start()
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        # every step the ranks all-gather the batch's last-position logits
        # (NCCL over NVLink), the only collective of the run; each rank keeps
        # decoding its own rows from its slice of the gathered logits
        gathered = (torch.empty(world * rows, c["vocab"], dtype=torch.bfloat16, device=dev)
                    if world > 1 else None)
        tok = nxt.clone()

        def decode_step(j=0):
            out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
            logits = gather_logits(out.logits[:, -1].contiguous(), gathered, world)
            tok.copy_(logits[rank * rows:(rank + 1) * rows].argmax(-1, keepdim=True))

        total = c["decode"] - 1
        # eager steps until the cache is in steady state (two evictions behind
        # it, at a period boundary), timed on their own
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        n_eager = 0
        while n_eager < total and not DecodeGraphs.ready(cache):
            decode_step()
            n_eager += 1
        e1.record(stream)
        graphs = None
        if total - n_eager >= 2 * DecodeGraphs.period_of(cache) and not args.e2e_eager:
            graphs = DecodeGraphs(cache, decode_step, stream=stream)
        torch.cuda.synchronize(dev)
        sampler = ClockSampler(dev.index if dev.index is not None else 0)
        sampler.start()
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_timed = total - n_eager
        with _no_gc():
            t0.record(stream)
            if graphs is not None:
                graphs.replay(n_timed)
            else:
                for _ in range(n_timed):
                    decode_step()
            t1.record(stream)
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        clocks = sampler.stop()
        used_graphs = graphs is not None
        del graphs
    handles.remove()
    dec_ms, pre_ms, eager_ms, peak = max_over_ranks(
        [t0.elapsed_time(t1), p0.elapsed_time(p1), e0.elapsed_time(e1), torch.cuda.max_memory_allocated(dev)],
        dev, world)
    if rank != 0:
        return None
    steps = n_timed
    total_rows = rows * world
    return {
        "metric": f"e2e decode tokens/s ({c['name']}, int4 tier)", "unit": "tokens/s",
        "value": total_rows * steps / (dec_ms * 1e-3), "n_gpus": world, "steps": steps,
        "ms_per_step": dec_ms / steps, "higher_is_better": True, "scaling": "strong",
        "dtype": "bf16 (int4 tier codes)", "data": "synthetic: random N(0,0.02) weights, uniform token ids",
        "config": {"workload": f"{c['name']}: decoder with random weights, greedy decode through "
                               "transformers with the windowed cache", "layers": c["layers"], "hidden": c["hidden"],
                   "q_heads": c["heads"], "kv_heads": c["kv_heads"], "head_dim": c["head_dim"],
                   "global_batch": total_rows, "rows_per_gpu": rows, "prompt": c["prompt"],
                   "decode_steps": c["decode"],
                   "cache_budget": budget, "retained_tokens": cache.get_seq_length(0),
                   "parallelism": f"{world} batch shards"},
        "prefill_ms": pre_ms, "ttft_ms": pre_ms, "tpot_ms": dec_ms / steps,
        "eager_steps": n_eager, "eager_tpot_ms": eager_ms / max(1, n_eager),
        "launch": ("timed steps replay CUDA graphs of the whole forward (steady state, after the "
                   f"{n_eager} eager steps that reach it)") if used_graphs else "eager",
        "nccl_ranks": world if world > 1 else None,
        "peak_mem_gib": peak / 2 ** 30, "clocks": clocks,
    }


def run_stock_e2e(args, rank, world, dev, model, c, rows):
    """The same model, rows and prompt through stock transformers: its own
    DynamicCache (every token kept, no eviction) and sdpa attention, decoded
    eagerly (a growing cache has no steady state to replay).  The comparison
    point a user of plain transformers gets: TTFT, TPOT, decode tokens/s and
    peak device memory."""
    import torch
    import torch.distributed as dist
    from transformers import DynamicCache
    model.config._attn_implementation = "sdpa"
    g = torch.Generator(device=dev).manual_seed(55 + rank)
    ids = torch.randint(0, c["vocab"], (rows, c["prompt"]), device=dev, generator=g)
    torch.cuda.reset_peak_memory_stats(dev)
    stream = torch.cuda.current_stream(dev)
    cache = DynamicCache()
    with torch.no_grad():
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        p1.record(stream)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = c["decode"] - 1
        t0.record(stream)
        for _ in range(steps):
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True, logits_to_keep=1)
            nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    dec_ms, pre_ms, peak = max_over_ranks(
        [t0.elapsed_time(t1), p0.elapsed_time(p1), torch.cuda.max_memory_allocated(dev)], dev, world)
    if rank != 0:
        return None
    return {
        "metric": "e2e decode tokens/s, stock transformers (DynamicCache, sdpa, no eviction)", "unit": "tokens/s",
        "value": rows * world * steps / (dec_ms * 1e-3), "n_gpus": world, "steps": steps,
        "ms_per_step": dec_ms / steps, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
        "data": "synthetic: random N(0,0.02) weights, uniform token ids",
        "config": {"workload": f"{c['name']}: decoder with random weights, greedy decode through stock "
                               "transformers",
                   "global_batch": rows * world, "prompt": c["prompt"], "decode_steps": c["decode"],
                   "retained_tokens": cache.get_seq_length(0)},
        "prefill_ms": pre_ms, "ttft_ms": pre_ms, "tpot_ms": dec_ms / steps, "peak_mem_gib": peak / 2 ** 30,
    }


def _all_host_threads():
    """BLAS thread pools sized to every host core (torchrun sets
    OMP_NUM_THREADS=1 for its ranks); returns (context, threads)."""
    n = os.cpu_count() or 1
    try:
        import threadpoolctl
        return threadpoolctl.threadpool_limits(limits=n), n
    except Exception:  # noqa: BLE001
        import contextlib
        return contextlib.nullcontext(), 1


def cpu_baseline(seconds: float = 10.0, rows: int = 1):
    ctx, cores = _all_host_threads()
    with ctx:
        oc, rng = cpu_reference_setup(rows)
        cpu_step(oc, rng)
        n = 0
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds or n < WS:
            cpu_step(oc, rng)
            n += 1
        dt = time.perf_counter() - t0
    return {"value": rows * n / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{rows} of {B} rows, {n} decode steps (incl. {n // WS} evictions), "
                      f"all-fp16 retained cache of {oc.seq_length} tokens (reference has no int4 tier); "
                      f"numpy restatement of the reference eager path (BLAS on {cores} threads)"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    ctx, cores = _all_host_threads()
    with ctx:
        oc, rng = cpu_reference_setup(1)
        for _ in range(args.warmup):
            cpu_step(oc, rng)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cpu_step(oc, rng)
        dt = time.perf_counter() - t0
    value = 1 * args.steps / dt
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": "decode-attention + eviction step of one layer, 32k context",
                   "global_batch": B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context": CTX,
                   "sample_rows": 1, "note": "reference CPU path (numpy restatement), all-fp16 tiers"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"1 of {B} rows per step, {args.steps} timed steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_tile_profile(dev):
    """Two decode-attention calls on the steady cache cut to its int4 part (all
    tier pages, then half of them) inside a profiler range: the difference of
    their counters is the cost of the int4 tiles alone, fixed per-block costs
    cancelling.  Run under `ncu --profile-from-start off`."""
    import ctypes as C

    import torch

    from stickykv_b200 import _lib
    cache = build_steady_cache(dev, 1, tier=True)
    st = cache._states[0]
    d = cache._desc(st, st.sides[st.cur])
    L = _lib.lib()
    q = torch.randn(B, HQ, D, device=dev, dtype=torch.float16)
    out = torch.empty_like(q)
    sc = torch.zeros(B, HQ, st.scores_cap, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    nb = L.skv_decode_workspace_size(C.byref(d), st.T)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    cases = [(SINKS + st.tier_pages * 8, st.tier_pages), (SINKS + (st.tier_pages // 2) * 8, st.tier_pages // 2)]

    def call(T, tp):
        _lib.check(L.skv_decode_attention(C.byref(d), T, tp, q.data_ptr(), q.stride(0), q.stride(1),
                                          out.data_ptr(), out.stride(0), out.stride(1), C.c_float(D ** -0.5),
                                          sc.data_ptr(), st.scores_cap, ws.data_ptr(), nb, s), "decode")

    for T, tp in cases:
        for _ in range(3):
            call(T, tp)
    torch.cuda.synchronize(dev)
    torch.cuda.profiler.start()
    for T, tp in cases:
        call(T, tp)
    torch.cuda.synchronize(dev)
    torch.cuda.profiler.stop()
    return {"tile_profile": [{"seq_len": T, "tier_pages": tp, "int4_tiles": B * HKV * (tp // 2)} for T, tp in cases]}


def first_evict_bytes(cache):
    """HBM bytes of the cache's first eviction, which the next update()
    runs: the accumulated scores read and the retained ones written, ids read
    and written, the fp tokens that stay fp (sinks and local windows) read and
    written, the kept evictable windows' K/V read and their int4 pages
    written, the page table written."""
    from stickykv_b200 import _lib
    st, r = cache._states[0], cache.resolved
    T = st.T + 1
    W = math.ceil((T - 1 - SINKS) / WS)
    plan = _lib.evict_plan(T, W, SINKS, WS, r.top_k_windows, cache.local_windows, cache.tier)
    fp_kept = plan.seq_len_new - plan.tier_pages_new * 8
    ent = plan.kept_evictable
    rows = st.B
    kv = rows * HKV * D * 2 * 2
    return (rows * HQ * W * 4 + rows * HQ * plan.retained_windows * 4 + rows * (W + plan.retained_windows) * 8
            + fp_kept * kv * 2 + ent * WS * kv + rows * HKV * ent * (WS // 8) * _lib.page_bytes(D)
            + rows * st.page_cap * 4)


def run_evict_first(args, dev):
    """The isolated evict + re-rotate step: the first eviction of a bf16
    cache of 16384 tokens (16 rows, 32/8 heads, head_dim 64, budget 0.40,
    int4 tier): the 613 kept evictable windows of every row (4904 tokens)
    are quantised into the tier, the sinks and local windows re-rotated into
    the compacted store.  Each repetition builds a fresh cache (eight decode
    steps after the prompt) and times its evicting update() with CUDA
    events: the head-mean keys, the radix top-k select and the apply (which
    also moves the step's one token into the compacted store) -- once as
    called from Python on an idle stream
    (host-driven) and once enqueued behind a sleep kernel (device time, the
    line's value).  The working set (the 268 MB store) exceeds the L2."""
    import statistics

    import torch
    peak, peak_kind = measured_hbm_peak()
    ctx, reps = 16384, max(3, min(args.steps, 10))
    us, host_us, dev_us, nbytes = [], [], [], 0
    for rep in range(2 * reps):
        # even repetitions: the update() called from Python with the stream
        # idle, the GPU waiting for each launch; odd ones: the same call
        # enqueued behind a bounded sleep kernel, so its kernels run back to
        # back and the events measure device time alone
        behind = rep % 2 == 1
        cache = build_steady_cache(dev, seed=1 + rep // 2, rows=B, tier=True, dtype=torch.bfloat16, ctx=ctx,
                                   steps=WS)
        st = cache._states[0]
        assert cache._generation_step[0] % WS == 0 and st.tier_pages == 0
        nbytes = first_evict_bytes(cache)
        kn = torch.randn(B, HKV, 1, D, device=dev, dtype=torch.bfloat16)
        # the eviction's workspace allocated before the timed call (an
        # allocation inside it would stall the launches behind it)
        import ctypes as C

        from stickykv_b200 import _lib
        cache._ensure_rope(st.T + 4096, D, dev)  # positions for the timed step, built beforehand
        W_ev = math.ceil((st.T - SINKS) / WS) + 1
        cache._workspace(_lib.lib().skv_evict_workspace_size(C.byref(cache._desc(st, st.sides[st.cur])), W_ev), dev)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        kv2 = kn.clone()
        if behind:
            torch.cuda._sleep(2_000_000)  # about 1 ms at 1.9 GHz, longer than the host's enqueue
        e0.record(s)
        th = time.perf_counter()
        cache.update(kn, kv2, 0)
        h = (time.perf_counter() - th) * 1e6
        e1.record(s)
        torch.cuda.synchronize(dev)
        assert st.tier_pages * 8 == cache.resolved.top_k_windows * WS  # every kept window demoted
        if behind:
            dev_us.append(e0.elapsed_time(e1) * 1e3)
        else:
            us.append(e0.elapsed_time(e1) * 1e3)
            host_us.append(h)
        del cache
    med, dmed = statistics.median(us), statistics.median(dev_us)
    achieved = nbytes / (dmed * 1e-6) / 1e9
    return {
        "metric": "first eviction, HBM GB/s (16k ctx, bf16, int4 demotion)", "value": achieved, "unit": "GB/s",
        "n_gpus": 1, "steps": reps, "higher_is_better": True, "device_us_per_eviction": dmed,
        "device_us_all": [round(x, 1) for x in dev_us],
        "host_driven_us_per_eviction": med, "host_driven_us_all": [round(x, 1) for x in us],
        "host_us_all": [round(x, 1) for x in host_us],
        "host_driven_gbs": nbytes / (med * 1e-6) / 1e9,
        "algorithmic_bytes": nbytes,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind},
        "dtype": "bf16 (int4 tier codes)", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "first eviction + re-rotation + int4 demotion of one layer", "global_batch": B,
                   "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context": ctx, "cache_budget": BUDGET,
                   "window_size": WS, "sinks": SINKS, "local": LOCAL,
                   "includes": "the evicting step's one-token append (inside the apply)"},
    }


def run_prefill(args, dev):
    """Prompt prefill through the C-ABI (`skv_prefill_attention`: causal
    attention, log-sum-exp and the prompt's window scores) on synthetic bf16
    q/k/v, timed with CUDA events; TFLOP/s counts three causal GEMMs (QK and
    PV of the forward, QK again for the column mass)."""
    import ctypes as C

    import torch

    from stickykv_b200 import _lib
    L = _lib.lib()
    Bp, T, Dp = args.prefill_batch, args.prefill_len, args.prefill_head_dim
    g = torch.Generator(device=dev).manual_seed(3)
    dt = torch.bfloat16
    q = torch.randn(Bp, HQ, T, Dp, device=dev, dtype=dt, generator=g)
    k = torch.randn(Bp, HKV, T, Dp, device=dev, dtype=dt, generator=g)
    v = torch.randn(Bp, HKV, T, Dp, device=dev, dtype=dt, generator=g)
    out = torch.empty(Bp, T, HQ, Dp, device=dev, dtype=dt)
    W = -(-(T - SINKS) // WS)
    sc = torch.zeros(Bp, HQ, W + 8, device=dev)
    d = _lib.LayerDesc()
    d.batch, d.num_kv_heads, d.num_q_heads, d.head_dim = Bp, HKV, HQ, Dp
    d.kv_dtype, d.window_size, d.num_sink, d.sink_pad = 2, WS, SINKS, 8
    d.fp_capacity, d.k_fp, d.v_fp = T, k.data_ptr(), v.data_ptr()
    nb = L.skv_prefill_workspace_size(C.byref(d), T)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream

    def call():
        _lib.check(L.skv_prefill_attention(C.byref(d), T, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           out.data_ptr(), C.c_float(Dp ** -0.5), sc.data_ptr(), sc.shape[-1],
                                           ws.data_ptr(), nb, s), "prefill")

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    flop = 3 * 2 * Bp * HQ * T * T * Dp / 2
    return {"metric": "prefill TFLOP/s (causal attention + column-mass scoring, 3 causal GEMMs)",
            "value": flop / ms / 1e9, "unit": "TFLOP/s", "ms_per_call": ms, "steps": args.steps,
            "warmup": args.warmup, "dtype": "bf16", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "prompt prefill", "batch": Bp, "q_heads": HQ, "kv_heads": HKV,
                       "head_dim": Dp, "prompt": T}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e", action="store_true",
                    help="end-to-end decode through a Llama-3.2-1B-shaped transformers model instead")
    ap.add_argument("--e2e-prompt", type=int, default=0)
    ap.add_argument("--e2e-decode", type=int, default=0)
    ap.add_argument("--e2e-budget", type=float, default=0.0)
    ap.add_argument("--e2e-stock", action="store_true",
                    help="with --e2e: the same model through stock transformers (DynamicCache, sdpa, no eviction)")
    ap.add_argument("--e2e-8b", action="store_true",
                    help="with --e2e: the Llama-3.1-8B-shaped configuration (64 rows, 32k prompt, 128 steps, "
                         "budget 0.25) instead of the Llama-3.2-1B one")
    ap.add_argument("--e2e-rows", type=int, default=0,
                    help="with --e2e: rows per GPU (default: the configuration's batch split over the GPUs)")
    ap.add_argument("--e2e-eager", action="store_true",
                    help="decode the model run eagerly (no CUDA-graph replay of its steps)")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU of the attention workload (default: the 16 rows partitioned over the GPUs)")
    ap.add_argument("--ctx", type=int, default=0,
                    help="context length of the decode-attention workload (default 32768; the parity tests "
                         "cover 4096/8192/16384/32768)")
    ap.add_argument("--no-model", action="store_true",
                    help="leave the Llama-3.2-1B-shaped model run out of the default line")
    ap.add_argument("--no-evict-first", action="store_true",
                    help="leave the isolated first eviction (16k bf16 cache) out of the default line")
    ap.add_argument("--no-tier", action="store_true",
                    help="keep every retained token in fp16 (reference mode) instead of the int4 tier")
    ap.add_argument("--tile-profile", action="store_true",
                    help="two decode calls on the int4 part of the cache in a profiler range (for ncu)")
    ap.add_argument("--prefill", action="store_true", help="time the prompt prefill kernels instead")
    ap.add_argument("--evict-first", action="store_true",
                    help="time the first eviction of a bf16 16k-token cache (16 rows) instead")
    ap.add_argument("--prefill-batch", type=int, default=4)
    ap.add_argument("--prefill-len", type=int, default=8192)
    ap.add_argument("--prefill-head-dim", type=int, default=64)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ctx:  # the decode-attention workload at another context length
        globals()["CTX"] = args.ctx
        globals()["METRIC"] = METRIC.replace("32k ctx", f"{args.ctx // 1024}k ctx")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    try:
        if args.tile_profile:
            line = run_tile_profile(dev)
        elif args.prefill:
            line = run_prefill(args, dev)
        elif args.evict_first:
            line = run_evict_first(args, dev)
        else:
            line = run_e2e(args, rank, world, dev) if args.e2e else run_ours(args, rank, world, dev)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
