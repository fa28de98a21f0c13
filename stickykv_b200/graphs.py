"""CUDA-graph replay of steady-state decode steps.

After its second eviction a windowed cache is in a steady state: every
eviction keeps the same number of tokens and the stores stop growing, so the
lengths, positions, buffer addresses and launch shapes of a decode step
repeat with a period of two evictions (``2 * window_size`` steps: the
ping-pong stores alternate).  ``DecodeGraphs`` captures one CUDA graph per
step of such a period (and, optionally, one of the whole period) from a
callable that runs one decode step on static buffers, then replays them in
phase order.  The host work of a step (the model's Python, the cache's
bookkeeping, the native calls) then runs once per phase, at capture, instead
of once per step; the device work of every replayed step is the full step.

Capture runs the step callable without device work, which advances the
cache's host counters: by one period for the per-step graphs and one more
for the whole-period graph.  Replays then perform exactly those steps on the
device first.  Host state and device state agree whenever the number of
replayed steps is a multiple of the period past the captured ones
(``finish_period``), which is when eager calls may resume.

Preconditions (checked by ``ready``): every layer has evicted at least twice,
all layers are at the same generation step, a multiple of the period, and no
telemetry is recorded (it would be recorded once, at capture).
"""

from __future__ import annotations

from typing import Callable, List, Optional

import torch


class DecodeGraphs:
    """Per-phase CUDA graphs of a steady-state decode step.

    ``step(j)`` must run one decode step (every layer's ``update`` and
    attention) reading its inputs from and writing its outputs to buffers
    that stay in place; ``j`` is the phase, 0 .. period - 1."""

    def __init__(self, cache, step: Callable[[int], None], stream: Optional[torch.cuda.Stream] = None,
                 whole_period: bool = True) -> None:
        if not self.ready(cache):
            raise RuntimeError("DecodeGraphs needs a cache in steady state at a period boundary "
                               "(see DecodeGraphs.ready)")
        if stream is not None and stream.cuda_stream == 0:
            stream = None  # capture needs a side stream; torch picks one for None
        self.period = self.period_of(cache)
        self.pos = 0
        self.graphs: List[torch.cuda.CUDAGraph] = []
        for j in range(self.period):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(j)
            self.graphs.append(g)
        self.whole: Optional[torch.cuda.CUDAGraph] = None
        if whole_period:
            self.whole = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.whole, stream=stream):
                for j in range(self.period):
                    step(j)
        # steps the host has accounted for that the device has not run yet
        self.behind = self.period * (2 if whole_period else 1)

    @staticmethod
    def period_of(cache) -> int:
        return 2 * cache.resolved.window_size

    @staticmethod
    def ready(cache) -> bool:
        states = [st for st in cache._states if st.allocated]
        if not states or any(st.evictions < 2 or st.pending is not None for st in states):
            return False
        steps = set(cache._generation_step)
        if len(steps) != 1 or next(iter(steps)) % DecodeGraphs.period_of(cache):
            return False
        return not bool(getattr(cache.telemetry, "enabled", False))

    def replay(self, n: int) -> None:
        """Run the next ``n`` steps on the device, in phase order."""
        while n > 0:
            if self.whole is not None and self.pos == 0 and n >= self.period:
                self.whole.replay()
                done = self.period
            else:
                self.graphs[self.pos].replay()
                self.pos = (self.pos + 1) % self.period
                done = 1
            n -= done
            self.behind = max(0, self.behind - done)

    @property
    def in_step(self) -> bool:
        """Host and device agree: every captured step has run and the replays
        stopped at a period boundary (eager calls may resume)."""
        return self.behind == 0 and self.pos == 0

    def finish_period(self) -> int:
        """Replay to the next period boundary; returns the steps replayed."""
        n = (self.period - self.pos) % self.period
        self.replay(n)
        return n
