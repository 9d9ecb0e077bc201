"""Opt-in CUDA phase timing for the quantized DiT path.

Mirrors the plugin's phase profiler (comfyui_turing_utils/profiling.py:28-95):
off by default (no events, no synchronisation); with
COMFYUI_TURING_UTILS_PROFILE_CALLS=N it records a CUDA event pair around
each phase of the first N attention calls (here: DiT block forwards), then
synchronises once, logs per-phase totals, averages and shares as one
"[Turing profile]" report and switches itself off.  While enabled each phase
is also an NVTX range, so an Nsight timeline shows the same names.
"""
from __future__ import annotations

import contextlib
import logging
import os
from collections import Counter
from collections.abc import Callable

import torch

LOG = logging.getLogger("comfyui-turing-utils")


def _profile_call_limit() -> int:
    value = os.environ.get("COMFYUI_TURING_UTILS_PROFILE_CALLS", "0").strip()
    try:
        return max(int(value), 0)
    except ValueError:
        LOG.warning("Ignoring invalid COMFYUI_TURING_UTILS_PROFILE_CALLS=%r; expected a "
                    "non-negative integer", value)
        return 0


class CudaPhaseProfiler:
    """Asynchronous event pairs per phase over one bounded window of calls."""

    def __init__(self, call_limit: int, event_factory: Callable | None = None,
                 nvtx: bool = True):
        self.call_limit = int(call_limit)
        self.calls = 0
        self.records: list[tuple[str, object, object]] = []
        self.shapes: Counter = Counter()
        self.reported = False
        self.last_report: dict[str, tuple[int, float]] = {}
        self._event = event_factory or (lambda: torch.cuda.Event(enable_timing=True))
        self._nvtx = nvtx

    @property
    def enabled(self) -> bool:
        return self.call_limit > 0 and not self.reported

    @contextlib.contextmanager
    def phase(self, name: str):
        """Times the enclosed launches as phase `name` (a no-op when off)."""
        if not self.enabled:
            yield
            return
        start, end = self._event(), self._event()
        if self._nvtx:
            torch.cuda.nvtx.range_push(name)
        start.record()
        try:
            yield
        finally:
            end.record()
            if self._nvtx:
                torch.cuda.nvtx.range_pop()
            self.records.append((str(name), start, end))

    def call(self, phase: str, function: Callable, /, *args, **kwargs):
        """function(*args, **kwargs) timed as `phase` (the plugin's form)."""
        with self.phase(phase):
            return function(*args, **kwargs)

    def complete_attention(self, query_or_shape) -> None:
        """Closes one call of the window; after `call_limit` calls, reports."""
        if not self.enabled:
            return
        self.calls += 1
        shape = (tuple(query_or_shape.shape) if isinstance(query_or_shape, torch.Tensor)
                 else tuple(query_or_shape))
        self.shapes[str(shape)] += 1
        if self.calls < self.call_limit:
            return
        self.reported = True
        if not self.records:
            return
        self.records[-1][2].synchronize()
        totals: Counter = Counter()
        counts: Counter = Counter()
        for name, start, end in self.records:
            totals[name] += start.elapsed_time(end)
            counts[name] += 1
        total = sum(totals.values())
        LOG.warning("[Turing profile] attention_calls=%d recorded_cuda=%.3f ms shapes=[%s]",
                    self.calls, total,
                    ",".join(f"{s}:{c}" for s, c in sorted(self.shapes.items())))
        for name, elapsed in totals.most_common():
            LOG.warning("  %-32s calls=%4d total=%10.3f ms avg=%8.3f ms %6.2f%%", name,
                        counts[name], elapsed, elapsed / counts[name],
                        elapsed * 100.0 / total if total else 0.0)
        self.last_report = {name: (counts[name], totals[name]) for name in totals}
        self.records.clear()


CUDA_PHASE_PROFILER = CudaPhaseProfiler(_profile_call_limit())
__all__ = ["CUDA_PHASE_PROFILER", "CudaPhaseProfiler"]
