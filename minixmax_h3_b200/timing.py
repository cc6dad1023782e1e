"""CUDA-event spans around named phases of a step (off by default).

``TIMER.span(name, flops, tag)`` brackets the launches made inside it with two
events on the current stream; when the timer is disabled it costs nothing and
records nothing.  The benchmark enables it for its timed steps to time the
dominant kernels live (attention, the NVFP4 GEMMs) and to break a sharded
step into phases per rank (norm/quant, GEMMs, the exchange barriers, RoPE,
attention).
"""
from __future__ import annotations

from contextlib import contextmanager
from typing import Iterator, Optional

import torch


class PhaseTimer:
    def __init__(self) -> None:
        self.enabled = False
        self._spans: list[tuple[str, torch.cuda.Event, torch.cuda.Event, float, Optional[tuple]]] = []

    @contextmanager
    def span(self, name: str, flops: float = 0.0, tag: Optional[tuple] = None) -> Iterator[None]:
        if not self.enabled:
            yield
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            self._spans.append((name, a, b, flops, tag))

    def drain(self) -> list[tuple[str, float, float, Optional[tuple]]]:
        """[(name, milliseconds, flops, tag)] of the recorded spans in launch
        order; synchronises the device and clears the record."""
        torch.cuda.synchronize()
        out = [(n, a.elapsed_time(b), f, t) for n, a, b, f, t in self._spans]
        self._spans.clear()
        return out


TIMER = PhaseTimer()
