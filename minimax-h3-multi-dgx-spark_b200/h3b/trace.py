"""Per-op CUDA-event spans and a kernel-launch counter (off unless a Trace is active).

While a Trace is active, every h3b op records a CUDA event pair on the stream
it launches on, tagged with the op name and its algorithmic work (bytes or
ops), and counts the kernels it launched.  bench.py uses this to report each
kernel's achieved throughput from the timed region itself.
"""
import contextlib

import torch

_active = None


class Trace:
    def __init__(self):
        self.spans = []  # (name, ev0, ev1, work)
        self.launches = 0

    def __enter__(self):
        global _active
        self._prev, _active = _active, self
        return self

    def __exit__(self, *exc):
        global _active
        _active = self._prev
        return False

    def summary(self, steps=1):
        """{name: {"ms": total ms per step, "calls": per step, "work": per step}} (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for name, e0, e1, work in self.spans:
            d = out.setdefault(name, {"ms": 0.0, "calls": 0, "work": 0.0})
            d["ms"] += e0.elapsed_time(e1)
            d["calls"] += 1
            d["work"] += work
        for d in out.values():
            d["ms"] /= steps
            d["calls"] /= steps
            d["work"] /= steps
        return out


@contextlib.contextmanager
def span(name, work=0.0, launches=1):
    t = _active
    if t is None:
        yield
        return
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    yield
    e1.record()
    t.spans.append((name, e0, e1, float(work)))
    t.launches += launches


def count(launches=1):
    if _active is not None:
        _active.launches += launches
