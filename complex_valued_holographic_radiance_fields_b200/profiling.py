"""Per-operator device timing with CUDA events on the launching (current) stream.

Disabled by default (zero cost).  ``with op_timing() as t: ...`` records a start and
end event around every instrumented operator call; ``t.summary()`` synchronises
and returns {name: (calls, mean_ms)}.
"""
import contextlib

import torch

_active = None


class OpTimes:
    def __init__(self):
        self.events = {}

    @contextlib.contextmanager
    def record(self, name):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self.events.setdefault(name, []).append((s, e))

    def summary(self):
        torch.cuda.synchronize()
        return {k: (len(v), sum(s.elapsed_time(e) for s, e in v) / len(v)) for k, v in self.events.items()}


def timed(name):
    return _active.record(name) if _active is not None else contextlib.nullcontext()


@contextlib.contextmanager
def op_timing():
    global _active
    prev, _active = _active, OpTimes()
    try:
        yield _active
    finally:
        _active = prev
