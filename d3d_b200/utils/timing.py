"""Host and device timers for the decode loop.

``StepProfiler`` accumulates host wall time per named phase and, for device
work, CUDA-event pairs recorded on the stream that ran it; ``summary()``
resolves the events (one synchronize) and reports milliseconds per phase.
Device numbers are what the GPU spent between the two events on that stream.

With ``D3D_NVTX=1`` every phase is also an NVTX range (``torch.cuda.nvtx``),
so external timeline tools see the coordinator's phases, enabled or not.
"""
from __future__ import annotations

import os
import time
from collections import defaultdict
from contextlib import contextmanager
from typing import Dict, List, Tuple


class StepProfiler:
    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self.host: Dict[str, float] = defaultdict(float)
        self.count: Dict[str, int] = defaultdict(int)
        self.dev: Dict[str, List[Tuple[object, object]]] = defaultdict(list)

    _nvtx = os.environ.get("D3D_NVTX") == "1"

    @contextmanager
    def phase(self, name: str):
        if self._nvtx:
            import torch
            torch.cuda.nvtx.range_push(name)
        try:
            if not self.enabled:
                yield
                return
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self.host[name] += time.perf_counter() - t0
                self.count[name] += 1
        finally:
            if self._nvtx:
                import torch
                torch.cuda.nvtx.range_pop()

    def dev_begin(self, name: str, stream):
        if not self.enabled:
            return None
        import torch
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        return (name, e0, stream)

    def dev_end(self, tok) -> None:
        if tok is None:
            return
        import torch
        name, e0, stream = tok
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        self.dev[name].append((e0, e1))

    def summary(self) -> dict:
        out = {"host_ms": {k: round(v * 1e3, 3) for k, v in self.host.items()},
               "calls": dict(self.count)}
        dev = {}
        for k, pairs in self.dev.items():
            tot = 0.0
            for e0, e1 in pairs:
                e1.synchronize()
                tot += e0.elapsed_time(e1)
            dev[k] = {"ms": round(tot, 3), "n": len(pairs), "ms_each": round(tot / max(1, len(pairs)), 4)}
        out["device"] = dev
        return out

    def reset(self):
        self.host.clear()
        self.count.clear()
        self.dev.clear()


NULL = StepProfiler(False)
