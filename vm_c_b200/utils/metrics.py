"""Engine metrics: per-step throughput, TTFT / ITL percentiles, prefix-cache and preemption counters.

The reference logs phase / tokens / requests / ms per forward (src/core/engine.cpp:1267-1274) and
keeps PrefixCacheStats (include/vm_c/core/scheduler.hpp:57-62) without exporting them; here the
counters are aggregated and exported (Prometheus text format on the server's /metrics route).
"""
from __future__ import annotations

import math
import threading
from collections import deque
from dataclasses import dataclass, field

# Latency samples kept for the percentiles: the most recent ones only, so a server that runs for
# days holds a bounded history (the serving bench's whole run fits in these windows).
TTFT_WINDOW = 1 << 16
ITL_WINDOW = 1 << 20


def percentile(xs, p: float) -> float:
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * p / 100.0
    f, c = math.floor(k), math.ceil(k)
    return s[int(k)] if f == c else s[f] + (s[c] - s[f]) * (k - f)


@dataclass
class EngineMetrics:
    steps: int = 0
    tokens_scheduled: int = 0
    tokens_generated: int = 0
    decode_tokens: int = 0
    cached_prompt_tokens: int = 0
    preemptions: int = 0
    finished: int = 0
    step_time_s: float = 0.0
    ttft_s: deque = field(default_factory=lambda: deque(maxlen=TTFT_WINDOW))
    itl_s: deque = field(default_factory=lambda: deque(maxlen=ITL_WINDOW))
    _lock: threading.Lock = field(default_factory=threading.Lock, repr=False)

    def record_step(self, T: int, S: int, nd: int, dt: float, cached: int) -> None:
        with self._lock:
            self.steps += 1
            self.tokens_scheduled += T
            self.tokens_generated += S
            self.decode_tokens += nd
            self.cached_prompt_tokens += cached
            self.step_time_s += dt

    def record_finish(self, req) -> None:
        with self._lock:
            self.finished += 1
            if req.token_times:
                self.ttft_s.append(req.token_times[0] - req.arrival_time)
                t = req.token_times
                self.itl_s.extend(b - a for a, b in zip(t, t[1:]))

    def summary(self) -> dict:
        with self._lock:
            return {
                "steps": self.steps,
                "tokens_scheduled": self.tokens_scheduled,
                "tokens_generated": self.tokens_generated,
                "preemptions": self.preemptions,
                "finished": self.finished,
                "p50_ttft_ms": percentile(self.ttft_s, 50) * 1e3,
                "p50_itl_ms": percentile(self.itl_s, 50) * 1e3,
                "p99_itl_ms": percentile(self.itl_s, 99) * 1e3,
            }

    def prometheus(self, prefix: str = "vmc") -> str:
        s = self.summary()
        lines = []
        for k, v in s.items():
            if isinstance(v, float) and math.isnan(v):
                continue
            lines.append(f"# TYPE {prefix}_{k} gauge")
            lines.append(f"{prefix}_{k} {v}")
        return "\n".join(lines) + "\n"
