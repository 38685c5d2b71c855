"""Hidden-state tracer: env-gated probes of intermediate activations (debugging numerics).

Counterpart of the reference's hidden-state log (src/official/llama/vm_c_hidden_log.cpp:71-103,
``hidden_log_register`` / ``hidden_log_dump_all``) and its logits log
(src/official/llama/llama-context.cpp:1635-1641). The environment interface is the reference's:

  VMC_LOG_HIDDEN=1         enable the probes (the runner then runs steps eagerly: a CUDA graph
                           replay has no host code between kernels to take the samples);
  VMC_LOG_HIDDEN_EVERY=N   0 or unset: log each (probe name, shape) the first time it is seen in the
                           process; N >= 1: every N-th time;
  VMC_LOG_LOGITS=1         also log the top-5 (token, logit) pairs of every sampled row.

A probe copies the first 8 values of the tensor on the device (no synchronisation); ``flush`` at the
end of a step reads every sample with one device-to-host copy and logs one line per probe.
"""
from __future__ import annotations

import os
from typing import Callable, Optional

import torch

from .logging import get_logger

log = get_logger("trace")


class HiddenTracer:
    def __init__(self, every: int = 0, logits: bool = False, sink: Optional[Callable[[str], None]] = None):
        self.every = max(0, int(every))
        self.logits = logits
        self.sink = sink or log.info
        self._count: dict[tuple, int] = {}
        self._pending: list[tuple[str, tuple, torch.Tensor]] = []
        self.step = 0

    @staticmethod
    def from_env() -> Optional["HiddenTracer"]:
        hidden = os.environ.get("VMC_LOG_HIDDEN", "") == "1"
        logits = os.environ.get("VMC_LOG_LOGITS", "") == "1"
        if not (hidden or logits):
            return None
        every = int(os.environ.get("VMC_LOG_HIDDEN_EVERY", "0") or 0)
        t = HiddenTracer(every=every, logits=logits)
        t.hidden = hidden
        return t

    hidden = True

    def _take(self, key: tuple) -> bool:
        n = self._count.get(key, 0) + 1
        self._count[key] = n
        return n == 1 if self.every == 0 else (n - 1) % self.every == 0

    def probe(self, name: str, t: torch.Tensor) -> None:
        """Sample the first 8 values of `t` (row-major) if this (name, shape) is due."""
        if not self.hidden:
            return
        shape = tuple(t.shape)
        if not self._take((name, shape)):
            return
        self._pending.append((name, shape, t.reshape(-1)[:8].float().clone()))

    def probe_logits(self, logits: torch.Tensor, rows: int) -> None:
        if not self.logits or rows <= 0:
            return
        v, i = torch.topk(logits[:rows].float(), k=min(5, logits.shape[-1]), dim=-1)
        self._pending.append(("logits_top5", (rows, logits.shape[-1]), torch.stack([i.float(), v], -1)))

    def flush(self) -> list[str]:
        """Log (and return) the lines of the samples taken since the last flush."""
        lines = []
        if self._pending:
            host = [p[2].cpu() for p in self._pending]  # one synchronisation for the whole step
            for (name, shape, _), h in zip(self._pending, host):
                if name == "logits_top5":
                    rows = ["[" + ", ".join(f"{int(tok)}:{val:.4f}" for tok, val in r.tolist()) + "]" for r in h]
                    lines.append(f"step {self.step} {name} rows={shape[0]} " + " ".join(rows))
                else:
                    vals = ", ".join(f"{x:.6g}" for x in h.tolist())
                    lines.append(f"step {self.step} hidden {name} shape={list(shape)} first8=[{vals}]")
            self._pending.clear()
            for ln in lines:
                self.sink(ln)
        self.step += 1
        return lines
