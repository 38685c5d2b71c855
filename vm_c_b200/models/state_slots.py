"""Per-request recurrent-state slots for hybrid (gated delta-net) models.

A GDN layer keeps, per running request, a conv history and a delta-rule state in slot-indexed pools
(the `slot` / `has_state` arguments of csrc/kernels/gdn.cu). The reference keeps them in llama's
recurrent memory, one cell per sequence (src/official/llama/models/qwen35moe.cpp:444-456,
get_r_l / get_s_l / build_rs). Here a slot is taken when a request is first scheduled, kept across
its prefill chunks and decode steps, and returned when it finishes or is preempted; a request whose
computed-token count is zero (new, or recomputed after preemption) starts from a zero state, so a
slot never needs clearing. The pool is sized by the scheduler's max_num_seqs.
"""
from __future__ import annotations

import numpy as np


class StateSlots:
    def __init__(self, num_slots: int):
        if num_slots <= 0:
            raise ValueError("num_slots must be positive")
        self.num_slots = num_slots
        self._free = list(range(num_slots - 1, -1, -1))
        self._of: dict[int, int] = {}

    @property
    def num_free(self) -> int:
        return len(self._free)

    def slot(self, req: int) -> int:
        return self._of[req]

    def release(self, req: int) -> None:
        """Return a finished or preempted request's slot (no-op for a request without one)."""
        s = self._of.pop(req, None)
        if s is not None:
            self._free.append(s)

    def step(self, reqs: list[int], num_computed: list[int]) -> tuple[np.ndarray, np.ndarray]:
        """Slots and has_state flags (int32) of one step's requests, in batch order. A request seen
        for the first time takes a free slot; has_state is 0 when it has no computed tokens yet."""
        slots = np.empty(len(reqs), np.int32)
        has = np.empty(len(reqs), np.int32)
        for i, (r, n) in enumerate(zip(reqs, num_computed)):
            s = self._of.get(r)
            if s is None:
                if not self._free:
                    raise RuntimeError("no free recurrent-state slot (more running requests than max_num_seqs)")
                s = self._free.pop()
                self._of[r] = s
            slots[i] = s
            has[i] = 1 if n > 0 else 0
        return slots, has
