"""Recurrent-state slot bookkeeping for hybrid models (host only)."""
import numpy as np
import pytest

from vm_c_b200.models.state_slots import StateSlots


def test_slots_follow_requests():
    ss = StateSlots(3)
    s, h = ss.step([10, 11], [0, 0])                 # two new prompts
    assert len(set(s.tolist())) == 2 and h.tolist() == [0, 0]
    s2, h2 = ss.step([11, 10, 12], [16, 32, 0])      # next chunk / decode keep their slots
    assert s2[0] == s[1] and s2[1] == s[0] and h2.tolist() == [1, 1, 0]
    with pytest.raises(RuntimeError):
        ss.step([13], [0])                           # pool exhausted
    ss.release(10)                                   # finished
    s3, h3 = ss.step([13], [0])
    assert s3[0] == s[0] and h3[0] == 0              # reused, starts from a zero state
    ss.release(11)                                   # preempted: recompute starts fresh
    s4, h4 = ss.step([11], [0])
    assert h4[0] == 0 and ss.num_free == 0
    ss.release(99)                                   # unknown request: no-op
    assert isinstance(s4, np.ndarray) and s4.dtype == np.int32
