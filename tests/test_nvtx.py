"""NVTX annotations (VMC_NVTX=1) on the host: balanced ranges around engine steps and layers, and no
calls at all when disabled."""
from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.utils import nvtx

from test_engine_cpu import make


class Recorder:
    def __init__(self):
        self.ev = []

    def push(self, name):
        self.ev.append(("push", name))

    def pop(self):
        self.ev.append(("pop", None))


def _balanced(ev):
    depth = 0
    for kind, _ in ev:
        depth += 1 if kind == "push" else -1
        assert depth >= 0
    return depth == 0


def test_ranges(monkeypatch):
    rec = Recorder()
    monkeypatch.setattr(nvtx, "backend", rec)
    monkeypatch.setattr(nvtx, "ENABLED", False)
    eng = make()
    eng.generate([[1, 2, 3]], SamplingParams.greedy_params(max_tokens=2))
    r = nvtx.LayerRanges()
    r.next(0)
    r.close()
    assert rec.ev == []

    monkeypatch.setattr(nvtx, "ENABLED", True)
    eng.generate([[4, 5]], SamplingParams.greedy_params(max_tokens=3))
    steps = [n for k, n in rec.ev if k == "push"]
    assert steps and all(n.startswith("engine.step ") for n in steps) and _balanced(rec.ev)
    rec.ev.clear()
    r = nvtx.LayerRanges()
    for i in range(3):
        r.next(i)
    r.close()
    assert [n for k, n in rec.ev if k == "push"] == ["layer 0", "layer 1", "layer 2"] and _balanced(rec.ev)
