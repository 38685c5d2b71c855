"""Hidden-state tracer: env interface, sampling cadence and line format (CPU tensors)."""
import torch

from vm_c_b200.utils.trace import HiddenTracer


def test_from_env(monkeypatch):
    monkeypatch.delenv("VMC_LOG_HIDDEN", raising=False)
    monkeypatch.delenv("VMC_LOG_LOGITS", raising=False)
    assert HiddenTracer.from_env() is None
    monkeypatch.setenv("VMC_LOG_HIDDEN", "1")
    monkeypatch.setenv("VMC_LOG_HIDDEN_EVERY", "3")
    t = HiddenTracer.from_env()
    assert t is not None and t.every == 3 and t.hidden and not t.logits


def test_first_time_only_and_every_n():
    lines = []
    t = HiddenTracer(every=0, sink=lines.append)
    x = torch.arange(20, dtype=torch.float32).view(4, 5)
    for _ in range(3):
        t.probe("l_out-0", x)
        t.flush()
    assert len(lines) == 1
    assert lines[0] == "step 0 hidden l_out-0 shape=[4, 5] first8=[0, 1, 2, 3, 4, 5, 6, 7]"
    t.probe("l_out-0", x[:2])  # a new shape is a new key
    assert len(t.flush()) == 1
    lines.clear()
    t = HiddenTracer(every=2, sink=lines.append)
    for _ in range(5):
        t.probe("a", x)
        t.flush()
    assert [ln.split()[1] for ln in lines] == ["0", "2", "4"]


def test_logits_top5():
    t = HiddenTracer(logits=True, sink=lambda s: None)
    t.hidden = False
    logits = torch.zeros(2, 10)
    logits[0, 7], logits[1, 3] = 5.0, 4.0
    t.probe("ignored", logits)
    t.probe_logits(logits, 2)
    out = t.flush()
    assert len(out) == 1 and out[0].startswith("step 0 logits_top5 rows=2 [7:5.0000")
    assert "[3:4.0000" in out[0]
