"""Engine metrics (vm_c_b200/utils/metrics.py): TTFT / ITL percentiles from finished requests, and a
bounded latency history (a long-running server keeps only the most recent samples)."""
from types import SimpleNamespace

from vm_c_b200.utils import metrics as M


def test_percentiles_from_token_times():
    m = M.EngineMetrics()
    m.record_finish(SimpleNamespace(token_times=[1.0, 1.5, 2.5], arrival_time=0.5))
    s = m.summary()
    assert s["p50_ttft_ms"] == 500.0
    assert s["p50_itl_ms"] == 750.0 and abs(s["p99_itl_ms"] - 995.0) < 1e-9
    assert m.finished == 1


def test_latency_history_is_bounded():
    m = M.EngineMetrics()
    n = M.ITL_WINDOW + 10
    m.record_finish(SimpleNamespace(token_times=[float(i * i) for i in range(n)], arrival_time=0.0))
    assert len(m.itl_s) == M.ITL_WINDOW
    # W + 9 gaps were recorded and the oldest 9 dropped: the first one kept is between tokens 9 and 10
    assert m.itl_s[0] == min(m.itl_s) == float(10 * 10 - 9 * 9)
    for _ in range(M.TTFT_WINDOW + 5):
        m.record_finish(SimpleNamespace(token_times=[2.0], arrival_time=1.0))
    assert len(m.ttft_s) == M.TTFT_WINDOW and m.finished == M.TTFT_WINDOW + 6
