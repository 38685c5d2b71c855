"""Scheduler semantics (reference: src/core/scheduler.cpp): decode-first, chunked prefill, budget,
prefix cache, preemption, stop rules, fair policy, batch metadata."""
import numpy as np
import pytest


def mk(host, blocks=64, bs=4, seqs=4, budget=16, model_len=64, policy_decode_first=True, prefix=True,
       threshold=0, chunked=True):
    cfg = host.SchedulerConfig()
    cfg.max_num_seqs = seqs
    cfg.max_num_batched_tokens = budget
    cfg.max_model_len = model_len
    cfg.decode_first = policy_decode_first
    cfg.long_prefill_token_threshold = threshold
    cfg.enable_chunked_prefill = chunked
    cfg.decode_latency_target_ms = 0
    bm = host.BlockManager(blocks, bs, prefix)
    return host.Scheduler(cfg, bm), bm


def params(host, max_tokens=4, eos=(), stop=(), min_tokens=0, ignore_eos=False):
    p = host.SeqParams()
    p.max_tokens = max_tokens
    p.eos_token_ids = list(eos)
    p.stop_token_ids = list(stop)
    p.min_tokens = min_tokens
    p.ignore_eos = ignore_eos
    return p


def run_step(s, tok=7):
    plan = s.schedule()
    ev = s.update(plan, np.full(plan.num_sample, tok, np.int32))
    return plan, ev


def test_budget_invariant(host):
    cfg = host.SchedulerConfig()
    cfg.max_num_seqs = 8
    cfg.max_num_batched_tokens = 4
    with pytest.raises(RuntimeError):
        host.Scheduler(cfg, host.BlockManager(8, 4, True))


def test_chunked_prefill_then_decode(host):
    s, _ = mk(host, budget=16)
    s.add_request(1, list(range(40)), params(host, max_tokens=3))
    plan, ev = run_step(s)
    assert [(e.num_tokens, e.start, e.sample) for e in plan.entries] == [(16, 0, False)]
    plan, _ = run_step(s)
    plan, ev = run_step(s)
    assert plan.entries[0].num_tokens == 8 and plan.entries[0].sample
    assert ev[0][1] == [7]
    plan, ev = run_step(s)
    assert plan.entries[0].is_decode and plan.entries[0].start == 40


def test_decode_first_ordering_and_budget(host):
    s, _ = mk(host, budget=10, seqs=4)
    s.add_request(1, list(range(5)), params(host, max_tokens=10))
    run_step(s)                               # prefill req 1 (5 tokens) -> first token
    s.add_request(2, list(range(30)), params(host, max_tokens=10))
    plan, _ = run_step(s)
    ents = plan.entries
    assert ents[0].id == 1 and ents[0].is_decode
    assert ents[1].id == 2 and ents[1].num_tokens == 9    # remaining budget goes to prefill
    assert plan.total_tokens == 10


def test_long_prefill_threshold(host):
    s, _ = mk(host, budget=32, threshold=5)
    s.add_request(1, list(range(20)), params(host))
    plan, _ = run_step(s)
    assert plan.entries[0].num_tokens == 5


def test_stop_rules(host):
    s, _ = mk(host)
    s.add_request(1, [1, 2, 3], params(host, max_tokens=5, eos=[9]))
    plan = s.schedule()
    ev = s.update(plan, np.array([9], np.int32))
    assert ev[0][2] and ev[0][3] == 0         # EOS -> STOP
    s.add_request(2, [1, 2, 3], params(host, max_tokens=5, eos=[9], min_tokens=2))
    plan = s.schedule()
    ev = s.update(plan, np.array([9], np.int32))
    assert not ev[0][2]                       # below min_tokens: EOS ignored
    s.add_request(3, [1, 2], params(host, max_tokens=1))
    plan = s.schedule()
    ev = s.update(plan, np.full(plan.num_sample, 4, np.int32))
    fin = {e[0]: e for e in ev}
    assert fin[3][2] and fin[3][3] == 1       # LENGTH
    s.add_request(4, [1], params(host, max_tokens=9, eos=[9], ignore_eos=True, stop=[8]))
    for tok, done in [(9, False), (8, True)]:
        plan = s.schedule()
        ev = {e[0]: e for e in s.update(plan, np.full(plan.num_sample, tok, np.int32))}
        assert ev[4][2] == done


def test_prefix_cache_hit_on_second_request(host):
    s, bm = mk(host, budget=64, bs=4)
    prompt = list(range(100, 118))
    s.add_request(1, prompt, params(host, max_tokens=1))
    run_step(s)
    s.add_request(2, prompt + [5, 6], params(host, max_tokens=1))
    plan = s.schedule()
    e = plan.entries[0]
    assert e.start == 16 and e.num_tokens == 4        # 4 full blocks cached (capped below num_tokens)
    assert plan.num_cached_tokens == 16
    assert s.prefix_hits == 1


def test_preemption_recompute(host):
    # 6 usable blocks of 4 tokens: two requests of 8-token prompts grow until one must be preempted
    s, bm = mk(host, blocks=7, bs=4, budget=32, seqs=2, prefix=False)
    s.add_request(1, list(range(8)), params(host, max_tokens=20))
    s.add_request(2, list(range(8)), params(host, max_tokens=20))
    preempted = []
    for _ in range(12):
        plan, ev = run_step(s)
        preempted += list(plan.preempted)
    assert 2 in preempted                     # the newest request is the victim
    info = s.seq_info(2)
    assert info["num_preemptions"] >= 1


def test_fair_policy(host):
    s, _ = mk(host, budget=8, policy_decode_first=False)
    s.add_request(1, list(range(20)), params(host))
    plan, _ = run_step(s)
    assert plan.entries[0].num_tokens == 8


def test_truncation_to_max_model_len(host):
    s, _ = mk(host, budget=64, model_len=10)
    s.add_request(1, list(range(30)), params(host, max_tokens=5))
    plan = s.schedule()
    assert plan.entries[0].num_tokens == 10
    ev = s.update(plan, np.array([3], np.int32))
    assert ev[0][2]                           # context full -> LENGTH


def test_abort(host):
    s, bm = mk(host)
    free0 = bm.num_free_blocks
    s.add_request(1, list(range(10)), params(host))
    run_step(s)
    assert s.abort_request(1)
    assert not s.abort_request(1)
    assert bm.num_free_blocks == free0


def test_build_batch_layout(host):
    s, bm = mk(host, budget=64, bs=4, seqs=4)
    s.add_request(1, [5, 6, 7], params(host, max_tokens=3))
    s.add_request(2, [8, 9], params(host, max_tokens=3))
    plan = s.schedule()
    L = host.BatchLayout(64, 8, 8)
    buf = np.zeros(L.total, np.int32)
    s.build_batch(plan, L, buf.ctypes.data, 0)
    assert buf[:5].tolist() == [5, 6, 7, 8, 9]
    assert buf[L.off_positions:L.off_positions + 5].tolist() == [0, 1, 2, 0, 1]
    assert buf[L.off_q_start:L.off_q_start + 3].tolist() == [0, 3, 5]
    assert buf[L.off_ctx_len:L.off_ctx_len + 2].tolist() == [3, 2]
    assert buf[L.off_logits_idx:L.off_logits_idx + 2].tolist() == [2, 4]
    b1 = bm.blocks_of(1)[0]
    assert buf[L.off_slot_mapping] == b1 * 4
    cnt = buf[L.off_counts:L.off_counts + 8].tolist()
    assert cnt[:4] == [5, 2, 2, 0]
    s.update(plan, np.array([1, 2], np.int32))
    plan = s.schedule()                       # two decodes, padded to a graph bucket of 4
    s.build_batch(plan, L, buf.ctypes.data, 4)
    cnt = buf[L.off_counts:L.off_counts + 8].tolist()
    assert cnt[6:] == [4, 4]
    assert buf[L.off_slot_mapping + 2] == -1 and buf[L.off_ctx_len + 3] == 0
