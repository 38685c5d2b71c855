"""Property-based test of the native scheduler and block manager (csrc/host/scheduler.cpp,
block_manager.cpp): hypothesis drives random interleavings of request arrivals (with shared prompt
prefixes, so the prefix cache hits), scheduling steps, aborts and host-side finishes against a KV
pool small enough to force preemption. The "model" is a deterministic rule (token after t at position
p = (31 t + 7 p + 11) mod V), so every request's output is known in advance.

Checked after every step: the token budget, the sequence limit and the decode-first order of the plan;
every entry starts where its request's computed prefix ends; exactly the entries that reach the last
known token sample; the KV pool never reports more free blocks than it has. At the end: every request
that was not aborted or finished by the host produced exactly its predicted tokens (through
preemptions and recomputation), and every block is free again."""
import numpy as np
from hypothesis import HealthCheck, settings
from hypothesis import strategies as st
from hypothesis.stateful import RuleBasedStateMachine, initialize, invariant, precondition, rule

from vm_c_b200 import _native

V = 97
EOS = 96
SEQS, BUDGET, MODEL_LEN, BLOCKS, BS = 4, 24, 80, 22, 4


def next_token(t, p):
    return (31 * t + 7 * p + 11) % V


def predict(prompt, max_tokens):
    """Tokens the scheduler must deliver for `prompt` (the scheduler's stop rules: EOS, max_tokens,
    max_model_len)."""
    known = list(prompt[:MODEL_LEN])  # prompts are truncated to max_model_len
    out = []
    while True:
        t = next_token(known[-1], len(known) - 1)
        out.append(t)
        known.append(t)
        if t == EOS or len(out) >= max_tokens or len(known) >= MODEL_LEN:
            return out


class SchedulerMachine(RuleBasedStateMachine):
    @initialize()
    def setup(self):
        h = _native.host()
        cfg = h.SchedulerConfig()
        cfg.max_num_seqs = SEQS
        cfg.max_num_batched_tokens = BUDGET
        cfg.max_model_len = MODEL_LEN
        cfg.decode_latency_target_ms = 0
        self.h = h
        self.s = h.Scheduler(cfg, h.BlockManager(BLOCKS, BS, True))
        self.reqs = {}      # id -> {"prompt", "max_tokens", "out", "state"}
        self.next_id = 1
        self.steps = 0
        self.preemptions = 0
        self.free_at_start = self.s.num_free_blocks

    def _params(self, max_tokens):
        p = self.h.SeqParams()
        p.max_tokens = max_tokens
        p.eos_token_ids = [EOS]
        return p

    def _live(self):
        return [i for i, r in self.reqs.items() if r["state"] == "live"]

    @rule(prefix=st.sampled_from([[], [1, 2, 3, 4, 5, 6, 7, 8], [1, 2, 3, 4, 9, 9, 9, 9, 9, 9, 9, 9]]),
          tail=st.lists(st.integers(0, V - 2), min_size=1, max_size=40), max_tokens=st.integers(1, 40))
    def add(self, prefix, tail, max_tokens):
        if len(self._live()) >= 12:
            return
        rid = self.next_id
        self.next_id += 1
        prompt = prefix + tail
        self.s.add_request(rid, prompt, self._params(max_tokens))
        self.reqs[rid] = {"prompt": prompt, "max_tokens": max_tokens, "out": [], "state": "live"}

    @precondition(lambda self: self.s.has_unfinished())
    @rule()
    def step(self):
        self._step()

    def _step(self):
        plan = self.s.schedule()
        self.steps += 1
        self.preemptions += len(plan.preempted)
        entries = list(plan.entries)
        assert plan.total_tokens <= BUDGET
        assert plan.total_tokens == sum(e.num_tokens for e in entries)
        assert len(entries) <= SEQS
        kinds = [e.is_decode for e in entries]
        assert kinds == sorted(kinds, reverse=True), "decodes come first"
        toks = []
        for e in entries:
            r = self.reqs[e.id]
            known = r["prompt"][:MODEL_LEN] + r["out"]
            info = self.s.seq_info(e.id)
            assert e.start + e.num_tokens <= len(known)
            assert e.sample == (e.start + e.num_tokens == len(known))
            if e.sample:
                p = len(known) - 1
                toks.append(next_token(known[p], p))
            assert info["num_computed"] == e.start
        events = self.s.update(plan, np.asarray(toks, dtype=np.int32))
        for rid, new, finished, _reason in events:
            r = self.reqs[rid]
            r["out"] += list(new)
            if finished:
                r["state"] = "finished"
                self.s.release(rid)

    @precondition(lambda self: any(r["state"] == "live" for r in self.reqs.values()))
    @rule(data=st.data(), host_finish=st.booleans(), dice=st.integers(0, 5))
    def stop_one(self, data, host_finish, dice):
        if dice:  # stops are rarer than steps, so that requests grow and the pool runs out
            return
        rid = data.draw(st.sampled_from(self._live()))
        if host_finish:  # a stop string matched on the host
            self.s.finish_request(rid, 0)
        else:            # the client went away
            self.s.abort_request(rid)
        self.s.release(rid)
        self.reqs[rid]["state"] = "stopped"

    @invariant()
    def pool_bounds(self):
        if hasattr(self, "s"):
            assert 0 <= self.s.num_free_blocks <= self.free_at_start

    def teardown(self):
        if not hasattr(self, "s"):
            return
        for _ in range(4000):
            if not self.s.has_unfinished():
                break
            self._step()
        assert not self.s.has_unfinished(), "every request finishes"
        for rid, r in self.reqs.items():
            if r["state"] == "finished":
                assert r["out"] == predict(r["prompt"], r["max_tokens"]), rid
            else:
                assert r["state"] == "stopped"
                want = predict(r["prompt"], r["max_tokens"])
                assert r["out"] == want[:len(r["out"])], rid  # a stopped request is a prefix
        assert self.s.num_free_blocks == self.free_at_start, "every KV block is free again"


SchedulerMachine.TestCase.settings = settings(max_examples=150, stateful_step_count=60, deadline=None,
                                              suppress_health_check=[HealthCheck.too_slow])
test_scheduler_state_machine = SchedulerMachine.TestCase
