"""The serving engine: request intake, scheduling, step execution, output handling.

Counterpart of the reference's Engine (src/core/engine.cpp: initialize :257, submit_request :465,
step :493, run_forward :556, sampling :1061-1155, finish logic :1219-1244). The scheduler, block
manager and per-step metadata builder are native (csrc/host/scheduler.cpp); this module moves the
step through a ModelRunner (models/runner.py on the GPU) and turns sampled tokens into per-request
outputs. Differences by design: any number of finished requests is released per step (the
reference frees one, engine.cpp:520-532), and sampling is seeded per request.
"""
from __future__ import annotations

import hashlib
import itertools
import os
import threading
import time
from collections import deque
from dataclasses import dataclass
from typing import Callable, Iterable, Optional

import numpy as np

from .. import _native
from ..config import VmCConfig
from ..utils.logging import get_logger
from ..utils.metrics import EngineMetrics
from .sampling_params import FinishReason, Request, RequestOutput, SamplingParams
from ..utils import nvtx

log = get_logger("engine")

SAMPLE_DTYPE = np.dtype([("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"), ("min_p", "<f4"),
                         ("repetition_penalty", "<f4"), ("frequency_penalty", "<f4"), ("presence_penalty", "<f4"),
                         ("step", "<i4"), ("seed", "<u8")])
assert SAMPLE_DTYPE.itemsize == 40


@dataclass
class StepCounts:
    T: int
    R: int
    S: int
    num_decode: int
    max_qlen: int
    max_ctx: int
    T_pad: int
    R_pad: int


class ModelRunner:
    """Executes one scheduled step. Implementations: models.runner.GpuModelRunner (sm_100a kernels)
    and test doubles."""
    num_kv_blocks: int
    max_model_len: int

    def max_graph_batch(self) -> int:
        return 0

    def execute(self, meta: np.ndarray, counts: StepCounts, params: np.ndarray, penalties=None) -> tuple[np.ndarray, np.ndarray]:
        raise NotImplementedError


class LLMEngine:
    def __init__(self, cfg: VmCConfig, runner: ModelRunner, eos_token_ids: Optional[list[int]] = None):
        self.cfg = cfg
        self.runner = runner
        self.h = _native.host()
        sc = self.h.SchedulerConfig()
        s = cfg.scheduler
        sc.max_num_seqs = s.max_num_seqs
        sc.max_num_batched_tokens = s.max_num_batched_tokens
        sc.max_model_len = cfg.model.max_model_len
        sc.enable_chunked_prefill = s.enable_chunked_prefill
        sc.long_prefill_token_threshold = s.long_prefill_token_threshold
        sc.decode_first = s.scheduling_policy == "decode_first"
        sc.max_prefill_per_batch = s.max_prefill_per_batch
        sc.decode_latency_target_ms = s.decode_latency_target_ms
        sc.preempt_prefill_on_latency = s.preempt_prefill_on_latency
        sc.decode_reserved_tokens = s.decode_reserved_tokens
        sc.num_lookahead_tokens = getattr(runner, "num_lookahead_tokens", 0)
        self.block_size = cfg.cache.block_size
        # Hybrid (recurrent-state) models cannot resume from cached KV blocks: no prefix caching there.
        self.bm = self.h.BlockManager(runner.num_kv_blocks, self.block_size,
                                      cfg.cache.enable_prefix_caching and not cfg.model.is_hybrid)
        self.sched = self.h.Scheduler(sc, self.bm)
        max_blocks = (cfg.model.max_model_len + sc.num_lookahead_tokens + self.block_size - 1) // self.block_size + 1
        max_tok = max(s.max_num_batched_tokens, s.max_num_seqs, runner.max_graph_batch())
        self.layout = self.h.BatchLayout(max_tok, max(s.max_num_seqs, runner.max_graph_batch()), max_blocks)
        self.meta = runner.alloc_meta(self.layout.total) if hasattr(runner, "alloc_meta") else \
            np.zeros(self.layout.total, dtype=np.int32)
        self.meta_np = self.meta.numpy() if hasattr(self.meta, "numpy") else self.meta
        self.meta_addr = self.meta.data_ptr() if hasattr(self.meta, "data_ptr") else self.meta.ctypes.data
        if hasattr(runner, "bind_layout"):
            runner.bind_layout(self.layout)
        self.eos = list(eos_token_ids if eos_token_ids is not None else cfg.model.eos_token_ids)
        self.requests: dict[int, Request] = {}
        self.by_name: dict[str, int] = {}
        self._ids = itertools.count(1)
        self._pending: deque[Request] = deque()
        self._aborts: deque[str] = deque()
        self._lock = threading.Lock()
        self.slot_params = np.zeros(sc.max_num_seqs, dtype=SAMPLE_DTYPE)
        self.slot_owner = np.full(sc.max_num_seqs, -1, dtype=np.int64)
        self.metrics = EngineMetrics()
        self.step_id = 0
        self.on_step: Optional[Callable] = None   # hook(plan, counts, dt)
        # hook(request ids, logits [S, vocab] on the host): full-vocabulary logits of every sampled row of
        # a non-speculative step (tests compare them with an fp32 oracle); None costs nothing.
        self.logits_hook: Optional[Callable] = None
        # Launch step n+1 before emitting step n's outputs (runners with launch / wait, no speculation;
        # VMC_PIPELINE=0 turns it off).
        self._inflight = None
        self._pen_ids: set[int] = set()  # running requests with repetition/frequency/presence penalties
        self._snapshots = True  # step() returns snapshots of running requests (generate() turns this off)
        self.pipelined = (hasattr(runner, "launch") and getattr(runner, "spec_k", 0) == 0
                          and os.environ.get("VMC_PIPELINE", "1") != "0")

    # -------------------------------------------------------------------------------------------
    # request intake (thread-safe: the server's HTTP threads call these)

    def add_request(self, prompt_token_ids: list[int], params: Optional[SamplingParams] = None,
                    request_id: Optional[str] = None, stream_callback=None, user_data=None) -> Request:
        params = params or SamplingParams()
        if not prompt_token_ids:
            raise ValueError("empty prompt")
        V = self.cfg.model.vocab
        if min(prompt_token_ids) < 0 or max(prompt_token_ids) >= V:
            raise ValueError(f"prompt token id out of range [0, {V})")
        rid = request_id or f"req-{next(self._ids)}"
        req = Request(rid, list(prompt_token_ids), params, stream_callback=stream_callback, user_data=user_data)
        # deterministic across processes (every tensor-parallel rank must draw the same samples)
        req.seed = params.seed if params.seed is not None else \
            int.from_bytes(hashlib.blake2b(rid.encode(), digest_size=8).digest(), "little") & 0x7fffffffffffffff
        with self._lock:
            self._pending.append(req)
        return req

    def abort_request(self, request_id: str) -> None:
        with self._lock:
            self._aborts.append(request_id)

    def _drain(self) -> None:
        with self._lock:
            pend, self._pending = self._pending, deque()
            aborts, self._aborts = self._aborts, deque()
        for req in pend:
            iid = next(self._ids)
            req.int_id = iid
            sp = self.h.SeqParams()
            p = req.params
            sp.max_tokens = max(1, p.max_tokens)
            sp.min_tokens = p.min_tokens
            sp.ignore_eos = p.ignore_eos
            sp.stop_token_ids = list(p.stop_token_ids)
            sp.eos_token_ids = self.eos
            self.sched.add_request(iid, req.prompt_token_ids, sp)
            self.requests[iid] = req
            if p.has_penalties:
                self._pen_ids.add(iid)
            self.by_name[req.request_id] = iid
        for name in aborts:
            iid = self.by_name.get(name)
            if iid is not None and self.sched.abort_request(iid):
                self._finish(self.requests[iid], FinishReason.ABORTED)

    def has_unfinished(self) -> bool:
        if self._inflight is not None:
            return True
        with self._lock:
            if self._pending:
                return True
        return self.sched.has_unfinished()

    @property
    def num_running(self) -> int:
        return self.sched.num_running

    @property
    def num_waiting(self) -> int:
        return self.sched.num_waiting + len(self._pending)

    # -------------------------------------------------------------------------------------------

    def _counts(self) -> StepCounts:
        c = self.meta_np[self.layout.off_counts:self.layout.off_counts + 8]
        return StepCounts(*[int(x) for x in c])

    def _sample_params(self, plan, S: int, R_pad_rows: int) -> np.ndarray:
        ids = np.asarray(plan.sample_ids(), dtype=np.int64)
        slots = np.asarray(plan.sample_slots(), dtype=np.int64)
        stale = np.nonzero(self.slot_owner[slots] != ids)[0]
        for k in stale:
            req = self.requests[int(ids[k])]
            p = req.params
            rec = self.slot_params[slots[k]]
            rec["temperature"] = 0.0 if p.greedy else p.temperature
            rec["top_k"] = p.top_k
            rec["top_p"] = p.top_p
            rec["min_p"] = p.min_p
            rec["repetition_penalty"] = p.repetition_penalty
            rec["frequency_penalty"] = p.frequency_penalty
            rec["presence_penalty"] = p.presence_penalty
            rec["seed"] = req.seed
            self.slot_params[slots[k]] = rec
            self.slot_owner[slots[k]] = ids[k]
        out = np.zeros(max(S, R_pad_rows), dtype=SAMPLE_DTYPE)
        out[:S] = self.slot_params[slots]
        reqs = self.requests
        out["step"][:S] = [len(reqs[i].output_token_ids) for i in ids.tolist()]
        return out

    def _penalties(self, plan, S: int):
        """CSR triples (row, token, output count) for rows that use penalties (None if none)."""
        if not self._pen_ids:
            return None
        rows, toks, cnts = [], [], []
        for k, iid in enumerate(plan.sample_ids()):
            req = self.requests[int(iid)]
            if not req.params.has_penalties:
                continue
            counts: dict[int, int] = {}
            for t in req.prompt_token_ids:
                counts.setdefault(t, 0)
            for t in req.output_token_ids:
                counts[t] = counts.get(t, 0) + 1
            for t, c in counts.items():
                rows.append(k)
                toks.append(t)
                cnts.append(c)
        if not rows:
            return None
        return (np.asarray(rows, np.int32), np.asarray(toks, np.int32), np.asarray(cnts, np.int32))

    def step(self) -> list[RequestOutput]:
        """Run one scheduler step; returns outputs of requests that produced tokens or finished."""
        if nvtx.ENABLED:
            with nvtx.nvtx_range(f"engine.step {self.step_id}"):
                return self._step()
        return self._step()

    def _step(self) -> list[RequestOutput]:
        # Pipelined steps: the previous step's kernels may still be running. Its tokens are applied
        # to the scheduler first (C++, cheap), the next step is scheduled and launched, and only then
        # are the previous step's outputs emitted (callbacks, finish bookkeeping, metrics), so that
        # host work overlaps the GPU instead of sitting between two steps.
        done = self._complete_inflight()
        self._drain()
        spec = getattr(self.runner, "spec", None)
        plan = self.sched.schedule()
        for iid in plan.preempted:
            self.metrics.preemptions += 1
            if spec is not None:
                spec.forget(int(iid))
        if len(plan) == 0:
            return self._emit(done) if done else []
        t0 = time.perf_counter()
        pen = self._penalties(plan, plan.num_sample)
        all_decode = plan.num_decode == len(plan)
        sample_ids = plan.sample_ids()
        # Speculate on all-decode, penalty-free steps: greedy batches by exact agreement, batches with
        # sampled requests by rejection sampling when the speculator supports it.
        all_greedy = all(self.requests[int(i)].params.greedy for i in sample_ids)
        speculate = spec is not None and all_decode and pen is None and \
            (all_greedy or getattr(spec, "supports_sampling", False))
        pad = 0
        if all_decode and pen is None and not speculate and hasattr(self.runner, "graph_bucket"):
            pad = self.runner.graph_bucket(len(plan))
        self.sched.build_batch(plan, self.layout, self.meta_addr, pad)
        counts = self._counts()
        if not pad:
            counts.R_pad = 0
        if self.pipelined and not speculate:
            params = self._sample_params(plan, counts.S, counts.R_pad)
            handle = self.runner.launch(self.meta, counts, params, pen)
            self._inflight = (plan, counts, sample_ids, handle, t0)
            return self._emit(done) if done else []
        outs = self._emit(done) if done else []
        lp_by_id = {}
        if speculate and all_greedy:
            new = spec.step(sample_ids, counts)
        elif speculate:
            reqs = [self.requests[int(i)] for i in sample_ids]
            seed = hash((self.step_id, tuple(rq.seed for rq in reqs))) & 0x7fffffffffffffff
            new = spec.sampled_step(sample_ids, counts, [rq.params for rq in reqs], seed)
        if speculate:
            flat = np.fromiter((t for row in new for t in row), dtype=np.int32)
            events = self.sched.update(plan, flat, [len(row) for row in new])
        else:
            params = self._sample_params(plan, counts.S, counts.R_pad)
            toks, lps = self.runner.execute(self.meta, counts, params, pen)
            if self.logits_hook is not None:
                self.logits_hook([int(i) for i in sample_ids], self.runner.full_logits(counts.S))
            if spec is not None:  # keep the draft's cache in step with the target's
                spec.set_batch([e.id for e in plan.entries])
                spec.shadow(counts)
            events = self.sched.update(plan, toks[:counts.S])
            for k, iid in enumerate(sample_ids):
                lp_by_id[int(iid)] = float(lps[k]) if lps is not None else 0.0
        return outs + self._emit(self._apply(events, lp_by_id, plan, counts, t0))

    def quiesce(self) -> list[RequestOutput]:
        """Finish the launched step (if any) and wait for the device, so that nothing of this rank is
        left in flight (a rank leaving a tensor-parallel job between steps calls this first)."""
        done = self._complete_inflight()
        outs = self._emit(done) if done else []
        if hasattr(self.runner, "synchronize"):
            self.runner.synchronize()
        return outs

    def _complete_inflight(self):
        """Wait for the launched step and apply its tokens (scheduler and per-request token lists)."""
        f = self._inflight
        if f is None:
            return None
        self._inflight = None
        plan, counts, sample_ids, handle, t0 = f
        toks, lps = self.runner.wait(handle)
        if self.logits_hook is not None:
            self.logits_hook([int(i) for i in sample_ids], self.runner.full_logits(counts.S))
        events = self.sched.update(plan, toks[:counts.S])
        lp_by_id = dict(zip(sample_ids, lps[:len(sample_ids)].tolist()))
        return self._apply(events, lp_by_id, plan, counts, t0)

    def _apply(self, events, lp_by_id, plan, counts, t0):
        now = time.perf_counter()
        reqs = self.requests
        for iid, new_toks, finished, reason in events:
            req = reqs.get(iid)
            if req is None:
                continue
            lp = lp_by_id.get(iid, 0.0)
            if len(new_toks) == 1:  # a decode step
                req.output_token_ids.append(new_toks[0])
                req.output_logprobs.append(lp)
                req.token_times.append(now)
            else:
                req.output_token_ids.extend(new_toks)
                req.output_logprobs.extend([lp] * len(new_toks))
                req.token_times.extend([now] * len(new_toks))
        return events, plan, counts, t0, now

    def _emit(self, done) -> list[RequestOutput]:
        """Callbacks, finish bookkeeping and metrics of a completed step."""
        events, plan, counts, t0, now = done
        outs = []
        for iid, new_toks, finished, reason in events:
            req = self.requests.get(int(iid))
            if req is None:
                continue
            if finished:
                self._finish(req, FinishReason(reason), new_toks)
            elif req.stream_callback:
                req.stream_callback(req, new_toks, False)
            outs.append(req.to_output() if (finished or (req.stream_callback is None and self._snapshots)) else None)
        dt = now - t0
        self.metrics.record_step(counts.T, counts.S, counts.num_decode, dt, plan.num_cached_tokens)
        self.step_id += 1
        if self.on_step:
            self.on_step(plan, counts, dt)
        return [o for o in outs if o is not None]

    def _finish(self, req: Request, reason: FinishReason, last_tokens: Optional[list[int]] = None) -> None:
        if req.finished:
            return
        req.finished = True
        req.finish_reason = reason
        self.sched.release(req.int_id)
        spec = getattr(self.runner, "spec", None)
        if spec is not None:
            spec.forget(req.int_id)
        self.requests.pop(req.int_id, None)
        self._pen_ids.discard(req.int_id)
        self.by_name.pop(req.request_id, None)
        self.metrics.record_finish(req)
        if req.stream_callback:
            req.stream_callback(req, list(last_tokens or []), True)

    def fail_all(self, reason: FinishReason = FinishReason.ERROR) -> int:
        """Finish every queued and running request with `reason` (after a rank or device failure).
        Returns how many requests were failed."""
        self._inflight = None
        self._drain()
        reqs = list(self.requests.values())
        for req in reqs:
            if self.sched.abort_request(req.int_id):
                pass
            self._finish(req, reason)
        return len(reqs)

    def finish_request(self, request_id: str, reason: FinishReason = FinishReason.STOP) -> None:
        """Finish a running request from the host (e.g. a stop string matched by the detokenizer)."""
        iid = self.by_name.get(request_id)
        if iid is None:
            return
        self.sched.finish_request(iid, int(reason))
        self._finish(self.requests[iid], reason)

    # -------------------------------------------------------------------------------------------

    def generate(self, prompts: Iterable[list[int]], params: SamplingParams | list[SamplingParams] | None = None,
                 ) -> list[RequestOutput]:
        """Offline batch generation: submit all prompts, step until done, return outputs in order."""
        prompts = list(prompts)
        plist = params if isinstance(params, list) else [params or SamplingParams()] * len(prompts)
        done: dict[str, RequestOutput] = {}
        reqs = [self.add_request(p, sp) for p, sp in zip(prompts, plist)]
        order = [r.request_id for r in reqs]
        # only finished outputs are read here: skip the per-step snapshots of running requests (a copy
        # of every token list each step, which grows with the output length)
        self._snapshots = False
        try:
            while self.has_unfinished():
                for o in self.step():
                    if o.finished:
                        done[o.request_id] = o
        finally:
            self._snapshots = True
        return [done[r] for r in order]
