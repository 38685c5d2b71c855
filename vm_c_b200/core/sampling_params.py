"""Request / sampling data model.

Same fields and defaults as the reference's SamplingParams and Request
(include/vm_c/core/request.hpp:28-42, :44-80: max_tokens 16, top_k 40, top_p 0.95,
temperature 0.8, penalties, stop ids / strings, ignore_eos, min_tokens, min_p, enable_thinking),
plus a per-request seed (the reference samples with seed 0 on every step).
"""
from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field
from typing import Callable, Optional


class FinishReason(enum.IntEnum):
    STOP = 0
    LENGTH = 1
    ERROR = 2
    ABORTED = 3

    @property
    def openai(self) -> str:
        return {0: "stop", 1: "length", 2: "error", 3: "abort"}[int(self)]


class RequestStatus(enum.IntEnum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2
    PREEMPTED = 3


@dataclass
class SamplingParams:
    max_tokens: int = 16
    top_k: int = 40
    top_p: float = 0.95
    temperature: float = 0.80
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    stop_token_ids: list[int] = field(default_factory=list)
    stop: list[str] = field(default_factory=list)
    ignore_eos: bool = False
    min_tokens: int = 0
    min_p: float = 0.0
    enable_thinking: bool = True
    seed: Optional[int] = None
    logprobs: bool = False

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1

    @property
    def has_penalties(self) -> bool:
        return (self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or self.presence_penalty != 0.0)

    @classmethod
    def greedy_params(cls, max_tokens: int = 16, **kw) -> "SamplingParams":
        return cls(max_tokens=max_tokens, temperature=0.0, top_k=1, top_p=1.0, **kw)


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: list[int]
    output_token_ids: list[int]
    output_logprobs: list[float]
    finished: bool
    finish_reason: Optional[FinishReason]
    text: str = ""
    arrival_time: float = 0.0
    first_token_time: float = 0.0
    finish_time: float = 0.0
    token_times: list[float] = field(default_factory=list)
    num_cached_tokens: int = 0

    @property
    def ttft(self) -> float:
        return self.first_token_time - self.arrival_time if self.first_token_time else float("nan")

    def itls(self) -> list[float]:
        t = self.token_times
        return [b - a for a, b in zip(t, t[1:])]


@dataclass
class Request:
    request_id: str
    prompt_token_ids: list[int]
    params: SamplingParams
    int_id: int = -1
    arrival_time: float = field(default_factory=time.perf_counter)
    output_token_ids: list[int] = field(default_factory=list)
    output_logprobs: list[float] = field(default_factory=list)
    token_times: list[float] = field(default_factory=list)
    finished: bool = False
    finish_reason: Optional[FinishReason] = None
    seed: int = 0
    stream_callback: Optional[Callable[["Request", list[int], bool], None]] = None
    user_data: object = None

    def to_output(self) -> RequestOutput:
        return RequestOutput(self.request_id, self.prompt_token_ids, list(self.output_token_ids),
                             list(self.output_logprobs), self.finished, self.finish_reason,
                             arrival_time=self.arrival_time,
                             first_token_time=self.token_times[0] if self.token_times else 0.0,
                             finish_time=self.token_times[-1] if self.token_times else 0.0,
                             token_times=list(self.token_times))
