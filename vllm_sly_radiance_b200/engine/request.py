"""Requests, sampling parameters and outputs (vLLM-compatible field names)."""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0            # 0 = disabled (vLLM uses -1; both accepted)
    min_p: float = 0.0
    max_tokens: int = 16
    min_tokens: int = 0
    seed: Optional[int] = None
    stop_token_ids: list = field(default_factory=list)
    stop: list = field(default_factory=list)
    ignore_eos: bool = False
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    logprobs: Optional[int] = None
    n: int = 1

    def __post_init__(self):
        if self.top_k is None or self.top_k < 0:
            self.top_k = 0
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError("top_p must be in (0, 1]")
        if self.max_tokens is not None and self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0 or self.top_k == 1


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED_STOPPED = "stop"
    FINISHED_LENGTH = "length"
    FINISHED_ABORTED = "abort"

    @property
    def finished(self) -> bool:
        return self in (RequestStatus.FINISHED_STOPPED, RequestStatus.FINISHED_LENGTH,
                        RequestStatus.FINISHED_ABORTED)


_ids = itertools.count()


class Request:
    def __init__(self, prompt_token_ids: list[int], params: SamplingParams,
                 request_id: Optional[str] = None, eos_token_id: Optional[int] = None,
                 arrival_time: Optional[float] = None):
        self.request_id = request_id if request_id is not None else f"req-{next(_ids)}"
        self.prompt_token_ids = list(prompt_token_ids)
        self.output_token_ids: list[int] = []
        self.output_logprobs: list[float] = []
        self.params = params
        self.eos_token_id = eos_token_id
        self.status = RequestStatus.WAITING
        self.num_computed_tokens = 0
        self.block_ids: list[int] = []
        self.state_slot: Optional[int] = None
        self.restore_snapshot: Optional[int] = None   # GDN snapshot slot to restore (prefix hit)
        self.arrival_time = arrival_time if arrival_time is not None else time.monotonic()
        self.first_token_time: Optional[float] = None
        self.finish_time: Optional[float] = None
        self.num_preemptions = 0
        self.seed = params.seed if params.seed is not None else hash(self.request_id) & 0x7FFFFFFF
        # speculative decoding
        self.draft_token_ids: list[int] = []
        self.num_draft_tokens = 0
        self.num_accepted_tokens = 0
        self.spec_width = None

    @property
    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def is_prefill(self) -> bool:
        return self.num_computed_tokens < self.num_tokens - 1 or (
            self.num_computed_tokens == 0 and self.num_tokens > 0)

    def append_token(self, tok: int, logprob: float = 0.0):
        if self.first_token_time is None:
            self.first_token_time = time.monotonic()
        self.output_token_ids.append(int(tok))
        self.output_logprobs.append(float(logprob))

    def check_stop(self, max_model_len: int) -> bool:
        """Sets a finished status if a stop condition holds; returns True when finished."""
        p = self.params
        n_out = len(self.output_token_ids)
        if n_out == 0:
            return False
        last = self.output_token_ids[-1]
        if n_out >= p.min_tokens:
            if (not p.ignore_eos) and self.eos_token_id is not None and last == self.eos_token_id:
                self.status = RequestStatus.FINISHED_STOPPED
            elif last in p.stop_token_ids:
                self.status = RequestStatus.FINISHED_STOPPED
        if not self.status.finished:
            if n_out >= p.max_tokens or self.num_tokens >= max_model_len:
                self.status = RequestStatus.FINISHED_LENGTH
        if self.status.finished:
            self.finish_time = time.monotonic()
            return True
        return False


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: list
    finish_reason: Optional[str]
    logprobs: Optional[list] = None


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: list
    outputs: list
    finished: bool
    prompt: Optional[str] = None
    metrics: Optional[dict] = None
