"""Engine metrics with vLLM-compatible Prometheus names (reference: the gate reads
``vllm:spec_decode_num_accepted_tokens_total``, ``vllm:num_preemptions_total``,
``vllm:num_requests_running`` ..., ``ci/accept/accept.py:162-207``)."""
from __future__ import annotations

import threading
import time


class EngineMetrics:
    def __init__(self):
        self.lock = threading.Lock()
        self.prompt_tokens_total = 0
        self.generation_tokens_total = 0
        self.requests_total = 0
        self.requests_finished = 0
        self.num_preemptions_total = 0
        self.spec_num_drafts_total = 0
        self.spec_num_draft_tokens_total = 0
        self.spec_num_accepted_tokens_total = 0
        self.spec_accepted_per_pos: list[int] = []
        self.num_requests_running = 0
        self.num_requests_waiting = 0
        self.kv_cache_usage = 0.0
        self.iteration_tokens_sum = 0
        self.iteration_tokens_count = 0
        self.step_time_sum = 0.0
        self.ttft: list[float] = []
        self.e2e: list[float] = []

    def on_arrival(self):
        with self.lock:
            self.requests_total += 1

    def on_step(self, sched, result, dt, kv_usage, running, waiting):
        with self.lock:
            self.iteration_tokens_sum += sched.num_tokens
            self.iteration_tokens_count += 1
            self.step_time_sum += dt
            self.num_preemptions_total += len(sched.preempted)
            self.kv_cache_usage = kv_usage
            self.num_requests_running = running
            self.num_requests_waiting = waiting
            for s in sched.seqs:
                if s.is_decode or s.samples:
                    pass
            self.generation_tokens_total += sum(len(v) for v in result.sampled.values())
            self.prompt_tokens_total += sum(s.num_new_tokens for s in sched.seqs if not s.is_decode)

    def on_spec(self, num_drafts, num_draft_tokens, accepted_lens, k):
        with self.lock:
            self.spec_num_drafts_total += num_drafts
            self.spec_num_draft_tokens_total += num_draft_tokens
            self.spec_num_accepted_tokens_total += sum(accepted_lens)
            if len(self.spec_accepted_per_pos) < k:
                self.spec_accepted_per_pos += [0] * (k - len(self.spec_accepted_per_pos))
            for a in accepted_lens:
                for p in range(min(a, k)):
                    self.spec_accepted_per_pos[p] += 1

    def on_finish(self, req):
        with self.lock:
            self.requests_finished += 1
            if req.first_token_time is not None:
                self.ttft.append(req.first_token_time - req.arrival_time)
            if req.finish_time is not None:
                self.e2e.append(req.finish_time - req.arrival_time)

    def prometheus(self, model_name: str = "model") -> str:
        lbl = f'{{model_name="{model_name}"}}'
        with self.lock:
            lines = [
                f"vllm:num_requests_running{lbl} {self.num_requests_running}",
                f"vllm:num_requests_waiting{lbl} {self.num_requests_waiting}",
                f"vllm:kv_cache_usage_perc{lbl} {self.kv_cache_usage}",
                f"vllm:prompt_tokens_total{lbl} {self.prompt_tokens_total}",
                f"vllm:generation_tokens_total{lbl} {self.generation_tokens_total}",
                f"vllm:num_preemptions_total{lbl} {self.num_preemptions_total}",
                f"vllm:request_success_total{lbl} {self.requests_finished}",
                f"vllm:iteration_tokens_total_sum{lbl} {self.iteration_tokens_sum}",
                f"vllm:iteration_tokens_total_count{lbl} {self.iteration_tokens_count}",
                f"vllm:spec_decode_num_drafts_total{lbl} {self.spec_num_drafts_total}",
                f"vllm:spec_decode_num_draft_tokens_total{lbl} {self.spec_num_draft_tokens_total}",
                f"vllm:spec_decode_num_accepted_tokens_total{lbl} {self.spec_num_accepted_tokens_total}",
            ]
            for p, n in enumerate(self.spec_accepted_per_pos):
                lines.append(f'vllm:spec_decode_num_accepted_tokens_per_pos_total{{model_name="{model_name}",position="{p}"}} {n}')
        return "\n".join(lines) + "\n"
