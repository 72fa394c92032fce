"""FCFS token-budget scheduler (host logic).

Behavioural mirror of the reference's ``TokenBudgetScheduler`` /
``InferenceRequest`` / ``ScheduleBatch`` (reference
``src/inferkernellab/scheduler.py:7-95``), because the runtime hooks of the
drop-in boundary depend on its exact packing decisions:

* prefill packs waiting requests first-come-first-served while the batch has
  fewer than ``max_num_seqs`` entries and token budget left;
* only the first request of a batch may be cut to fit the budget (a chunked
  prefill continues at the head of the queue in the next batch);
* when nothing is waiting, the decode batch is ``running[:max_num_seqs]``.

``tests/golden/runtime_events.json`` pins the packing against the reference.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field


@dataclass
class InferenceRequest:
    request_id: int
    prompt_tokens: int
    max_new_tokens: int
    generated_tokens: int = 0
    cached_tokens: int = 0
    status: str = "waiting"
    block_table: list[int] = field(default_factory=list)

    @property
    def prompt_remaining(self) -> int:
        return max(0, self.prompt_tokens - self.cached_tokens)

    @property
    def finished(self) -> bool:
        return self.generated_tokens >= self.max_new_tokens


@dataclass(frozen=True)
class ScheduleBatch:
    requests: tuple[InferenceRequest, ...]
    phase: str
    scheduled_tokens: int


class TokenBudgetScheduler:
    def __init__(self, max_num_seqs: int = 32, max_num_batched_tokens: int = 2048):
        if max_num_seqs <= 0 or max_num_batched_tokens <= 0:
            raise ValueError("scheduler limits must be positive")
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.waiting: deque[InferenceRequest] = deque()
        self.running: list[InferenceRequest] = []
        self.finished: list[InferenceRequest] = []

    def add(self, request: InferenceRequest) -> None:
        if request.status != "waiting":
            raise ValueError("only waiting requests can be added")
        self.waiting.append(request)

    def _take_prefill(self) -> tuple[list[InferenceRequest], int]:
        batch: list[InferenceRequest] = []
        used = 0
        while self.waiting and len(batch) < self.max_num_seqs:
            budget_left = self.max_num_batched_tokens - used
            if budget_left <= 0:
                break
            head = self.waiting[0]
            want = head.prompt_remaining
            if want == 0:  # nothing left to prefill: promote without scheduling
                self.waiting.popleft()
                head.status = "running"
                self.running.append(head)
                continue
            if batch and want > budget_left:  # only the first entry may be chunked
                break
            self.waiting.popleft()
            grant = min(want, budget_left)
            head.cached_tokens += grant
            used += grant
            batch.append(head)
            if head.prompt_remaining == 0:
                head.status = "running"
                self.running.append(head)
            else:
                head.status = "waiting"
                self.waiting.appendleft(head)  # the rest goes first next time
        return batch, used

    def schedule(self) -> ScheduleBatch:
        batch, used = self._take_prefill()
        if batch:
            return ScheduleBatch(tuple(batch), "prefill", used)
        decode = tuple(self.running[: self.max_num_seqs])
        if not decode:
            return ScheduleBatch((), "idle", 0)
        return ScheduleBatch(decode, "decode", len(decode))

    def mark_decode_step(self, requests: tuple[InferenceRequest, ...]) -> None:
        stepped = {id(r) for r in requests}
        for request in list(self.running):
            if id(request) not in stepped:
                continue
            request.generated_tokens += 1
            if request.finished:
                request.status = "finished"
                self.running.remove(request)
                self.finished.append(request)
