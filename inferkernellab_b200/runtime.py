"""Model-independent runtime: the hook boundary the attention backends plug into.

Behavioural mirror of the reference's ``InferenceRuntime`` (reference
``src/inferkernellab/runtime.py:10-113``): the same three hook types
(``prefill_fn(request, start, end)``, ``prefill_batch_fn(requests, starts,
ends)``, ``decode_fn(requests)``), the same block-growth rules and the same
order of hook calls and accounting, so a model runner written for the
reference drives this runtime unchanged.

* ``submit`` allocates ``ceil(max(1, prompt) / block_size)`` blocks.
* A prefill step snapshots every request's ``cached_tokens`` before the
  scheduler runs and hands each request its newly scheduled range
  ``[before, after)``.
* A decode step first reserves the slot of the token the step will write
  (``prompt + generated + 1`` tokens of capacity), then calls ``decode_fn``,
  then advances the scheduler and frees the blocks of finished requests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from .scheduler import InferenceRequest, ScheduleBatch, TokenBudgetScheduler

PrefillFn = Callable[[InferenceRequest, int, int], None]
PrefillBatchFn = Callable[[tuple[InferenceRequest, ...], tuple[int, ...], tuple[int, ...]], None]
DecodeFn = Callable[[tuple[InferenceRequest, ...]], None]


@dataclass(frozen=True)
class RuntimeStats:
    waiting: int
    running: int
    finished: int
    free_blocks: int
    used_blocks: int


class InferenceRuntime:
    def __init__(self, cache, scheduler: TokenBudgetScheduler, *,
                 prefill_fn: PrefillFn | None = None,
                 prefill_batch_fn: PrefillBatchFn | None = None,
                 decode_fn: DecodeFn | None = None):
        if prefill_fn is not None and prefill_batch_fn is not None:
            raise ValueError("prefill_fn and prefill_batch_fn are mutually exclusive")
        self.cache = cache
        self.scheduler = scheduler
        self.prefill_fn = prefill_fn
        self.prefill_batch_fn = prefill_batch_fn
        self.decode_fn = decode_fn
        self._requests: dict[int, InferenceRequest] = {}

    def submit(self, request_id: int, prompt_tokens: int, max_new_tokens: int) -> InferenceRequest:
        if request_id in self._requests:
            raise ValueError(f"duplicate request_id: {request_id}")
        request = InferenceRequest(request_id, prompt_tokens, max_new_tokens)
        request.block_table = self.cache.allocate_request(request_id, max(1, prompt_tokens))
        self._requests[request_id] = request
        self.scheduler.add(request)
        return request

    def _ensure_capacity(self, request: InferenceRequest, num_tokens: int) -> None:
        block_size = self.cache.layout.block_size
        short = -(-num_tokens // block_size) - len(request.block_table)
        if short > 0:
            request.block_table.extend(
                self.cache.allocator.allocate(short, owner=request.request_id))

    def _run_prefill(self, batch: ScheduleBatch, before: dict[int, int]) -> None:
        ranges = []
        for request in batch.requests:
            self._ensure_capacity(request, max(1, request.cached_tokens))
            start, end = before[id(request)], request.cached_tokens
            if start < end:
                ranges.append((request, start, end))
        if ranges and self.prefill_batch_fn is not None:
            requests, starts, ends = zip(*ranges)
            self.prefill_batch_fn(tuple(requests), tuple(starts), tuple(ends))
        elif self.prefill_fn is not None:
            for request, start, end in ranges:
                self.prefill_fn(request, start, end)

    def _run_decode(self, batch: ScheduleBatch) -> None:
        for request in batch.requests:
            # Reserve the KV slot that this step's model call will write.
            self._ensure_capacity(request, request.prompt_tokens + request.generated_tokens + 1)
        if self.decode_fn is not None:
            self.decode_fn(batch.requests)
        self.scheduler.mark_decode_step(batch.requests)
        for request in batch.requests:
            if request.finished:
                self.cache.release_request(request.block_table, request_id=request.request_id)
                request.block_table = []

    def step(self) -> ScheduleBatch:
        before = {id(r): r.cached_tokens for r in self._requests.values()}
        batch = self.scheduler.schedule()
        if batch.phase == "prefill":
            self._run_prefill(batch, before)
        elif batch.phase == "decode":
            self._run_decode(batch)
        return batch

    def stats(self) -> RuntimeStats:
        allocator = self.cache.allocator
        return RuntimeStats(
            waiting=len(self.scheduler.waiting),
            running=len(self.scheduler.running),
            finished=len(self.scheduler.finished),
            free_blocks=allocator.num_free_blocks,
            used_blocks=allocator.num_used_blocks,
        )
