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

Prefix sharing (not in the reference; ``prefix_cache.py``): with a
``PrefixCache`` and the prompt's token ids at ``submit``, a request gets its
blocks when it first reaches the prefill budget instead of at ``submit``: its
table starts with the cached blocks of its longest cached prefix, its
``cached_tokens`` starts after them (so the prefill hooks only see the rest),
and once its prompt is prefilled its full prompt blocks are indexed for later
requests.  When the pool runs short the runtime evicts unused cached blocks
before it gives up.  Without a ``PrefixCache`` nothing changes.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from .prefix_cache import PrefixCache
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
                 decode_fn: DecodeFn | None = None,
                 prefix_cache: PrefixCache | None = None):
        if prefill_fn is not None and prefill_batch_fn is not None:
            raise ValueError("prefill_fn and prefill_batch_fn are mutually exclusive")
        self.cache = cache
        self.scheduler = scheduler
        self.prefill_fn = prefill_fn
        self.prefill_batch_fn = prefill_batch_fn
        self.decode_fn = decode_fn
        self.prefix_cache = prefix_cache
        self._requests: dict[int, InferenceRequest] = {}
        self._unplaced: dict[int, tuple[int, ...]] = {}  # prompt ids of requests without blocks
        self._prompt_ids: dict[int, tuple[int, ...]] = {}
        self.prefix_cached_tokens = 0  # prompt tokens served from shared blocks

    def submit(self, request_id: int, prompt_tokens: int, max_new_tokens: int,
               token_ids=None) -> InferenceRequest:
        if request_id in self._requests:
            raise ValueError(f"duplicate request_id: {request_id}")
        request = InferenceRequest(request_id, prompt_tokens, max_new_tokens)
        if self.prefix_cache is not None and token_ids is not None:
            ids = tuple(int(t) for t in token_ids)
            if len(ids) != prompt_tokens:
                raise ValueError("token_ids must hold prompt_tokens entries")
            self._unplaced[request_id] = ids  # blocks come when the request is scheduled
            self._prompt_ids[request_id] = ids
        else:
            request.block_table = self.cache.allocate_request(request_id, max(1, prompt_tokens))
        self._requests[request_id] = request
        self.scheduler.add(request)
        return request

    def _allocate(self, count: int, owner: int) -> list[int]:
        allocator = self.cache.allocator
        if self.prefix_cache is not None and count > allocator.num_free_blocks:
            self.prefix_cache.evict(count - allocator.num_free_blocks)
        return allocator.allocate(count, owner=owner)

    def _place(self) -> None:
        """Give blocks to the waiting requests the next prefill batch can take: the
        cached blocks of their longest cached prefix first, then new ones."""
        budget = self.scheduler.max_num_batched_tokens
        block_size = self.cache.layout.block_size
        for count, request in enumerate(self.scheduler.waiting):
            if budget <= 0 or count >= self.scheduler.max_num_seqs:
                break
            ids = self._unplaced.get(request.request_id)
            if ids is None:
                want = request.prompt_remaining
            else:
                want = request.prompt_tokens - len(self.prefix_cache.lookup(ids)) * block_size
            if count > 0 and want > budget:  # the scheduler only chunks the head request
                break
            if ids is not None:
                del self._unplaced[request.request_id]
                shared = self.prefix_cache.match(ids)
                request.cached_tokens = len(shared) * block_size
                self.prefix_cached_tokens += request.cached_tokens
                need = -(-max(1, request.prompt_tokens) // block_size) - len(shared)
                request.block_table = shared + self._allocate(need, request.request_id)
            budget -= want

    def _ensure_capacity(self, request: InferenceRequest, num_tokens: int) -> None:
        block_size = self.cache.layout.block_size
        short = -(-num_tokens // block_size) - len(request.block_table)
        if short > 0:
            request.block_table.extend(self._allocate(short, request.request_id))

    def _run_prefill(self, batch: ScheduleBatch, before: dict[int, int]) -> None:
        for request in batch.requests:  # scheduled before placement: plain blocks below
            self._unplaced.pop(request.request_id, None)
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
        if self.prefix_cache is not None:
            for request, _, end in ranges:
                ids = self._prompt_ids.get(request.request_id)
                if ids is not None and end == request.prompt_tokens:
                    self.prefix_cache.insert(ids, request.block_table, end)

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
                self._prompt_ids.pop(request.request_id, None)

    def step(self) -> ScheduleBatch:
        if self._unplaced:
            self._place()
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
