"""Synthetic single-layer decoder driven through the paged runtime (b200 backend).

Mirror of the reference's ``SyntheticDecoderConfig`` / ``SyntheticDecodeRunner``
/ ``DecodeRunResult`` (reference ``src/inferkernellab/decode.py:23-592``): the same
seeded weights, the same request and block-table set-up (round-robin repack
with a reserved block between logical rounds), the same prefill/decode hooks
and the same timing and result record -- with attention and KV append on the
sm_100a kernels.  Two things differ by design:

* backend names: ``backend="b200_paged"``, ``append_backend="b200"`` (the only
  ones; there is no CPU or Triton path here);
* metadata: block tables live in a persistent device buffer that grows
  incrementally (like the reference's ``_metadata_tensors``, ``:361-391``) and
  every slot mapping -- prefill ranges and the decode step's new token -- is
  built on the device by one ``build_slot_mapping`` launch instead of a
  per-request host ``slot_mapping`` + ``torch.cat`` (``:330-335,453-462``).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn.functional as F

from .cache import PagedKVCache
from .ops import append_kv, build_slot_mapping, paged_decode_attention
from .runtime import InferenceRuntime
from .scheduler import InferenceRequest, TokenBudgetScheduler

_ATTENTION_BACKENDS = {"b200_paged"}
_APPEND_BACKENDS = {"b200"}


@dataclass(frozen=True)
class SyntheticDecoderConfig:
    vocab_size: int = 256
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 64
    block_size: int = 16
    dtype: torch.dtype = torch.float16
    device: torch.device | str = "cuda"
    seed: int = 0
    backend: str = "b200_paged"
    append_backend: str = "b200"
    max_num_seqs: int = 32
    max_num_batched_tokens: int = 2048
    num_blocks: int | None = None
    prefill_mode: str = "batched"

    def __post_init__(self) -> None:
        device = torch.device(self.device)
        object.__setattr__(self, "device", device)
        if self.vocab_size <= 1:
            raise ValueError("vocab_size must be greater than one")
        if min(self.num_heads, self.num_kv_heads, self.head_dim, self.block_size) <= 0:
            raise ValueError("model and cache dimensions must be positive")
        if self.num_heads % self.num_kv_heads != 0:
            raise ValueError("num_heads must be divisible by num_kv_heads")
        if self.backend not in _ATTENTION_BACKENDS:
            raise ValueError(f"unsupported attention backend: {self.backend}")
        if self.append_backend not in _APPEND_BACKENDS:
            raise ValueError(f"unsupported append backend: {self.append_backend}")
        if self.max_num_seqs <= 0 or self.max_num_batched_tokens <= 0:
            raise ValueError("scheduler limits must be positive")
        if self.prefill_mode not in {"batched", "token"}:
            raise ValueError("prefill_mode must be batched or token")
        if self.num_blocks is not None and self.num_blocks <= 0:
            raise ValueError("num_blocks must be positive when provided")
        if self.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("the b200 backend runs float16 or bfloat16 models")
        if device.type != "cuda":
            raise ValueError(f"{self.backend} requires a CUDA device")
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA was requested but is unavailable")


def _percentile(values: Sequence[float], percentile: float) -> float:
    if not values:
        return 0.0
    ordered = sorted(values)
    position = (len(ordered) - 1) * percentile
    lower, upper = math.floor(position), math.ceil(position)
    if lower == upper:
        return ordered[lower]
    weight = position - lower
    return ordered[lower] * (1.0 - weight) + ordered[upper] * weight


@dataclass(frozen=True)
class DecodeRunResult:
    backend: str
    append_backend: str
    prompt_lengths: tuple[int, ...]
    max_new_tokens: int
    generated_tokens: tuple[tuple[int, ...], ...]
    logits: tuple[torch.Tensor, ...]
    prefill_wall_ms: float
    decode_step_wall_ms: tuple[float, ...]
    ttft_wall_ms: float
    tpot_wall_ms: float
    tokens_per_sec: float
    end_to_end_tokens_per_sec: float
    prefill_device_ms: float
    decode_step_device_ms: tuple[float, ...]
    ttft_device_ms: float
    tpot_device_ms: float
    device_tokens_per_sec: float
    end_to_end_device_tokens_per_sec: float
    peak_memory_allocated_bytes: int
    used_blocks_peak: int
    prefill_step_wall_ms: tuple[float, ...] = ()
    prefill_mode: str = "token"
    prefill_batch_count: int = 0
    prefill_tokens: int = 0
    prefill_padding_tokens: int = 0

    @property
    def decode_step_p50_ms(self) -> float:
        return _percentile(self.decode_step_wall_ms, 0.50)

    @property
    def decode_step_p95_ms(self) -> float:
        return _percentile(self.decode_step_wall_ms, 0.95)

    @property
    def decode_step_device_p50_ms(self) -> float:
        return _percentile(self.decode_step_device_ms, 0.50)

    @property
    def decode_step_device_p95_ms(self) -> float:
        return _percentile(self.decode_step_device_ms, 0.95)

    @property
    def prefill_p50_ms(self) -> float:
        return _percentile(self.prefill_step_wall_ms, 0.50)

    @property
    def prefill_p95_ms(self) -> float:
        return _percentile(self.prefill_step_wall_ms, 0.95)


class DeviceBlockTables:
    """Persistent device copy of every request's block table (+ lengths).

    Rows are request ids; columns fill in as tables grow.  Only the new entries
    of a grown table are copied host-to-device (the reference's incremental
    ``_metadata_tensors``); unused columns stay 0, which the kernels never read.
    """

    def __init__(self, num_requests: int, width: int, device: torch.device):
        self.width = width
        self.tables = torch.zeros((num_requests, width), dtype=torch.int32, device=device)
        self._synced = [0] * num_requests
        self.device = device

    def sync(self, requests: Sequence[InferenceRequest]) -> None:
        for request in requests:
            n = len(request.block_table)
            if n > self.width:
                raise RuntimeError("request block table exceeds preallocated metadata capacity")
            done = self._synced[request.request_id]
            if n > done:
                fresh = torch.tensor(request.block_table[done:n], dtype=torch.int32)
                self.tables[request.request_id, done:n].copy_(fresh, non_blocking=True)
                self._synced[request.request_id] = n

    def rows(self, requests: Sequence[InferenceRequest]) -> torch.Tensor:
        ids = [r.request_id for r in requests]
        if ids == list(range(len(ids))):
            return self.tables[: len(ids)]
        return self.tables.index_select(0, torch.tensor(ids, dtype=torch.long, device=self.device))

    def slots(self, requests, starts, ends, block_size: int, num_blocks: int) -> torch.Tensor:
        """Device-built int32 slots of positions starts[i]..ends[i]-1, packed."""
        total = int(sum(e - s for s, e in zip(starts, ends)))
        meta = torch.tensor([list(starts), list(ends)], dtype=torch.int32).to(self.device,
                                                                             non_blocking=True)
        slots, _ = build_slot_mapping(self.rows(requests), meta[0], meta[1], block_size=block_size,
                                      num_blocks=num_blocks, total_tokens=total,
                                      with_cu_seqlens=False)
        return slots


@dataclass(frozen=True)
class _SyntheticWeights:
    embedding: torch.Tensor
    q_proj: torch.Tensor
    k_proj: torch.Tensor
    v_proj: torch.Tensor
    out_proj: torch.Tensor
    lm_head: torch.Tensor


class SyntheticDecodeRunner:
    """Deterministic single-layer decoder through the paged runtime, b200 kernels."""

    def __init__(self, config: SyntheticDecoderConfig, prompts: Sequence[Sequence[int]],
                 max_new_tokens: int = 16):
        if not prompts:
            raise ValueError("at least one prompt is required")
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        if len(prompts) > config.max_num_seqs:
            raise ValueError("the scheduler max_num_seqs is smaller than the batch")
        self.config = config
        self.device = config.device
        self.max_new_tokens = max_new_tokens
        self.prompts = tuple(tuple(int(t) for t in p) for p in prompts)
        if any(not p for p in self.prompts):
            raise ValueError("prompts must be non-empty")
        if any(t < 0 or t >= config.vocab_size for p in self.prompts for t in p):
            raise ValueError("prompt token is outside the configured vocabulary")
        self.prompt_lengths = tuple(len(p) for p in self.prompts)
        self.weights = self._make_weights()
        bs = config.block_size
        initial = tuple(-(-n // bs) for n in self.prompt_lengths)
        total_blocks = sum(-(-(n + max_new_tokens) // bs) for n in self.prompt_lengths)
        minimum = total_blocks + max(0, max(initial, default=0) - 1)
        num_blocks = config.num_blocks if config.num_blocks is not None else minimum
        if num_blocks < minimum:
            raise ValueError(f"num_blocks is insufficient: requested={num_blocks}, minimum={minimum}")
        self.cache = PagedKVCache(num_blocks, bs, config.num_kv_heads, config.head_dim,
                                  dtype=config.dtype, device=self.device)
        scheduler = TokenBudgetScheduler(max_num_seqs=config.max_num_seqs,
                                         max_num_batched_tokens=config.max_num_batched_tokens)
        self.runtime = InferenceRuntime(
            self.cache, scheduler,
            prefill_fn=self._prefill if config.prefill_mode == "token" else None,
            prefill_batch_fn=self._prefill_batch if config.prefill_mode == "batched" else None,
            decode_fn=self._decode)
        self.requests: list[InferenceRequest] = [
            self.runtime.submit(rid, len(p), max_new_tokens) for rid, p in enumerate(self.prompts)]
        self._reserved_blocks: list[int] = []
        self._repack_initial_block_tables(initial)
        width = max(1, max(-(-(n + max_new_tokens) // bs) for n in self.prompt_lengths))
        self.meta = DeviceBlockTables(len(self.requests), width, self.device)
        self._last_tokens: dict[int, torch.Tensor] = {}
        self._generated: dict[int, list[torch.Tensor]] = {r.request_id: [] for r in self.requests}
        self._step_logits: list[torch.Tensor] = []
        self._has_run = False

    def _repack_initial_block_tables(self, block_counts: Sequence[int]) -> None:
        """Round-robin allocation with a reserved block between rounds (decode.py:245-259)."""
        for request in self.requests:
            self.cache.release_request(list(request.block_table), request_id=request.request_id)
            request.block_table = []
        rounds = max(block_counts, default=0)
        for logical in range(rounds):
            for request, count in zip(self.requests, block_counts):
                if logical < count:
                    request.block_table.extend(
                        self.cache.allocator.allocate(1, owner=request.request_id))
            if logical + 1 < rounds:
                self._reserved_blocks.extend(self.cache.allocator.allocate(1, owner=-1))

    def _make_weights(self) -> _SyntheticWeights:
        """Seeded weights, same draws and scales as the reference (decode.py:261-279)."""
        gen = torch.Generator(device="cpu")
        gen.manual_seed(self.config.seed)
        hidden = self.config.num_heads * self.config.head_dim
        kv = self.config.num_kv_heads * self.config.head_dim

        def w(shape, scale):
            value = torch.randn(shape, generator=gen, dtype=torch.float32) * scale
            return value.to(device=self.device, dtype=self.config.dtype)

        hs = hidden ** -0.5
        return _SyntheticWeights(
            embedding=w((self.config.vocab_size, hidden), 0.02), q_proj=w((hidden, hidden), hs),
            k_proj=w((kv, hidden), hs), v_proj=w((kv, hidden), hs),
            out_proj=w((hidden, hidden), hs), lm_head=w((self.config.vocab_size, hidden), hs))

    def _project_query(self, token_ids: torch.Tensor) -> torch.Tensor:
        hidden = F.embedding(token_ids.to(torch.long), self.weights.embedding)
        return F.linear(hidden, self.weights.q_proj).reshape(-1, self.config.num_heads,
                                                             self.config.head_dim)

    def _project_kv(self, token_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        hidden = F.embedding(token_ids.to(torch.long), self.weights.embedding)
        shape = (-1, self.config.num_kv_heads, self.config.head_dim)
        return (F.linear(hidden, self.weights.k_proj).reshape(shape),
                F.linear(hidden, self.weights.v_proj).reshape(shape))

    def _append_ranges(self, requests, starts, ends, key, value) -> None:
        self.meta.sync(requests)
        slots = self.meta.slots(requests, starts, ends, self.cache.layout.block_size,
                                self.cache.layout.num_blocks)
        append_kv(key, value, self.cache, slots)

    def _prefill(self, request: InferenceRequest, start: int, end: int) -> None:
        ids = torch.tensor(self.prompts[request.request_id][start:end], dtype=torch.long)
        key, value = self._project_kv(ids.to(self.device, non_blocking=True))
        self._append_ranges((request,), (start,), (end,), key, value)

    def _prefill_batch(self, requests, starts, ends) -> None:
        ids = torch.tensor([t for r, s, e in zip(requests, starts, ends)
                            for t in self.prompts[r.request_id][s:e]], dtype=torch.long)
        key, value = self._project_kv(ids.to(self.device, non_blocking=True))
        self._append_ranges(requests, starts, ends, key, value)

    def _decode(self, requests: tuple[InferenceRequest, ...]) -> None:
        current = []
        for request in requests:
            if request.generated_tokens == 0:
                current.append(torch.tensor(self.prompts[request.request_id][-1]).to(self.device))
            else:
                current.append(self._last_tokens[request.request_id])
        tokens = torch.stack(current).to(torch.long)
        query = self._project_query(tokens)
        positions = [r.prompt_tokens + r.generated_tokens for r in requests]
        self.meta.sync(requests)
        lens = torch.tensor(positions, dtype=torch.int32).to(self.device, non_blocking=True)
        attended = paged_decode_attention(query, self.cache, self.meta.rows(requests), lens,
                                          validate_inputs=False)
        hidden = F.linear(attended.reshape(attended.shape[0], -1), self.weights.out_proj)
        logits = F.linear(hidden, self.weights.lm_head)
        next_tokens = logits.argmax(dim=-1)
        next_key, next_value = self._project_kv(next_tokens)
        # The new token goes to position prompt + generated (capacity reserved by the runtime).
        self._append_ranges(requests, positions, [p + 1 for p in positions], next_key, next_value)
        self._step_logits.append(logits.detach().float().cpu())
        for row, request in enumerate(requests):
            token = next_tokens[row]
            self._last_tokens[request.request_id] = token
            self._generated[request.request_id].append(token)

    def _timed_step(self):
        wall_start = time.perf_counter()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        batch = self.runtime.step()
        end.record()
        end.synchronize()
        return batch, (time.perf_counter() - wall_start) * 1000.0, float(start.elapsed_time(end))

    def run(self) -> DecodeRunResult:
        if self._has_run:
            raise RuntimeError("a SyntheticDecodeRunner instance can only be run once")
        self._has_run = True
        torch.cuda.reset_peak_memory_stats(self.device)
        prefill_wall = prefill_dev = 0.0
        prefill_steps: list[float] = []
        decode_wall: list[float] = []
        decode_dev: list[float] = []
        used_peak = self.cache.allocator.num_used_blocks
        try:
            with torch.inference_mode():
                while self.runtime.scheduler.waiting or self.runtime.scheduler.running:
                    batch, wall_ms, dev_ms = self._timed_step()
                    used_peak = max(used_peak, self.cache.allocator.num_used_blocks)
                    if batch.phase == "prefill":
                        prefill_wall += wall_ms
                        prefill_dev += dev_ms
                        prefill_steps.append(wall_ms)
                    elif batch.phase == "decode":
                        decode_wall.append(wall_ms)
                        decode_dev.append(dev_ms)
                    else:
                        raise RuntimeError("scheduler became idle before all requests finished")
        finally:
            if self._reserved_blocks:
                self.cache.allocator.free(self._reserved_blocks, owner=-1)
                self._reserved_blocks = []
        generated = tuple(
            tuple(int(t) for t in torch.stack(self._generated[r.request_id]).cpu().tolist())
            for r in self.requests)
        expected = len(self.requests) * self.max_new_tokens
        if sum(len(t) for t in generated) != expected:
            raise RuntimeError("decoder finished with an unexpected number of generated tokens")
        if not decode_wall:
            raise RuntimeError("decoder produced no decode steps")
        total_wall = prefill_wall + sum(decode_wall)
        total_dev = prefill_dev + sum(decode_dev)
        count = float(expected)
        return DecodeRunResult(
            backend=self.config.backend, append_backend=self.config.append_backend,
            prompt_lengths=self.prompt_lengths, max_new_tokens=self.max_new_tokens,
            generated_tokens=generated, logits=tuple(self._step_logits),
            prefill_wall_ms=prefill_wall, prefill_step_wall_ms=tuple(prefill_steps),
            prefill_mode=self.config.prefill_mode, prefill_batch_count=len(prefill_steps),
            prefill_tokens=sum(self.prompt_lengths), prefill_padding_tokens=0,
            decode_step_wall_ms=tuple(decode_wall), ttft_wall_ms=prefill_wall + decode_wall[0],
            tpot_wall_ms=sum(decode_wall) / len(decode_wall),
            tokens_per_sec=count / (sum(decode_wall) / 1000.0),
            end_to_end_tokens_per_sec=count / (total_wall / 1000.0),
            prefill_device_ms=prefill_dev, decode_step_device_ms=tuple(decode_dev),
            ttft_device_ms=prefill_dev + decode_dev[0],
            tpot_device_ms=sum(decode_dev) / len(decode_dev),
            device_tokens_per_sec=count / (sum(decode_dev) / 1000.0),
            end_to_end_device_tokens_per_sec=count / (total_dev / 1000.0),
            peak_memory_allocated_bytes=int(torch.cuda.max_memory_allocated(self.device)),
            used_blocks_peak=used_peak)
