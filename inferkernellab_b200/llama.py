"""Transformers Llama decoder over the paged KV cache, on the b200 kernels.

Mirror of the reference's ``LlamaPagedDecodeRunner`` / ``LlamaPagedRunResult``
(reference ``src/inferkernellab/hf_benchmark.py:88-695``) for backend
``"b200_paged"`` / append ``"b200"``.  The layer computes what the reference's
Transformers modules compute, with the launches cut down:

* the q/k/v projections run as one GEMM over a packed ``[q | k | v]`` weight
  and gate/up as one GEMM over ``[gate | up]``; the model's own ``Linear``
  weights are re-pointed at views of the packed tensors, so the model keeps
  working unchanged and no weight memory is duplicated;
* every ``LlamaRMSNorm`` (with the residual add in front of it) is one
  ``add_rmsnorm`` launch and ``act_fn(gate) * up`` one ``silu_mul`` launch,
  both rounding like the torch ops they replace;
* o_proj, down_proj, the embedding, the rotary table and lm_head are the
  model's own modules.

Logits therefore differ from the eager model only through attention and GEMM
summation order.  Attention-side work is on the sm_100a kernels:

* batched prefill is *packed*: the scheduled ranges of a budget batch are
  concatenated (no padding rows, unlike the reference's ``_prefill_batch``
  ``:522-547``), slots and ``cu_seqlens`` come from one device
  ``build_slot_mapping`` launch per batch and the causal attention runs in
  ``paged_prefill_attention_varlen``;
* decode runs ``paged_decode_attention_append``: the attention launch itself
  applies the rotary embedding to q and to the new k and writes the new K/V
  into the cache (bit-identical to the reference's ``_apply_rotary`` + append);
  the step's slots and lengths are built once and reused by all layers;
* prefill runs one ``rope_append_kv`` launch per layer (rotary on q and k, K/V
  into the cache) before the prefill attention;
* ``cuda_graph=True`` captures the whole decode step (every layer, lm_head)
  into one CUDA graph with device-resident metadata and replays it each step,
  instead of re-launching ~35 kernels per layer from Python every step as the
  reference runner does.

Multi-GPU: requests are partitioned over ranks by the caller; each rank runs its
own runner (own block pool) and passes ``token_exchange`` -- e.g.
``allgather_token_exchange`` -- which all-gathers the sampled token ids of every
decode step over NCCL (the only collective on this path).
"""

from __future__ import annotations

import math
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

import torch

from .cache import PagedKVCache
from .decode import DeviceBlockTables, _percentile
from .prefix_cache import PrefixCache
from .ops import (
    add_rmsnorm,
    build_slot_mapping,
    paged_decode_attention,
    paged_decode_attention_append,
    paged_prefill_attention_varlen,
    rope_append_kv,
    silu_mul,
)
from .runtime import InferenceRuntime
from .scheduler import InferenceRequest, TokenBudgetScheduler


@dataclass(frozen=True)
class LlamaPagedRunResult:
    backend: str
    append_backend: str
    prompt_lengths: tuple[int, ...]
    max_new_tokens: int
    generated_tokens: tuple[tuple[int, ...], ...]
    prompt_logits: torch.Tensor
    decode_logits: tuple[torch.Tensor, ...]
    prefill_wall_ms: float
    decode_step_wall_ms: tuple[float, ...]
    ttft_wall_ms: float
    tpot_wall_ms: float
    peak_memory_allocated_bytes: int
    peak_kv_memory_bytes: int
    used_blocks_peak: int
    cache_released: bool
    prefill_step_wall_ms: tuple[float, ...] = ()
    prefill_mode: str = "token"
    prefill_batch_count: int = 0
    prefill_tokens: int = 0
    prefill_padding_tokens: int = 0
    token_logprobs: tuple[tuple[float, ...], ...] = ()
    sampling_logprobs: tuple[tuple[float, ...], ...] = ()
    finish_reasons: tuple[str, ...] = ()
    prefix_cached_tokens: int = 0  # prompt tokens served from shared blocks (prefix_caching)

    @property
    def decode_p50_ms(self) -> float:
        return _percentile(self.decode_step_wall_ms, 0.50)

    @property
    def decode_p95_ms(self) -> float:
        return _percentile(self.decode_step_wall_ms, 0.95)

    @property
    def prefill_p50_ms(self) -> float:
        return _percentile(self.prefill_step_wall_ms, 0.50)

    @property
    def prefill_p95_ms(self) -> float:
        return _percentile(self.prefill_step_wall_ms, 0.95)


TokenExchange = Callable[[torch.Tensor], None]


class LlamaPagedDecodeRunner:
    """Run a Transformers Llama one token at a time over the paged cache (b200 backend)."""

    def __init__(self, model: Any, prompts: Sequence[Sequence[int]], *, max_new_tokens: int,
                 backend: str = "b200_paged", block_size: int = 16, append_backend: str = "b200",
                 max_num_batched_tokens: int = 2048, prefill_mode: str = "batched",
                 temperature: float = 0.0, top_p: float = 1.0, seed: int = 2026,
                 eos_token_ids: Sequence[int] | None = None,
                 token_exchange: TokenExchange | None = None, collect_logits: bool = True,
                 cuda_graph: bool = False, prefix_caching: bool = False,
                 sync_steps: bool = True, fused_decode: bool | str = "auto"):
        if not prompts:
            raise ValueError("at least one prompt is required")
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        if block_size <= 0 or max_num_batched_tokens <= 0:
            raise ValueError("block-size and max-num-batched-tokens must be positive")
        if backend != "b200_paged":
            raise ValueError(f"unsupported backend: {backend}")
        if append_backend != "b200":
            raise ValueError(f"unsupported append backend: {append_backend}")
        if prefill_mode not in {"batched", "token"}:
            raise ValueError("prefill_mode must be batched or token")
        if (not math.isfinite(temperature) or temperature < 0 or not math.isfinite(top_p)
                or not 0 < top_p <= 1):
            raise ValueError("temperature must be non-negative and top_p must be in (0, 1]")
        self.model = model
        param = next(model.parameters())
        self.device, self.dtype = param.device, param.dtype
        if self.device.type != "cuda":
            raise ValueError("the b200 backend needs the model on a CUDA device")
        self.prompts = tuple(tuple(int(t) for t in p) for p in prompts)
        if any(not p for p in self.prompts):
            raise ValueError("prompts must be non-empty")
        vocab = int(model.config.vocab_size)
        if any(t < 0 or t >= vocab for p in self.prompts for t in p):
            raise ValueError("prompt token is outside the configured vocabulary")
        self.backend, self.append_backend, self.prefill_mode = backend, append_backend, prefill_mode
        self.max_new_tokens = max_new_tokens
        self.temperature, self.top_p = temperature, top_p
        self.eos_token_ids = set(eos_token_ids or ())
        if any(t < 0 or t >= vocab for t in self.eos_token_ids):
            raise ValueError("EOS token id is outside the configured vocabulary")
        self.token_exchange = token_exchange
        self.collect_logits = collect_logits
        self.cuda_graph = cuda_graph
        # sync_steps=True times every step to its device completion (the
        # reference's per-step wall clock); False lets the host prepare the next
        # step while the device still runs this one (throughput measurement; the
        # per-step figures then split the same total differently).
        self.sync_steps = sync_steps
        # fused_decode: rotary + append inside the attention launch
        # (paged_decode_attention_append); False: rope_append_kv, then
        # paged_decode_attention (two launches per layer, same results).  "auto"
        # fuses when the step has at most two (request, kv head) segments per
        # resident decode CTA: the fused kernel stages every segment's rotated
        # q before it streams, which pays off for few long segments (one B200:
        # 193.3 vs 196.2 us at 64 requests of ctx U[1,8192]) but not for many
        # short ones (122.8 vs 119.1 us at 256 requests of ctx ~540).
        if fused_decode not in (True, False, "auto"):
            raise ValueError("fused_decode must be True, False or 'auto'")
        self.fused_decode = fused_decode
        self._host_tokens = torch.empty(len(prompts), dtype=torch.long, pin_memory=True)
        self._tokens_ready = torch.cuda.Event()
        self._graph: _DecodeGraph | None = None
        self.prompt_lengths = tuple(len(p) for p in self.prompts)
        cfg = model.config
        self.num_layers = int(cfg.num_hidden_layers)
        self.num_heads = int(cfg.num_attention_heads)
        self.num_kv_heads = int(cfg.num_key_value_heads)
        self.head_dim = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // self.num_heads)
        if self.num_heads % self.num_kv_heads != 0:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        total_blocks = sum(-(-(n + max_new_tokens) // block_size) for n in self.prompt_lengths)
        self.cache = PagedKVCache(total_blocks, block_size, self.num_kv_heads, self.head_dim,
                                  num_layers=self.num_layers, dtype=self.dtype, device=self.device)
        scheduler = TokenBudgetScheduler(max_num_seqs=len(self.prompts),
                                         max_num_batched_tokens=max_num_batched_tokens)
        self.prefix_cache = PrefixCache(self.cache.allocator, block_size) if prefix_caching else None
        self.runtime = InferenceRuntime(
            self.cache, scheduler,
            prefill_fn=self._prefill if prefill_mode == "token" else None,
            prefill_batch_fn=self._prefill_batch if prefill_mode == "batched" else None,
            decode_fn=self._decode, prefix_cache=self.prefix_cache)
        self.requests = [self.runtime.submit(rid, len(p), max_new_tokens,
                                             token_ids=p if prefix_caching else None)
                         for rid, p in enumerate(self.prompts)]
        width = max(1, max(-(-(n + max_new_tokens) // block_size) for n in self.prompt_lengths))
        self.meta = DeviceBlockTables(len(self.requests), width, self.device)
        self._prompt_logits: dict[int, torch.Tensor] = {}
        self._next_logits: dict[int, torch.Tensor] = {}
        self._batch_logits: tuple[tuple[int, ...], torch.Tensor] | None = None
        self._decode_logits: list[torch.Tensor] = []
        self._generated: dict[int, list[int]] = {r.request_id: [] for r in self.requests}
        self._token_logprobs: dict[int, list[float]] = {r.request_id: [] for r in self.requests}
        self._sampling_logprobs: dict[int, list[float]] = {r.request_id: [] for r in self.requests}
        self._finish_reasons = {r.request_id: "length" for r in self.requests}
        self._generators = {}
        for r in self.requests:
            gen = torch.Generator(device=self.device)
            gen.manual_seed(seed + r.request_id)
            self._generators[r.request_id] = gen
        self._has_run = False
        self._pack_weights()

    # ------------------------------------------------------------------ layers
    def _pack_weights(self) -> None:
        """Pack each layer's q/k/v and gate/up weights into one tensor each.

        The model's ``Linear`` modules are re-pointed at views of the packed
        tensors (same values), so the eager model still works and the weights
        are not held twice."""
        act = getattr(self.model.config, "hidden_act", "silu")
        if act != "silu":
            raise ValueError(f"the b200 runner supports SiLU-gated MLPs, not {act!r}")
        self._qkv, self._gate_up = [], []
        for layer in self.model.model.layers:
            attn, mlp = layer.self_attn, layer.mlp
            self._qkv.append(_pack_linears((attn.q_proj, attn.k_proj, attn.v_proj)))
            self._gate_up.append(_pack_linears((mlp.gate_proj, mlp.up_proj)))

    def _forward(self, token_ids: torch.Tensor, positions: torch.Tensor, attend) -> torch.Tensor:
        """Shared layer loop on a flat token batch ``[N]``; returns the final-norm
        hidden ``[N, H]``.

        Per layer: one q|k|v GEMM, ``attend(layer, q, k, v, cos, sin)`` (rotary,
        K/V append and attention; q/k/v are views of the GEMM output), o_proj,
        ``add_rmsnorm`` (residual add + post-attention norm), one gate|up GEMM,
        ``silu_mul``, down_proj and ``add_rmsnorm`` into the next layer's input
        norm."""
        n = token_ids.shape[0]
        inner = self.model.model
        hidden = inner.embed_tokens(token_ids.to(torch.long))
        cos, sin = inner.rotary_emb(hidden.unsqueeze(0), positions.view(1, -1))
        cos, sin = cos[0], sin[0]
        layers = inner.layers
        qd = self.num_heads * self.head_dim
        kvd = self.num_kv_heads * self.head_dim
        normed, residual = add_rmsnorm(None, hidden, *_norm_args(layers[0].input_layernorm))
        for index, layer in enumerate(layers):
            weight, bias = self._qkv[index]
            qkv = torch.nn.functional.linear(normed, weight, bias)
            q = qkv[:, :qd].view(n, self.num_heads, self.head_dim)
            k = qkv[:, qd:qd + kvd].view(n, self.num_kv_heads, self.head_dim)
            v = qkv[:, qd + kvd:].view(n, self.num_kv_heads, self.head_dim)
            attended = attend(index, q, k, v, cos, sin)
            out = layer.self_attn.o_proj(attended.reshape(n, qd))
            normed, residual = add_rmsnorm(out, residual,
                                           *_norm_args(layer.post_attention_layernorm))
            weight, bias = self._gate_up[index]
            act = silu_mul(torch.nn.functional.linear(normed, weight, bias))
            out = layer.mlp.down_proj(act)
            following = layers[index + 1].input_layernorm if index + 1 < len(layers) else inner.norm
            normed, residual = add_rmsnorm(out, residual, *_norm_args(following))
        return normed

    def _decode_body(self, token_ids: torch.Tensor, positions: torch.Tensor,
                     tables: torch.Tensor) -> torch.Tensor:
        """One decode step from device tensors only (capturable in a CUDA graph).

        ``positions`` int32 ``[B]``: where each request's new token goes; the
        step appends its K/V there and attends over ``positions + 1`` tokens."""
        bs, nb = self.cache.layout.block_size, self.cache.layout.num_blocks
        lens = positions + 1
        slots, _ = build_slot_mapping(tables, positions, lens, block_size=bs, num_blocks=nb,
                                      total_tokens=positions.shape[0], with_cu_seqlens=False)

        fused = self.fused_decode
        if fused == "auto":
            fused = positions.shape[0] * self.num_kv_heads <= 2 * _decode_ctas(self.device)

        def attend(layer, q, k, v, cos, sin):
            if not fused:
                q = rope_append_kv(q, k, v, cos, sin, self.cache, slots, layer=layer)
                return paged_decode_attention(q, self.cache, tables, lens, layer=layer,
                                              validate_inputs=False)
            return paged_decode_attention_append(q, k, v, self.cache, tables, lens, slots,
                                                 cos=cos, sin=sin, layer=layer)

        hidden = self._forward(token_ids, positions.to(torch.long), attend)
        return self.model.lm_head(hidden)

    def _forward_decode(self, token_ids, requests, positions: Sequence[int]) -> torch.Tensor:
        self.meta.sync(requests)
        pos = torch.tensor(list(positions), dtype=torch.int32).to(self.device, non_blocking=True)
        return self._decode_body(token_ids, pos, self.meta.rows(requests))

    def _forward_prefill_packed(self, requests, starts, ends) -> torch.Tensor:
        """Packed ranges of one budget batch; returns hidden of every token ``[sum T, H]``."""
        self.meta.sync(requests)
        bs, nb = self.cache.layout.block_size, self.cache.layout.num_blocks
        meta = torch.tensor([list(starts), list(ends)], dtype=torch.int32).to(self.device,
                                                                            non_blocking=True)
        total = int(sum(e - s for s, e in zip(starts, ends)))
        tables = self.meta.rows(requests)
        slots, cu = build_slot_mapping(tables, meta[0], meta[1], block_size=bs, num_blocks=nb,
                                       total_tokens=total)
        ids = torch.tensor([t for r, s, e in zip(requests, starts, ends)
                            for t in self.prompts[r.request_id][s:e]], dtype=torch.long)
        pos = torch.tensor([p for s, e in zip(starts, ends) for p in range(s, e)],
                           dtype=torch.long)
        ids = ids.to(self.device, non_blocking=True)
        pos = pos.to(self.device, non_blocking=True)

        def attend(layer, q, k, v, cos, sin):
            q = rope_append_kv(q, k, v, cos, sin, self.cache, slots, layer=layer)
            return paged_prefill_attention_varlen(q, self.cache, tables, cu, meta[0], meta[1],
                                                  layer=layer)

        return self._forward(ids, pos, attend)

    # ------------------------------------------------------------------- hooks
    def _prefill(self, request: InferenceRequest, start: int, end: int) -> None:
        hidden = self._forward_prefill_packed((request,), (start,), (end,))
        if end == len(self.prompts[request.request_id]):
            logits = self.model.lm_head(hidden[-1:])[0].detach()
            self._prompt_logits[request.request_id] = logits
            self._next_logits[request.request_id] = logits

    def _prefill_batch(self, requests, starts, ends) -> None:
        lengths = [int(e) - int(s) for s, e in zip(starts, ends)]
        if not requests or any(n <= 0 for n in lengths):
            raise ValueError("prefill batch must contain non-empty ranges")
        hidden = self._forward_prefill_packed(requests, starts, ends)
        last, rows, offset = [], [], 0
        for request, end, n in zip(requests, ends, lengths):
            offset += n
            if end == len(self.prompts[request.request_id]):
                last.append(offset - 1)
                rows.append(request.request_id)
        if last:
            logits = self.model.lm_head(hidden[torch.tensor(last, device=self.device)]).detach()
            for rid, row in zip(rows, logits):
                self._prompt_logits[rid] = row
                self._next_logits[rid] = row

    def _sample_token(self, logits: torch.Tensor, generator: torch.Generator):
        """Temperature / top-p sampling as the reference does (hf_benchmark.py:581-605)."""
        values = logits.float()
        if self.temperature > 0:
            values = values / self.temperature
        policy_logprobs = torch.log_softmax(values, dim=-1)
        if self.top_p < 1.0:
            sorted_logits, sorted_indices = torch.sort(values, descending=True)
            sorted_probs = torch.softmax(sorted_logits, dim=-1)
            remove = sorted_probs.cumsum(dim=-1) - sorted_probs > self.top_p
            sorted_logits = sorted_logits.masked_fill(remove, float("-inf"))
            values = torch.full_like(values, float("-inf")).scatter(-1, sorted_indices,
                                                                     sorted_logits)
        log_probs = torch.log_softmax(values, dim=-1)
        if self.temperature == 0:
            token = values.argmax(dim=-1)
        else:
            token = torch.multinomial(log_probs.exp(), num_samples=1, generator=generator).squeeze(-1)
        return (token, policy_logprobs.gather(-1, token.view(1)).squeeze(0),
                log_probs.gather(-1, token.view(1)).squeeze(0))

    def _logits_for(self, requests) -> torch.Tensor:
        """``[B, V]`` next-token logits of ``requests``: the previous decode step's
        batch tensor as is when the batch is unchanged, else gathered per request."""
        ids = tuple(r.request_id for r in requests)
        if self._batch_logits is not None:
            batch_ids, logits = self._batch_logits
            if batch_ids == ids:
                return logits
            for row, rid in enumerate(batch_ids):
                self._next_logits[rid] = logits[row].clone()
            self._batch_logits = None
        return torch.stack([self._next_logits[rid] for rid in ids], dim=0)

    def _decode(self, requests: tuple[InferenceRequest, ...]) -> None:
        used = self._logits_for(requests)
        if self.collect_logits:
            self._decode_logits.append(used.detach().float().cpu())
        sampled = None
        if self.temperature == 0 and not self.eos_token_ids:
            next_tokens = used.argmax(dim=-1).to(torch.long)
        else:
            sampled = [self._sample_token(used[i], self._generators[r.request_id])
                       for i, r in enumerate(requests)]
            next_tokens = torch.stack([s[0] for s in sampled]).to(torch.long)
        if self.token_exchange is not None:
            self.token_exchange(next_tokens)
        # Copy the sampled ids out before the step's model work is queued, so the
        # host waits for the sampling only, not for the whole forward pass.
        host_tokens = self._host_tokens[:len(requests)]
        host_tokens.copy_(next_tokens, non_blocking=True)
        self._tokens_ready.record()
        positions = [r.prompt_tokens + r.generated_tokens for r in requests]
        ids = [r.request_id for r in requests]
        if self.cuda_graph and ids == list(range(len(ids))):
            if self._graph is None or self._graph.batch != len(ids):
                self._graph = _DecodeGraph(self, requests, next_tokens, positions)
            self.meta.sync(requests)
            next_logits = self._graph.replay(next_tokens, positions)
        else:
            next_logits = self._forward_decode(next_tokens, requests, positions)
        self._tokens_ready.synchronize()
        tokens = host_tokens.tolist()
        for row, request in enumerate(requests):
            token = int(tokens[row])
            self._generated[request.request_id].append(token)
            if sampled is not None:
                self._token_logprobs[request.request_id].append(float(sampled[row][1].item()))
                self._sampling_logprobs[request.request_id].append(float(sampled[row][2].item()))
            if token in self.eos_token_ids:
                self._finish_reasons[request.request_id] = "eos"
                request.max_new_tokens = request.generated_tokens + 1
        self._batch_logits = (tuple(ids), next_logits.detach())

    # --------------------------------------------------------------------- run
    def _timed_step(self):
        started = time.perf_counter()
        batch = self.runtime.step()
        if self.sync_steps or batch.phase != "decode":
            torch.cuda.synchronize(self.device)
        return batch, (time.perf_counter() - started) * 1000

    def run(self) -> LlamaPagedRunResult:
        if self._has_run:
            raise RuntimeError("a LlamaPagedDecodeRunner instance can only be run once")
        self._has_run = True
        torch.cuda.reset_peak_memory_stats(self.device)
        prefill_ms, prefill_steps, decode_ms = 0.0, [], []
        used_peak = self.cache.allocator.num_used_blocks
        with torch.inference_mode():
            while self.runtime.scheduler.waiting or self.runtime.scheduler.running:
                batch, elapsed = self._timed_step()
                used_peak = max(used_peak, self.cache.allocator.num_used_blocks)
                if batch.phase == "prefill":
                    prefill_ms += elapsed
                    prefill_steps.append(elapsed)
                elif batch.phase == "decode":
                    decode_ms.append(elapsed)
                else:
                    raise RuntimeError("scheduler became idle before all requests finished")
            if decode_ms and not self.sync_steps:  # the last step's device work
                started = time.perf_counter()
                torch.cuda.synchronize(self.device)
                decode_ms[-1] += (time.perf_counter() - started) * 1000
        if self.prefix_cache is not None:
            self.prefix_cache.clear()  # the index holds one reference per cached block
        cache_released = self.cache.allocator.num_used_blocks == 0
        if len(self._prompt_logits) != len(self.requests):
            raise RuntimeError("prefill did not produce one final logits tensor per request")
        generated = tuple(tuple(self._generated[r.request_id]) for r in self.requests)
        if any(not t or len(t) > self.max_new_tokens for t in generated):
            raise RuntimeError("decoder finished with an invalid generated sequence length")
        element = torch.tensor([], dtype=self.dtype).element_size()
        lay = self.cache.layout
        peak_kv = (used_peak * lay.block_size * lay.num_layers * lay.num_kv_heads * lay.head_dim
                   * 2 * element)
        return LlamaPagedRunResult(
            backend=self.backend, append_backend=self.append_backend,
            prompt_lengths=self.prompt_lengths, max_new_tokens=self.max_new_tokens,
            generated_tokens=generated,
            prompt_logits=torch.stack([self._prompt_logits[r.request_id]
                                       for r in self.requests]).float().cpu(),
            decode_logits=tuple(self._decode_logits), prefill_wall_ms=prefill_ms,
            prefill_step_wall_ms=tuple(prefill_steps), prefill_mode=self.prefill_mode,
            prefill_batch_count=len(prefill_steps), prefill_tokens=sum(self.prompt_lengths),
            prefill_padding_tokens=0,
            token_logprobs=tuple(tuple(self._token_logprobs[r.request_id]) for r in self.requests),
            sampling_logprobs=tuple(tuple(self._sampling_logprobs[r.request_id])
                                    for r in self.requests),
            finish_reasons=tuple(self._finish_reasons[r.request_id] for r in self.requests),
            decode_step_wall_ms=tuple(decode_ms), ttft_wall_ms=prefill_ms + decode_ms[0],
            tpot_wall_ms=sum(decode_ms) / len(decode_ms),
            peak_memory_allocated_bytes=int(torch.cuda.max_memory_allocated(self.device)),
            peak_kv_memory_bytes=peak_kv, used_blocks_peak=used_peak,
            cache_released=cache_released and self.cache.allocator.num_used_blocks == 0,
            prefix_cached_tokens=self.runtime.prefix_cached_tokens)


class _DecodeGraph:
    """The whole decode step of a fixed batch (all layers + lm_head) as one CUDA graph.

    Inputs live in static device buffers: the token ids and positions are
    copied in before each replay, the block tables are the runner's persistent
    device table rows (grown in place by ``DeviceBlockTables.sync``).  The
    slots and lengths are derived on the device inside the graph.  Capture
    runs on a side stream after one eager warm-up step that sets up the
    kernels' workspaces, as CUDA graph capture requires.
    """

    def __init__(self, runner: "LlamaPagedDecodeRunner", requests, tokens: torch.Tensor,
                 positions: Sequence[int]):
        self.batch = len(requests)
        device = runner.device
        runner.meta.sync(requests)
        self.tables = runner.meta.rows(requests)
        self.tokens = tokens.detach().clone().to(torch.long)
        self.positions = torch.tensor(list(positions), dtype=torch.int32, device=device)
        # Two pinned staging buffers, used in turn: with the runner's sync_steps=False
        # the host writes step N+1's positions while step N's copy may still be
        # queued; it last used this buffer two steps ago, whose copy has run (the
        # host has since waited for a later step's sampled tokens).
        self._host_pos = [torch.empty(self.batch, dtype=torch.int32, pin_memory=True)
                          for _ in range(2)]
        self._turn = 0
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            # Warm-up (eager) on the capture stream; it writes the same K/V the
            # replay below rewrites, so it has no effect on results.
            runner._decode_body(self.tokens, self.positions, self.tables)
        stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.logits = runner._decode_body(self.tokens, self.positions, self.tables)
        torch.cuda.current_stream(device).wait_stream(stream)

    def replay(self, tokens: torch.Tensor, positions: Sequence[int]) -> torch.Tensor:
        host = self._host_pos[self._turn]
        self._turn ^= 1
        host.copy_(torch.tensor(list(positions), dtype=torch.int32))
        self.positions.copy_(host, non_blocking=True)
        self.tokens.copy_(tokens)
        self.graph.replay()
        return self.logits


# ------------------------------------------------------------------ helpers

def _decode_ctas(device: torch.device) -> int:
    """Resident CTAs of the decode kernel on ``device`` (two per SM)."""
    return 2 * torch.cuda.get_device_properties(device).multi_processor_count


def _pack_linears(modules) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Concatenate ``Linear`` weights (and biases) along the output dimension and
    re-point each module's parameters at its slice of the packed tensors."""
    biases = [m.bias for m in modules]
    if any(b is None for b in biases) and not all(b is None for b in biases):
        raise ValueError("cannot pack projections where only some have a bias")
    with torch.no_grad():
        weight = torch.cat([m.weight.detach() for m in modules], dim=0).contiguous()
        bias = None if biases[0] is None else torch.cat([b.detach() for b in biases]).contiguous()
        offset = 0
        for m in modules:
            rows = m.weight.shape[0]
            m.weight = torch.nn.Parameter(weight[offset:offset + rows], requires_grad=False)
            if bias is not None:
                m.bias = torch.nn.Parameter(bias[offset:offset + rows], requires_grad=False)
            offset += rows
    return weight, bias


def _norm_args(norm) -> tuple[torch.Tensor, float]:
    """(weight, eps) of a ``LlamaRMSNorm``."""
    eps = getattr(norm, "variance_epsilon", None)
    if eps is None:
        eps = getattr(norm, "eps")
    return norm.weight, float(eps)


def load_random_llama(*, vocab_size: int, hidden_size: int, intermediate_size: int,
                      num_layers: int, num_attention_heads: int, num_kv_heads: int,
                      max_position_embeddings: int, rope_theta: float, seed: int,
                      device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16,
                      init_on_device: bool = False):
    """Random-init ``LlamaForCausalLM`` like the reference's ``_load_model`` (hf_benchmark.py:698-745).

    ``init_on_device=False`` reproduces the reference bit for bit (CPU float32
    init after ``torch.manual_seed(seed)``, then cast); ``True`` initialises on
    the GPU in ``dtype`` (same N(0, 0.02) scheme, different random stream),
    which is the practical way to build an 8B-parameter model.
    """
    from transformers import LlamaConfig, LlamaForCausalLM

    config = LlamaConfig(vocab_size=vocab_size, hidden_size=hidden_size,
                         intermediate_size=intermediate_size, num_hidden_layers=num_layers,
                         num_attention_heads=num_attention_heads, num_key_value_heads=num_kv_heads,
                         max_position_embeddings=max_position_embeddings, rope_theta=rope_theta,
                         attention_bias=False, mlp_bias=False, tie_word_embeddings=False)
    config._attn_implementation = "eager"
    torch.manual_seed(seed)
    if init_on_device:
        previous = torch.get_default_dtype()
        torch.set_default_dtype(dtype)
        try:
            with torch.device(device):
                model = LlamaForCausalLM(config)
        finally:
            torch.set_default_dtype(previous)
    else:
        model = LlamaForCausalLM(config)
    model.config._attn_implementation = "eager"
    model = model.to(device=device, dtype=dtype).eval()
    for parameter in model.parameters():
        parameter.requires_grad_(False)
    return model


def eager_reference_logits(model, prompts, generated_tokens) -> tuple[torch.Tensor, ...]:
    """Full-sequence eager forward per step, the reference's oracle (hf_benchmark.py:764-779)."""
    device = next(model.parameters()).device
    outputs = []
    for step in range(len(generated_tokens[0]) + 1):
        with torch.inference_mode():
            rows = []
            for prompt, tokens in zip(prompts, generated_tokens):
                sequence = tuple(prompt) + tuple(tokens[:step])
                ids = torch.tensor([sequence], dtype=torch.long, device=device)
                rows.append(model(ids, use_cache=False, return_dict=True).logits[0, -1, :])
        outputs.append(torch.stack(rows).float().cpu())
    return tuple(outputs)


def correctness(model, prompts, result: LlamaPagedRunResult) -> dict:
    """Logit error and greedy-token match against the eager model (hf_benchmark.py:782-823)."""
    refs = eager_reference_logits(model, prompts, result.generated_tokens)
    prompt_err = float((result.prompt_logits.float() - refs[0].float()).abs().max())
    decode_errs = [float((a.float() - b.float()).abs().max())
                   for a, b in zip(result.decode_logits, refs[:-1])]
    errs = [prompt_err, *decode_errs]
    ours = torch.stack([l.argmax(-1) for l in result.decode_logits], dim=1)
    theirs = torch.stack([l.argmax(-1) for l in refs[:-1]], dim=1)
    matches = int((ours == theirs).sum())
    dtype = next(model.parameters()).dtype
    tol = 3e-2 if dtype == torch.bfloat16 else 5e-3 if dtype == torch.float16 else 1e-4
    # Smallest top-2 margin of the eager logits where the tokens disagree (0 if none).
    flips = [(float(r.topk(2).values[0] - r.topk(2).values[1]))
             for step, ref in enumerate(refs[:-1]) for i, r in enumerate(ref)
             if int(ours[i, step]) != int(theirs[i, step])]
    return {"logits_max_error": max(errs), "prefill_logits_max_error": errs[0],
            "decode_logits_max_error": max(errs[1:]) if len(errs) > 1 else 0.0,
            "token_match_rate": matches / max(int(theirs.numel()), 1), "token_matches": matches,
            "token_count": int(theirs.numel()), "logits_tolerance": tol,
            "flip_margins": flips,
            "status": "ok" if max(errs) <= tol and matches == theirs.numel() else "failed",
            "oracle": "Transformers Llama eager full-sequence path"}


def partition_requests(num_requests: int, world: int, rank: int) -> range:
    """The contiguous slice of request indices rank ``rank`` of ``world`` serves.

    Every rank gets ``ceil(num_requests / world)`` requests except the last
    ones, which may get fewer (or none); each rank then runs its own runner with
    its own block pool over ``prompts[slice]``.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    per = -(-num_requests // world)
    return range(min(rank * per, num_requests), min((rank + 1) * per, num_requests))


def allgather_token_exchange(group=None, max_local: int | None = None) -> TokenExchange:
    """All-gather of every rank's sampled token ids (one collective per decode step).

    Returns a callable for ``LlamaPagedDecodeRunner(token_exchange=...)``; the
    gathered ids of the last step are kept in ``callable.last`` (``[world, max_local]``,
    ``-1`` = padding).  The gather runs into a flat ``[world * max_local]``
    buffer, the form every backend takes (NCCL on GPUs, gloo for host tests).
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    state = {"buf": None}

    def exchange(tokens: torch.Tensor) -> None:
        width = max_local or tokens.numel()
        local = torch.full((width,), -1, dtype=torch.int32, device=tokens.device)
        local[: tokens.numel()] = tokens.to(torch.int32)
        if state["buf"] is None or state["buf"].numel() != world * width:
            state["buf"] = torch.empty((world * width,), dtype=torch.int32, device=tokens.device)
        dist.all_gather_into_tensor(state["buf"], local, group=group)
        exchange.last = state["buf"].view(world, width)

    exchange.last = None
    return exchange
