"""Scheduler and runtime host logic, pinned to the reference's traces.

tests/golden/runtime_events.json holds the hook calls, phases and stats the
reference InferenceRuntime produced (tests/golden/make_golden.py); replaying the
same scenarios here must produce identical sequences.
"""

import json
from pathlib import Path

import pytest
import torch

from inferkernellab_b200 import InferenceRequest, InferenceRuntime, PagedKVCache, TokenBudgetScheduler

TRACES = json.loads((Path(__file__).resolve().parent / "golden" / "runtime_events.json").read_text())


def _replay(t):
    cache = PagedKVCache(t["num_blocks"], t["block_size"], 1, 16)
    events = []

    def prefill(request, start, end):
        events.append(["prefill", request.request_id, start, end, request.cached_tokens,
                       list(request.block_table)])

    def prefill_batch(reqs, starts, ends):
        events.append(["prefill_batch", [r.request_id for r in reqs], list(starts), list(ends),
                       [list(r.block_table) for r in reqs]])

    def decode(reqs):
        events.append(["decode", [r.request_id for r in reqs], [r.generated_tokens for r in reqs],
                       [list(r.block_table) for r in reqs]])

    rt = InferenceRuntime(cache, TokenBudgetScheduler(max_num_seqs=t["max_num_seqs"],
                                                      max_num_batched_tokens=t["budget"]),
                          prefill_fn=None if t["batched"] else prefill,
                          prefill_batch_fn=prefill_batch if t["batched"] else None,
                          decode_fn=decode)
    for rid, prompt, new in t["requests"]:
        rt.submit(rid, prompt, new)
    phases, stats = [], []
    for _ in range(200):
        batch = rt.step()
        phases.append([batch.phase, [r.request_id for r in batch.requests], batch.scheduled_tokens])
        s = rt.stats()
        stats.append([s.waiting, s.running, s.finished, s.free_blocks, s.used_blocks])
        if batch.phase == "idle":
            break
    return events, phases, stats


@pytest.mark.parametrize("name", sorted(TRACES))
def test_runtime_replays_reference_trace(name):
    t = TRACES[name]
    events, phases, stats = _replay(t)
    assert events == t["events"]
    assert phases == t["phases"]
    assert stats == t["stats"]


def test_runtime_rejects_two_prefill_callback_shapes():
    cache = PagedKVCache(4, 4, 1, 16)
    with pytest.raises(ValueError, match="mutually exclusive"):
        InferenceRuntime(cache, TokenBudgetScheduler(), prefill_fn=lambda r, s, e: None,
                         prefill_batch_fn=lambda r, s, e: None)


def test_runtime_rejects_duplicate_request():
    rt = InferenceRuntime(PagedKVCache(8, 4, 1, 16), TokenBudgetScheduler())
    rt.submit(1, 3, 1)
    with pytest.raises(ValueError, match="duplicate"):
        rt.submit(1, 3, 1)


def test_scheduler_chunks_prefill_then_decodes():
    scheduler = TokenBudgetScheduler(max_num_seqs=4, max_num_batched_tokens=4)
    request = InferenceRequest(1, prompt_tokens=7, max_new_tokens=2)
    scheduler.add(request)
    batch = scheduler.schedule()
    assert (batch.phase, batch.scheduled_tokens, request.cached_tokens) == ("prefill", 4, 4)
    batch = scheduler.schedule()
    assert (batch.phase, request.cached_tokens) == ("prefill", 7)
    batch = scheduler.schedule()
    assert batch.phase == "decode"
    scheduler.mark_decode_step(batch.requests)
    assert request.generated_tokens == 1


def test_scheduler_marks_finished_and_validates():
    scheduler = TokenBudgetScheduler()
    request = InferenceRequest(1, prompt_tokens=1, max_new_tokens=1)
    scheduler.add(request)
    scheduler.schedule()
    batch = scheduler.schedule()
    scheduler.mark_decode_step(batch.requests)
    assert request.status == "finished" and scheduler.finished == [request]
    with pytest.raises(ValueError, match="waiting"):
        scheduler.add(request)
    with pytest.raises(ValueError, match="positive"):
        TokenBudgetScheduler(max_num_seqs=0)


def test_synthetic_config_validation_needs_no_gpu():
    from inferkernellab_b200.decode import SyntheticDecoderConfig

    with pytest.raises(ValueError, match="unsupported attention backend"):
        SyntheticDecoderConfig(backend="paged_reference")
    with pytest.raises(ValueError, match="unsupported append backend"):
        SyntheticDecoderConfig(append_backend="torch")
    with pytest.raises(ValueError, match="divisible"):
        SyntheticDecoderConfig(num_heads=6, num_kv_heads=4)
    with pytest.raises(ValueError, match="CUDA device"):
        SyntheticDecoderConfig(device="cpu")
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        SyntheticDecoderConfig(dtype=torch.float32)


def test_llama_runner_validation_needs_no_gpu():
    pytest.importorskip("transformers")
    from inferkernellab_b200.llama import LlamaPagedDecodeRunner, load_random_llama

    model = load_random_llama(vocab_size=32, hidden_size=32, intermediate_size=64, num_layers=1,
                              num_attention_heads=2, num_kv_heads=1, max_position_embeddings=32,
                              rope_theta=10_000.0, seed=1, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="unsupported backend"):
        LlamaPagedDecodeRunner(model, [[1, 2]], max_new_tokens=1, backend="triton_paged")
    with pytest.raises(ValueError, match="CUDA device"):
        LlamaPagedDecodeRunner(model, [[1, 2]], max_new_tokens=1)
    with pytest.raises(ValueError, match="top_p"):
        LlamaPagedDecodeRunner(model, [[1, 2]], max_new_tokens=1, top_p=0.0)
