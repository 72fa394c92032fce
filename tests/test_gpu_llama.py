"""Transformers Llama over the paged cache on the b200 kernels, end to end.

Mirrors the reference's tests/test_hf_benchmark.py: random-init Llama models
built exactly like the reference's _load_model (CPU float32 init after
torch.manual_seed, then cast), decoded greedily through the runtime, and
checked against the Transformers eager full-sequence forward (the reference's
own oracle, hf_benchmark.py:764-823) with its logit tolerances (bf16 3e-2,
fp16 5e-3) and greedy-token match.
"""

import pytest
import torch

from inferkernellab_b200.llama import LlamaPagedDecodeRunner, correctness, load_random_llama

pytestmark = pytest.mark.gpu


def _model(dtype, num_kv_heads=2, num_layers=2, hidden=64, heads=4, vocab=128, seed=2026):
    return load_random_llama(vocab_size=vocab, hidden_size=hidden, intermediate_size=2 * hidden,
                             num_layers=num_layers, num_attention_heads=heads,
                             num_kv_heads=num_kv_heads, max_position_embeddings=256,
                             rope_theta=10_000.0, seed=seed, device="cuda", dtype=dtype)


def _prompts(batch, length, vocab, seed=2026):
    # The reference's arithmetic prompt generator (hf_benchmark.py:748-761).
    base = torch.arange(length, dtype=torch.long)
    return tuple(tuple(((base + seed + row * 17) % vocab).tolist()) for row in range(batch))


def _assert_ok(report):
    tol = report["logits_tolerance"]
    assert report["logits_max_error"] <= tol, report
    # Greedy tokens match, except possible flips where the eager top-2 margin is tiny.
    assert report["token_match_rate"] == 1.0 or all(m < 2 * tol for m in report["flip_margins"]), report


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("num_kv_heads,num_layers", [(4, 1), (2, 2), (1, 2)])
def test_llama_runner_matches_eager(dtype, num_kv_heads, num_layers):
    model = _model(dtype, num_kv_heads=num_kv_heads, num_layers=num_layers)
    prompts = _prompts(2, 5, 128)
    result = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=3, block_size=4).run()
    _assert_ok(correctness(model, prompts, result))
    assert result.cache_released
    assert result.decode_p95_ms >= result.decode_p50_ms > 0


def test_llama_runner_ragged_batched_prefill_ignores_nan_slots():
    """Reference test_hf_benchmark.py:101-123 with the cache poisoned by NaN."""
    model = _model(torch.bfloat16)
    prompts = ((1, 2, 3, 4, 5, 9, 11, 3, 2), (6, 7, 8), tuple(range(20, 57)))
    runner = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=3, block_size=4,
                                    max_num_batched_tokens=16)
    runner.cache.k.fill_(float("nan"))
    runner.cache.v.fill_(float("nan"))
    result = runner.run()
    _assert_ok(correctness(model, prompts, result))
    assert result.prefill_batch_count >= 2  # the budget chunks the long prompt
    assert result.cache_released


def test_llama_token_and_batched_prefill_agree():
    model = _model(torch.float16)
    prompts = _prompts(3, 9, 128)
    token = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=3, block_size=4,
                                   prefill_mode="token").run()
    batched = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=3, block_size=4,
                                     prefill_mode="batched").run()
    assert token.generated_tokens == batched.generated_tokens
    assert torch.allclose(token.prompt_logits, batched.prompt_logits, atol=5e-3, rtol=0)


def test_llama_runner_head_dim_128_gqa_long_prompts():
    model = _model(torch.bfloat16, num_kv_heads=2, num_layers=2, hidden=512, heads=4)
    prompts = tuple(tuple((7 * i + j) % 128 for j in range(n)) for i, n in enumerate([130, 64, 7]))
    result = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=4, block_size=16,
                                    max_num_batched_tokens=128).run()
    _assert_ok(correctness(model, prompts, result))


def test_llama_sampling_is_seeded():
    model = _model(torch.bfloat16)
    prompts = _prompts(2, 6, 128)
    a = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=4, block_size=4, temperature=0.8,
                               top_p=0.9, seed=7).run()
    b = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=4, block_size=4, temperature=0.8,
                               top_p=0.9, seed=7).run()
    assert a.generated_tokens == b.generated_tokens
    assert all(len(x) == 4 for x in a.token_logprobs)


def test_llama_cuda_graph_decode_matches_eager_decode():
    model = _model(torch.bfloat16, num_kv_heads=2, num_layers=2, hidden=256, heads=2)
    prompts = tuple(tuple((5 * i + j) % 128 for j in range(n)) for i, n in enumerate([40, 7, 33]))
    eager = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=20, block_size=16).run()
    graph = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=20, block_size=16,
                                   cuda_graph=True).run()
    assert graph.generated_tokens == eager.generated_tokens
    for a, b in zip(graph.decode_logits, eager.decode_logits):
        assert torch.allclose(a, b, atol=1e-3, rtol=0)
    assert graph.cache_released
    _assert_ok(correctness(model, prompts, graph))


def test_llama_prefix_caching_gives_the_unshared_results():
    """Prompts with a common 40-token prefix: with prefix caching the later budget
    batches reuse the first request's blocks and prefill only their own tokens;
    tokens and logits match the unshared run (and the eager oracle)."""
    model = _model(torch.bfloat16, num_kv_heads=2, num_layers=2, hidden=128, heads=4)
    common = [(3 * j + 1) % 128 for j in range(40)]
    prompts = (tuple(common + [5, 6, 7]), tuple(common + [9] * 12), tuple(common),
               tuple(common[:20] + [1, 2, 3]))
    kwargs = dict(max_new_tokens=4, block_size=8, max_num_batched_tokens=48)
    plain = LlamaPagedDecodeRunner(model, prompts, **kwargs).run()
    shared = LlamaPagedDecodeRunner(model, prompts, prefix_caching=True, **kwargs).run()
    assert shared.prefix_cached_tokens > 0
    assert shared.generated_tokens == plain.generated_tokens
    assert torch.allclose(shared.prompt_logits, plain.prompt_logits, atol=3e-2, rtol=0)
    _assert_ok(correctness(model, prompts, shared))
    assert shared.cache_released


def test_llama_unsynchronised_steps_give_the_same_tokens():
    """sync_steps=False (the host prepares step N+1 while step N runs, with
    double-buffered staging) must not change anything the device computes."""
    model = _model(torch.bfloat16, num_kv_heads=2, num_layers=2, hidden=128, heads=4)
    prompts = _prompts(6, 21, 128)
    kwargs = dict(max_new_tokens=6, block_size=8, cuda_graph=True)
    synced = LlamaPagedDecodeRunner(model, prompts, **kwargs).run()
    free = LlamaPagedDecodeRunner(model, prompts, sync_steps=False, **kwargs).run()
    assert free.generated_tokens == synced.generated_tokens
    for a, b in zip(free.decode_logits, synced.decode_logits):
        assert torch.equal(a, b)


@pytest.mark.parametrize("fused", [True, False])
def test_llama_fused_and_unfused_decode_agree(fused):
    """The decode step with the rotary append inside the attention launch and the
    two-launch step leave identical caches, hence identical tokens and logits."""
    model = _model(torch.bfloat16, num_kv_heads=2, num_layers=2, hidden=128, heads=4)
    prompts = _prompts(5, 19, 128)
    kwargs = dict(max_new_tokens=5, block_size=8, cuda_graph=True)
    ref = LlamaPagedDecodeRunner(model, prompts, fused_decode=False, **kwargs).run()
    got = LlamaPagedDecodeRunner(model, prompts, fused_decode=fused, **kwargs).run()
    assert got.generated_tokens == ref.generated_tokens
    for a, b in zip(got.decode_logits, ref.decode_logits):
        assert torch.allclose(a, b, atol=1e-5, rtol=0)


def test_llama3_8b_shape_greedy_tokens_match_eager():
    """Config-5 shape (32 layers, hidden 4096, 32/8 heads, D128, intermediate
    14336, vocab 128256, RoPE theta 5e5, bf16): 8 seeded prompts U[64, 1024]
    (the e2e benchmark's generator) and 8 greedy steps through the CUDA-graph
    decode step, against the Transformers eager full-sequence forward of every
    step (reference hf_benchmark.py:764-823).  Weights are initialised on the
    GPU (N(0, 0.02), the e2e benchmark's scheme).

    At this depth bf16 rounding alone moves the logits far more than the small
    models' 3e-2 bar, so the bar is the reference's own: the same eager model
    run in float32 is the truth, and this path must stay as close to it as the
    bf16 eager model (the reference's oracle) does -- logit error at most 1.5x
    the eager bf16 error, and greedy tokens equal to the float32 model's except
    where its top-2 margin is inside twice that eager bf16 error."""
    import copy

    from inferkernellab_b200.e2e_bench import make_prompts
    from inferkernellab_b200.llama import eager_reference_logits

    vocab = 128256
    model = load_random_llama(vocab_size=vocab, hidden_size=4096, intermediate_size=14336,
                              num_layers=32, num_attention_heads=32, num_kv_heads=8,
                              max_position_embeddings=1024 + 8, rope_theta=5e5, seed=0,
                              device="cuda", dtype=torch.bfloat16, init_on_device=True)
    prompts = make_prompts(8, 64, 1024, vocab, seed=0)
    result = LlamaPagedDecodeRunner(model, prompts, max_new_tokens=8, block_size=16,
                                    cuda_graph=True).run()
    assert result.cache_released
    # decode_logits[s] are the logits step s sampled from: the eager forward of
    # the prompt plus the first s generated tokens (truth[s]); prompt_logits
    # are the prefill's, truth[0] too.
    ours = [l.float() for l in result.decode_logits]
    eager16 = eager_reference_logits(model, prompts, result.generated_tokens)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        model32 = copy.deepcopy(model).float()
        truth = eager_reference_logits(model32, prompts, result.generated_tokens)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
        model32 = None
    steps = len(result.decode_logits)
    err_ours = max([float((result.prompt_logits.float() - truth[0]).abs().max())]
                   + [float((a - b).abs().max()) for a, b in zip(ours, truth)])
    err_eager = max(float((a - b).abs().max()) for a, b in zip(eager16, truth))
    err_vs_eager = max(float((a - b).abs().max()) for a, b in zip(ours, eager16))
    # greedy tokens of each decode step (the runner samples from the logits it
    # used at that step, i.e. ours[s] for s < steps)
    tokens = torch.tensor(result.generated_tokens)
    flips, margins = 0, []
    for s in range(steps):
        top2 = truth[s].topk(2, dim=-1).values
        margin = top2[:, 0] - top2[:, 1]
        for i in range(len(prompts)):
            if int(tokens[i, s]) != int(truth[s][i].argmax()):
                flips += 1
                margins.append(float(margin[i]))
    eager_flips = sum(int((eager16[s].argmax(-1) != truth[s].argmax(-1)).sum())
                      for s in range(steps))
    print("config-5 shape parity:", {
        "err_ours_vs_f32": err_ours, "err_eager_bf16_vs_f32": err_eager,
        "err_ours_vs_eager_bf16": err_vs_eager, "token_flips_vs_f32": flips,
        "eager_bf16_token_flips_vs_f32": eager_flips, "tokens": steps * len(prompts),
        "flip_margins": margins})
    assert err_ours <= 1.5 * err_eager, (err_ours, err_eager)
    assert all(m < 2 * err_eager for m in margins), (margins, err_eager)
    del model
    torch.cuda.empty_cache()
