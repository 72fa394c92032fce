"""The synthetic single-layer decoder on the b200 backend, end to end.

The runner mirrors the reference's SyntheticDecodeRunner (decode.py:152-592)
with attention and append on the sm_100a kernels.  Its logits are checked
teacher-forced against the float32 numpy restatement of the same decoder
(oracle/synthetic_ref.py, itself pinned to the reference runner's golden run):
for the token history the runner produced, every step's logits must agree
within the fp16 tolerance, and every greedy token must match wherever the
oracle's top-2 margin is larger than that tolerance.
"""

import numpy as np
import pytest
import torch

from inferkernellab_b200.decode import SyntheticDecodeRunner, SyntheticDecoderConfig
from oracle import synthetic_ref

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-3  # logits are ~0.06 in magnitude; fp16 weights, fp32 oracle


def _config(**kw):
    base = dict(vocab_size=256, num_heads=32, num_kv_heads=8, head_dim=64, block_size=16,
                dtype=torch.float16, seed=0, max_num_seqs=8, max_num_batched_tokens=64)
    base.update(kw)
    return SyntheticDecoderConfig(**base)


def _prompts(lengths, vocab=256):
    return [[(7 * i + 3 * j) % vocab for j in range(n)] for i, n in enumerate(lengths)]


def _check_against_oracle(cfg, prompts, result):
    w = synthetic_ref.make_weights(cfg.vocab_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                   cfg.seed)
    w = {k: torch.from_numpy(v).to(cfg.dtype).float().numpy() for k, v in w.items()}
    want = synthetic_ref.decode_logits(w, prompts, result.generated_tokens, cfg.num_heads,
                                       cfg.num_kv_heads, cfg.head_dim)
    checked = 0
    for step, (got, ref) in enumerate(zip(result.logits, want)):
        got = got.numpy()
        assert np.abs(got - ref).max() < LOGIT_ATOL, f"step {step}"
        top2 = np.sort(ref, axis=-1)[:, -2:]
        sure = (top2[:, 1] - top2[:, 0]) > 2 * LOGIT_ATOL
        toks = np.array([g[step] for g in result.generated_tokens])
        assert (toks[sure] == ref.argmax(-1)[sure]).all(), f"step {step}"
        checked += int(sure.sum())
    return checked


@pytest.mark.parametrize("num_kv_heads", [8, 32, 1])
def test_synthetic_runner_matches_oracle(num_kv_heads):
    cfg = _config(num_kv_heads=num_kv_heads)
    prompts = _prompts([5, 17, 40, 1, 33])
    result = SyntheticDecodeRunner(cfg, prompts, max_new_tokens=6).run()
    assert all(len(t) == 6 for t in result.generated_tokens)
    _check_against_oracle(cfg, prompts, result)
    assert result.used_blocks_peak > 0
    assert result.tpot_device_ms > 0 and result.device_tokens_per_sec > 0


def test_synthetic_runner_bf16_and_long_prompts():
    cfg = _config(dtype=torch.bfloat16, head_dim=128, num_heads=32, num_kv_heads=8,
                  max_num_batched_tokens=512)
    prompts = _prompts([300, 64, 513, 2])
    result = SyntheticDecodeRunner(cfg, prompts, max_new_tokens=4).run()
    w = synthetic_ref.make_weights(cfg.vocab_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                   cfg.seed)
    w = {k: torch.from_numpy(v).to(cfg.dtype).float().numpy() for k, v in w.items()}
    want = synthetic_ref.decode_logits(w, prompts, result.generated_tokens, cfg.num_heads,
                                       cfg.num_kv_heads, cfg.head_dim)
    for got, ref in zip(result.logits, want):
        assert np.abs(got.numpy() - ref).max() < 1e-2  # bf16 weights/activations


def test_token_and_batched_prefill_agree():
    prompts = _prompts([5, 3, 21])
    token = SyntheticDecodeRunner(_config(prefill_mode="token", max_num_batched_tokens=5),
                                  prompts, max_new_tokens=3).run()
    batched = SyntheticDecodeRunner(_config(prefill_mode="batched", max_num_batched_tokens=5),
                                    prompts, max_new_tokens=3).run()
    assert batched.generated_tokens == token.generated_tokens
    assert batched.prefill_batch_count == token.prefill_batch_count
    for a, b in zip(token.logits, batched.logits):
        assert torch.allclose(a, b, atol=1e-6, rtol=0)


def test_runner_releases_blocks_and_uses_non_contiguous_tables():
    runner = SyntheticDecodeRunner(_config(max_num_batched_tokens=8, block_size=4),
                                   _prompts([5, 6]), max_new_tokens=20)
    # Round-robin repack with reserved holes (reference decode.py:245-259).
    assert all(len(r.block_table) > 1 and any(b - a != 1 for a, b in zip(r.block_table,
                                                                         r.block_table[1:]))
               for r in runner.requests)
    result = runner.run()
    assert all(len(t) == 20 for t in result.generated_tokens)
    assert runner.runtime.stats().used_blocks == 0
    assert runner.runtime.stats().finished == 2
    with pytest.raises(RuntimeError, match="only be run once"):
        runner.run()
