"""The b200 operators dropped into the reference's own objects and runner.

Everything here drives the UNMODIFIED reference package installed under
``baseline/_ref`` (skipped when that install is absent):

* the operators take the reference's own ``PagedKVCache`` (``cache.py:67-200``)
  and are compared on the GPU with the reference's own functions on the same
  storage: ``append_kv`` with ``PagedKVCache.write_slots`` (bit-exact),
  ``paged_decode_attention`` with the ``paged_reference`` backend
  (``attention.py:134-175``, float32 math) and ``paged_prefill_attention``
  with ``paged_prefill_attention_sdpa`` (``attention.py:230-321``);
* the reference's ``SyntheticDecodeRunner`` (``decode.py:152-592``) runs with
  the two backend branches a maintainer adds (one name per backend set, one
  branch per dispatch, exactly the lines of the integration guide) against the
  same runner on its stock ``paged_reference`` / ``torch`` backends: the
  generated tokens and every step's logits must agree.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

import inferkernellab_b200 as b200
from tests.helpers import TOL

pytestmark = pytest.mark.gpu

_REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
LOGIT_ATOL = 2e-3  # the synthetic decoder's logits are ~0.06; fp16 activations


@pytest.fixture(scope="module")
def ref():
    if not (_REF / "inferkernellab").is_dir():
        pytest.skip("the reference is not installed under baseline/_ref")
    if str(_REF) not in sys.path:
        sys.path.insert(0, str(_REF))
    import inferkernellab  # the reference package
    from inferkernellab import decode

    return inferkernellab, decode


def _filled_cache(ref_pkg, *, num_blocks, block_size, kv_heads, head_dim, dtype, seed):
    """A reference PagedKVCache on cuda:0 with every slot set (no stale NaN)."""
    cache = ref_pkg.PagedKVCache(num_blocks, block_size, kv_heads, head_dim, dtype=dtype,
                                 device="cuda")
    gen = torch.Generator(device="cpu").manual_seed(seed)
    cache.k.copy_(torch.randn(cache.k.shape, generator=gen).to(dtype))
    cache.v.copy_(torch.randn(cache.v.shape, generator=gen).to(dtype))
    return cache


def _tables(cache, lens, seed):
    """Shuffled block tables allocated through the reference's own allocator."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    tables = [cache.allocate_request(i, n) for i, n in enumerate(lens)]
    return [[t[j] for j in torch.randperm(len(t), generator=gen).tolist()] for t in tables]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_append_into_reference_cache_equals_write_slots(ref, dtype):
    ref_pkg, _ = ref
    a = _filled_cache(ref_pkg, num_blocks=40, block_size=16, kv_heads=8, head_dim=128,
                      dtype=dtype, seed=1)
    b = ref_pkg.PagedKVCache(40, 16, 8, 128, dtype=dtype, device="cuda")
    b.k.copy_(a.k)
    b.v.copy_(a.v)
    gen = torch.Generator(device="cpu").manual_seed(2)
    tokens = 301
    slots = torch.randperm(40 * 16, generator=gen)[:tokens].to("cuda")
    key = torch.randn(tokens, 8, 128, generator=gen).to(dtype).cuda()
    value = torch.randn(tokens, 8, 128, generator=gen).to(dtype).cuda()
    a.write_slots(0, slots, key, value)
    b200.append_kv(key, value, b, slots.to(torch.int32))
    torch.cuda.synchronize()
    assert torch.equal(a.k, b.k) and torch.equal(a.v, b.v)


@pytest.mark.parametrize("num_heads,kv_heads,head_dim,block_size,dtype", [
    (32, 8, 128, 16, torch.bfloat16),   # GQA, the Llama-3 head shape
    (32, 32, 64, 16, torch.float16),    # MHA
    (16, 1, 128, 32, torch.float16),    # MQA
])
def test_decode_on_reference_cache_matches_paged_reference(ref, num_heads, kv_heads, head_dim,
                                                           block_size, dtype):
    ref_pkg, _ = ref
    lens = [1, 17, 300, 1024, 2049, 64]
    need = sum(-(-n // block_size) for n in lens)
    cache = _filled_cache(ref_pkg, num_blocks=need + 5, block_size=block_size, kv_heads=kv_heads,
                          head_dim=head_dim, dtype=dtype, seed=3)
    tables = _tables(cache, lens, seed=4)
    gen = torch.Generator(device="cpu").manual_seed(5)
    query = torch.randn(len(lens), num_heads, head_dim, generator=gen).to(dtype).cuda()
    want = ref_pkg.paged_decode_attention(query, cache, tables, lens)
    # The paged_reference backend passes ragged Python lists; the Triton
    # backends pass padded int32 device tensors.  Both forms are accepted.
    got_lists = b200.paged_decode_attention(query, cache, tables, lens)
    width = max(len(t) for t in tables)
    table_t = torch.tensor([t + [0] * (width - len(t)) for t in tables], dtype=torch.int32,
                           device="cuda")
    got_dev = b200.paged_decode_attention(query, cache, table_t,
                                          torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                          validate_inputs=True)
    torch.cuda.synchronize()
    torch.testing.assert_close(got_lists.float(), want.float(), **TOL[dtype])
    assert torch.equal(got_lists, got_dev)
    assert b200.check_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_on_reference_cache_matches_reference_sdpa(ref, dtype):
    ref_pkg, _ = ref
    num_heads, kv_heads, head_dim, block_size = 32, 8, 128, 16
    starts = [0, 5, 0, 100, 31]
    ends = [37, 6, 160, 228, 31 + 77]
    need = sum(-(-e // block_size) for e in ends)
    cache = _filled_cache(ref_pkg, num_blocks=need + 3, block_size=block_size, kv_heads=kv_heads,
                          head_dim=head_dim, dtype=dtype, seed=6)
    ragged = _tables(cache, ends, seed=7)
    # the reference's prefill takes a rectangular table; ours also takes the ragged rows
    tables = [t + [0] * (max(map(len, ragged)) - len(t)) for t in ragged]
    width = max(e - s for s, e in zip(starts, ends))
    gen = torch.Generator(device="cpu").manual_seed(8)
    query = torch.randn(len(ends), num_heads, width, head_dim, generator=gen).to(dtype).cuda()
    want = ref_pkg.paged_prefill_attention_sdpa(query, cache, tables, starts, ends)
    got = b200.paged_prefill_attention(query, cache, tables, starts, ends)
    got_ragged = b200.paged_prefill_attention(query, cache, ragged, starts, ends)
    torch.cuda.synchronize()
    assert torch.equal(got, got_ragged)
    for b, (s, e) in enumerate(zip(starts, ends)):  # padded rows are unspecified
        torch.testing.assert_close(got[b, :, :e - s].float(), want[b, :, :e - s].float(),
                                   **TOL[dtype])
    assert b200.check_device_errors() == 0


def _b200_runner_class(decode):
    """The reference runner with the b200 branches of the integration guide."""

    class Runner(decode.SyntheticDecodeRunner):
        def _attention(self, query, requests, context_lengths):
            if self.config.backend == "b200_paged":
                table_tensor, length_tensor = self._metadata_tensors(requests, context_lengths)
                return b200.paged_decode_attention(query, self.cache, table_tensor,
                                                   length_tensor, validate_inputs=True)
            return super()._attention(query, requests, context_lengths)

        def _slots(self, requests, starts, lengths):
            return torch.cat([self.cache.slot_mapping(r.block_table, s, n)
                              for r, s, n in zip(requests, starts, lengths)]).to(torch.int32)

        def _append_ranges(self, requests, starts, ends, key, value):
            if self.config.append_backend == "b200":
                lengths = [e - s for s, e in zip(starts, ends)]
                b200.append_kv(key, value, self.cache, self._slots(requests, starts, lengths))
                return
            super()._append_ranges(requests, starts, ends, key, value)

        def _append_batch(self, requests, key, value):
            if self.config.append_backend == "b200":
                starts = [r.prompt_tokens + r.generated_tokens for r in requests]
                b200.append_kv(key, value, self.cache,
                               self._slots(requests, starts, [1] * len(requests)))
                return
            super()._append_batch(requests, key, value)

    return Runner


@pytest.mark.parametrize("num_kv_heads", [8, 32, 1])
def test_reference_runner_on_b200_backends_matches_its_stock_backends(ref, monkeypatch,
                                                                      num_kv_heads):
    _, decode = ref
    monkeypatch.setattr(decode, "_ATTENTION_BACKENDS",
                        decode._ATTENTION_BACKENDS | {"b200_paged"})
    monkeypatch.setattr(decode, "_APPEND_BACKENDS", decode._APPEND_BACKENDS | {"b200"})
    prompts = [[(7 * i + 3 * j) % 256 for j in range(n)] for i, n in enumerate([5, 17, 40, 1, 33])]

    def run(backend, append_backend, cls):
        cfg = decode.SyntheticDecoderConfig(
            vocab_size=256, num_heads=32, num_kv_heads=num_kv_heads, head_dim=64, block_size=16,
            dtype=torch.float16, device="cuda", seed=0, backend=backend,
            append_backend=append_backend, max_num_seqs=8, max_num_batched_tokens=64)
        return cls(cfg, prompts, max_new_tokens=6).run()

    stock = run("paged_reference", "torch", decode.SyntheticDecodeRunner)
    ours = run("b200_paged", "b200", _b200_runner_class(decode))
    assert ours.backend == "b200_paged" and ours.append_backend == "b200"
    assert len(ours.logits) == len(stock.logits) == 6
    # Every decode step batches all requests in the same order in both runs, so
    # row r of a step's logits is the same request throughout.
    same = [True] * len(prompts)  # rows whose token history still agrees
    for step, (want, got) in enumerate(zip(stock.logits, ours.logits)):
        assert want.shape == got.shape == (len(prompts), 256)
        for r in range(len(prompts)):
            if not same[r]:
                continue
            assert (got[r] - want[r]).abs().max().item() < LOGIT_ATOL, f"step {step} row {r}"
            if int(got[r].argmax()) != int(want[r].argmax()):
                top2 = torch.topk(want[r], 2).values  # only a near tie may flip the token
                assert (top2[0] - top2[1]).item() <= 2 * LOGIT_ATOL, f"step {step} row {r}"
                same[r] = False
    assert sum(same) >= len(prompts) - 1
    if all(same):
        assert ours.generated_tokens == stock.generated_tokens
    assert ours.used_blocks_peak == stock.used_blocks_peak
    assert b200.check_device_errors() == 0
