"""Pin the numpy oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by importing the reference project itself
(tests/golden/make_golden.py); these tests need no GPU.
"""

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_slot_mapping_matches_reference_vectors():
    data = np.load(GOLDEN / "slot_mapping.npz")
    for name in data["cases"]:
        got = oracle.slot_mapping(data[f"{name}_table"].tolist(), int(data[f"{name}_start"]),
                                  int(data[f"{name}_length"]), int(data[f"{name}_block_size"]),
                                  int(data[f"{name}_num_blocks"]))
        np.testing.assert_array_equal(got, data[f"{name}_slots"])
    # The reference's own literal (tests/test_cache.py:8-12).
    assert oracle.slot_mapping([6, 2, 5], 2, 6, 4, 8).tolist() == [26, 27, 8, 9, 10, 11]


def test_slot_mapping_errors_match_reference():
    with pytest.raises(ValueError, match="invalid physical block"):
        oracle.slot_mapping([-1], 0, 1, 4, 4)
    with pytest.raises(ValueError, match="shorter"):
        oracle.slot_mapping([2], 4, 1, 4, 4)
    with pytest.raises(ValueError, match="non-negative"):
        oracle.slot_mapping([0], -1, 1, 4, 4)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("decode_*.npz")), ids=lambda p: p.stem)
def test_decode_oracle_matches_reference(path):
    d = np.load(path)
    kind = str(d["kind"])
    scale = None if np.isnan(d["scale"]) else float(d["scale"])
    got = oracle.paged_decode_attention(d["query"], d["k"], d["v"], kind, d["block_tables"].tolist(),
                                        d["context_lens"].tolist(), scale=scale, layer=int(d["layer"]))
    np.testing.assert_allclose(got, d["out_f32"], atol=2e-6, rtol=2e-5)
    # The reference's native-dtype output is the fp32 result rounded once.
    native = oracle.to_f32(d["out_native"], kind)
    tol = 1e-2 if kind == "bf16" else 2e-3
    np.testing.assert_allclose(got, native, atol=tol, rtol=tol)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("prefill_*.npz")), ids=lambda p: p.stem)
def test_prefill_oracle_matches_reference(path):
    d = np.load(path)
    got = oracle.paged_prefill_attention(d["query"], d["k"], d["v"], str(d["kind"]),
                                         d["block_tables"].tolist(), d["query_starts"].tolist(),
                                         d["context_lens"].tolist())
    # Every row, padded rows included (they attend key 0 in both).
    np.testing.assert_allclose(got, d["out_f32"], atol=2e-6, rtol=2e-5)


def test_append_oracle_matches_reference():
    d = np.load(GOLDEN / "append.npz")
    k = np.zeros_like(d["k_after"])
    v = np.zeros_like(d["v_after"])
    oracle.write_slots(k, v, int(d["layer"]), d["slots"], d["key"], d["value"])
    np.testing.assert_array_equal(k.view(np.uint16), d["k_after"].view(np.uint16))
    np.testing.assert_array_equal(v.view(np.uint16), d["v_after"].view(np.uint16))


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_rotary_oracle_matches_reference_bit_exact(kind):
    """The rounded-elementwise rotary restatement equals the reference's
    ``_apply_rotary`` output bit for bit (hf_benchmark.py:69-85)."""
    d = np.load(GOLDEN / "rotary.npz")
    for src, want in (("query", "q_rot"), ("key", "k_rot")):
        got = oracle.rotary_embed(d[f"{kind}_{src}"], d[f"{kind}_cos"], d[f"{kind}_sin"], kind)
        np.testing.assert_array_equal(got.view(np.uint16), d[f"{kind}_{want}"].view(np.uint16))


def test_bf16_round_trip_is_exact_and_rounds_to_nearest_even():
    bits = np.arange(0, 1 << 16, 7, dtype=np.uint16)
    f = oracle.bf16_bits_to_f32(bits)
    finite = np.isfinite(f)
    np.testing.assert_array_equal(oracle.f32_to_bf16_bits(f[finite]), bits[finite])
    # 1 + 2^-8 is exactly between two bf16 values: ties go to the even mantissa (1.0).
    assert oracle.f32_to_bf16_bits(np.array([1.0 + 2 ** -8], np.float32))[0] == 0x3F80
    assert oracle.f32_to_bf16_bits(np.array([1.0 + 3 * 2 ** -8], np.float32))[0] == 0x3F82


def test_synthetic_decoder_oracle_matches_reference():
    """The numpy synthetic-decoder restatement reproduces the reference runner's
    float32 logits and greedy tokens (tests/golden/synthetic_decoder.json)."""
    import json

    from oracle import synthetic_ref

    data = json.loads((GOLDEN / "synthetic_decoder.json").read_text())
    for name, case in data.items():
        cfg = case["cfg"]
        weights = synthetic_ref.make_weights(cfg["vocab_size"], cfg["num_heads"],
                                             cfg["num_kv_heads"], cfg["head_dim"], cfg["seed"])
        logits = synthetic_ref.decode_logits(weights, case["prompts"], case["generated"],
                                             cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"])
        assert len(logits) == case["max_new"]
        for step, (got, want) in enumerate(zip(logits, case["logits"])):
            np.testing.assert_allclose(got, np.asarray(want, np.float32), atol=2e-6, rtol=1e-5,
                                       err_msg=f"{name} step {step}")
            assert got.argmax(-1).tolist() == [g[step] for g in case["generated"]]


def _pack_padded(query, query_starts, context_lens):
    """[B, Hq, T, D] padded rows -> [sum T, Hq, D] packed rows (unpadded only)."""
    rows = [query[b, :, :e - s, :].transpose(1, 0, 2)
            for b, (s, e) in enumerate(zip(query_starts, context_lens))]
    return np.concatenate(rows, axis=0)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("prefill_*.npz")), ids=lambda p: p.stem)
def test_packed_prefill_oracle_matches_reference_and_loop_form(path):
    d = np.load(path)
    starts, ends = d["query_starts"].tolist(), d["context_lens"].tolist()
    packed = _pack_padded(d["query"], starts, ends)
    got = oracle.paged_prefill_attention_packed(packed, d["k"], d["v"], str(d["kind"]),
                                                d["block_tables"].tolist(), starts, ends)
    want = _pack_padded(d["out_f32"], starts, ends)
    np.testing.assert_allclose(got, want, atol=2e-6, rtol=2e-5)


@pytest.mark.parametrize("kind,group", [("bf16", 4), ("f16", 1), ("bf16", 8)])
def test_packed_prefill_oracle_matches_loop_form_on_ragged_chunks(kind, group):
    rng = np.random.default_rng(7 + group)
    hkv, dim, bs = 2, 32, 8
    starts, ends = [0, 5, 30, 11], [9, 21, 47, 12]  # chunked ranges, one single-token range
    need = [-(-e // bs) for e in ends]
    nb = sum(need) + 3
    perm = rng.permutation(nb).tolist()
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [0] * (max(need) - n))
        cur += n

    def store(shape):
        x = rng.standard_normal(shape, dtype=np.float32)
        return oracle.f32_to_bf16_bits(x) if kind == "bf16" else x.astype(np.float16)

    k = store((1, nb, bs, hkv, dim))
    v = store((1, nb, bs, hkv, dim))
    width = max(e - s for s, e in zip(starts, ends))
    query = store((len(ends), hkv * group, width, dim))
    loop = oracle.paged_prefill_attention(query, k, v, kind, tables, starts, ends, scale=0.3)
    packed = oracle.paged_prefill_attention_packed(_pack_padded(query, starts, ends), k, v, kind,
                                                   tables, starts, ends, scale=0.3)
    np.testing.assert_allclose(packed, _pack_padded(loop, starts, ends), atol=2e-6, rtol=2e-5)
