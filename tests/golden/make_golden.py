"""Regenerate the golden fixtures in this folder from the reference project.

Run in a container that has the reference checked out (read-only is fine)::

    python tests/golden/make_golden.py --reference /path/to/InferKernelLab

It imports the reference's own ``inferkernellab`` package (pure Python +
torch, CPU) and records, for seeded inputs, what the reference computes:

* ``slot_mapping.npz``   -- ``PagedKVCache.slot_mapping`` (``cache.py:113-129``);
* ``decode_*.npz``       -- ``paged_decode_attention`` (``attention.py:134-175``)
                            on a float32 copy of an fp16/bf16 cache (the oracle
                            form) and on the native-dtype cache;
* ``prefill_*.npz``      -- ``paged_prefill_attention_sdpa`` (``attention.py:230-321``);
* ``append.npz``         -- ``PagedKVCache.write_slots`` (``cache.py:156-189``);
* ``rotary.npz``         -- ``_apply_rotary`` (``hf_benchmark.py:69-85``) in fp16
                            and bf16, with cos/sin from a Llama rotary table;
* ``runtime_events.json``-- ``InferenceRuntime`` hook traces (``runtime.py:65-104``)
                            and ``TokenBudgetScheduler`` packing (``scheduler.py:50-84``);
* ``synthetic_decoder.json`` -- ``SyntheticDecodeRunner`` tokens and logits
                            (``decode.py:152-592``), float32 on CPU.

The GPU box has no reference checkout, so only the resulting ``.npz``/``.json``
files travel; nothing at test time imports the reference.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy, bfloat16 kept as raw uint16 bits."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


_KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}


def _slot_cases(ikl):
    cache_mod = ikl["cache"]
    out = {}
    cache = cache_mod.PagedKVCache(8, 4, 2, 3, dtype=torch.float32)
    out["t0_table"] = np.array([6, 2, 5], dtype=np.int64)
    out["t0_start"] = np.array(2)
    out["t0_length"] = np.array(6)
    out["t0_block_size"] = np.array(4)
    out["t0_num_blocks"] = np.array(8)
    out["t0_slots"] = cache.slot_mapping([6, 2, 5], 2, 6).numpy()
    gen = torch.Generator().manual_seed(1234)
    cases = []
    for i, (bs, nb) in enumerate([(16, 97), (8, 40), (1, 33), (32, 20), (4, 256)]):
        cache = cache_mod.PagedKVCache(nb, bs, 1, 2, dtype=torch.float32)
        width = int(torch.randint(1, 12, (1,), generator=gen))
        table = torch.randperm(nb, generator=gen)[:width].tolist()
        cap = width * bs
        start = int(torch.randint(0, cap, (1,), generator=gen))
        length = int(torch.randint(0, cap - start + 1, (1,), generator=gen))
        slots = cache.slot_mapping(table, start, length)
        name = f"r{i}"
        out[f"{name}_table"] = np.array(table, dtype=np.int64)
        out[f"{name}_start"] = np.array(start)
        out[f"{name}_length"] = np.array(length)
        out[f"{name}_block_size"] = np.array(bs)
        out[f"{name}_num_blocks"] = np.array(nb)
        out[f"{name}_slots"] = slots.numpy()
        cases.append(name)
    out["cases"] = np.array(["t0"] + cases)
    np.savez_compressed(HERE / "slot_mapping.npz", **out)


def _make_decode_case(ikl, name, *, batch, num_heads, num_kv_heads, head_dim, block_size,
                      num_blocks, lengths, dtype, seed, layers=1, layer=0, scale=None,
                      width=None):
    cache_mod = ikl["cache"]
    attn = ikl["attention"]
    gen = torch.Generator().manual_seed(seed)
    cache = cache_mod.PagedKVCache(num_blocks, block_size, num_kv_heads, head_dim,
                                   num_layers=layers, dtype=dtype)
    # Fill every slot (also unused ones) with finite noise so the fixture is deterministic.
    cache.k.copy_(torch.randn(cache.k.shape, generator=gen).to(dtype))
    cache.v.copy_(torch.randn(cache.v.shape, generator=gen).to(dtype))
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    need = [(n + block_size - 1) // block_size for n in lengths]
    width = width or max(need)
    tables = []
    cursor = 0
    for n in need:
        row = perm[cursor:cursor + n]
        cursor += n
        row = row + [0] * (width - len(row))  # zero padding like _metadata_tensors
        tables.append(row)
    query = torch.randn(batch, num_heads, head_dim, generator=gen).to(dtype)
    cache32 = cache_mod.PagedKVCache(num_blocks, block_size, num_kv_heads, head_dim,
                                     num_layers=layers, dtype=torch.float32)
    cache32.k.copy_(cache.k.float())
    cache32.v.copy_(cache.v.float())
    out32 = attn.paged_decode_attention(query.float(), cache32, tables, lengths, scale=scale,
                                        layer=layer)
    out_native = attn.paged_decode_attention(query, cache, tables, lengths, scale=scale,
                                             layer=layer)
    np.savez_compressed(
        HERE / f"decode_{name}.npz",
        kind=np.array(_KIND[dtype]), query=_np(query), k=_np(cache.k), v=_np(cache.v),
        block_tables=np.array(tables, dtype=np.int64), context_lens=np.array(lengths, dtype=np.int64),
        layer=np.array(layer), scale=np.array(np.nan if scale is None else scale),
        out_f32=_np(out32), out_native=_np(out_native),
    )


def _decode_cases(ikl):
    # The reference's own Triton parity shape (tests/test_attention.py:119-137).
    for hkv in (4, 2, 1):
        for dt in (torch.float16, torch.bfloat16):
            _make_decode_case(ikl, f"tri_h{hkv}_{_KIND[dt]}", batch=2, num_heads=4, num_kv_heads=hkv,
                              head_dim=16, block_size=8, num_blocks=16, lengths=[19, 23], dtype=dt,
                              seed=100 + hkv)
    # Grouped shape with a layer index (tests/test_attention.py:140-173).
    for hkv in (8, 4, 1):
        _make_decode_case(ikl, f"grp_h{hkv}_bf16", batch=2, num_heads=32, num_kv_heads=hkv,
                          head_dim=16, block_size=8, num_blocks=32, lengths=[19, 23],
                          dtype=torch.bfloat16, seed=200 + hkv, layers=2, layer=1)
    # Ragged, block-crossing, length 1, custom scale, D64/D128.
    _make_decode_case(ikl, "ragged_d64_f16", batch=5, num_heads=8, num_kv_heads=2, head_dim=64,
                      block_size=16, num_blocks=40, lengths=[1, 15, 16, 17, 130], dtype=torch.float16,
                      seed=7)
    _make_decode_case(ikl, "ragged_d128_bf16", batch=4, num_heads=8, num_kv_heads=1, head_dim=128,
                      block_size=16, num_blocks=30, lengths=[33, 1, 64, 200], dtype=torch.bfloat16,
                      seed=8, scale=0.1)
    _make_decode_case(ikl, "bs4_d32_f16", batch=3, num_heads=6, num_kv_heads=3, head_dim=32,
                      block_size=4, num_blocks=40, lengths=[5, 9, 41], dtype=torch.float16, seed=9)


def _prefill_cases(ikl):
    cache_mod = ikl["cache"]
    attn = ikl["attention"]

    def case(name, *, num_heads, num_kv_heads, head_dim, block_size, num_blocks, tables, starts,
             ends, width, dtype, seed):
        gen = torch.Generator().manual_seed(seed)
        cache = cache_mod.PagedKVCache(num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype)
        cache.k.copy_(torch.randn(cache.k.shape, generator=gen).to(dtype))
        cache.v.copy_(torch.randn(cache.v.shape, generator=gen).to(dtype))
        query = torch.randn(len(tables), num_heads, width, head_dim, generator=gen).to(dtype)
        cache32 = cache_mod.PagedKVCache(num_blocks, block_size, num_kv_heads, head_dim,
                                         dtype=torch.float32)
        cache32.k.copy_(cache.k.float())
        cache32.v.copy_(cache.v.float())
        out32 = attn.paged_prefill_attention_sdpa(query.float(), cache32, tables, starts, ends)
        np.savez_compressed(
            HERE / f"prefill_{name}.npz",
            kind=np.array(_KIND[dtype]), query=_np(query), k=_np(cache.k), v=_np(cache.v),
            block_tables=np.array(tables, dtype=np.int64), query_starts=np.array(starts, dtype=np.int64),
            context_lens=np.array(ends, dtype=np.int64), out_f32=_np(out32),
        )

    # The reference's own ragged prefill case (tests/test_attention.py:90-116), in fp16.
    case("ref_ragged_f16", num_heads=4, num_kv_heads=2, head_dim=16, block_size=4, num_blocks=24,
         tables=[[17, 3, 12], [5, 21, 8]], starts=[0, 2], ends=[5, 7], width=5,
         dtype=torch.float16, seed=11)
    # GQA bf16, D64, chunked continuation (start > 0) and padding rows.
    case("gqa_d64_bf16", num_heads=8, num_kv_heads=2, head_dim=64, block_size=16, num_blocks=20,
         tables=[[3, 7, 1, 9], [12, 0, 5, 2], [4, 18, 6, 11]], starts=[0, 20, 33], ends=[37, 50, 35],
         width=37, dtype=torch.bfloat16, seed=12)


def _append_case(ikl):
    cache_mod = ikl["cache"]
    gen = torch.Generator().manual_seed(5)
    cache = cache_mod.PagedKVCache(8, 8, 2, 16, num_layers=2, dtype=torch.float16)
    cache.k.zero_()
    cache.v.zero_()
    table = [6, 1, 3]
    key = torch.randn(11, 2, 16, generator=gen).to(torch.float16)
    value = torch.randn(11, 2, 16, generator=gen).to(torch.float16)
    slots = torch.cat((cache.slot_mapping(table, 0, 5), cache.slot_mapping(table, 13, 6)))
    cache.write_slots(1, slots, key, value)
    np.savez_compressed(HERE / "append.npz", key=_np(key), value=_np(value), slots=_np(slots),
                        layer=np.array(1), k_after=_np(cache.k), v_after=_np(cache.v))


def _rotary_case(ikl):
    hf = ikl["hf_benchmark"]
    gen = torch.Generator().manual_seed(77)
    out = {}
    tokens, hq, hkv, dim = 37, 8, 2, 64
    positions = torch.randint(0, 8192, (tokens,), generator=gen).double()
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    angles = positions[:, None] * inv_freq[None, :]
    emb = torch.cat((angles, angles), dim=-1)
    for dtype in (torch.float16, torch.bfloat16):
        kind = _KIND[dtype]
        query = (torch.randn(tokens, hq, dim, generator=gen) * 3).to(dtype)
        key = (torch.randn(tokens, hkv, dim, generator=gen) * 3).to(dtype)
        cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
        q_rot, k_rot = hf._apply_rotary(query, key, cos, sin)
        for name, t in (("query", query), ("key", key), ("cos", cos), ("sin", sin),
                        ("q_rot", q_rot), ("k_rot", k_rot)):
            out[f"{kind}_{name}"] = _np(t)
    np.savez_compressed(HERE / "rotary.npz", **out)


def _runtime_traces(ikl):
    cache_mod = ikl["cache"]
    runtime_mod = ikl["runtime"]
    sched_mod = ikl["scheduler"]
    traces = {}

    def run(name, *, num_blocks, block_size, max_num_seqs, budget, requests, batched):
        cache = cache_mod.PagedKVCache(num_blocks, block_size, 1, 2)
        events = []

        def prefill(request, start, end):
            events.append(["prefill", request.request_id, start, end, request.cached_tokens,
                           list(request.block_table)])

        def prefill_batch(reqs, starts, ends):
            events.append(["prefill_batch", [r.request_id for r in reqs], list(starts), list(ends),
                           [list(r.block_table) for r in reqs]])

        def decode(reqs):
            events.append(["decode", [r.request_id for r in reqs],
                           [r.generated_tokens for r in reqs], [list(r.block_table) for r in reqs]])

        rt = runtime_mod.InferenceRuntime(
            cache, sched_mod.TokenBudgetScheduler(max_num_seqs=max_num_seqs,
                                                  max_num_batched_tokens=budget),
            prefill_fn=None if batched else prefill,
            prefill_batch_fn=prefill_batch if batched else None, decode_fn=decode)
        for rid, prompt, new in requests:
            rt.submit(rid, prompt, new)
        phases = []
        stats = []
        for _ in range(200):
            batch = rt.step()
            phases.append([batch.phase, [r.request_id for r in batch.requests], batch.scheduled_tokens])
            s = rt.stats()
            stats.append([s.waiting, s.running, s.finished, s.free_blocks, s.used_blocks])
            if batch.phase == "idle":
                break
        traces[name] = {"num_blocks": num_blocks, "block_size": block_size,
                        "max_num_seqs": max_num_seqs, "budget": budget, "requests": requests,
                        "batched": batched, "events": events, "phases": phases, "stats": stats}

    run("ref_chunked", num_blocks=8, block_size=4, max_num_seqs=32, budget=4,
        requests=[[9, 5, 2]], batched=False)
    run("ref_batch", num_blocks=12, block_size=4, max_num_seqs=2, budget=8,
        requests=[[3, 4, 1], [7, 3, 1]], batched=True)
    gen = torch.Generator().manual_seed(21)
    lens = torch.randint(17, 513, (24,), generator=gen).tolist()
    run("c4_budget2048", num_blocks=2048, block_size=16, max_num_seqs=32, budget=2048,
        requests=[[i, int(n), 3] for i, n in enumerate(lens)], batched=True)
    run("mixed_seqcap", num_blocks=64, block_size=4, max_num_seqs=3, budget=10,
        requests=[[0, 7, 2], [1, 3, 3], [2, 12, 1], [3, 1, 2], [4, 5, 1]], batched=False)
    (HERE / "runtime_events.json").write_text(json.dumps(traces, indent=1) + "\n")


def _synthetic_cases(ikl):
    """Reference SyntheticDecodeRunner (decode.py:152-592), float32 on CPU."""
    dec = ikl["decode"]
    cases = {
        "ref_small": dict(cfg=dict(vocab_size=32, num_heads=4, num_kv_heads=2, head_dim=8,
                                   block_size=4, seed=19, max_num_seqs=2,
                                   max_num_batched_tokens=4),
                          prompts=[[1, 2, 3], [7, 8, 9, 10]], max_new=3),
        "gqa_d64": dict(cfg=dict(vocab_size=256, num_heads=32, num_kv_heads=8, head_dim=64,
                                 block_size=16, seed=0, max_num_seqs=8,
                                 max_num_batched_tokens=64),
                        prompts=[[(7 * i + 3 * j) % 256 for j in range(n)]
                                 for i, n in enumerate([5, 17, 40, 1, 33])], max_new=6),
    }
    out = {}
    for name, c in cases.items():
        cfg = dec.SyntheticDecoderConfig(dtype=torch.float32, device="cpu",
                                         backend="paged_reference", **c["cfg"])
        res = dec.SyntheticDecodeRunner(cfg, c["prompts"], max_new_tokens=c["max_new"]).run()
        out[name] = {"cfg": c["cfg"], "prompts": c["prompts"], "max_new": c["max_new"],
                     "generated": [list(t) for t in res.generated_tokens],
                     "logits": [l.tolist() for l in res.logits]}
    (HERE / "synthetic_decoder.json").write_text(json.dumps(out) + "\n")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", required=True, help="path of the reference project checkout")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import importlib

    ikl = {m: importlib.import_module(f"inferkernellab.{m}")
           for m in ("cache", "attention", "runtime", "scheduler", "decode", "hf_benchmark")}
    torch.set_num_threads(4)
    _slot_cases(ikl)
    _decode_cases(ikl)
    _prefill_cases(ikl)
    _append_case(ikl)
    _rotary_case(ikl)
    _runtime_traces(ikl)
    _synthetic_cases(ikl)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
