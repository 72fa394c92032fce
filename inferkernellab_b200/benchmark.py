"""Attention microbenchmark and shape sweeps for the sm_100a paged-KV kernels.

``python -m inferkernellab_b200.benchmark`` mirrors the reference's
``python -m inferkernellab.benchmark`` (reference ``src/inferkernellab/benchmark.py``):
same arguments and defaults, same interleaved block-table layout with a
reserved block between logical rounds (``benchmark.py:73-123``), CUDA events
with one synchronisation per sample (``:46-70``), and a JSON record with the
environment, the configuration, P50/P95 timings and the estimated K/V read
bandwidth (``:271-287``).  It adds what the reference could not measure:

* ``amortised`` -- the kernel replayed from a CUDA graph over ``--rotate``
  cache copies so the working set exceeds the 126 MB L2, giving achieved HBM
  GB/s of the algorithmic bytes (K/V + Q + O + table + lengths);
* ``--append`` -- config 2's step: append one token per request through its
  slot, then attend over context + 1;
* ``--sweep config2`` -- the 36-shape config-2 sweep as JSON lines;
* ``--prefill`` -- config 4: ragged causal prefill + KV append under a token
  budget, reported as achieved TFLOP/s of the causal attention.

Correctness is not re-checked here: the parity tests (``tests/``) compare every
kernel with the float32 oracle on the same seeded inputs.
"""

from __future__ import annotations

import argparse
import json
import math
import platform
import statistics
import sys
import time
from pathlib import Path

import torch

from . import _lib
from .cache import PagedKVCache
from .ops import (
    append_kv,
    rope_append_kv,
    paged_decode_attention,
    paged_decode_attention_append,
    paged_prefill_attention_varlen,
)
from .scheduler import InferenceRequest, TokenBudgetScheduler


def _percentile(values, q):
    values = sorted(values)
    pos = (len(values) - 1) * q
    lo, hi = math.floor(pos), math.ceil(pos)
    return values[lo] if lo == hi else values[lo] * (hi - pos) + values[hi] * (pos - lo)


def _cuda_device(name: str) -> torch.device:
    device = torch.device(name)
    if device.type != "cuda":
        raise RuntimeError("the B200 kernels need a CUDA device")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def _environment(device: torch.device) -> dict:
    return {
        "python": platform.python_version(),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "library": _lib.version(),
        "gpu": torch.cuda.get_device_name(device),
        "compute_capability": list(torch.cuda.get_device_capability(device)),
    }


def _interleaved_tables(batch: int, blocks_per_req: int, allocator) -> list[list[int]]:
    """Reference benchmark.py:89-93: one block per request per round, plus a reserved hole."""
    tables = [[] for _ in range(batch)]
    for logical in range(blocks_per_req):
        for r in range(batch):
            tables[r].extend(allocator.allocate(1, owner=r))
        if logical + 1 < blocks_per_req:
            allocator.allocate(1, owner=-1)
    return tables


class DecodeCase:
    def __init__(self, args, device, copies: int = 1):
        dtype = getattr(torch, args.dtype)
        self.args = args
        bs = args.block_size
        need = -(-(args.context_len + (1 if args.append else 0)) // bs)
        minimum = args.batch_size * need + need - 1
        num_blocks = max(args.num_blocks, minimum)
        torch.manual_seed(args.seed)
        self.caches, self.tables = [], None
        for _ in range(copies):
            cache = PagedKVCache(num_blocks, bs, args.num_kv_heads, args.head_dim, dtype=dtype,
                                 device=device)
            cache.k.normal_()
            cache.v.normal_()
            self.caches.append(cache)
        if args.layout == "interleaved":
            tables = _interleaved_tables(args.batch_size, need, self.caches[0].allocator)
        else:
            gen = torch.Generator().manual_seed(args.seed)
            perm = torch.randperm(num_blocks, generator=gen).tolist()
            tables = [perm[i * need:(i + 1) * need] for i in range(args.batch_size)]
        self.tables = torch.tensor(tables, dtype=torch.int32, device=device)
        ctx = args.context_len + (1 if args.append else 0)
        self.ctx = ctx
        self.lens = torch.full((args.batch_size,), ctx, dtype=torch.int32, device=device)
        self.query = torch.randn(args.batch_size, args.num_heads, args.head_dim, device=device,
                                 dtype=dtype)
        self.out = torch.empty_like(self.query)
        pos = ctx - 1
        self.slots = (self.tables[:, pos // bs].long() * bs + pos % bs).to(torch.int32)
        self.new_k = torch.randn(args.batch_size, args.num_kv_heads, args.head_dim, device=device,
                                 dtype=dtype)
        self.new_v = torch.randn_like(self.new_k)

    def bytes_per_call(self) -> int:
        a = self.args
        es = torch.tensor([], dtype=getattr(torch, a.dtype)).element_size()
        kv = 2 * a.batch_size * self.ctx * a.num_kv_heads * a.head_dim * es
        qo = 2 * a.batch_size * a.num_heads * a.head_dim * es
        table = a.batch_size * (-(-self.ctx // a.block_size)) * 4 + a.batch_size * 4
        append = (4 * a.batch_size * a.num_kv_heads * a.head_dim * es + a.batch_size * 4
                  if a.append else 0)
        return kv + qo + table + append

    def call(self, cache):
        # Default: append_kv, then decode (two launches).  --fused-append times
        # the one-launch form (the append inside the decode kernel): it saves a
        # launch, but on these small shapes its producer waits for the append
        # before loading the tile that holds the new token (config-2 sweep mean
        # 20.1 us fused against 18.8 us unfused, graph-replayed).
        if self.args.append and getattr(self.args, "fused_append", False):
            paged_decode_attention_append(self.query, self.new_k, self.new_v, cache, self.tables,
                                          self.lens, self.slots, out=self.out)
            return
        if self.args.append:
            append_kv(self.new_k, self.new_v, cache, self.slots)
        paged_decode_attention(self.query, cache, self.tables, self.lens, validate_inputs=False,
                               out=self.out)


def run(args) -> dict:
    device = _cuda_device(args.device)
    torch.cuda.set_device(device)
    kv_bytes = 2 * args.batch_size * (args.context_len + args.append) * args.num_kv_heads * \
        args.head_dim * torch.tensor([], dtype=getattr(torch, args.dtype)).element_size()
    rotate = args.rotate or max(1, math.ceil(4 * 128e6 / max(kv_bytes, 1)))
    rotate = min(rotate, 64)
    case = DecodeCase(args, device, copies=rotate)
    # per-call latency, the reference's method (events + sync per sample)
    for _ in range(args.warmup):
        case.call(case.caches[0])
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    samples = []
    for i in range(args.iterations):
        start.record()
        case.call(case.caches[i % rotate])
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end))
    # amortised: CUDA graph of rotate x repeat calls, caches rotated to defeat L2
    repeat = max(1, args.graph_calls // rotate)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for c in case.caches:
            case.call(c)  # warm the workspaces on this stream before capture
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(repeat):
            for c in case.caches:
                case.call(c)
    calls = repeat * rotate
    graph.replay()
    torch.cuda.synchronize(device)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(args.graph_replays):
        graph.replay()
    g1.record()
    g1.synchronize()
    per_call_ms = g0.elapsed_time(g1) / (args.graph_replays * calls)
    nbytes = case.bytes_per_call()
    return {
        "schema_version": 2,
        "environment": _environment(device),
        "config": {
            "device": str(device), "dtype": args.dtype, "batch_size": args.batch_size,
            "context_len": args.context_len, "num_heads": args.num_heads,
            "num_kv_heads": args.num_kv_heads, "head_dim": args.head_dim,
            "block_size": args.block_size, "num_blocks": case.caches[0].layout.num_blocks,
            "block_table_layout": args.layout, "append": bool(args.append),
            "append_mode": ("none" if not args.append else
                            "fused into the decode launch" if args.fused_append else
                            "append_kv + decode (two launches)"),
            "attended_context": case.ctx, "warmup": args.warmup, "iterations": args.iterations,
            "seed": args.seed,
            "timing": "CUDA events with per-sample synchronization; amortised = CUDA graph replay",
        },
        "kernel_config": {"decode": "paged_decode_kernel (stream-K split-KV, TMA + mma.sync)",
                          "rotated_cache_copies": rotate, "graph_calls": calls},
        "estimated_kv_read_bytes": kv_bytes,
        "algorithmic_bytes_per_call": nbytes,
        "results": {
            "b200_paged": {
                "timing": {"mean_ms": statistics.fmean(samples),
                           "p50_ms": _percentile(samples, 0.5),
                           "p95_ms": _percentile(samples, 0.95)},
                "estimated_kv_read_gbps": kv_bytes / (statistics.fmean(samples) * 1e-3) / 1e9,
                "amortised_ms_per_call": per_call_ms,
                "amortised_gbps": nbytes / (per_call_ms * 1e-3) / 1e9,
            }
        },
    }


def sweep_config2(args):
    """B x ctx x Hkv x dtype with a one-token append per step."""
    for dtype in ("float16", "bfloat16"):
        for batch in (1, 4, 16):
            for ctx in (128, 512):
                for hkv in (32, 8, 1):
                    ns = argparse.Namespace(**vars(args))
                    ns.dtype, ns.batch_size, ns.context_len, ns.num_kv_heads = dtype, batch, ctx, hkv
                    ns.num_heads, ns.head_dim, ns.block_size, ns.append = 32, 64, 16, 1
                    ns.layout = "shuffled"
                    yield run(ns)


def config4_plan(seed: int, prompts: int = 24, min_len: int = 17, max_len: int = 512,
                 budget: int = 2048, block_size: int = 16):
    """BASELINE config 4's batches: seeded prompt lengths packed under the token budget.

    Returns ``(lens, batches, tables, num_blocks)``: ``batches`` lists, per
    budget batch the ``TokenBudgetScheduler`` forms (FCFS, only the head request
    chunked), ``(request, start, end)`` of each scheduled range; ``tables`` are
    the requests' block-table rows over a shuffled pool of ``num_blocks``.
    """
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (prompts,), generator=gen).tolist()
    sched = TokenBudgetScheduler(max_num_seqs=max(32, prompts), max_num_batched_tokens=budget)
    reqs = [InferenceRequest(i, n, 1) for i, n in enumerate(lens)]
    for r in reqs:
        sched.add(r)
    batches = []
    while True:
        before = {r.request_id: r.cached_tokens for r in reqs}
        b = sched.schedule()
        if b.phase != "prefill":
            break
        batches.append([(r.request_id, before[r.request_id], r.cached_tokens) for r in b.requests])
    need = [-(-n // block_size) for n in lens]
    num_blocks = sum(need) + 8
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    width = max(need)
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [0] * (width - n))
        cur += n
    return lens, batches, tables, num_blocks


def run_prefill(args) -> dict:
    """24 prompts U[17,512], token budget 2048, packed prefill + append."""
    device = _cuda_device(args.device)
    torch.cuda.set_device(device)
    dtype = torch.bfloat16
    hq, hkv, dim, bs = 32, 8, 128, 16
    lens, batches, tables, num_blocks = config4_plan(
        args.seed, args.prefill_prompts, args.prefill_min_len, args.prefill_max_len)
    cache = PagedKVCache(num_blocks, bs, hkv, dim, dtype=dtype, device=device)
    tables = torch.tensor(tables, dtype=torch.int32, device=device)
    work = []
    flops = 0.0
    from .ops import build_slot_mapping

    for batch in batches:
        ids = [rid for rid, _, _ in batch]
        starts = torch.tensor([s for _, s, _ in batch], dtype=torch.int32, device=device)
        ends = torch.tensor([e for _, _, e in batch], dtype=torch.int32, device=device)
        total = int(sum(e - s for _, s, e in batch))
        q = torch.randn(total, hq, dim, device=device, dtype=dtype)
        k = torch.randn(total, hkv, dim, device=device, dtype=dtype)
        v = torch.randn(total, hkv, dim, device=device, dtype=dtype)
        btab = tables[ids].contiguous()
        rot = None
        if args.rope:  # Llama-3 rotary rows (theta 5e5) of every scheduled position
            pos = torch.tensor([t for _, s, e in batch for t in range(s, e)], dtype=torch.float64)
            inv = 1.0 / (5e5 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
            ang = pos[:, None] * inv[None, :]
            emb = torch.cat((ang, ang), dim=-1)
            rot = (emb.cos().to(dtype).to(device), emb.sin().to(dtype).to(device),
                   torch.empty_like(q))
        work.append((btab, starts, ends, total, q, k, v, rot))
        for _, s, e in batch:
            flops += sum(2.0 * 2.0 * dim * hq * (p + 1) for p in range(s, e))

    def step():
        for btab, starts, ends, total, q, k, v, rot in work:
            slots, cu = build_slot_mapping(btab, starts, ends, block_size=bs,
                                           num_blocks=num_blocks, total_tokens=total)
            if rot is None:
                append_kv(k, v, cache, slots)
                qr = q
            else:
                qr = rope_append_kv(q, k, v, rot[0], rot[1], cache, slots, out=rot[2])
            paged_prefill_attention_varlen(qr, cache, btab, cu, starts, ends,
                                           kernel=args.prefill_kernel)

    metas = []
    for btab, starts, ends, total, q, k, v, rot in work:
        slots, cu = build_slot_mapping(btab, starts, ends, block_size=bs,
                                       num_blocks=num_blocks, total_tokens=total)
        metas.append(cu)

    def attention_only():
        for (btab, starts, ends, total, q, k, v, rot), cu in zip(work, metas):
            paged_prefill_attention_varlen(q, cache, btab, cu, starts, ends,
                                           kernel=args.prefill_kernel)

    def timed(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iterations):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / args.iterations

    ms = timed(step)
    attn_ms = timed(attention_only)
    # The same launches replayed from a CUDA graph: device time without the
    # host's per-launch cost (the eager figures above include it when the host
    # is slower than the kernels).
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        attention_only()
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        attention_only()
    torch.cuda.current_stream(device).wait_stream(side)
    attn_graph_ms = timed(graph.replay)
    return {
        "schema_version": 2, "benchmark": "config4_prefill",
        "environment": _environment(device),
        "config": {"prompts": lens, "budget": 2048, "batches": len(batches), "num_heads": hq,
                   "num_kv_heads": hkv, "head_dim": dim, "block_size": bs, "dtype": "bfloat16",
                   "kernel": args.prefill_kernel,
                   "append": "rope_append_kv" if args.rope else "append_kv"},
        "prefill_ms": ms, "causal_attention_flops": flops,
        "achieved_tflops": flops / (ms * 1e-3) / 1e12,
        "attention_only_ms": attn_ms,
        "attention_only_tflops": flops / (attn_ms * 1e-3) / 1e12,
        "attention_graph_ms": attn_graph_ms,
        "attention_graph_tflops": flops / (attn_graph_ms * 1e-3) / 1e12,
        "tokens_per_s": sum(lens) / (ms * 1e-3),
    }


def _reference_modules():
    """The reference project installed under ``baseline/_ref`` (repository root)."""
    path = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (path / "inferkernellab").is_dir():
        raise RuntimeError("the reference is not installed under baseline/_ref")
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    from inferkernellab import attention, cache, triton_ops  # the reference's own modules

    return attention, cache, triton_ops


def run_reference_gpu(args) -> list[dict]:
    """The reference's own GPU decode backends beside this library's kernel.

    Configs 1 and 3 on the same B200, the same inputs in one cache object (the
    reference's ``PagedKVCache``, which this library's ops also accept):
    ``triton_paged`` (reference ``triton_ops.py:404-478``),
    ``triton_paged_grouped`` (``:481-610``), ``paged_sdpa``
    (``attention.py:178-227``) and ``b200_paged``.  Each backend is timed two
    ways with CUDA events: one call at a time with a synchronisation between
    calls (median), and ``--iterations`` calls back to back (mean).  Inputs
    validation is off where a backend has the switch.  The outputs are checked
    against this library's before timing.
    """
    from .workloads import workload_tensors

    ref_attention, ref_cache, ref_triton = _reference_modules()
    device = _cuda_device(args.device)
    torch.cuda.set_device(device)
    cases = []
    # config 1: B4, ctx 512, Hq32/Hkv8, D64, BS16, 159 blocks, fp16, seeded shuffled tables
    gen = torch.Generator().manual_seed(args.seed)
    c1 = ref_cache.PagedKVCache(159, 16, 8, 64, dtype=torch.float16, device=device)
    c1.k.copy_(torch.randn(c1.k.shape, generator=gen).half())
    c1.v.copy_(torch.randn(c1.v.shape, generator=gen).half())
    perm = torch.randperm(159, generator=gen)
    tables1 = perm[:4 * 32].view(4, 32).to(torch.int32).to(device)
    lens1 = torch.full((4,), 512, dtype=torch.int32, device=device)
    q1 = torch.randn(4, 32, 64, generator=gen).half().to(device)
    cases.append(("config1", c1, q1, tables1, lens1, [512] * 4, 16))
    # config 3: the bench's seed-0 batch
    t = workload_tensors(args.seed, device)
    c3 = ref_cache.PagedKVCache(t["num_blocks"], 16, 8, 128, dtype=torch.bfloat16, device=device)
    c3.k, c3.v = t["k"], t["v"]
    cases.append(("config3", c3, t["query"], t["tables"].to(device),
                  torch.tensor(t["lens"], dtype=torch.int32, device=device), t["lens"], 16))
    records = []
    for name, cache, q, tables, lens, lens_list, bs in cases:
        lay = cache.layout
        es = q.element_size()
        nbytes = (sum(lens_list) * lay.num_kv_heads * lay.head_dim * es * 2
                  + 2 * q.numel() * es + sum(-(-n // bs) for n in lens_list) * 4 + 4 * len(lens_list))
        backends = {
            "b200_paged": lambda: paged_decode_attention(q, cache, tables, lens,
                                                         validate_inputs=False),
            "triton_paged": lambda: ref_triton.paged_decode_attention_triton(
                q, cache, tables, lens, validate_inputs=False),
            "triton_paged_grouped": lambda: ref_triton.paged_decode_attention_triton_grouped(
                q, cache, tables, lens, validate_inputs=False),
            "paged_sdpa": lambda: ref_attention.paged_decode_attention_sdpa(q, cache, tables, lens),
        }
        want = backends["b200_paged"]().float()
        for backend, fn in backends.items():
            diff = float((fn().float() - want).abs().max())
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize(device)
            single = []
            for _ in range(args.iterations):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                e1.synchronize()
                single.append(e0.elapsed_time(e1))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iterations):
                fn()
            e1.record()
            e1.synchronize()
            b2b = e0.elapsed_time(e1) / args.iterations
            p50 = statistics.median(single)
            records.append({
                "benchmark": "reference_gpu_decode", "config": name, "backend": backend,
                "per_call_p50_ms": round(p50, 5), "back_to_back_ms": round(b2b, 5),
                "algorithmic_bytes": nbytes,
                "per_call_gbs": round(nbytes / (p50 * 1e-3) / 1e9, 1),
                "back_to_back_gbs": round(nbytes / (b2b * 1e-3) / 1e9, 1),
                "max_abs_diff_vs_b200_paged": diff,
                "l2_note": "working set fits in the 126 MB L2" if nbytes < 64e6 else
                           "working set exceeds L2",
                "device": torch.cuda.get_device_name(device),
            })
    return records


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="B200 paged decode attention microbenchmark")
    p.add_argument("--device", default="cuda")
    p.add_argument("--dtype", choices=("float16", "bfloat16"), default="float16")
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--context-len", type=int, default=128)
    p.add_argument("--num-heads", type=int, default=8)
    p.add_argument("--num-kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--num-blocks", type=int, default=4096)
    p.add_argument("--layout", choices=("interleaved", "shuffled"), default="interleaved")
    p.add_argument("--append", type=int, choices=(0, 1), default=0)
    p.add_argument("--fused-append", action="store_true",
                   help="with --append: one launch (append inside the decode kernel)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iterations", type=int, default=30)
    p.add_argument("--rotate", type=int, default=0, help="cache copies (0 = enough to defeat L2)")
    p.add_argument("--graph-calls", type=int, default=256)
    p.add_argument("--graph-replays", type=int, default=5)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--sweep", choices=("config2",), default=None)
    p.add_argument("--prefill", action="store_true", help="config-4 ragged prefill benchmark")
    p.add_argument("--prefill-kernel", choices=("auto", "tcgen05", "mma_sync"), default="auto")
    p.add_argument("--prefill-prompts", type=int, default=24)
    p.add_argument("--prefill-min-len", type=int, default=17)
    p.add_argument("--prefill-max-len", type=int, default=512)
    p.add_argument("--rope", action="store_true",
                   help="with --prefill: rotary + append in one rope_append_kv launch per batch")
    p.add_argument("--profile-kernel", action="store_true",
                   help="one decode launch between cudaProfilerStart/Stop (ncu --profile-from-start off)")
    p.add_argument("--reference-gpu", action="store_true",
                   help="time the reference's own GPU decode backends (baseline/_ref) beside "
                        "b200_paged on configs 1 and 3")
    p.add_argument("--output", type=Path)
    return p


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    if args.profile_kernel:
        device = _cuda_device(args.device)
        case = DecodeCase(args, device)
        case.call(case.caches[0])
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()
        case.call(case.caches[0])
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        print(json.dumps({"profile_mode": "single b200 paged-decode launch"}))
        return
    records = []
    if args.reference_gpu:
        records.extend(run_reference_gpu(args))
    elif args.prefill:
        records.append(run_prefill(args))
    elif args.sweep == "config2":
        records.extend(sweep_config2(args))
    else:
        records.append(run(args))
    text = "\n".join(json.dumps(r) for r in records)
    print(text)
    if args.output:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(text + "\n")


if __name__ == "__main__":
    main(sys.argv[1:])
