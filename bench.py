#!/usr/bin/env python
"""Benchmark of the paged-KV decode hot path on B200 (one JSON line on stdout).

Workload ("long ragged decode with split-KV"): per GPU a
batch of 64 requests with context lengths drawn uniformly from [1, 8192]
(seeded), 32 query heads, 8 KV heads, head_dim 128, block_size 16, bfloat16,
physical pool = total blocks + 10 %, shuffled allocation.  One *step* is one
decode step of the hot path for the batch:

  1. append the new token's K/V of every request through its slot
     (reshape-and-cache), and
  2. paged decode attention of every request over its whole context,
     context length = drawn length (the new token is the last position),

both in one launch: ``paged_decode_attention_append`` (the attention kernel's
producer warp writes each new token just before it loads the tile that holds
it; bit-identical to ``append_kv`` followed by ``paged_decode_attention``).

The step is idempotent (the same slots are rewritten), so K timed steps are
K identical passes over a 1.08 GB working set -- far larger than the 126 MB
L2, so no flush is needed between steps.

``value`` = algorithmic bytes of a step (K/V + Q + O + block table + lengths of
the attention, plus the append's read and write) x steps x GPUs / the max over
ranks of the device time of the K steps.  ``e2e`` repeats the measurement
through the same public API with every step's inputs copied from pinned host
memory and the output copied back inside the timed region (the copies run on
side streams against two device buffer sets, overlapping the neighbouring
steps' kernels, as a serving loop overlaps them).  ``roofline`` is the
step's kernel, timed with CUDA events around each of its launches.

``--impl reference`` times the reference's own CPU implementation of the step
-- ``PagedKVCache.write_slots`` + ``paged_decode_attention`` (the
``paged_reference`` backend) of the reference project installed under
``baseline/_ref`` -- on the same seed-0 batch copied to the host, with all host
threads (the numpy restatement in ``oracle/`` stands in when that install is
absent).  ``cpu_baseline`` is the same path on a bounded sample.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): every rank owns
its own 64-request batch and its own block pool (requests are partitioned by
rank, weak scaling); there is no collective on the data path.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

from inferkernellab_b200.workloads import workload_lens, workload_tensors

ROOT = Path(__file__).resolve().parent
METRIC = "paged-decode-attn achieved HBM GB/s"
WORKLOAD = ("config3: ragged paged decode step, B=64/GPU, ctx~U[1,8192], Hq32/Hkv8, D128, "
            "BS16, bf16, pool=1.1x shuffled, 1-token KV append + split-KV attention")


# --------------------------------------------------------------- workload

class Workload:
    def __init__(self, seed: int, device: torch.device, batch=64, num_heads=32, num_kv_heads=8,
                 head_dim=128, block_size=16, max_ctx=8192, dtype=torch.bfloat16):
        from inferkernellab_b200 import PagedKVCache

        t = workload_tensors(seed, device, batch, num_heads, num_kv_heads, head_dim, block_size,
                             max_ctx, dtype)
        self.batch, self.num_heads, self.num_kv_heads = batch, num_heads, num_kv_heads
        self.head_dim, self.block_size, self.dtype = head_dim, block_size, dtype
        self.lens_list = t["lens"]
        self.tables_host = t["tables"]
        self.cache = PagedKVCache(t["num_blocks"], block_size, num_kv_heads, head_dim, dtype=dtype,
                                  device=device)
        self.cache.k.copy_(t["k"])
        self.cache.v.copy_(t["v"])
        del t["k"], t["v"]
        self.query, self.new_k, self.new_v = t["query"], t["new_k"], t["new_v"]
        self.slots_host = t["slots"]
        self.tables = t["tables"].to(device)
        self.lens = torch.tensor(self.lens_list, dtype=torch.int32, device=device)
        self.slots = self.slots_host.to(device)
        self.out = torch.empty_like(self.query)

    # Algorithmic bytes (what the step must move at minimum).
    def decode_bytes(self) -> int:
        es = 2
        kv = sum(self.lens_list) * self.num_kv_heads * self.head_dim * es * 2
        qo = 2 * self.batch * self.num_heads * self.head_dim * es
        table = sum(-(-n // self.block_size) for n in self.lens_list) * 4
        return kv + qo + table + self.batch * 4

    def append_bytes(self) -> int:
        return 2 * 2 * self.batch * self.num_kv_heads * self.head_dim * 2 + self.batch * 4

    def step(self):
        from inferkernellab_b200 import paged_decode_attention_append

        paged_decode_attention_append(self.query, self.new_k, self.new_v, self.cache,
                                      self.tables, self.lens, self.slots, out=self.out)


# ---------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "clocks.mem,clocks.max.mem")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""
        return False

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(",") for r in getattr(self, "out", "").strip().splitlines() if r.strip()]
        sm, smax, reasons, mem, mem_max = [], None, set(), [], None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, flag in zip(names, r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
            if len(r) >= 11:
                try:
                    mem.append(float(r[9]))
                    mem_max = float(r[10])
                except ValueError:
                    pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "mem_mhz": statistics.median(mem) if mem else None, "mem_max_mhz": mem_max,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "nvidia-smi every 50 ms over a 1 s untimed soak of the step, the timed steps and the per-launch event pass"}


# ------------------------------------------------------------------ helpers

def _peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _ncu_traffic() -> float | None:
    """DRAM bytes per decode launch from the committed ncu summary, if present."""
    path = ROOT / "profiles" / "decode_config3_ncu.md"
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", path.read_text())
        return float(m.group(1)) if m else None
    except OSError:
        return None


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _barrier_sync(world):
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ arms

def run_ours(args, world, rank, local) -> dict | None:
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = Workload(seed=args.seed + 1000 * rank, device=device)
    step_bytes = wl.decode_bytes() + wl.append_bytes()
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        wl.step()
    from inferkernellab_b200 import check_device_errors, paged_decode_attention_append

    if check_device_errors() & ~8:
        raise RuntimeError("device error word set during warm-up")
    # ---- device-resident timed region ----
    k_steps = args.steps
    dec_start = [torch.cuda.Event(enable_timing=True) for _ in range(k_steps)]
    dec_end = [torch.cuda.Event(enable_timing=True) for _ in range(k_steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # An untimed soak of at least a second inside the sampler's window, so
        # that the clock record holds samples under load even when the timed
        # region itself is a few milliseconds.
        soak_end = time.perf_counter() + 1.0
        while time.perf_counter() < soak_end:
            for _ in range(64):
                wl.step()
            torch.cuda.synchronize(device)
        _barrier_sync(world)
        t0.record(stream)
        for i in range(k_steps):
            paged_decode_attention_append(wl.query, wl.new_k, wl.new_v, wl.cache, wl.tables,
                                          wl.lens, wl.slots, out=wl.out)
        t1.record(stream)
        _barrier_sync(world)
        # The roofline's per-launch time: a second pass with an event pair around
        # every launch (kept out of the timed region above, where the events
        # themselves would add a few microseconds per step).
        for i in range(k_steps):
            dec_start[i].record(stream)
            paged_decode_attention_append(wl.query, wl.new_k, wl.new_v, wl.cache, wl.tables,
                                          wl.lens, wl.slots, out=wl.out)
            dec_end[i].record(stream)
        torch.cuda.synchronize(device)
    elapsed_ms = _max_over_ranks(t0.elapsed_time(t1), world, device)
    dec_ms = sum(a.elapsed_time(b) for a, b in zip(dec_start, dec_end)) / k_steps
    # ---- end-to-end through the public API with host buffers ----
    # Every step copies its inputs from pinned host memory and its output back,
    # inside the timed region.  As a serving loop does, the copies run on their
    # own streams against two device buffer sets: step i+1's inputs go up and
    # step i-1's output comes down while step i's kernel runs.
    pin = dict(pin_memory=True)
    q_h = wl.query.cpu().pin_memory()
    k_h, v_h = wl.new_k.cpu().pin_memory(), wl.new_v.cpu().pin_memory()
    tab_h = wl.tables_host.pin_memory()
    len_h = torch.tensor(wl.lens_list, dtype=torch.int32).pin_memory()
    slot_h = wl.slots_host.pin_memory()
    hosts = (q_h, k_h, v_h, tab_h, len_h, slot_h)
    out_hs = [torch.empty(wl.query.shape, dtype=wl.dtype, **pin) for _ in range(2)]
    sets = [[torch.empty(t.shape, dtype=t.dtype, device=device) for t in hosts]
            + [torch.empty_like(wl.query)] for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in hosts)
    d2h = out_hs[0].numel() * out_hs[0].element_size()
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    inputs_in = [torch.cuda.Event() for _ in range(2)]
    kernel_done = [torch.cuda.Event() for _ in range(2)]
    output_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i & 1
        d_q, d_k, d_v, d_tab, d_len, d_slot, d_out = sets[b]
        with torch.cuda.stream(up):
            up.wait_event(kernel_done[b])  # the last kernel that read this set is done
            for dst, src in zip(sets[b], hosts):
                dst.copy_(src, non_blocking=True)
            inputs_in[b].record(up)
        stream.wait_event(inputs_in[b])
        stream.wait_event(output_out[b])  # this set's last output has been copied out
        paged_decode_attention_append(d_q, d_k, d_v, wl.cache, d_tab, d_len, d_slot, out=d_out)
        kernel_done[b].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(kernel_done[b])
            out_hs[b].copy_(d_out, non_blocking=True)
            output_out[b].record(down)

    for i in range(4):
        e2e_step(i)
    stream.wait_stream(down)
    _barrier_sync(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_stream(stream)  # no copy of the timed steps starts before e0
    for i in range(k_steps):
        e2e_step(i)
    stream.wait_stream(down)  # ... and the last output copy ends before e1
    e1.record(stream)
    _barrier_sync(world)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world, device)
    if not torch.equal(out_hs[(k_steps - 1) & 1].to(device), wl.out):
        raise RuntimeError("end-to-end output differs from the device-resident step")
    errors = check_device_errors()
    if errors & ~8:
        raise RuntimeError(f"device error word {errors:#x} after the timed region")

    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    achieved = step_bytes / (dec_ms * 1e-3) / 1e9
    total_bytes = step_bytes * k_steps * world
    value = total_bytes / (elapsed_ms * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    record = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": k_steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / k_steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/Q, seeded U[1,8192] context lengths)",
        "config": {
            "workload": WORKLOAD,
            "batch_per_gpu": wl.batch,
            "sum_ctx_rank0": sum(wl.lens_list),
            "num_blocks_rank0": wl.cache.layout.num_blocks,
            "step_bytes_rank0": step_bytes,
            "l2": "no flush: 1.08 GB working set per step is >8x the 126 MB L2",
            "parallelism": f"request-partitioned dp{world}, no data-path collective",
            "seed": args.seed,
        },
        "decode_tok_s": round(wl.batch * world * k_steps / (elapsed_ms * 1e-3), 1),
        "roofline": {
            "bound": "hbm",
            "kernel": "paged_decode_kernel<BF16,128,-1,true> (append fused; G=4: keys as M)",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6650 GB/s",
            "traffic": _ncu_traffic(),
            "algorithmic_bytes_per_launch": step_bytes,
            "avg_launch_ms": round(dec_ms, 5),
            "frac_of_nominal_8TBs": round(achieved / 8000.0, 4),
        },
        "e2e": {
            "value": round(e2e_value, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": round(e2e_ms / k_steps, 5),
            "api": "inferkernellab_b200.paged_decode_attention_append, pinned host buffers; "
                   "H2D/D2H on side streams overlap the neighbouring steps' kernels",
        },
        "gpu_launches": k_steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        record["cpu_baseline"] = cpu_baseline(wl, budget_s=args.cpu_budget, seed=args.seed)
    return record


def _bits(t: torch.Tensor) -> np.ndarray:
    """bfloat16 tensor -> numpy uint16 bit patterns (the oracle's bf16 storage)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_sample_from(wl: Workload, max_tokens: int):
    """Copy the first requests of a GPU workload (up to max_tokens of context) to host numpy."""
    chosen, total = [], 0
    for b, n in enumerate(wl.lens_list):
        if chosen and total + n > max_tokens:
            break
        chosen.append(b)
        total += n
    bs = wl.block_size
    blocks, tables = [], []
    for b in chosen:
        need = -(-wl.lens_list[b] // bs)
        tables.append(list(range(len(blocks), len(blocks) + need)))
        blocks.extend(wl.tables_host[b, :need].tolist())
    idx = torch.tensor(blocks, dtype=torch.long, device=wl.cache.k.device)
    return (_bits(wl.query[chosen]), _bits(wl.cache.k[:, idx]), _bits(wl.cache.v[:, idx]), tables,
            [wl.lens_list[b] for b in chosen])


def _oracle_sample_from_host(seed: int, max_tokens: int, num_heads=32, num_kv_heads=8,
                             head_dim=128, block_size=16):
    """Leading requests of the config-3 batch with host-drawn values (numpy)."""
    lens_all = workload_lens(seed)
    lens, total = [], 0
    for n in lens_all:
        if lens and total + n > max_tokens:
            break
        lens.append(n)
        total += n
    need = [-(-n // block_size) for n in lens]
    rng = np.random.default_rng(seed)
    nb = sum(need)
    perm = rng.permutation(nb)
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n].tolist())
        cur += n
    shape = (1, nb, block_size, num_kv_heads, head_dim)
    k = _bits(torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).bfloat16())
    v = _bits(torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).bfloat16())
    q = _bits(torch.from_numpy(
        rng.standard_normal((len(lens), num_heads, head_dim), dtype=np.float32)).bfloat16())
    return q, k, v, tables, lens


def _oracle_bytes(lens, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16) -> int:
    es = 2
    return (sum(lens) * num_kv_heads * head_dim * es * 2 + 2 * len(lens) * num_heads * head_dim * es
            + sum(-(-n // block_size) for n in lens) * 4 + len(lens) * 4)


def _time_oracle(q, k, v, tables, lens, threads: int) -> float:
    import oracle  # the CPU restatement: only the baseline legs of this file use it

    def one(b):
        return oracle.paged_decode_attention(q[b:b + 1], k, v, "bf16", [tables[b]], [lens[b]])

    t = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as pool:
        list(pool.map(one, range(len(lens))))
    return time.perf_counter() - t


def _reference_package():
    """The reference project installed under baseline/_ref, or (None, why)."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "inferkernellab").is_dir():
        return None, "baseline/_ref holds no reference install"
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    try:
        from inferkernellab import attention, cache  # the reference's own modules
    except Exception as exc:  # noqa: BLE001 -- any import failure means "not available"
        return None, f"reference import failed: {type(exc).__name__}: {exc}"
    return (attention, cache), ""


class ReferenceStep:
    """One config-3 step through the reference's own CPU path, on host tensors.

    ``PagedKVCache.write_slots`` appends the new token of every request
    (reference ``cache.py:156-189``), then ``paged_decode_attention`` -- the
    reference's ``paged_reference`` backend, a per-request gather and a float32
    dense attention (``attention.py:134-175``) -- attends over the whole context.
    The inputs are the GPU arm's tensors of the same seed, copied to the host.
    """

    def __init__(self, modules, seed: int):
        attention, cache_mod = modules
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
            else torch.device("cpu")
        t = workload_tensors(seed, device)
        self._all = dict(lens=t["lens"], tables=t["tables"], query=t["query"].cpu(),
                         new_k=t["new_k"].cpu(), new_v=t["new_v"].cpu(), slots=t["slots"].cpu())
        self.cache = cache_mod.PagedKVCache(t["num_blocks"], t["block_size"], t["num_kv_heads"],
                                            t["head_dim"], dtype=t["dtype"], device="cpu")
        self.cache.k.copy_(t["k"].cpu())
        self.cache.v.copy_(t["v"].cpu())
        del t
        self.attention = attention
        self.same_data = device.type == "cuda"
        self.restrict(len(self._all["lens"]))

    def restrict(self, requests: int) -> "ReferenceStep":
        """Make a step cover the leading ``requests`` requests of the batch."""
        a, n = self._all, requests
        self.lens, self.tables, self.query = a["lens"][:n], a["tables"][:n], a["query"][:n]
        self.new_k, self.new_v, self.slots = a["new_k"][:n], a["new_v"][:n], a["slots"][:n]
        self.bytes = _oracle_bytes(self.lens) + 2 * 2 * n * 8 * 128 * 2 + n * 4
        return self

    def seconds_per_token(self) -> float:
        """Times one step over the first 4 requests (warms the code path too)."""
        n = len(self.lens)
        self.restrict(4)
        t = time.perf_counter()
        self()
        per_token = (time.perf_counter() - t) / max(1, sum(self.lens))
        self.restrict(n)
        return per_token

    def __call__(self):
        self.cache.write_slots(0, self.slots, self.new_k, self.new_v)
        return self.attention.paged_decode_attention(self.query, self.cache, self.tables,
                                                     self.lens)


def _reference_requests(seed: int, budget_s: float, per_step_probe) -> int:
    """How many leading requests of the batch fit in ``budget_s`` per step."""
    lens = workload_lens(seed)
    per_token = per_step_probe
    total, n = 0, 0
    for length in lens:
        if n and (total + length) * per_token > budget_s:
            break
        total += length
        n += 1
    return n


def cpu_baseline(wl: Workload, budget_s: float, seed: int) -> dict:
    """The reference's own CPU path (baseline/_ref) on host cores, bounded sample.

    Falls back to the numpy restatement in ``oracle/`` (``kind: "port"``) when
    the reference install is absent.
    """
    threads = os.cpu_count() or 1
    modules, why = _reference_package()
    if modules is not None:
        torch.set_num_threads(threads)
        step = ReferenceStep(modules, seed)
        n = _reference_requests(seed, budget_s, step.seconds_per_token())
        step.restrict(n)
        t = time.perf_counter()
        step()
        secs = time.perf_counter() - t
        return {"value": round(step.bytes / secs / 1e9, 4), "unit": "GB/s",
                "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"first {n} of the 64 requests of rank 0 ({sum(step.lens)} context "
                          f"tokens): the reference's write_slots + paged_decode_attention "
                          f"(baseline/_ref, torch CPU, bf16 cache, fp32 math), "
                          f"{torch.get_num_threads()} threads, {secs:.2f} s"}
    q, k, v, tables, lens = _oracle_sample_from(wl, max_tokens=4096)
    probe = _time_oracle(q, k, v, tables, lens, threads)
    per_token = probe / max(1, sum(lens))
    target_tokens = int(budget_s / max(per_token, 1e-9))
    q, k, v, tables, lens = _oracle_sample_from(wl, max_tokens=max(4096, target_tokens))
    secs = _time_oracle(q, k, v, tables, lens, threads)
    gbs = _oracle_bytes(lens) / secs / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"first {len(lens)} of the 64 requests of rank 0 ({sum(lens)} context "
                      f"tokens), numpy float32 restatement of paged_decode_attention, "
                      f"{threads} threads, {secs:.2f} s ({why})"}


def run_reference(args, world, rank) -> dict | None:
    """CPU reference arm: the reference's own CPU path, same metric and config.

    With the reference installed under baseline/_ref, every step is
    ``write_slots`` + ``paged_decode_attention`` of the reference itself on the
    GPU arm's seed-0 batch (the whole batch when warm-up + steps fit in about
    two minutes, else its leading requests); without it, the numpy
    restatement of the same algorithm.  Rank 0 alone runs it.
    """
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    warm = min(args.warmup, 3)
    per_step_s = 120.0 / (args.steps + warm)
    modules, why = _reference_package()
    if modules is not None:
        torch.set_num_threads(threads)
        step = ReferenceStep(modules, args.seed)
        n = _reference_requests(args.seed, per_step_s, step.seconds_per_token())
        step.restrict(n)
        for _ in range(warm):
            step()
        secs = []
        for _ in range(args.steps):
            t = time.perf_counter()
            step()
            secs.append(time.perf_counter() - t)
        kind, cores, step_bytes = "reference", torch.get_num_threads(), step.bytes
        same = n == 64 and step.same_data
        sample = (f"{'all' if n == 64 else f'first {n} of the'} 64 requests of the config-3 "
                  f"batch ({sum(step.lens)} context tokens{'' if step.same_data else ', CPU-drawn values'}) per step: "
                  f"the reference's PagedKVCache.write_slots + paged_decode_attention "
                  f"(baseline/_ref, torch CPU, bf16 cache, fp32 math), {cores} threads")
    else:
        q, k, v, tables, lens = _oracle_sample_from_host(args.seed, max_tokens=2048)
        per_token = _time_oracle(q, k, v, tables, lens, threads) / max(1, sum(lens))
        tokens = int(min(8192 * 4, max(64, per_step_s / max(per_token, 1e-9))))
        q, k, v, tables, lens = _oracle_sample_from_host(args.seed, max_tokens=tokens)
        for _ in range(warm):
            _time_oracle(q, k, v, tables, lens, threads)
        secs = [_time_oracle(q, k, v, tables, lens, threads) for _ in range(args.steps)]
        kind, cores, step_bytes, same = "port", threads, _oracle_bytes(lens), False
        sample = (f"first {len(lens)} requests of the config-3 batch ({sum(lens)} context "
                  f"tokens) per step, numpy float32 restatement of the reference "
                  f"paged_decode_attention, {threads} threads ({why})")
    total = sum(secs)
    gbs = step_bytes * len(secs) / total / 1e9
    return {
        "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / len(secs) * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": WORKLOAD, "sample": sample, "same_config": same,
                   "seed": args.seed},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def _json_stdout():
    """Keep stdout for this program's JSON line alone.

    Libraries may print to stdout (NCCL prints a version banner when the
    environment sets NCCL_DEBUG=VERSION, as the GPU boxes here do): file
    descriptor 1 is pointed at stderr for the rest of the run, and the JSON line
    goes to a duplicate of the original stdout.
    """
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main(argv=None) -> int:
    json_out = _json_stdout()
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--cpu-budget", type=float, default=10.0,
                        help="seconds of CPU work for the cpu_baseline sample")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    world, rank, local = _dist()
    if world != args.gpus and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        record = run_reference(args, world, rank)
        if record:
            print(json.dumps(record), file=json_out, flush=True)
        return 0
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    try:
        record = run_ours(args, world, rank, local)
        if record:
            print(json.dumps(record), file=json_out, flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
