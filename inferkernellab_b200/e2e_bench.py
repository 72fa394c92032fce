"""Config-5 end-to-end decoder benchmark: Llama-3-8B shape on 1..8 B200s.

``python -m inferkernellab_b200.e2e_bench`` (one GPU) or
``torchrun --nproc-per-node N -m inferkernellab_b200.e2e_bench`` (N GPUs).

Workload: a random-init Llama-3-8B-shaped decoder --
32 layers, hidden 4096, 32 query / 8 KV heads, head_dim 128, intermediate
14336, vocab 128256, RMSNorm, RoPE theta 5e5, bf16 weights ~ N(0, 0.02) --
serving 256 requests whose prompt token ids and lengths (uniform in
[64, 1024]) are drawn from a seeded generator: batched prefill under a
2048-token budget, then 128 greedy decode steps.

Parallelism: the requests are partitioned contiguously over the ranks (one
process per GPU, each with its own weights replica and block pool); every
decode step all-gathers the sampled token ids over NCCL -- the only collective.
``value`` = all generated tokens of all ranks / the max over ranks of the
decode-phase time (strong scaling: the 256 requests are fixed).  The weights
are initialised on the GPU (same N(0, 0.02) scheme as the reference's
``_load_model``, GPU random stream), which is the practical way to build an
8B model; correctness at this scale is covered by the small-model parity tests.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

import torch

from .llama import LlamaPagedDecodeRunner, allgather_token_exchange, load_random_llama


def make_prompts(num_requests: int, min_len: int, max_len: int, vocab: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (num_requests,), generator=gen).tolist()
    return [torch.randint(0, vocab, (n,), generator=gen).tolist() for n in lens]


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--min-prompt", type=int, default=64)
    p.add_argument("--max-prompt", type=int, default=1024)
    p.add_argument("--max-new-tokens", type=int, default=128)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--intermediate", type=int, default=14336)
    p.add_argument("--vocab", type=int, default=128256)
    p.add_argument("--rope-theta", type=float, default=5e5)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--max-num-batched-tokens", type=int, default=2048)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cuda-graph", action="store_true",
                   help="launch the decode step eagerly instead of replaying one CUDA graph")
    args = p.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=device)
    try:
        prompts = make_prompts(args.requests, args.min_prompt, args.max_prompt, args.vocab,
                               args.seed)
        per = -(-len(prompts) // world)
        mine = prompts[rank * per:(rank + 1) * per]
        t0 = time.perf_counter()
        model = load_random_llama(vocab_size=args.vocab, hidden_size=args.hidden,
                                  intermediate_size=args.intermediate, num_layers=args.layers,
                                  num_attention_heads=args.heads, num_kv_heads=args.kv_heads,
                                  max_position_embeddings=args.max_prompt + args.max_new_tokens,
                                  rope_theta=args.rope_theta, seed=args.seed, device=device,
                                  dtype=torch.bfloat16, init_on_device=True)
        init_s = time.perf_counter() - t0
        exchange = allgather_token_exchange(max_local=per) if world > 1 else None
        runner = LlamaPagedDecodeRunner(model, mine, max_new_tokens=args.max_new_tokens,
                                        block_size=args.block_size,
                                        max_num_batched_tokens=args.max_num_batched_tokens,
                                        token_exchange=exchange, collect_logits=False,
                                        cuda_graph=not args.no_cuda_graph)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        result = runner.run()
        decode_ms = sum(result.decode_step_wall_ms)
        stats = torch.tensor([decode_ms, result.prefill_wall_ms, result.tpot_wall_ms,
                              float(sum(len(t) for t in result.generated_tokens))],
                             dtype=torch.float64, device=device)
        if world > 1:
            gathered = [torch.empty_like(stats) for _ in range(world)]
            torch.distributed.all_gather(gathered, stats)
        else:
            gathered = [stats]
        if rank == 0:
            g = torch.stack(gathered).cpu()
            decode_max = float(g[:, 0].max())
            tokens = float(g[:, 3].sum())
            record = {
                "metric": "decode tok/s (config5 Llama-3-8B-shaped, 256 requests)",
                "value": round(tokens / (decode_max / 1e3), 1),
                "unit": "tok/s", "n_gpus": world, "scaling": "strong",
                "decode_ms_max_over_ranks": round(decode_max, 2),
                "prefill_ms_max_over_ranks": round(float(g[:, 1].max()), 2),
                "tpot_ms_max_over_ranks": round(float(g[:, 2].max()), 3),
                "generated_tokens": int(tokens),
                "requests_per_rank": per, "prompt_tokens_total": sum(len(x) for x in prompts),
                "model_init_s": round(init_s, 2),
                "peak_memory_gb_rank0": round(result.peak_memory_allocated_bytes / 1e9, 2),
                "peak_kv_gb_rank0": round(result.peak_kv_memory_bytes / 1e9, 2),
                "config": {"layers": args.layers, "hidden": args.hidden, "heads": args.heads,
                           "kv_heads": args.kv_heads, "intermediate": args.intermediate,
                           "vocab": args.vocab, "rope_theta": args.rope_theta,
                           "block_size": args.block_size, "budget": args.max_num_batched_tokens,
                           "prompt_len": [args.min_prompt, args.max_prompt],
                           "max_new_tokens": args.max_new_tokens, "seed": args.seed,
                           "dtype": "bf16", "backend": "b200_paged",
                           "decode_step": "eager" if args.no_cuda_graph else "cuda_graph"},
            }
            print(json.dumps(record), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
