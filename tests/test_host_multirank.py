"""Request partitioning and the per-step token exchange, as 2 gloo ranks on CPU.

The multi-GPU decoder (``e2e_bench`` under torchrun) partitions the requests
contiguously over the ranks (``llama.partition_requests``); every rank serves
its slice with its own block pool and runtime, and every decode step
all-gathers the sampled token ids of all ranks (``llama.allgather_token_exchange``,
the only collective on the path).  Here each rank is a CPU process on the gloo
backend and the model is a deterministic stand-in (the next token is a hash of
the request's sequence), so the test checks the host side exactly: the
gathered ids of every step must equal a single-process run over all requests.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferkernellab_b200.cache import PagedKVCache
from inferkernellab_b200.llama import allgather_token_exchange, partition_requests
from inferkernellab_b200.runtime import InferenceRuntime
from inferkernellab_b200.scheduler import TokenBudgetScheduler

VOCAB = 1000
MAX_NEW = 6
BLOCK = 4


def _prompts():
    return [tuple((7 * i + 3 * j) % VOCAB for j in range(5 + (i * 13) % 40)) for i in range(11)]


def _next_token(prompt, generated) -> int:
    """Stand-in model: a deterministic function of the whole sequence."""
    h = 0
    for t in tuple(prompt) + tuple(generated):
        h = (h * 1000003 + t + 1) % (2 ** 31)
    return h % VOCAB


def _serve(prompts, ids, exchange=None, record=None):
    """One rank's serving loop over requests ``ids``: own pool, own runtime."""
    need = sum(-(-(len(prompts[i]) + MAX_NEW) // BLOCK) for i in ids)
    cache = PagedKVCache(max(1, need), BLOCK, 1, 8, device="cpu")
    sched = TokenBudgetScheduler(max_num_seqs=max(1, len(ids)), max_num_batched_tokens=32)
    generated = {rid: [] for rid in ids}

    def decode(requests):
        tokens = torch.tensor([_next_token(prompts[r.request_id], generated[r.request_id])
                               for r in requests], dtype=torch.long)
        if exchange is not None:
            exchange(tokens)
            record.append(exchange.last.clone())
        for r, t in zip(requests, tokens.tolist()):
            generated[r.request_id].append(t)

    runtime = InferenceRuntime(cache, sched, prefill_batch_fn=lambda *args: None,
                               decode_fn=decode)
    for rid in ids:
        runtime.submit(rid, len(prompts[rid]), MAX_NEW)
    while sched.waiting or sched.running:
        runtime.step()
    return generated, cache.allocator.num_used_blocks


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = _prompts()
        part = partition_requests(len(prompts), world, rank)
        per = -(-len(prompts) // world)
        record = []
        generated, used = _serve(prompts, list(part), allgather_token_exchange(max_local=per),
                                 record)
        torch.save({"part": (part.start, part.stop), "record": record, "generated": generated,
                    "used_blocks": used}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_is_contiguous_and_covers_every_request():
    for n, world in [(256, 8), (11, 2), (11, 4), (3, 8), (1, 1)]:
        parts = [partition_requests(n, world, r) for r in range(world)]
        flat = [i for p in parts for i in p]
        assert flat == list(range(n))
        assert max(len(p) for p in parts) == -(-n // world)
    with pytest.raises(ValueError):
        partition_requests(4, 2, 2)


@pytest.mark.parametrize("world", [2])
def test_gloo_ranks_gather_the_single_process_tokens(world, tmp_path):
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    prompts = _prompts()
    single, used = _serve(prompts, list(range(len(prompts))))
    assert used == 0
    per = -(-len(prompts) // world)
    results = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r, res in enumerate(results):
        assert res["used_blocks"] == 0  # each rank's own pool is released
        start, stop = res["part"]
        assert {rid: single[rid] for rid in range(start, stop)} == res["generated"]
        assert len(res["record"]) == MAX_NEW  # one exchange per decode step
    for step in range(MAX_NEW):
        want = torch.full((world, per), -1, dtype=torch.int32)
        for r in range(world):
            part = partition_requests(len(prompts), world, r)
            want[r, :len(part)] = torch.tensor([single[rid][step] for rid in part])
        for res in results:  # every rank holds the same gathered matrix
            assert torch.equal(res["record"][step], want)
