"""Multi-process request sharding on CPU ranks (gloo, world size 2).

Each rank decodes its contiguous slice of the requests with the CPU oracle; gathering the
slices reproduces a single-process run over all requests (tokens and history exactly, logits
within float32 tolerance), so sharding needs no collective inside the step.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from ckl.workloads.sharding import request_range, shard_prompts

CONFIG = dict(batch=6, hidden=32, heads=2, layers=2, ffn=48, vocab=64, context=5, steps=4)


def test_request_ranges_partition_the_job():
    for total, world in ((4096, 8), (7, 2), (5, 4), (1, 1)):
        ranges = [request_range(total, world, r) for r in range(world)]
        covered = [i for a, b in ranges for i in range(a, b)]
        assert covered == list(range(total))
    with pytest.raises(ValueError):
        request_range(4, 2, 2)


def _decode_shard(config, seed, world, rank):
    from oracle import decoder as ref

    full = ref.Config(**config)
    arrays, rng = ref.make_weights(full, seed)
    prompts = ref.make_prompts(full, rng)
    local = shard_prompts(prompts, world, rank)
    shard = ref.Config(**{**config, "batch": local.shape[1]})
    state = {k: v for k, v in arrays.items()}
    state.update(ref.empty_state(shard))
    state["tokens"] = local[0].copy()
    for i in range(shard.context - 1):
        ref.decode_step(state, shard)
        state["tokens"][:] = local[i + 1]
    for _ in range(shard.steps):
        ref.decode_step(state, shard)
    return state


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        state = _decode_shard(CONFIG, 9, world, rank)
        history = torch.from_numpy(state["history"].T.copy())          # [local, T]
        logits = torch.from_numpy(state["logits"].copy())
        gathered_h = [torch.zeros_like(history) for _ in range(world)]
        gathered_l = [torch.zeros_like(logits) for _ in range(world)]
        dist.all_gather(gathered_h, history)
        dist.all_gather(gathered_l, logits)
        elapsed = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)                  # bench's max over ranks
        if rank == 0:
            queue.put((torch.cat(gathered_h).numpy(), torch.cat(gathered_l).numpy(),
                       float(elapsed.item())))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_the_single_process_job():
    from oracle import decoder as ref

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    processes = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in processes:
        p.start()
    history, logits, slowest = queue.get(timeout=120)
    for p in processes:
        p.join(timeout=60)
        assert p.exitcode == 0
    single = _decode_shard(CONFIG, 9, 1, 0)
    assert np.array_equal(history, single["history"].T)
    assert np.allclose(logits, single["logits"], rtol=1e-4, atol=1e-5)
    assert slowest == 2.0
