"""The multi-GPU plumbing of bench.py on CPU: LPT sharding of clips across ranks
and the single all-gather of finished embeddings, run as two gloo ranks (no GPU).
The GPU path uses the same functions with NCCL (one process per GPU)."""
import os
import socket

import numpy as np
import pytest

import bench


def test_lpt_shard_covers_every_clip_once_and_balances():
    lengths = bench.global_lengths(4, 1000)
    shards = bench.lpt_shard(lengths, 4)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lengths)))
    loads = [int(lengths[s].sum()) for s in map(np.array, shards)]
    assert max(loads) - min(loads) <= int(lengths.max())
    assert max(len(s) for s in shards) <= 1000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_clips, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = bench.global_lengths(world, n_clips // world)
        shards = bench.lpt_shard(lengths, world)
        n_max = max(len(s) for s in shards)
        local = torch.zeros(n_max, 4)
        for k, clip in enumerate(shards[rank]):  # stand-in "embedding": the clip id
            local[k] = float(clip)
        gathered = torch.empty(world * n_max, 4)
        bench.gather_embeddings(local, gathered, world)
        ordered = bench.restore_order(gathered, shards, n_max)
        ok = bool(torch.equal(ordered[:, 0], torch.arange(len(lengths), dtype=torch.float32)))
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_in_clip_order():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, 64, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(res) == [(0, True), (1, True)]
