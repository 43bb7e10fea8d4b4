"""Multi-rank host logic on CPU: image sharding and the ordered gather of
pooled embeddings, run as world_size-2 gloo process groups (the GPU run uses
the same code over NCCL)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b2q import synth
from b2q.shard import gather_in_order, per_rank_capacity, shard_images, shard_rows


def test_shard_images_is_a_balanced_partition():
    grids = synth.naflex_grids(512, seed=0)
    for world in (1, 2, 4, 8):
        parts = [shard_images(grids, r, world) for r in range(world)]
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(grids)))
        tokens = [sum(grids[i][0] * grids[i][1] for i in p) for p in parts]
        assert max(tokens) - min(tokens) <= 1024          # one image's worth at most
        assert max(len(p) for p in parts) <= per_rank_capacity(len(grids), world)


def test_shard_rows_covers_prompts():
    for n, world in ((1000, 8), (5, 2), (3, 4)):
        parts = [list(shard_rows(n, r, world)) for r in range(world)]
        assert [i for p in parts for i in p] == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_images, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        grids = synth.naflex_grids(n_images, seed=3)
        mine = shard_images(grids, rank, world)
        # stand-in embedding of image i: its index in every column
        local = torch.tensor([[float(i)] * 4 for i in mine], dtype=torch.float32).reshape(-1, 4)
        out = gather_in_order(local, mine, n_images)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_images", [7, 64])
def test_gather_in_order_two_ranks(n_images):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_images, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = np.repeat(np.arange(n_images, dtype=np.float32)[:, None], 4, axis=1)
    for r in range(2):
        np.testing.assert_array_equal(results[r], expect)
