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


# ---- zero-shot scoring sharded over two ranks ------------------------------
def _zs_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    from datetime import timedelta
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    import oracle as O
    from b2q.zeroshot import zero_shot
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        H, n_img, n_txt = 48, 11, 7
        emb_i = np.random.default_rng(1).standard_normal((n_img, H)).astype(np.float32)
        emb_t = np.random.default_rng(2).standard_normal((n_txt, H)).astype(np.float32)
        seen = {}

        def enc_img(rows):
            seen["img"] = list(rows)
            return torch.from_numpy(emb_i[rows.start:rows.stop].copy())

        def enc_txt(rows):
            seen["txt"] = list(rows)
            return torch.from_numpy(emb_t[rows.start:rows.stop].copy())

        def score(img, txt):
            return torch.from_numpy(O.score(img.numpy(), txt.numpy(), np.log(10.0), -10.0))

        out = zero_shot(enc_img, enc_txt, score, n_img, n_txt, rank, world)
        q.put((rank, out.numpy(), seen))
    finally:
        if world > 1:
            dist.destroy_process_group()


def test_zero_shot_two_ranks_matches_one(oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_zs_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, out, seen = q.get(timeout=120)
        results[r] = (out, seen)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # each rank encoded a disjoint contiguous share of images and of prompts
    assert sorted(results[0][1]["img"] + results[1][1]["img"]) == list(range(11))
    assert sorted(results[0][1]["txt"] + results[1][1]["txt"]) == list(range(7))
    # every rank holds the full score matrix in image order, equal to one process scoring everything
    emb_i = np.random.default_rng(1).standard_normal((11, 48)).astype(np.float32)
    emb_t = np.random.default_rng(2).standard_normal((7, 48)).astype(np.float32)
    ref = oracle.score(emb_i, emb_t, np.log(10.0), -10.0)
    for r in range(2):
        np.testing.assert_array_equal(results[r][0], ref)


# ---- a rank that fails between steps ---------------------------------------
def _fail_worker(rank, world, port, mode, q):
    """Two steps of the embedding gather.  Rank 1 leaves after the first step
    (mode "exit": the process ends; mode "hang": it stops taking part); rank 0
    must get an error from its next collective within the process-group
    timeout and exit non-zero."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import time
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    local = torch.full((2, 4), float(rank))
    mine = [2 * rank, 2 * rank + 1]
    def report(*msg):
        q.put(msg)
        q.close()
        q.join_thread()                      # flushed before a hard exit

    gather_in_order(local, mine, 4)          # step 1: every rank takes part
    if rank == 1:
        report(1, "left", 0.0)
        if mode == "exit":
            os._exit(3)
        time.sleep(600)                      # never joins step 2 (the test ends this process)
        os._exit(4)
    t0 = time.monotonic()
    try:
        gather_in_order(local, mine, 4)      # step 2: the peer is gone
    except Exception as e:                   # noqa: BLE001 - any collective error counts
        report(0, f"error: {type(e).__name__}", time.monotonic() - t0)
        os._exit(1)
    report(0, "completed", time.monotonic() - t0)
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "hang"])
def test_failed_rank_ends_the_survivor_with_an_error(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = {}
        for _ in procs:
            r, what, dt = q.get(timeout=90)
            got[r] = (what, dt)
        assert got[1][0] == "left"
        assert got[0][0].startswith("error"), got[0]
        assert got[0][1] < 60.0, got[0]       # bounded by the 5 s process-group timeout, not a hang
        procs[0].join(timeout=30)
        assert procs[0].exitcode == 1
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()                     # this test's own child process
            p.join(timeout=30)
    if mode == "exit":
        assert procs[1].exitcode == 3
