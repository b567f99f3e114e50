"""Multi-process (gloo, world_size 2) tests of the batch-sharding host logic.

Each rank computes the oracle forward of its shard of a GPT2 batch and the
shards are gathered over the gloo group; the gathered logits must equal the
unsharded forward.  Also checks that a rank that never joins ends the others
with an error instead of a hang (short process-group timeout)."""

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
        import torch
        import torch.distributed as dist

        from oracle import init, models
        from wxx_b200.distributed import init_host_group, shard_bounds

        init_host_group(timeout_s=60)
        sd = init.gpt2_state_dict(0, 64, 32, 4, 2, 16)
        ids = init.token_ids(1, 6, 16, 64)
        lo, hi = shard_bounds(6, world, rank)
        local = models.gpt2_forward(sd, ids[lo:hi], 4, 2, fast=True)
        parts = [torch.zeros((hi - lo,) + local.shape[1:]) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(local))
        full = np.concatenate([p.numpy() for p in parts], axis=0)
        ref = models.gpt2_forward(sd, ids, 4, 2, fast=True)
        q.put((rank, float(np.abs(full - ref).max())))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, repr(e)))


def test_sharded_forward_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(v, float) and v < 1e-6 for v in results.values()), results


def test_shard_bounds_cover_batch_once():
    from wxx_b200.distributed import shard_bounds

    for batch in (4, 7, 64, 256):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _lonely(port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0",
                          WORLD_SIZE="2", LOCAL_RANK="0")
        from wxx_b200.distributed import init_host_group

        init_host_group(timeout_s=5)
        q.put("joined")
    except Exception as e:
        q.put("error:" + type(e).__name__)


def test_missing_rank_errors_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    assert res.startswith("error:"), res
