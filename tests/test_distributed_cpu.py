"""Multi-process (gloo) tests of the batch-sharding host logic.

Each rank computes the oracle forward of its shard of a GPT2 batch and the
shards are gathered over the gloo group; the gathered logits must equal the
unsharded forward.  ``wxx_b200.distributed.HostGather`` runs the same slot
padding and rank-order assembly as the device path (``gather_layout`` /
``assemble_slots``), so uneven shards and idle ranks (batch < world) are
covered here.  Also checks that a rank that never joins, or that leaves
between steps, ends the others with an error instead of a hang (short
process-group timeout)."""

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


def _uneven_worker(rank, world, port, batch, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
        from oracle import init, models
        from wxx_b200.distributed import HostGather, init_host_group, shard_bounds

        dist = init_host_group(timeout_s=60)
        sd = init.gpt2_state_dict(0, 64, 32, 4, 2, 16)
        ids = init.token_ids(1, batch, 16, 64)
        lo, hi = shard_bounds(batch, world, rank)
        local = models.gpt2_forward(sd, ids[lo:hi], 4, 2, fast=True) if hi > lo else None
        g = HostGather(dist, world)
        full = g.allgather_rows(local, batch, (16, 64), np.float32)
        # token ids (u32) go through the same path
        am = None if local is None else local.argmax(-1).astype(np.uint32)
        full_ids = g.allgather_rows(am, batch, (16,), np.uint32)
        ref = models.gpt2_forward(sd, ids, 4, 2, fast=True)
        ok_ids = bool(np.array_equal(full_ids, ref.argmax(-1).astype(np.uint32)))
        q.put((rank, (float(np.abs(full - ref).max()), full.shape[0], ok_ids)))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,batch", [(3, 5), (3, 2), (2, 7)])
def test_uneven_and_idle_shards_assemble_in_rank_order(world, batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_uneven_worker, args=(r, world, port, batch, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in results.items():
        assert isinstance(v, tuple), (r, v)
        err, rows, ok_ids = v
        assert err < 1e-6 and rows == batch and ok_ids, (r, v)


def test_gather_layout_and_assembly():
    from wxx_b200.distributed import assemble_slots, gather_layout

    rows, spans = gather_layout(5, 3)
    assert rows == 2 and spans == [(0, 2), (2, 4), (4, 5)]
    rows, spans = gather_layout(2, 4)           # two idle ranks still send one row
    assert rows == 1 and spans[2] == (2, 2) and spans[3] == (2, 2)
    slots = np.arange(4 * 1 * 3).reshape(4, 3)
    out = assemble_slots(slots, 2, 4)
    assert np.array_equal(out, slots[:2])
    slots = np.array([[0], [1], [2], [3], [4], [-1]])  # rank 2's second slot row is padding
    assert assemble_slots(slots, 5, 3)[:, 0].tolist() == [0, 1, 2, 3, 4]
    with pytest.raises(ValueError):
        assemble_slots(slots[:5], 5, 3)


def _leaver(rank, port, q):
    """Rank 1 takes part in step 1 and exits between steps; rank 0's step-2
    gather must end in an error within the process-group timeout."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE="2", LOCAL_RANK=str(rank))
        from wxx_b200.distributed import HostGather, init_host_group

        dist = init_host_group(timeout_s=5)
        g = HostGather(dist, 2)
        first = g.allgather_rows(np.full((1, 3), rank, np.float32), 2, (3,), np.float32)
        if rank == 1:
            q.put((rank, "left after step 1"))
            q.close()
            q.join_thread()          # the message is sent before the process goes
            os._exit(0)
        try:
            g.allgather_rows(np.zeros((1, 3), np.float32), 2, (3,), np.float32)
            q.put((rank, "step 2 completed without its peer"))
        except Exception as e:
            q.put((rank, "error:" + type(e).__name__ + ":" + str(first[:, 0].tolist())))
    except Exception as e:  # pragma: no cover
        q.put((rank, "setup:" + repr(e)))


def test_rank_leaving_between_steps_errors_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1] == "left after step 1", results
    assert results[0].startswith("error:") and results[0].endswith("[0.0, 1.0]"), results
