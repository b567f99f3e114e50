"""Batch-sharded inference across the GPUs of one node.

One process per GPU (launched by ``torch.distributed.run``; RANK, WORLD_SIZE,
LOCAL_RANK from the environment).  Every rank holds the full, replicated
model, runs the forward of its slice of the batch, and the per-rank outputs
are collected with one NCCL all-gather over NVLink / NVSwitch on the kernel
library's stream.  The inference path has no other exchange step: batch
rows are independent (eval-mode BatchNorm, no cross-sample attention).

Host-side coordination (the NCCL unique id, barriers, timing reductions)
goes through a ``torch.distributed`` process group, normally ``gloo``, with a
short timeout so that a missing rank ends in an error instead of a hang.
"""

import ctypes
import datetime
import os

from .backend import device as _dev
from .backend.lib import F, check


def env_rank_world():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def shard_bounds(global_batch, world, rank):
    """Rows [start, stop) of the batch owned by ``rank`` (equal split; the
    first ``global_batch % world`` ranks take one extra row)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(int(global_batch), world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def gather_layout(global_batch, world):
    """(rows_per_slot, spans) for gathering a batch split by ``shard_bounds``:
    every rank sends a slot of ``rows_per_slot`` rows (its shard, zero-padded
    when shorter; at least one row so idle ranks still take part), so the
    all-gather moves equal blocks; ``spans[r]`` = (start, stop) of rank r's
    rows in the assembled batch."""
    spans = [shard_bounds(global_batch, world, r) for r in range(world)]
    rows = max(1, max(hi - lo for lo, hi in spans))
    return rows, spans


def assemble_slots(gathered, global_batch, world):
    """Rank-ordered batch from gathered padded slots (numpy): ``gathered`` is
    (world * rows_per_slot, ...) as the all-gather returns it; the padding rows
    of short shards are dropped."""
    import numpy as np

    rows, spans = gather_layout(global_batch, world)
    gathered = np.asarray(gathered)
    if gathered.shape[0] != world * rows:
        raise ValueError(f"gathered {gathered.shape[0]} rows, expected {world} x {rows}")
    parts = [gathered[r * rows:r * rows + (hi - lo)] for r, (lo, hi) in enumerate(spans)]
    return np.concatenate(parts, axis=0)


class HostGather:
    """The sharded all-gather over the host process group (gloo), on numpy
    arrays, with the same slot padding and rank-order assembly as the device
    path (``NcclCommunicator.allgather_rows``).  Used where no GPU is present:
    CPU tests of the multi-rank logic, host-side result collection."""

    def __init__(self, dist, world):
        self.dist = dist
        self.world = world

    def allgather_rows(self, shard, global_batch, row_shape, dtype):
        import numpy as np
        import torch

        rows, _ = gather_layout(global_batch, self.world)
        slot = np.zeros((rows,) + tuple(row_shape), dtype)
        if shard is not None and len(shard):
            slot[:len(shard)] = shard
        # moved as raw bytes, so any element type (u32 ids, f32 logits) works
        raw = torch.from_numpy(slot.reshape(rows, -1).view(np.uint8).copy())
        parts = [torch.zeros_like(raw) for _ in range(self.world)]
        self.dist.all_gather(parts, raw)
        gathered = np.concatenate([t.numpy() for t in parts]).view(dtype)
        gathered = gathered.reshape((self.world * rows,) + tuple(row_shape))
        return assemble_slots(gathered, global_batch, self.world)


def init_host_group(timeout_s=120):
    """Initialises the gloo process group used for host-side coordination."""
    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
    return dist


class NcclCommunicator:
    """Device all-gather over NCCL (the library's own communicator)."""

    def __init__(self, rank, world, dist):
        import torch

        self.rank = rank
        self.world = world
        _dev.ensure_init()
        uid = (ctypes.c_uint8 * 128)()
        if rank == 0:
            check(F.wxx_nccl_unique_id(uid), "ncclGetUniqueId")
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8)
        dist.broadcast(t, src=0)
        uid = (ctypes.c_uint8 * 128)(*t.tolist())
        check(F.wxx_nccl_init(uid, world, rank), "ncclCommInitRank")
        self._alive = True

    def allgather(self, tensor):
        """[rows, ...] on every rank -> [world * rows, ...] (equal shards)."""
        from .Tensor import Tensor

        src = tensor if tensor.is_dense() else tensor.contiguous()
        shape = [src.shape[0] * self.world] + list(src.shape[1:])
        out = Tensor._empty(shape, src.type)
        check(F.wxx_nccl_allgather(out.buffer.ptr, src.ptr, src.nbytes), "ncclAllGather")
        return out

    def allgather_rows(self, shard, global_batch, row_shape, dtype="f32", slot=None):
        """Gathers a batch split by ``shard_bounds`` (shards may differ by a
        row; a rank with no rows passes ``shard=None``) into
        [global_batch, *row_shape] on every rank, in rank order.  Each rank
        sends a slot of ``gather_layout`` rows (its shard, padded), so unequal
        shards need no second collective.

        ``slot=None``: on the library stream; returns the gathered tensor.
        ``slot=k`` (0..3): on the communication stream while the library stream
        goes on; returns a ``PendingGather`` whose ``wait()`` orders the library
        stream after the gather and returns the tensor."""
        from . import functional
        from .Tensor import Tensor

        rows, spans = gather_layout(global_batch, self.world)
        row_shape = list(row_shape)
        n_mine = 0 if shard is None else shard.shape[0]
        if n_mine != spans[self.rank][1] - spans[self.rank][0]:
            raise ValueError(f"rank {self.rank} holds {n_mine} rows, its shard has "
                             f"{spans[self.rank][1] - spans[self.rank][0]}")
        if shard is not None and n_mine == rows and shard.is_dense():
            send = shard
        else:
            send = Tensor._empty([rows] + row_shape, dtype)
            if n_mine:
                functional.assign(send.narrow(0, 0, n_mine), shard)
        recv = Tensor._empty([self.world * rows] + row_shape, dtype)
        uneven = any(hi - lo != rows for lo, hi in spans)

        def assemble():
            if not uneven:
                return recv
            out = Tensor._empty([global_batch] + row_shape, dtype)
            for r, (lo, hi) in enumerate(spans):
                if hi > lo:
                    functional.assign(out.narrow(0, lo, hi - lo), recv.narrow(0, r * rows, hi - lo))
            return out

        if slot is None:
            check(F.wxx_nccl_allgather(recv.buffer.ptr, send.ptr, send.nbytes), "ncclAllGather")
            return assemble()
        check(F.wxx_nccl_allgather_async(recv.buffer.ptr, send.ptr, send.nbytes, int(slot)),
              "ncclAllGather (async)")
        return PendingGather(slot, send, recv, assemble)

    def async_error(self):
        code = ctypes.c_int(0)
        check(F.wxx_nccl_async_error(ctypes.byref(code)))
        return code.value

    def destroy(self, abort=False):
        if self._alive:
            self._alive = False
            check(F.wxx_nccl_destroy(1 if abort else 0), "nccl destroy")


class PendingGather:
    """An all-gather running on the communication stream.  Holds the send and
    receive buffers until ``wait()`` has ordered the library stream after the
    gather (so the stream-ordered allocator cannot hand them out early)."""

    def __init__(self, slot, send, recv, assemble):
        self.slot = slot
        self._send = send
        self._recv = recv
        self._assemble = assemble
        self._out = None

    def wait(self):
        if self._out is None:
            check(F.wxx_nccl_wait(int(self.slot)), "nccl wait")
            self._out = self._assemble()
            self._send = None
        return self._out


def assemble(parts):
    """Host-side concatenation of per-rank shards in rank order (numpy)."""
    import numpy as np

    return np.concatenate(list(parts), axis=0)
