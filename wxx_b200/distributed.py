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

    def async_error(self):
        code = ctypes.c_int(0)
        check(F.wxx_nccl_async_error(ctypes.byref(code)))
        return code.value

    def destroy(self, abort=False):
        if self._alive:
            self._alive = False
            check(F.wxx_nccl_destroy(1 if abort else 0), "nccl destroy")


def assemble(parts):
    """Host-side concatenation of per-rank shards in rank order (numpy)."""
    import numpy as np

    return np.concatenate(list(parts), axis=0)
