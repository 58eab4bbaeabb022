"""Sharding set-up for the engine (B200 extension; no reference counterpart).

The model/context/generation layer is the reference's own Python runtime (sardyne.runtime over
sardyne.capi), which runs this library unchanged with SARDYNE_LIB pointing at it. What it cannot
express is that one process is rank r of a tensor/expert-parallel group: set_shard (or
shard_from_torch) configures the next engine_model_load of this process.
"""
import ctypes

from . import capi


NCCL_ID_BYTES = 128


def set_shard(rank: int, world: int, nccl_id: bytes | None = None) -> None:
    """Configure the next Model load of this process as rank `rank` of `world` (one GPU per process;
    world 1 = unsharded). Sharded ranks keep attention and the router, split the FFN rows, the
    experts and the vocabulary, and all return the one-GPU logits. Every rank must then load the
    same model and run the same eval calls."""
    lib = capi.lib()
    buf = (ctypes.c_char * NCCL_ID_BYTES).from_buffer_copy(nccl_id) if nccl_id else None
    if lib.sdy_engine_set_shard(rank, world, buf) != 0:
        raise ValueError(capi.last_error())


def new_nccl_id() -> bytes:
    buf = (ctypes.c_char * NCCL_ID_BYTES)()
    if capi.lib().sdy_nccl_unique_id(buf) != 0:
        raise RuntimeError(capi.last_error())
    return bytes(buf)


def shard_from_torch(group=None) -> tuple[int, int]:
    """set_shard from a torch.distributed process group: rank 0 creates the NCCL id and
    broadcasts it. Returns (rank, world)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nccl_id = None
    if world > 1:
        obj = [new_nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        nccl_id = obj[0]
    set_shard(rank, world, nccl_id)
    return rank, world
