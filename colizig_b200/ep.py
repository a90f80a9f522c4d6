"""Expert parallelism over the GPUs of one node (one process per GPU).

The reference evaluates every expert independently (forwardGrouped,
src/qwen38/moe.zig:637-664), so the experts partition: rank r holds experts
[r*E/W, (r+1)*E/W) and rank 0 also the shared expert.  Router and top-k run
replicated on every rank (identical, bit-exact); each rank adds the outputs of
the experts it holds, and one all-reduce (sum) over the ranks completes every
forward.  The all-reduce runs inside the library (NCCL) on the call's stream.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

from . import _abi

UNIQUE_ID_BYTES = 128


def expert_range(rank: int, world: int, experts: int) -> Tuple[int, int]:
    """Experts [lo, hi) held by `rank` (contiguous, sizes differ by at most one)."""
    if not (0 <= rank < world) or world > experts:
        raise ValueError("need 0 <= rank < world <= experts")
    return rank * experts // world, (rank + 1) * experts // world


def unique_id() -> bytes:
    """A fresh NCCL unique id (call on one rank, hand the bytes to all)."""
    buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
    _abi.check("colizig_cuda_ep_unique_id", _abi.load().colizig_cuda_ep_unique_id(buf))
    return buf.raw


def share_unique_id(make=unique_id, group=None) -> bytes:
    """Rank 0 makes the id, every rank of the torch.distributed group receives it."""
    import torch.distributed as dist

    obj = [make() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != UNIQUE_ID_BYTES:
        raise RuntimeError("bad unique id")
    return bytes(uid)


def init(rank: Optional[int] = None, world: Optional[int] = None, uid: Optional[bytes] = None) -> None:
    """colizig_cuda_ep_init for this process (after gpu.init).  Without arguments
    the rank, world size and id come from the torch.distributed default group."""
    if rank is None or world is None:
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
    if world > 1 and uid is None:
        uid = share_unique_id()
    buf = ctypes.create_string_buffer(bytes(uid), UNIQUE_ID_BYTES) if uid is not None else None
    _abi.check("colizig_cuda_ep_init", _abi.load().colizig_cuda_ep_init(int(rank), int(world), buf))


def shutdown() -> None:
    _abi.check("colizig_cuda_ep_shutdown", _abi.load().colizig_cuda_ep_shutdown())
