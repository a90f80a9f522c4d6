"""Expert parallelism over the GPUs of one node (one process per GPU).

The reference evaluates every expert independently (forwardGrouped,
src/qwen38/moe.zig:637-664), so the experts partition: rank r holds experts
[r*E/W, (r+1)*E/W) and rank 0 also the shared expert.  Router and top-k run
replicated on every rank (identical, bit-exact); each rank adds the outputs of
the experts it holds, and the ranks' outputs are summed: for decode batches
inside the decode kernel (each rank stores its partial rows into every rank's
peer-mapped receive buffer and adds the ranks' rows in rank order), otherwise
by one NCCL all-reduce inside the library on the call's stream.

Failure detection (no reference counterpart: the reference runs on one
process).  The library's host waits are watched while its communicator is
active (set_timeout): one that runs out aborts the communicator and the call
raises ColizigError(-9) instead of waiting for a peer that never comes.  A host
that steps in lockstep can learn earlier, before it launches anything:
Heartbeat.step() checks through the torch.distributed store that every peer
has reached the same step, and aborts (abort()) and raises -9 when one has not
within its timeout.
"""

from __future__ import annotations

import ctypes
import datetime
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


def set_timeout(ms: int) -> None:
    """Deadline of the library's host waits while the EP communicator is active
    (colizig_cuda_ep_set_timeout; <= 0 waits without one)."""
    _abi.check("colizig_cuda_ep_set_timeout", _abi.load().colizig_cuda_ep_set_timeout(int(ms)))


def combine_mode() -> int:
    """1 when expert-parallel decode calls sum the ranks inside the decode kernel
    (peer stores into every rank's receive buffer), 0 when by an NCCL all-reduce."""
    return int(_abi.load().colizig_cuda_ep_combine_mode())


def set_combine(in_kernel: bool) -> None:
    """Choose the decode combine (colizig_cuda_ep_set_combine); every rank must
    make the same choice before its next EP call."""
    _abi.check("colizig_cuda_ep_set_combine", _abi.load().colizig_cuda_ep_set_combine(1 if in_kernel else 0))


def abort() -> None:
    """Abort the EP communicator now (colizig_cuda_ep_abort): EP calls raise -9
    until shutdown() and init()."""
    _abi.check("colizig_cuda_ep_abort", _abi.load().colizig_cuda_ep_abort())


class Heartbeat:
    """Lockstep liveness check between EP steps over a torch.distributed store.

    step() marks this rank as having reached step n, then waits (at most
    `timeout_s`) until every other rank has marked step n too.  A peer that has
    exited or stopped stepping makes step() call `on_lost` (default: abort the
    library's communicator) and raise ColizigError(-9); nothing has been
    launched for that step on this rank.  Ranks leave only between steps."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "cz_hb",
                 on_lost=None):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.timeout = datetime.timedelta(seconds=float(timeout_s))
        self.prefix = prefix
        self.on_lost = abort if on_lost is None else on_lost
        self.n = 0

    def step(self) -> int:
        self.n += 1
        self.store.set(f"{self.prefix}/{self.n}/{self.rank}", b"1")
        peers = [f"{self.prefix}/{self.n}/{r}" for r in range(self.world) if r != self.rank]
        try:
            if peers:
                self.store.wait(peers, self.timeout)
        except Exception as e:  # the store's timeout (or a lost store connection)
            self.on_lost()
            raise _abi.ColizigError(f"heartbeat step {self.n}: a peer did not arrive ({type(e).__name__})",
                                    -9) from e
        return self.n
