"""Failure detection on the host, with no GPU (no reference counterpart: the
reference runs on one process).

- The library's watched host wait (colizig_cuda_debug_watch_wait runs the same
  watch_wait that guards its stream waits while an EP communicator is active):
  fakes of the stream query, the communicator's error report and the abort
  stand in for CUDA and NCCL.  A wait that finishes returns 0 and aborts
  nothing; one that runs out of time, or meets a communicator error, aborts
  once and returns -9; a failed query returns -5.
- ep.Heartbeat over world-size-2 gloo ranks: a rank that leaves between steps
  is noticed by the other on its next step, before it launches anything: the
  lost-peer action runs and ColizigError(-9) is raised.
"""

import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from colizig_b200 import _abi, ep


class _Fake:
    def __init__(self, done_after=None, error_after=None, fail_after=None):
        self.polls = 0
        self.aborts = 0
        self.done_after, self.error_after, self.fail_after = done_after, error_after, fail_after

    def query(self, _ctx):
        self.polls += 1
        if self.fail_after is not None and self.polls > self.fail_after:
            return -1
        if self.done_after is not None and self.polls > self.done_after:
            return 0
        return 1

    def error(self, _ctx):
        return int(self.error_after is not None and self.polls > self.error_after)

    def abort(self, _ctx):
        self.aborts += 1


def _watch(fake, timeout_ms):
    L = _abi.load()
    q = _abi.WATCH_QUERY(fake.query)
    e = _abi.WATCH_QUERY(fake.error)
    a = _abi.WATCH_ABORT(fake.abort)
    t0 = time.perf_counter()
    rc = L.colizig_cuda_debug_watch_wait(q, e, a, None, timeout_ms)
    return rc, time.perf_counter() - t0


def test_watch_wait_returns_when_the_work_completes():
    f = _Fake(done_after=3)
    rc, _ = _watch(f, 10_000)
    assert rc == 0 and f.aborts == 0 and f.polls == 4


def test_watch_wait_aborts_once_at_the_deadline():
    f = _Fake()
    rc, dt = _watch(f, 200)
    assert rc == -9
    assert f.aborts == 1
    assert 0.19 <= dt < 5.0


def test_watch_wait_aborts_on_a_communicator_error():
    f = _Fake(error_after=2)
    rc, dt = _watch(f, 60_000)
    assert rc == -9 and f.aborts == 1 and dt < 5.0


def test_watch_wait_reports_a_failed_query_without_abort():
    f = _Fake(fail_after=1)
    rc, _ = _watch(f, 60_000)
    assert rc == -5 and f.aborts == 0


def test_watch_wait_rejects_missing_callbacks():
    L = _abi.load()
    assert L.colizig_cuda_debug_watch_wait(_abi.WATCH_QUERY(0), _abi.WATCH_QUERY(0), _abi.WATCH_ABORT(0), None,
                                           10) == -1


def test_abort_and_timeout_need_no_device():
    ep.set_timeout(1234)
    ep.abort()  # no communicator: nothing to abort
    ep.set_timeout(60_000)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _hb_worker(rank, world, port, leave_after, q):
    try:
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0)
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world)
        lost = []
        hb = ep.Heartbeat(store, rank, world, timeout_s=1.0, on_lost=lambda: lost.append(True))
        steps = 0
        try:
            for _ in range(3):
                if leave_after is not None and rank == 1 and steps == leave_after:
                    break  # this rank leaves between steps
                hb.step()
                steps += 1
            q.put((rank, steps, None, len(lost)))
        except _abi.ColizigError as e:
            q.put((rank, steps, e.rc, len(lost)))
        if leave_after is None:
            dist.barrier()
        if rank == 0:
            time.sleep(0.5)  # rank 1 (a store client) leaves first
        dist.destroy_process_group()
    except Exception as e:  # surface the failure in the parent
        q.put((rank, -1, repr(e), 0))
        raise


@pytest.mark.parametrize("leave_after", [None, 2])
def test_heartbeat_world2_gloo(leave_after):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_hb_worker, args=(2, _free_port(), leave_after, q), nprocs=2, join=True,
                       start_method="spawn")
    res = {}
    for _ in range(2):
        r, steps, err, lost = q.get()
        assert steps >= 0, err
        res[r] = (steps, err, lost)
    if leave_after is None:
        assert res == {0: (3, None, 0), 1: (3, None, 0)}
    else:
        assert res[1] == (2, None, 0)       # left after two steps
        assert res[0] == (2, -9, 1)         # its third step noticed: lost-peer action, -9
