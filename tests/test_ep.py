"""Expert parallelism: host logic on CPU with world-size-2 gloo ranks.

The partition of experts over ranks (colizig_b200.ep.expert_range, the same
rule as colizig_cuda_moe_register_layer with COLIZIG_EP), the exchange of the
NCCL unique id through torch.distributed, and the combine: every rank adds the
outputs of the experts it holds (plus the shared expert on rank 0) and one
all-reduce sums the ranks.  The per-rank partials are formed with the oracle's
own block-FP8 matmul and route (the reference's forwardDense restricted to a
rank's experts, moe.zig:481-539), summed with a gloo all-reduce, and compared
with the oracle's full layer output.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from colizig_b200 import ep
from tests.util import OUT_TOL, golden, oracle_layer, rel_err


def test_expert_range_partitions_every_expert_once():
    for E in (16, 128, 512):
        for W in (1, 2, 3, 4, 8):
            seen = []
            for r in range(W):
                lo, hi = ep.expert_range(r, W, E)
                assert hi - lo in (E // W, E // W + 1)
                seen.extend(range(lo, hi))
            assert seen == list(range(E))
    with pytest.raises(ValueError):
        ep.expert_range(2, 2, 16)
    with pytest.raises(ValueError):
        ep.expert_range(0, 32, 16)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_partial(w, d, od, x, rank, world):
    """Sum over this rank's experts of gate * down(silu(gate(x)) * up(x)), shared
    expert (sigmoid(x . sh_gate) * shared(x)) on rank 0 only."""
    lw = oracle_layer(w)
    lo, hi = ep.expert_range(rank, world, d["E"])
    out = np.zeros_like(x)
    silu = np.vectorize(oracle.silu, otypes=[np.float32])
    for t in range(x.shape[0]):
        xt = x[t:t + 1]
        idx, gates = oracle.route(lw, od, xt[0])
        for z, e in enumerate(idx.tolist()):
            if not lo <= e < hi:
                continue
            g = oracle.matmul_fp8(xt, w["gate_w"][e], w["gate_s"][e])
            u = oracle.matmul_fp8(xt, w["up_w"][e], w["up_s"][e])
            h = (silu(g) * u).astype(np.float32)
            out[t] += gates[z] * oracle.matmul_fp8(h, w["down_w"][e], w["down_s"][e])[0]
        if d["SI"] and rank == 0:
            sg = oracle.sigmoid(oracle.dot_f32(xt[0], w["sh_gate"]))
            g = oracle.matmul_fp8(xt, w["sh_gate_w"], w["sh_gate_s"])
            u = oracle.matmul_fp8(xt, w["sh_up_w"], w["sh_up_s"])
            h = (silu(g) * u).astype(np.float32)
            out[t] += np.float32(sg) * oracle.matmul_fp8(h, w["sh_down_w"], w["sh_down_s"])[0]
    return out


def _worker(rank, world, port, name, shared, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        # the unique id travels through torch.distributed exactly as ep.init does it
        uid = ep.share_unique_id(make=lambda: bytes(range(128)))
        assert uid == bytes(range(128))
        z = golden(name)
        d = {"H": int(z["H"]), "E": int(z["E"]), "K": int(z["K"]), "I": int(z["I"]),
             "SI": int(z["SI"]) if shared else 0}
        w = {k: np.ascontiguousarray(z[k]) for k in z.files if not k.isupper() and k not in ("x", "out", "idx")}
        od = oracle.Dims(d["H"], d["E"], d["K"], d["I"], d["SI"], True)
        x = np.ascontiguousarray(z["x"], np.float32).reshape(-1, d["H"])
        part = torch.from_numpy(_rank_partial(w, d, od, x, rank, world))
        dist.all_reduce(part)
        if rank == 0:
            full, _, _ = oracle.moe_forward(oracle_layer(w), od, x)
            q.put(rel_err(part.numpy(), full))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surface the failure in the parent
        q.put(repr(e))
        raise


@pytest.mark.parametrize("name,shared", [("moe_c1.npz", False), ("moe_shared_tiny.npz", True)])
def test_ep_combine_world2_gloo_matches_full_layer(name, shared):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, name, shared, q), nprocs=2, join=True, start_method="spawn")
    res = q.get()
    assert not isinstance(res, str), res
    assert res <= OUT_TOL, res
