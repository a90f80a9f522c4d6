"""One rank of the 2-GPU expert-parallel check (launched by tests/test_gpu_ep.py
through torch.distributed.run).  Rank r holds experts [r*E/2, (r+1)*E/2) of
every layer; the layer outputs (summed over ranks inside the decode kernel,
and again by the library's NCCL all-reduce: both must agree) are compared with the CPU oracle (top-k bit-exact, outputs within
the layer tolerance) and with the same layer run whole on one GPU.  Then the
sharded-token path (each rank its own batch, rows exchanged with NCCL
send/recv), the batches together against the oracle and the one-GPU layer,
and the same for a two-layer sharded stack (rms + MoE + residual per layer)."""

import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import colizig_b200 as cz  # noqa: E402
import oracle  # noqa: E402
from colizig_b200 import ep, moe, synth  # noqa: E402
from tests.util import OUT_TOL, rel_err  # noqa: E402


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    cz.gpu.init(local)
    ep.init()
    oracle.set_threads(os.cpu_count() or 1)
    ok = True
    lid = 700
    # decode calls sum the ranks inside the kernel (peer stores) on an NVLink box
    mode = ep.combine_mode()
    print(f"rank {rank}: decode combine mode {mode}", flush=True)
    ok &= mode == 1
    for cfg, Ts in (("c2", (1, 4, 16)), ("c5", (1, 5))):
        d = synth.CONFIGS[cfg]
        w = synth.make_layer(d, seed=11, device="cuda")
        Lep = moe.Layer.from_weights(lid, d, w, ep=True)
        Lfull = moe.Layer.from_weights(lid + 1, d, w)
        lid += 2
        wn = synth.to_numpy_layer(w) if rank == 0 else None
        for T in Ts:
            x = synth.make_tokens(T, d.hidden, 300 + T, device="cuda", dtype=torch.bfloat16)
            out, idx, gates = moe.forward(Lep, x)
            ref, ridx, rg = moe.forward(Lfull, x)
            # the same call with the NCCL all-reduce combine: a two-rank sum commutes,
            # so both combines give the same bits
            ep.set_combine(False)
            out_nccl, _, _ = moe.forward(Lep, x)
            ep.set_combine(True)
            torch.cuda.synchronize()
            moe.check()
            # two ranks: a + b commutes, so the bits agree; more ranks: NCCL's summation
            # order is its own, so within a few f32 roundings of the output
            diff = (out - out_nccl).abs().max().item()
            if (world == 2 and diff != 0.0) or diff > 1e-6 * out.abs().max().item():
                print(f"rank {rank} {cfg} T={T}: in-kernel and NCCL combines differ by {diff:.3e}", flush=True)
                ok = False
            if rank == 0:
                ol = oracle.layer_from_dict(wn)
                od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
                oo, oi, _ = oracle.moe_forward(ol, od, synth.tokens_f32(x.cpu()))
                e_or = rel_err(out.cpu().numpy(), oo)
                e_one = rel_err(out.cpu().numpy(), ref.cpu().numpy())
                same = np.array_equal(idx.cpu().numpy().view(np.uint32), oi)
                print(f"{cfg} T={T}: top-k exact {same}, vs oracle {e_or:.2e}, vs one GPU {e_one:.2e}", flush=True)
                ok &= same and e_or <= OUT_TOL and e_one <= OUT_TOL and torch.equal(idx, ridx) and torch.equal(gates, rg)
        if cfg == "c2":
            # many calls back to back (receive slots reused every second call, the
            # decode launches of a 9-token call each exchanging): each equals its first result
            xs = [synth.make_tokens(T, d.hidden, 500 + T, device="cuda", dtype=torch.bfloat16) for T in (1, 9, 3)]
            firsts = [moe.forward(Lep, x)[0] for x in xs]
            same = True
            for k in range(60):
                o = moe.forward(Lep, xs[k % 3])[0]
                same &= bool(torch.equal(o, firsts[k % 3]))
            torch.cuda.synchronize()
            moe.check()
            print(f"rank {rank}: 60 back-to-back EP decode calls repeat their results: {same}", flush=True)
            ok &= same
        Lep.unregister()
        Lfull.unregister()
    # sharded tokens (prefill): each rank its own batch (one rank may have none); the
    # batches together against the oracle and against the whole layer on one GPU
    d = synth.CONFIGS["c2"]
    w = synth.make_layer(d, seed=13, device="cuda")
    Lep = moe.Layer.from_weights(lid, d, w, ep=True)
    Lfull = moe.Layer.from_weights(lid + 1, d, w)
    wn = synth.to_numpy_layer(w) if rank == 0 else None
    # per-rank batch sizes (two-rank cases extended to `world` ranks)
    for Ts in [tuple((b[r] if r < 2 else (17 * r + 5) % 60) for r in range(world))
               for b in ((40, 72), (48, 0), (3, 5))]:
        xs = [synth.make_tokens(t, d.hidden, 900 + 17 * i + t, device="cuda", dtype=torch.bfloat16)
              for i, t in enumerate(Ts)]
        xall = torch.cat(xs)
        out, idx, gates = moe.forward(Lep, xs[rank], sharded=True)
        torch.cuda.synchronize()
        moe.check()
        parts = [None] * world
        dist.all_gather_object(parts, (out.cpu(), idx.cpu(), gates.cpu()))
        if rank == 0:
            o = torch.cat([p[0] for p in parts]).numpy()
            i_ = torch.cat([p[1] for p in parts]).numpy().view(np.uint32)
            ref, ridx, _ = moe.forward(Lfull, xall)
            ol = oracle.layer_from_dict(wn)
            od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
            oo, oi, _ = oracle.moe_forward(ol, od, synth.tokens_f32(xall.cpu()))
            same = np.array_equal(i_, oi)
            e_or = rel_err(o, oo)
            e_one = rel_err(o, ref.cpu().numpy())
            print(f"sharded c2 T={Ts}: top-k exact {same}, vs oracle {e_or:.2e}, vs one GPU {e_one:.2e}", flush=True)
            ok &= same and e_or <= OUT_TOL and e_one <= OUT_TOL
    Lep.unregister()
    Lfull.unregister()
    # the sharded stack (rms + MoE + residual per layer, rows exchanged in every layer),
    # teacher-forced per layer against the oracle and the one-GPU layer on the same input
    # (a chain of layers amplifies rounding differences through later top-k picks)
    lid += 2
    NL = 2
    ws = [synth.make_layer(d, seed=60 + l, device="cuda") for l in range(NL)]
    eps_l = [moe.Layer.from_weights(lid + l, d, ws[l], ep=True) for l in range(NL)]
    full_l = [moe.Layer.from_weights(lid + 10 + l, d, ws[l]) for l in range(NL)]
    rng = np.random.default_rng(5)
    norm_w = (1.0 + 0.05 * rng.standard_normal((NL, d.hidden))).astype(np.float32)
    Ts = tuple((40, 24)[r] if r < 2 else 8 * r for r in range(world))
    h0 = [rng.standard_normal((t, d.hidden)).astype(np.float32) for t in Ts]
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    h = h0[rank].copy()
    for l in range(NL):
        h_in = [None] * world
        dist.all_gather_object(h_in, h)
        h = moe.stack_forward(lid + l, 1, h.copy(), norm_w[l:l + 1], 1e-6, sharded=True)
        h_out = [None] * world
        dist.all_gather_object(h_out, h)
        if rank == 0:
            hi, ho = np.concatenate(h_in), np.concatenate(h_out)
            ref = moe.stack_forward(lid + 10 + l, 1, hi.copy(), norm_w[l:l + 1], 1e-6)
            b, _, _ = oracle.moe_forward(oracle.layer_from_dict(synth.to_numpy_layer(ws[l])), od,
                                         oracle.rms(hi, norm_w[l], 1e-6))
            # h + b is rounded to f32: allow the layer tolerance plus one rounding of the
            # residual add (two for the GPU-vs-GPU comparison)
            want = (hi + b).astype(np.float32)
            ulp = np.spacing(np.maximum(np.abs(hi), np.abs(want))).astype(np.float64)
            e_or = float(np.max((np.abs(ho.astype(np.float64) - want) - ulp) / (OUT_TOL * np.abs(b).max())))
            e_one = float(np.max((np.abs(ho.astype(np.float64) - ref) - 2 * ulp) /
                                 (OUT_TOL * np.abs(ref.astype(np.float64) - hi).max())))
            print(f"sharded c2 stack layer {l} T={Ts}: error / bound vs one GPU {e_one:.2e}, vs oracle {e_or:.2e}",
                  flush=True)
            ok &= e_one <= 1.0 and e_or <= 1.0
    # the two-layer call equals the chain of one-layer calls on every rank
    h2 = moe.stack_forward(lid, NL, h0[rank].copy(), norm_w, 1e-6, sharded=True)
    same = bool(np.array_equal(h2, h))
    if not same:
        print(f"rank {rank}: sharded stack of {NL} differs from its layer-by-layer chain", flush=True)
    ok &= same
    for lay in eps_l + full_l:
        lay.unregister()
    torch.cuda.synchronize()
    ep.shutdown()
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
