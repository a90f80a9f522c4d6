"""Parity at every configuration's stated size, against the CPU oracle (the C
restatement of the reference's Zig path, moe.zig:435-665 and model.zig:227-232):

  * config 3: the config-2 layer with Zipf(1.1)-skewed routing, prefill batches of
    2048 and 8192 tokens (groups of thousands of positions: the grouped GEMMs'
    multi-tile schedule, the chunked counting sort, the 64-position tails);
  * config 5: the large layer with its shared expert, a 4096-token prefill;
  * config 4: the 48-layer stack of config-2 layers (29 GB of E4M3 weights,
    attention = identity) through colizig_cuda_moe_stack_forward at T = 1 and at
    T = 4096 (prefill), teacher-forced layer by layer against the oracle (T = 4096:
    on 64 tokens spread over the batch), and the fused 48-layer call equal to the
    layer-by-layer chain.

Bars: router top-k ids and gates bit-exact; outputs within max-abs <=
1e-3 * ||out||_inf (OUT_TOL).  This file sorts just before the no-allocation test,
after every other parity test, so a failure here cannot hide the other rows in a
run that stops at the first failure.
"""

import os

import numpy as np
import pytest
import torch

import colizig_b200 as cz
import oracle
from colizig_b200 import moe, synth
from tests.util import OUT_TOL, assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    torch.cuda.init()
    cz.gpu.init()
    oracle.set_threads(os.cpu_count() or 1)
    yield
    oracle.set_threads(1)


def _odims(d):
    return oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)


@pytest.mark.parametrize("T", [2048, 8192])
def test_c3_prefill_zipf_full_size(T):
    d = synth.CONFIGS["c3"]
    w = synth.make_layer(d, seed=3, device="cuda")
    synth.zipf_router(w, 3)
    L = moe.Layer.from_weights(7000 + T, d, w)
    try:
        x = synth.zipf_tokens(T, d.hidden, 60000 + T, device="cuda", dtype=torch.bfloat16)
        out, idx, gates = moe.forward(L, x)
        out2, _, _ = moe.forward(L, x)
        torch.cuda.synchronize()
        moe.check()
        assert torch.equal(out, out2)  # deterministic
        ids = idx.cpu().numpy().view(np.uint32)
        counts = np.bincount(ids.ravel(), minlength=d.experts)
        pairs = T * d.topk
        share = counts.max() / pairs
        print(f"c3 T={T}: top expert {counts.max()} of {pairs} pairs ({share:.3f}), "
              f"{(counts > 0).sum()} distinct experts")
        # the skew the config asks for: the hottest expert far above the uniform 1/E share
        assert counts.max() > 4 * pairs / d.experts
        assert (counts > 0).sum() > d.topk
        wn = synth.to_numpy_layer(w)
        del w
        oo, oi, og = oracle.moe_forward(oracle.layer_from_dict(wn), _odims(d), synth.tokens_f32(x))
        assert np.array_equal(ids, oi), "top-k differs"
        np.testing.assert_array_equal(gates.cpu().numpy(), og)
        e = assert_close(out.cpu().numpy(), oo, OUT_TOL, f"c3 T={T}")
        print(f"c3 T={T}: rel err {e:.2e}")
    finally:
        L.unregister()


def test_c5_prefill_shared_expert_t4096():
    d = synth.CONFIGS["c5"]
    w = synth.make_layer(d, seed=5, device="cuda")
    L = moe.Layer.from_weights(7100, d, w)
    try:
        x = synth.make_tokens(4096, d.hidden, 61000, device="cuda", dtype=torch.bfloat16)
        out, idx, gates = moe.forward(L, x)
        torch.cuda.synchronize()
        moe.check()
        wn = synth.to_numpy_layer(w)
        del w
        oo, oi, og = oracle.moe_forward(oracle.layer_from_dict(wn), _odims(d), synth.tokens_f32(x))
        assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi), "top-k differs"
        np.testing.assert_array_equal(gates.cpu().numpy(), og)
        e = assert_close(out.cpu().numpy(), oo, OUT_TOL, "c5 T=4096")
        print(f"c5 T=4096: rel err {e:.2e}")
    finally:
        L.unregister()


def _layer_check(h_in, h_out, w_l, wn_l, od, what):
    """One teacher-forced layer: h_out must equal h_in + moe(rms(h_in, w_l)) up to
    the layer tolerance plus one rounding of the residual add."""
    n = oracle.rms(h_in, w_l, 1e-6)
    b, _, _ = oracle.moe_forward(oracle.layer_from_dict(wn_l), od, n)
    want = (h_in + b).astype(np.float32)
    ulp = np.spacing(np.maximum(np.abs(h_in), np.abs(want))).astype(np.float64)
    bound = OUT_TOL * np.abs(b).max() + ulp
    diff = np.abs(h_out.astype(np.float64) - want)
    assert np.all(diff <= bound), f"{what}: max excess {np.max(diff - bound):.3e}"
    return float(np.max(diff) / np.abs(b).max())


def test_c4_stack_48_layers_teacher_forced():
    d = synth.CONFIGS["c2"]
    NL, base = 48, 5000
    layers = []
    g = torch.Generator(device="cpu").manual_seed(48)
    norm_w = (1.0 + 0.05 * torch.randn(NL, d.hidden, generator=g)).float()
    try:
        for l in range(NL):
            layers.append(moe.Layer.from_weights(base + l, d, synth.make_layer(d, seed=100 + l, device="cuda")))
        nw_dev = norm_w.cuda()
        od = _odims(d)
        rng = np.random.default_rng(4)
        h1 = rng.standard_normal((1, d.hidden)).astype(np.float32)
        hP = torch.from_numpy(rng.standard_normal((4096, d.hidden)).astype(np.float32)).cuda()
        sample = np.arange(0, 4096, 64)  # 64 tokens spread over the prefill batch

        # fused calls over all 48 layers
        fused1 = moe.stack_forward(base, NL, h1.copy(), norm_w.numpy(), 1e-6)
        fusedP = hP.clone()
        moe.stack_forward(base, NL, fusedP, nw_dev, 1e-6)
        torch.cuda.synchronize()
        moe.check()

        # layer by layer, each layer checked against the oracle on the GPU's own input
        c1, cP = h1.copy(), hP.clone()
        worst1 = worstP = 0.0
        for l in range(NL):
            n1 = moe.stack_forward(base + l, 1, c1.copy(), norm_w[l:l + 1].numpy(), 1e-6)
            nP = cP.clone()
            moe.stack_forward(base + l, 1, nP, nw_dev[l:l + 1].contiguous(), 1e-6)
            torch.cuda.synchronize()
            wn = synth.to_numpy_layer(_layer_weights(d, l))
            wl = norm_w[l].numpy()
            worst1 = max(worst1, _layer_check(c1, n1, wl, wn, od, f"T=1 layer {l}"))
            inP = cP[sample].cpu().numpy()
            worstP = max(worstP, _layer_check(inP, nP[sample].cpu().numpy(), wl, wn, od, f"T=4096 layer {l}"))
            c1, cP = n1, nP
        print(f"c4 48 layers: worst layer rel err T=1 {worst1:.2e}, T=4096 sample {worstP:.2e}")
        moe.check()
        assert np.array_equal(fused1, c1)  # the fused stack equals the layer-by-layer chain
        assert torch.equal(fusedP, cP)
    finally:
        for L in layers:
            L.unregister()


def _layer_weights(d, l):
    """The weights of stack layer l, regenerated with the same seed (the library
    keeps its own resident copy; regenerating avoids holding 29 GB twice)."""
    return synth.make_layer(d, seed=100 + l, device="cuda")
