"""Prefill path (token batches of 32 or more: tcgen05 grouped GEMMs) against the
CPU oracle's grouped forward (moe.zig:597-665): top-k ids bit-exact, outputs
within max-abs <= 1e-3 * ||out||_inf, deterministic; and against the decode
kernel on the same tokens at a larger batch."""

import os

import numpy as np
import pytest
import torch

import colizig_b200 as cz
import oracle
from colizig_b200 import moe, synth
from tests.util import OUT_TOL, assert_close, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    torch.cuda.init()
    cz.gpu.init()
    oracle.set_threads(os.cpu_count() or 1)
    yield
    oracle.set_threads(1)


def _oracle(d, w, x):
    ol = oracle.layer_from_dict(synth.to_numpy_layer(w))
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    return oracle.moe_forward(ol, od, synth.tokens_f32(x.cpu()) if x.dtype == torch.bfloat16 else x.cpu().numpy())


@pytest.mark.parametrize("cfg,T,dtype", [("c1", 64, torch.bfloat16), ("c2", 256, torch.bfloat16),
                                         ("c2", 48, torch.float32), ("c5", 40, torch.bfloat16)])
def test_prefill_matches_oracle(cfg, T, dtype):
    d = synth.CONFIGS[cfg]
    w = synth.make_layer(d, seed=21, device="cuda")
    L = moe.Layer.from_weights(800, d, w)
    try:
        x = synth.make_tokens(T, d.hidden, 4000 + T, device="cuda", dtype=dtype)
        out, idx, gates = moe.forward(L, x)
        out2, _, _ = moe.forward(L, x)
        torch.cuda.synchronize()
        moe.check()
        oo, oi, og = _oracle(d, w, x)
        assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi)
        assert np.array_equal(gates.cpu().numpy(), og)
        e = assert_close(out.cpu().numpy(), oo, OUT_TOL, f"{cfg} T={T}")
        print(f"{cfg} T={T} {dtype}: rel err {e:.2e}")
        assert torch.equal(out, out2)  # deterministic
    finally:
        L.unregister()


def test_prefill_agrees_with_decode_kernel_c2_t512():
    """T=512 through the prefill path vs the same tokens 4 at a time through the
    decode kernel (colizig_cuda_moe_forward on slices below the prefill size)."""
    d = synth.CONFIGS["c2"]
    w = synth.make_layer(d, seed=22, device="cuda")
    L = moe.Layer.from_weights(801, d, w)
    try:
        x = synth.make_tokens(512, d.hidden, 777, device="cuda", dtype=torch.bfloat16)
        out, idx, _ = moe.forward(L, x)
        parts = [moe.forward(L, x[i:i + 16]) for i in range(0, 512, 16)]
        torch.cuda.synchronize()
        moe.check()
        ref = torch.cat([p[0] for p in parts])
        ridx = torch.cat([p[1] for p in parts])
        assert torch.equal(idx, ridx)
        assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= OUT_TOL
    finally:
        L.unregister()


def test_kernel_timer_records_decode_and_prefill_gemms():
    """The benchmark timer: one decode launch (T=3) gives one kind-1 pair, one
    prefill forward (T=64) a kind-2 and a kind-3 pair, all with positive device
    time; a full timer reports the dropped pairs instead of wrapping."""
    d = synth.CONFIGS["c1"]
    w = synth.make_layer(d, seed=5, device="cuda")
    L = moe.Layer.from_weights(801, d, w)
    try:
        moe.kernel_timer(3)
        moe.forward(L, synth.make_tokens(3, d.hidden, 1, device="cuda"))
        moe.forward(L, synth.make_tokens(64, d.hidden, 2, device="cuda"))
        rec = moe.kernel_timer_read()
        assert [k for k, _ in rec] == [moe.TIMER_DECODE, moe.TIMER_PREFILL_GATE_UP, moe.TIMER_PREFILL_DOWN]
        assert all(ms > 0 for _, ms in rec)
        moe.forward(L, synth.make_tokens(3, d.hidden, 3, device="cuda"))  # no room left
        with pytest.raises(cz.ColizigError):
            moe.kernel_timer_read()
        moe.kernel_timer(0)
        moe.forward(L, synth.make_tokens(3, d.hidden, 4, device="cuda"))
        assert moe.kernel_timer_read() == []
        moe.check()
    finally:
        moe.kernel_timer(0)
        L.unregister()
