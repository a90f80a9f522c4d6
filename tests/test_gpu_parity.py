"""GPU parity: libcolizig_cuda.so (through its C ABI) against the CPU oracle and
the reference's golden fixtures.

Bars (north_star): router top-k indices bit-exact; layer outputs within
max-abs <= 1e-3 * ||out||_inf (OUT_TOL in tests/util.py) with fp32 accumulation.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

import colizig_b200 as cz
import oracle
from colizig_b200 import _abi, moe, synth
from tests.util import OUT_TOL, assert_close, golden, oracle_layer, rel_err

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module", autouse=True)
def _init():
    torch.cuda.init()
    cz.gpu.init()
    oracle.set_threads(os.cpu_count() or 1)
    yield
    oracle.set_threads(1)


def test_device_name():
    name = cz.gpu.device_name()
    assert "sm_100" in name, name


def test_router_exp_bit_identical_to_oracle():
    rng = np.random.default_rng(5)
    xs = np.concatenate([
        rng.uniform(-104, 89, 1 << 20), rng.uniform(-20, 0, 1 << 20), -np.abs(rng.standard_normal(1 << 18)) * 1e-3,
        [0.0, -0.0, 1.0, -1.0, 88.72, -103.97, -110.5, 100.5, np.inf, -np.inf],
    ]).astype(np.float32)
    x = torch.from_numpy(xs).cuda()
    y = torch.empty_like(x)
    _abi.check("debug_expf", _abi.load().colizig_cuda_debug_expf(x.data_ptr(), y.data_ptr(), x.numel()))
    got = y.cpu().numpy()
    want = oracle.expf(xs)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- legacy per-matrix op (colizig_cuda_matmul_fp8) ----------------------------

@pytest.mark.parametrize("name", ["two_blocks", "all_finite_bytes", "c1_gate", "ragged"])
def test_matmul_fp8_kat(name):
    k = golden("fp8_matmul_kat.npz")
    x, w, s, y = (k[f"{name}_{t}"] for t in "xwsy")
    got = cz.fp8.matmul_fp8(x, w, s)
    assert rel_err(got, y) < 1e-5
    assert rel_err(got, oracle.matmul_fp8(x, w, s)) < 1e-5


def test_matmul_fp8_keyed_store():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 2048)).astype(np.float32)
    w = rng.integers(0, 256, (768, 2048), dtype=np.uint8)
    w[(w == 0x7F) | (w == 0xFF)] = 0x00
    s = rng.uniform(1e-3, 3e-3, (6, 16)).astype(np.float32)
    want = oracle.matmul_fp8(x, w, s)
    h0, m0, _, _ = cz.gpu.stats()
    cz.gpu.set_vram_budget(0)
    y0 = cz.fp8.matmul_fp8_keyed(x, w, s, key=5)  # budget 0: uncached
    cz.gpu.set_vram_budget(1 << 30)
    y1 = cz.fp8.matmul_fp8_keyed(x, w, s, key=5)  # miss
    y2 = cz.fp8.matmul_fp8_keyed(x, w, s, key=5)  # hit: no upload
    h1, m1, up, res = cz.gpu.stats()
    assert (h1 - h0, m1 - m0) == (1, 1) and res >= 1
    assert np.array_equal(y0, y1) and np.array_equal(y1, y2)
    assert_close(y2, want, 1e-5)
    cz.gpu.set_vram_budget(0)  # evicts everything
    assert cz.gpu.stats()[3] == 0


REF_SO = os.path.join(ROOT, "oracle", "_ref", "libcolizig_cuda_ref.so")


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference CUDA backend not built (oracle/_ref)")
def test_matmul_fp8_matches_reference_cuda_backend():
    """The reference's own mm_fp8_kernel, compiled from its source for sm_100a."""
    R = ctypes.CDLL(REF_SO)
    R.colizig_cuda_init.restype = ctypes.c_int
    R.colizig_cuda_matmul_fp8.restype = ctypes.c_int
    R.colizig_cuda_matmul_fp8.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_uint64]
    assert R.colizig_cuda_init() == 0
    k = golden("fp8_matmul_kat.npz")
    for name in ["two_blocks", "all_finite_bytes", "c1_gate", "ragged"]:
        x, w, s = (np.ascontiguousarray(k[f"{name}_{t}"]) for t in "xws")
        S, I = x.shape
        O = w.shape[0]
        yr = np.empty((S, O), np.float32)
        assert R.colizig_cuda_matmul_fp8(yr.ctypes.data, x.ctypes.data, w.ctypes.data, s.ctypes.data, S, I, O, 0) == 0
        assert rel_err(cz.fp8.matmul_fp8(x, w, s), yr) < 1e-5


# ---- MoE layer ------------------------------------------------------------------

def _register_golden(name, layer_id, shared=False):
    z = golden(name)
    d = moe.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]) if shared else 0, True)
    w = {k: np.ascontiguousarray(z[k]) for k in z.files if not k.isupper() and k not in ("x", "out", "idx")}
    return z, d, moe.Layer.from_weights(layer_id, d, w), w


def test_moe_c1_golden():
    z, d, L, w = _register_golden("moe_c1.npz", 100)
    ol = oracle_layer(w)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, 0, True)
    for t in range(z["x"].shape[0]):
        out, idx, gates = moe.forward(L, z["x"][t:t + 1])
        oo, oi, og = oracle.moe_forward(ol, od, z["x"][t])
        assert np.array_equal(idx[0], z["idx"][t]) and np.array_equal(idx, oi)
        np.testing.assert_array_equal(gates, og)  # norm_topk gates are bit-exact too
        assert_close(out, oo)
        assert_close(out[0], z["out"][t])
    out, idx, _ = moe.forward(L, z["x"])  # T = 5
    oo, oi, _ = oracle.moe_forward(ol, od, z["x"])
    assert np.array_equal(idx, z["idx"]) and np.array_equal(idx, oi)
    assert_close(out, oo)
    L.unregister()


def test_moe_shared_expert_golden():
    z, d, L, w = _register_golden("moe_shared_tiny.npz", 101, shared=True)
    ol = oracle_layer(w)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, True)
    out, idx, _ = moe.forward(L, z["x"])
    oo, oi, _ = oracle.moe_forward(ol, od, z["x"])
    assert np.array_equal(idx, z["idx"]) and np.array_equal(idx, oi)
    assert_close(out, oo)
    assert_close(out, z["out"])
    L.unregister()


def _device_layer(cfg, seed, layer_id):
    d = synth.CONFIGS[cfg]
    w = synth.make_layer(d, seed=seed, device="cuda")
    L = moe.Layer.from_weights(layer_id, d, w)
    return d, w, L


def _check_layer(d, w, L, Ts, seed0=1000, bf16=True):
    wn = synth.to_numpy_layer(w)
    ol = oracle_layer(wn)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    errs = {}
    for T in Ts:
        x = synth.make_tokens(T, d.hidden, seed0 + T, device="cuda",
                              dtype=torch.bfloat16 if bf16 else torch.float32)
        out, idx, gates = moe.forward(L, x)
        torch.cuda.synchronize()
        moe.check()
        oo, oi, og = oracle.moe_forward(ol, od, synth.tokens_f32(x))
        gi = idx.cpu().numpy().view(np.uint32)
        assert np.array_equal(gi, oi), f"T={T}: top-k differs"
        np.testing.assert_array_equal(gates.cpu().numpy(), og)
        errs[T] = assert_close(out.cpu().numpy(), oo, OUT_TOL, f"T={T}")
    return errs


def test_moe_c2_decode_full_size():
    d, w, L = _device_layer("c2", 0, 200)
    errs = _check_layer(d, w, L, [1, 4, 16])
    print("c2 rel err", errs)
    L.unregister()


def test_moe_c2_chunked_and_odd_token_counts():
    d, w, L = _device_layer("c2", 1, 201)
    _check_layer(d, w, L, [3, 5, 32, 33, 70], seed0=77, bf16=False)
    L.unregister()


def test_moe_c5_shared_full_size():
    d, w, L = _device_layer("c5", 0, 202)
    errs = _check_layer(d, w, L, [1, 16])
    print("c5 rel err", errs)
    L.unregister()


def test_moe_host_and_device_paths_agree_and_deterministic():
    d, w, L = _device_layer("c2", 2, 203)
    x = synth.make_tokens(8, d.hidden, 5, device="cuda")
    o1, i1, g1 = moe.forward(L, x)
    o2, i2, g2 = moe.forward(L, x)
    oh, ih, gh = moe.forward(L, x.cpu())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(i1, i2)
    assert np.array_equal(o1.cpu().numpy(), oh) and np.array_equal(i1.cpu().numpy().view(np.uint32), ih)
    L.unregister()


def test_moe_router_ties_and_nan_tokens():
    z = golden("moe_c1.npz")
    w = {k: np.array(z[k]) for k in ("router", "gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}
    w["router"][5] = w["router"][9]
    w["router"][3] = w["router"][9]
    w["router"][12] = w["router"][9]
    d = moe.Dims(256, 16, 8, 128, 0, True)
    L = moe.Layer.from_weights(104, d, w)
    ol = oracle_layer(w)
    od = oracle.Dims(256, 16, 8, 128, 0, True)
    x = z["x"]
    out, idx, gates = moe.forward(L, x)
    oo, oi, og = oracle.moe_forward(ol, od, x)
    assert np.array_equal(idx, oi)
    assert_close(out, oo)
    xn = np.full((2, 256), np.nan, np.float32)
    out, idx, gates = moe.forward(L, xn)  # every logit NaN: reference picks id 0 each round
    oo, oi, og = oracle.moe_forward(ol, od, xn)
    assert np.array_equal(idx, oi) and not idx.any()
    assert np.isnan(gates).all() and np.isnan(og).all()
    L.unregister()


def test_stack_forward_teacher_forced():
    """model.zig:227-232 loop (attention = identity) over 3 C1-sized layers."""
    d = synth.CONFIGS["c1"]
    layers, ws = [], []
    for l in range(3):
        w = synth.make_layer(d, seed=40 + l, device="cuda")
        layers.append(moe.Layer.from_weights(300 + l, d, w))
        ws.append(synth.to_numpy_layer(w))
    rng = np.random.default_rng(9)
    norm_w = (1.0 + 0.1 * rng.standard_normal((3, d.hidden))).astype(np.float32)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, 0, True)
    for T in (1, 6):
        h0 = rng.standard_normal((T, d.hidden)).astype(np.float32)
        h_all = moe.stack_forward(300, 3, h0.copy(), norm_w, 1e-6)
        h = h0.copy()
        for l in range(3):
            h_gpu = moe.stack_forward(300 + l, 1, h.copy(), norm_w[l:l + 1], 1e-6)
            n = oracle.rms(h, norm_w[l], 1e-6)
            b, _, _ = oracle.moe_forward(oracle_layer(ws[l]), od, n)
            # h += b in f32: the GPU result may differ from fl(h + b_oracle) by the
            # layer tolerance plus one rounding of the residual add
            want = (h + b).astype(np.float32)
            ulp = np.spacing(np.maximum(np.abs(h), np.abs(want))).astype(np.float64)
            bound = OUT_TOL * np.abs(b).max() + ulp
            assert np.all(np.abs(h_gpu.astype(np.float64) - want) <= bound), f"layer {l}"
            h = h_gpu
        assert np.array_equal(h_all, h)  # the fused stack equals the layer-by-layer chain
    for L in layers:
        L.unregister()


def test_error_codes():
    L = _abi.load()
    x = torch.zeros((2, 256), device="cuda")
    out = torch.empty_like(x)
    assert L.colizig_cuda_moe_forward(9999, x.data_ptr(), 0, 2, out.data_ptr(), None, None, 1, None) == -6
    assert L.colizig_cuda_moe_forward(9999, x.data_ptr(), 7, 2, out.data_ptr(), None, None, 1, None) == -1
    d = _abi.MoeDims(250, 16, 4, 128, 0, 1)  # hidden not a multiple of 16
    exp = (_abi.MoeExpert * 16)()
    r = np.zeros((16, 250), np.float32)
    assert L.colizig_cuda_moe_register_layer(1, ctypes.byref(d), r.ctypes.data, exp, None, None, 0) == -8


def test_host_pointer_calls_replayed_from_graph_match_device_calls():
    """Host-pointer decode calls are run directly the first time and replayed from
    a captured CUDA graph afterwards; every call must equal the device-pointer
    forward on its own tokens, and a re-registered layer must not reuse a graph
    captured for the old weights."""
    d, w, L = _device_layer("c2", 4, 205)
    try:
        for T in (1, 3):
            for i in range(5):
                x = synth.make_tokens(T, d.hidden, 7000 + 10 * T + i, device="cuda", dtype=torch.bfloat16)
                od, idd, gd = moe.forward(L, x)
                oh, ih, gh = moe.forward(L, x.cpu())
                torch.cuda.synchronize()
                assert np.array_equal(od.cpu().numpy(), oh), (T, i)
                assert np.array_equal(idd.cpu().numpy().view(np.uint32), ih) and np.array_equal(gd.cpu().numpy(), gh)
        x = synth.make_tokens(1, d.hidden, 7100, device="cpu", dtype=torch.bfloat16)
        before, _, _ = moe.forward(L, x)
        w2 = synth.make_layer(d, seed=5, device="cuda")
        L2 = moe.Layer.from_weights(205, d, w2)  # same id, new weights
        after, _, _ = moe.forward(L2, x)
        want, _, _ = moe.forward(L2, x.cuda())
        torch.cuda.synchronize()
        assert np.array_equal(after, want.cpu().numpy()) and not np.array_equal(after, before)
    finally:
        L.unregister()
