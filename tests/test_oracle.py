"""The CPU oracle against the reference's own known answers (CPU only).

Pins: the reference's Zig test constants (fp8.zig:261-384, activation.zig:42-47,
matmul.zig:133-216, moe.zig:673-742) and golden fixtures produced by the
reference's NumPy implementation (tests/golden/make_golden.py).
"""

import numpy as np
import pytest

import oracle
from tests.util import LAYER_KEYS, SHARED_KEYS, assert_close, golden

DEMO_BYTES = np.array([0x38, 0x34, 0x30, 0x3C, 0xB8, 0xB4, 0x40, 0x2C], np.uint8)
DEMO_VALUES = np.array([1.0, 0.75, 0.5, 1.5, -1.0, -0.75, 2.0, 0.375], np.float32)


def test_e4m3_demo_bytes_decode_exactly():  # fp8.zig:266-271
    lut = oracle.e4m3_lut()
    assert np.array_equal(lut[DEMO_BYTES], DEMO_VALUES)
    assert lut[0] == 0.0


def test_e4m3_all_256_match_reference_decoder():
    want = golden("e4m3_decode_all256.npy")
    lut = oracle.e4m3_lut()
    nan = np.isnan(want)
    assert np.array_equal(np.nonzero(nan)[0], [0x7F, 0xFF])
    assert np.array_equal(np.isnan(lut), nan)
    assert np.array_equal(lut[~nan].view(np.uint32), want[~nan].view(np.uint32))  # bit-exact, incl. -0


def test_nblk():  # fp8.zig:379-384
    assert [oracle.nblk(v) for v in (1, 128, 129, 2560)] == [1, 1, 2, 20]


def test_dequant_row_bit_identical_to_lut():  # fp8.zig:355-377
    I = 128 + 77
    w = (np.arange(I) % 256).astype(np.uint8)
    scale_row = np.array([0.5, 1.75], np.float32)
    got = oracle.dequant_row(w, scale_row)
    lut = oracle.e4m3_lut()
    want = (lut[w] * scale_row[np.arange(I) // 128]).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan], want[~nan])


def _dequant(w, s):
    lut = oracle.e4m3_lut()
    O, I = w.shape
    return (lut[w] * np.repeat(np.repeat(s, 128, 0), 128, 1)[:O, :I]).astype(np.float32)


@pytest.mark.parametrize("name", ["two_blocks", "all_finite_bytes", "c1_gate", "ragged"])
def test_matmul_fp8_matches_reference_numpy(name):
    k = golden("fp8_matmul_kat.npz")
    x, w, s, y = (k[f"{name}_{t}"] for t in "xwsy")
    got = oracle.matmul_fp8(x, w, s)
    np.testing.assert_allclose(got, y, rtol=1e-4, atol=1e-4 * np.abs(y).max())
    # fp8.zig:273-311: equals the plain f32 matmul on dequantised weights
    ref = oracle.matmul_f32(x, _dequant(w, s))
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())


def test_dot_fp8_row_all_finite_bytes():  # fp8.zig:313-353 (S == 1 fused path, I=384, O=6)
    rng = np.random.default_rng(0x5115)
    I, O = 384, 6
    x = (rng.random(I) * 2 - 1).astype(np.float32)
    w = rng.integers(0, 256, (O, I), dtype=np.uint8)
    w[(w == 0x7F) | (w == 0xFF)] = 0
    s = (0.25 + rng.random((1, 3))).astype(np.float32)
    y1 = oracle.matmul_fp8(x, w, s)[0]
    y2 = oracle.matmul_f32(x[None], _dequant(w, s))[0]
    np.testing.assert_allclose(y1, y2, rtol=1e-4)


def test_dot_f32_matches_naive():  # matmul.zig:133-155 (I = 37, not a multiple of the width)
    rng = np.random.default_rng(0xC0FFEE)
    x = (rng.random((5, 37)) * 2 - 1).astype(np.float32)
    w = (rng.random((9, 37)) * 2 - 1).astype(np.float32)
    np.testing.assert_allclose(oracle.matmul_f32(x, w), x.astype(np.float64) @ w.T.astype(np.float64), rtol=1e-4)


def test_dot_f32_lane_order():
    """dotF32 = 4 chains x 8 lanes, total=((a0+a1)+a2)+a3, ordered lane sum, FMA tail."""
    rng = np.random.default_rng(7)
    for n in (1, 7, 8, 31, 32, 33, 200, 2048):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        acc = np.zeros((4, 8), np.float32)
        i = 0
        fma = lambda p, q, r: np.float32(np.float64(p) * np.float64(q) + np.float64(r))  # exact-product f32 fma
        while i + 32 <= n:
            for k in range(4):
                for l in range(8):
                    acc[k, l] = fma(a[i + 8 * k + l], b[i + 8 * k + l], acc[k, l])
            i += 32
        while i + 8 <= n:
            for l in range(8):
                acc[0, l] = fma(a[i + l], b[i + l], acc[0, l])
            i += 8
        total = np.zeros(8, np.float32)
        for k in range(4):
            total = (total + acc[k]).astype(np.float32)
        s = np.float32(total[0])
        for l in range(1, 8):
            s = np.float32(s + total[l])
        while i < n:
            s = fma(a[i], b[i], s)
            i += 1
        assert oracle.dot_f32(a, b) == s, n


def test_threaded_matches_serial_bit_exact():  # matmul.zig:191-216
    rng = np.random.default_rng(0xA11)
    x = (rng.random((2, 256)) * 2 - 1).astype(np.float32)
    w = (rng.random((512, 256)) * 2 - 1).astype(np.float32)
    wq = rng.integers(0, 256, (512, 256), dtype=np.uint8)
    wq[(wq == 0x7F) | (wq == 0xFF)] = 0
    s = (0.5 + rng.random((4, 2))).astype(np.float32)
    oracle.set_threads(1)
    ys, qs = oracle.matmul_f32(x, w), oracle.matmul_fp8(x, wq, s)
    q1 = oracle.matmul_fp8(x[:1], wq, s)
    oracle.set_threads(8)
    try:
        yp, qp = oracle.matmul_f32(x, w), oracle.matmul_fp8(x, wq, s)
        q1p = oracle.matmul_fp8(x[:1], wq, s)
    finally:
        oracle.set_threads(1)
    assert np.array_equal(ys, yp) and np.array_equal(qs, qp) and np.array_equal(q1, q1p)


def test_activation_reference_points():  # activation.zig:42-47
    assert abs(oracle.sigmoid(0.0) - 0.5) < 1e-6
    assert abs(oracle.sigmoid(1.0) - 0.7310586) < 1e-5
    assert abs(oracle.silu(0.0)) < 1e-6
    assert abs(oracle.sigmoid(-3.0) - (1.0 - oracle.sigmoid(3.0))) < 1e-6


def test_expf_is_correctly_rounded():
    """The restatement of @exp(f32) equals exp in f64 rounded once to f32."""
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.uniform(-103, 88, 200000), rng.uniform(-1, 1, 100000), rng.uniform(-30, 0, 100000),
                         [0.0, -0.0, 1.0, -1.0, 88.7, -87.0, -103.9]]).astype(np.float32)
    got = oracle.expf(xs)
    want = np.exp(xs.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, want)
    special = oracle.expf(np.array([np.nan, np.inf, -np.inf, 200.0, -200.0], np.float32))
    assert np.isnan(special[0]) and special[1] == np.inf and special[2] == 0 and special[3] == np.inf
    assert special[4] == 0


def _layer(z, shared=False):
    kw = {k: z[k] for k in LAYER_KEYS}
    if shared:
        kw.update({k: z[k] for k in SHARED_KEYS})
    return oracle.LayerWeights(**kw)


def test_moe_c1_matches_reference_numpy():
    """C1 tiny layer vs the reference's qwen3moe_ref.Model.moe (f64 accumulation)."""
    z = golden("moe_c1.npz")
    d = oracle.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), 0, True)
    L = _layer(z)
    for t in range(z["x"].shape[0]):  # decode path, one token at a time
        out, idx, _ = oracle.moe_forward(L, d, z["x"][t])
        assert np.array_equal(idx[0], z["idx"][t])
        assert_close(out[0], z["out"][t], 1e-5)
    out, idx, _ = oracle.moe_forward(L, d, z["x"])  # grouped prefill path
    assert np.array_equal(idx, z["idx"])
    assert_close(out, z["out"], 1e-5)


def test_moe_shared_expert_matches_reference_numpy():
    """Always-on shared expert with sigmoid gate vs qwen38_ref.Model.moe."""
    z = golden("moe_shared_tiny.npz")
    d = oracle.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]), True)
    L = _layer(z, shared=True)
    out, idx, _ = oracle.moe_forward(L, d, z["x"])
    assert np.array_equal(idx, z["idx"])
    assert_close(out, z["out"], 1e-5)
    for t in range(z["x"].shape[0]):
        o1, i1, _ = oracle.moe_forward(L, d, z["x"][t])
        assert np.array_equal(i1[0], z["idx"][t])
        assert_close(o1[0], z["out"][t], 1e-5)


def _layer_bf16_shared(z):
    kw = {k: z[k] for k in LAYER_KEYS}
    kw.update({k: np.ascontiguousarray(z[k]) for k in ("sh_gate_bf16", "sh_up_bf16", "sh_down_bf16", "sh_gate")})
    return oracle.LayerWeights(**kw)


def test_moe_bf16_shared_expert_matches_reference_numpy():
    """BF16 NativeMatrix shared expert (moe.zig:297-338, dotBf16 matmul.zig:84-106)
    vs qwen38_ref.Model.moe on the same weights widened to f32."""
    z = golden("moe_shared_bf16_tiny.npz")
    assert z["sh_gate_bf16"].dtype == np.uint16
    d = oracle.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]), True)
    L = _layer_bf16_shared(z)
    out, idx, _ = oracle.moe_forward(L, d, z["x"])
    assert np.array_equal(idx, z["idx"])
    assert_close(out, z["out"], 1e-5)
    for t in range(z["x"].shape[0]):
        o1, i1, _ = oracle.moe_forward(L, d, z["x"][t])
        assert np.array_equal(i1[0], z["idx"][t])
        assert_close(o1[0], z["out"][t], 1e-5)


def test_dot_bf16_widens_exactly():
    """dotBf16 equals dotF32 on the same weights widened to f32 (both 4 chains x 8 lanes)."""
    rng = np.random.default_rng(3)
    for n in (256, 200, 37):
        a = rng.standard_normal(n).astype(np.float32)
        b = (rng.standard_normal(n) * 0.1).astype(np.float32)
        bits = (b.view(np.uint32) >> 16).astype(np.uint16)
        wide = (bits.astype(np.uint32) << 16).view(np.float32)
        y = oracle.matmul_bf16(a[None, :], bits[None, :])
        assert y[0, 0] == np.float32(oracle.dot_f32(a, wide))


def test_grouped_prefill_close_to_dense():  # moe.zig:720-728
    z = golden("moe_c1.npz")
    d = oracle.Dims(256, 16, 4, 128, 0, True)
    L = _layer(z)
    og, ig, _ = oracle.moe_forward(L, d, z["x"])
    for t in range(z["x"].shape[0]):
        od, idd, _ = oracle.moe_forward(L, d, z["x"][t])
        assert np.array_equal(ig[t], idd[0])
        assert np.max(np.abs(od[0] - og[t])) <= 1e-3


def test_route_ties_pick_lowest_id_and_nan_picks_zero():
    """moe.zig:447-460: strict > from e = 0 (ties -> lowest id); no candidate -> id 0."""
    z = golden("moe_c1.npz")
    L = _layer(z)
    router = np.array(L.router)
    router[5] = router[9]  # identical rows -> identical logits
    router[3] = router[9]
    L.router = router
    d = oracle.Dims(256, 16, 16, 128, 0, True)  # select all: forces the tie order to show
    x = z["x"][0]
    idx, gates = oracle.route(L, d, x)
    pos = {e: i for i, e in enumerate(idx)}
    assert pos[3] < pos[5] < pos[9]
    xn = np.full(256, np.nan, np.float32)
    idx, gates = oracle.route(L, oracle.Dims(256, 16, 4, 128, 0, True), xn)
    assert list(idx) == [0, 0, 0, 0] and np.all(np.isnan(gates))


def test_rms_matches_formula():  # rmsnorm.zig:32-40
    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    got = oracle.rms(x, w, 1e-6)
    for r in range(3):
        ss = 0.0
        for v in x[r].astype(np.float64):
            ss += v * v
        mean = np.float32(ss / 256)
        rr = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(1e-6)))
        want = (x[r] * rr * w).astype(np.float32)
        assert np.array_equal(got[r], want)
