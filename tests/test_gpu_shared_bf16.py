"""BF16 shared expert (the reference's NativeMatrix shared expert,
src/qwen38/moe.zig:297-338 and 467-479, dotBf16 in src/ops/matmul.zig:84-110),
registered with COLIZIG_SHARED_BF16 beside the block-FP8 routed experts: the
golden fixture made by the reference's numpy model, a config-5-shaped layer
(hidden 4096, 512 experts, top-10, shared_inter 1024) through the decode and
prefill paths, the stack caller (rms + MoE + residual), and host pointers.
Top-k ids and gates bit-exact; outputs within 1e-3 * ||out||_inf."""

import numpy as np
import pytest
import torch

import oracle
from colizig_b200 import moe, synth
from tests.util import OUT_TOL, assert_close, golden, oracle_layer

pytestmark = pytest.mark.gpu


def test_bf16_shared_golden():
    z = golden("moe_shared_bf16_tiny.npz")
    d = moe.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]), True)
    w = {k: np.ascontiguousarray(z[k]) for k in z.files if not k.isupper() and k not in ("x", "out", "idx")}
    assert w["sh_gate_bf16"].dtype == np.uint16
    L = moe.Layer.from_weights(150, d, w)
    ol = oracle_layer(w)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, True)
    oo, oi, _ = oracle.moe_forward(ol, od, z["x"])
    out, idx, _ = moe.forward(L, z["x"])  # host pointers, 3 tokens
    assert np.array_equal(idx, z["idx"]) and np.array_equal(idx, oi)
    assert_close(out, z["out"], OUT_TOL, "vs reference numpy")
    assert_close(out, oo, OUT_TOL, "vs oracle")
    for t in range(z["x"].shape[0]):  # one token per call (graph-replayed after the first two)
        for _ in range(3):
            o1, i1, _ = moe.forward(L, z["x"][t:t + 1])
            assert np.array_equal(i1[0], z["idx"][t])
            assert_close(o1[0], z["out"][t], OUT_TOL, f"token {t}")
    L.unregister()


def _c5_bf16_layer(layer_id, seed):
    d = synth.CONFIGS["c5"]
    w = synth.bf16_shared(synth.make_layer(d, seed=seed, device="cuda"), d, seed=seed)
    return d, w, moe.Layer.from_weights(layer_id, d, w)


@pytest.mark.parametrize("T", [1, 16, 40])
def test_bf16_shared_c5_matches_oracle(T):
    d, w, L = _c5_bf16_layer(151, 3)
    ol = oracle_layer(synth.to_numpy_layer(w))
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    x = synth.make_tokens(T, d.hidden, 4000 + T, device="cuda", dtype=torch.bfloat16)
    out, idx, gates = moe.forward(L, x)
    out2, _, _ = moe.forward(L, x)
    torch.cuda.synchronize()
    moe.check()
    oo, oi, og = oracle.moe_forward(ol, od, synth.tokens_f32(x))
    assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi)
    np.testing.assert_array_equal(gates.cpu().numpy(), og)
    e = assert_close(out.cpu().numpy(), oo, OUT_TOL, f"T={T}")
    assert torch.equal(out, out2)  # deterministic
    # the shared expert's own share is visible in the output: dropping it fails the check
    d0 = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, 0, d.norm_topk)
    o_routed, _, _ = oracle.moe_forward(oracle_layer({k: v for k, v in synth.to_numpy_layer(w).items()
                                                      if not k.startswith("sh_")}), d0, synth.tokens_f32(x))
    assert np.max(np.abs(oo - o_routed)) > 10 * OUT_TOL * np.max(np.abs(oo))
    print(f"c5 bf16 shared T={T}: rel err {e:.2e}")
    L.unregister()


def test_bf16_shared_stack_caller():
    """model.zig:227-232 with a BF16-shared layer: n = rms(h); h += moe(n)."""
    d, w, L = _c5_bf16_layer(152, 4)
    ol = oracle_layer(synth.to_numpy_layer(w))
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    rng = np.random.default_rng(21)
    norm_w = (1.0 + 0.05 * rng.standard_normal((1, d.hidden))).astype(np.float32)
    for T in (2, 40):
        h = rng.standard_normal((T, d.hidden)).astype(np.float32)
        h_gpu = moe.stack_forward(152, 1, h.copy(), norm_w, 1e-6)
        b, _, _ = oracle.moe_forward(ol, od, oracle.rms(h, norm_w[0], 1e-6))
        want = (h + b).astype(np.float32)
        ulp = np.spacing(np.maximum(np.abs(h), np.abs(want))).astype(np.float64)
        bound = OUT_TOL * np.abs(b).max() + ulp
        assert np.all(np.abs(h_gpu.astype(np.float64) - want) <= bound), f"T={T}"
    L.unregister()
