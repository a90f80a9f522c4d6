"""The checkpoint loader on the GPU: a layer registered straight from
safetensors shards (colizig_cuda_moe_load_safetensors) gives the same outputs
and top-k, bit for bit, as the same tensors registered from arrays, and agrees
with the CPU oracle; BF16 routers and BF16 block scales are widened exactly
(matmul.zig:84-110 dotBf16 multiplies the f32 widening of the bf16 bits)."""

import os

import numpy as np
import pytest
import torch

import colizig_b200 as cz
import oracle
from colizig_b200 import checkpoint, moe, synth
from tests.safetensors_util import bf16_bits, layer_tensors, write_safetensors
from tests.util import OUT_TOL, assert_close, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    torch.cuda.init()
    cz.gpu.init()
    oracle.set_threads(os.cpu_count() or 1)
    yield
    oracle.set_threads(1)


def _widen_bf16(a):
    return (bf16_bits(a).astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("router_bf16,scales_bf16,split", [(False, False, False), (True, True, True)])
def test_loaded_layer_equals_registered_layer(tmp_path, router_bf16, scales_bf16, split):
    d = synth.CONFIGS["c2"]
    w = synth.to_numpy_layer(synth.make_layer(d, seed=12, device="cpu"))
    t = layer_tensors(w, 3, prefix="model.language_model", router_bf16=router_bf16, scales_bf16=scales_bf16)
    if split:
        names = list(t)
        shards = []
        for i in range(3):
            p = tmp_path / f"model-{i:05d}-of-00003.safetensors"
            write_safetensors(p, {k: t[k] for k in names[i::3]})
            shards.append(p)
    else:
        shards = [tmp_path / "model.safetensors"]
        write_safetensors(shards[0], t)
    # what the loader must hold: the widened values
    wr = dict(w)
    if router_bf16:
        wr["router"] = _widen_bf16(w["router"])
    if scales_bf16:
        for k in ("gate_s", "up_s", "down_s"):
            wr[k] = _widen_bf16(w[k])
    A = checkpoint.load_layer(9201, shards, 3, d, prefix="model.language_model")
    B = moe.Layer.from_weights(9202, d, {k: np.ascontiguousarray(v) for k, v in wr.items()})
    try:
        for T in (1, 4, 64):
            x = synth.make_tokens(T, d.hidden, 500 + T, device="cuda", dtype=torch.bfloat16)
            oa, ia, ga = moe.forward(A, x)
            ob, ib, gb = moe.forward(B, x)
            torch.cuda.synchronize()
            moe.check()
            assert torch.equal(ia, ib) and torch.equal(ga, gb) and torch.equal(oa, ob), T
        oo, oi, _ = oracle.moe_forward(oracle.layer_from_dict(wr), oracle.Dims(d.hidden, d.experts, d.topk, d.inter, 0,
                                                                               True), synth.tokens_f32(x))
        assert np.array_equal(ia.cpu().numpy().view(np.uint32), oi)
        assert_close(oa.cpu().numpy(), oo, OUT_TOL, "loaded layer vs oracle")
    finally:
        A.unregister()
        B.unregister()


def test_loaded_shared_expert_layer_matches_golden(tmp_path):
    """The tiny shared-expert layer made by the reference's own numpy tools."""
    z = golden("moe_shared_tiny.npz")
    d = moe.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]), True)
    w = {k: np.ascontiguousarray(z[k]) for k in z.files if not k.isupper() and k not in ("x", "out", "idx")}
    p = tmp_path / "tiny.safetensors"
    write_safetensors(p, layer_tensors(w, 0, prefix=None))
    A = checkpoint.load_layer(9203, [p], 0, d, prefix="model")  # bare names: the prefixed lookup misses first
    try:
        out, idx, _ = moe.forward(A, z["x"])
        assert np.array_equal(idx, z["idx"])
        assert_close(out, z["out"])
    finally:
        A.unregister()


def test_loaded_bf16_shared_expert_layer_matches_golden(tmp_path):
    """A BF16 shared expert as real Qwen4-Exp checkpoints hold it (no scales),
    from the fixture made by the reference's numpy model."""
    z = golden("moe_shared_bf16_tiny.npz")
    d = moe.Dims(int(z["H"]), int(z["E"]), int(z["K"]), int(z["I"]), int(z["SI"]), True)
    w = {k: np.ascontiguousarray(z[k]) for k in z.files if not k.isupper() and k not in ("x", "out", "idx")}
    p = tmp_path / "tiny_bf16.safetensors"
    write_safetensors(p, layer_tensors(w, 0))
    A = checkpoint.load_layer(9204, [p], 0, d, prefix="model")
    try:
        out, idx, _ = moe.forward(A, z["x"])
        assert np.array_equal(idx, z["idx"])
        assert_close(out, z["out"])
    finally:
        A.unregister()
