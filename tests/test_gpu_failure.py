"""Failure path on one GPU, in the form allowed on a shared pool: a bounded
device wait that runs out.  colizig_cuda_debug_hold_router makes the next decode
launch withhold router row 0's logits, so every CTA's wait for them gives up
after a short poll limit; the launch ends early with the error word set.  The
reference's contract is "an error code, never a wrong number" (its exports
return -1..-5, colizig_cuda.cu:228-284): here the call returns -7 (host
pointers), moe.check() raises it (device pointers), and the next call starts
clean and matches the undisturbed result.  No trap, no fault, no endless wait.
"""

import numpy as np
import pytest
import torch

import colizig_b200 as cz
from colizig_b200 import _abi, moe, synth

pytestmark = pytest.mark.gpu

HOLD_POLLS = 4000  # about a millisecond of polling before the waits give up


@pytest.fixture(scope="module")
def layer():
    torch.cuda.init()
    cz.gpu.init()
    d = synth.CONFIGS["c2"]
    L = moe.Layer.from_weights(9301, d, synth.make_layer(d, seed=31, device="cuda"))
    yield d, L
    L.unregister()


def _hold():
    _abi.check("colizig_cuda_debug_hold_router", _abi.load().colizig_cuda_debug_hold_router(HOLD_POLLS))


@pytest.mark.parametrize("T", [1, 3])
def test_host_call_reports_timeout_then_recovers(layer, T):
    d, L = layer
    x = synth.make_tokens(T, d.hidden, 70 + T, device="cpu", dtype=torch.float32).numpy()
    want, wi, wg = moe.forward(L, x)
    _hold()
    with pytest.raises(cz.ColizigError) as ei:
        moe.forward(L, x)
    assert ei.value.rc == -7
    got, gi, gg = moe.forward(L, x)  # the next call is clean and exact
    assert np.array_equal(gi, wi) and np.array_equal(gg, wg) and np.array_equal(got, want)


def test_device_call_reports_timeout_through_check_then_recovers(layer):
    d, L = layer
    x = synth.make_tokens(2, d.hidden, 91, device="cuda", dtype=torch.bfloat16)
    want, wi, _ = moe.forward(L, x)
    torch.cuda.synchronize()
    moe.check()
    _hold()
    moe.forward(L, x)
    with pytest.raises(cz.ColizigError) as ei:
        moe.check()
    assert ei.value.rc == -7
    moe.check()  # the error word was cleared by the read
    got, gi, _ = moe.forward(L, x)
    torch.cuda.synchronize()
    moe.check()
    assert torch.equal(gi, wi) and torch.equal(got, want)


def test_hold_is_one_shot_and_rejects_zero_limit(layer):
    d, L = layer
    assert _abi.load().colizig_cuda_debug_hold_router(0) == -1
    x = synth.make_tokens(1, d.hidden, 5, device="cpu", dtype=torch.float32).numpy()
    _hold()
    with pytest.raises(cz.ColizigError):
        moe.forward(L, x)
    for _ in range(3):
        moe.forward(L, x)  # no error: the hold applied to one launch only
