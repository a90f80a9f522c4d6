"""colizig_cuda_moe_forward_noalloc (no counterpart in the reference): the
device-pointer MoE forward with its scratch in a static device array, so that
no call allocates device memory.

Checked against colizig_cuda_moe_forward on the same registered layer and the
same tokens: two calls in a row after the set-up call, each within the layer
output tolerance (top-k ids and gates identical).  Device free memory and
torch's allocator are unchanged across those two calls.  A layer beyond the
static scratch's limits is rejected before anything runs.

This file is collected last on purpose (its name), so it runs both after every
other test in one session and alone in a fresh process.
"""

import pytest
import torch

import colizig_b200 as cz
from colizig_b200 import _abi, moe, synth
from tests.util import OUT_TOL, assert_close

pytestmark = pytest.mark.gpu

LAYER_C2 = 9101
LAYER_BIG = 9102


@pytest.fixture(scope="module")
def c2_layer():
    torch.cuda.init()
    cz.gpu.init()
    d = synth.CONFIGS["c2"]
    layer = moe.Layer.from_weights(LAYER_C2, d, synth.make_layer(d, seed=77, device="cuda"))
    yield d, layer
    layer.unregister()


def _outputs(T, d):
    return (torch.empty((T, d.hidden), dtype=torch.float32, device="cuda"),
            torch.empty((T, d.topk), dtype=torch.int32, device="cuda"),
            torch.empty((T, d.topk), dtype=torch.float32, device="cuda"))


@pytest.mark.parametrize("T,dtype", [(1, torch.float32), (4, torch.bfloat16), (6, torch.float32)])
def test_noalloc_matches_forward_two_calls_in_a_row(c2_layer, T, dtype):
    d, layer = c2_layer
    xs = [synth.make_tokens(T, d.hidden, seed=900 + 10 * T + i, device="cuda", dtype=dtype) for i in range(3)]
    want = [moe.forward(layer, x) for x in xs]
    outs = [_outputs(T, d) for _ in xs]
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    # first call: set-up (scratch address, kernel attributes)
    moe.forward_noalloc(layer, xs[0], *outs[0], status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    free0 = torch.cuda.mem_get_info()[0]
    torch0 = torch.cuda.memory_allocated()
    for i in (1, 2):
        moe.forward_noalloc(layer, xs[i], *outs[i], status=status)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == torch0
    assert status.item() == 0
    for i in range(3):
        w_out, w_idx, w_g = want[i]
        out, idx, g = outs[i]
        assert torch.equal(idx, w_idx), i
        assert torch.equal(g, w_g), i
        assert_close(out.cpu().numpy(), w_out.cpu().numpy(), OUT_TOL, f"call {i}")


def test_noalloc_recovers_after_a_wait_gave_up(c2_layer):
    """A launch whose bounded waits give up (router row 0 withheld by the
    failure-path hook) reports it in status; the shared static scratch is left
    ready, so the next call is clean and matches colizig_cuda_moe_forward."""
    d, layer = c2_layer
    x = synth.make_tokens(2, d.hidden, seed=4242, device="cuda", dtype=torch.bfloat16)
    w_out, w_idx, w_g = moe.forward(layer, x)
    out, idx, g = _outputs(2, d)
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _abi.check("colizig_cuda_debug_hold_router", _abi.load().colizig_cuda_debug_hold_router(4000))
    moe.forward_noalloc(layer, x, out, idx, g, status=status)
    torch.cuda.synchronize()
    assert status.item() != 0
    moe.forward_noalloc(layer, x, out, idx, g, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(idx, w_idx) and torch.equal(g, w_g)
    assert_close(out.cpu().numpy(), w_out.cpu().numpy(), OUT_TOL, "after recovery")


def test_noalloc_rejects_layer_beyond_static_scratch():
    torch.cuda.init()
    cz.gpu.init()
    d = moe.Dims(hidden=4112, experts=4, topk=2, inter=16, shared_inter=0, norm_topk=True)
    layer = moe.Layer.from_weights(LAYER_BIG, d, synth.make_layer(d, seed=3, device="cuda"))
    try:
        x = synth.make_tokens(1, d.hidden, seed=5, device="cuda", dtype=torch.float32)
        out, idx, g = _outputs(1, d)
        status = torch.full((1,), 0x5A5A, dtype=torch.int32, device="cuda")
        with pytest.raises(_abi.ColizigError) as ei:
            moe.forward_noalloc(layer, x, out, idx, g, status=status)
        assert ei.value.rc == -8
        torch.cuda.synchronize()
        assert status.item() == 0x5A5A  # nothing launched
    finally:
        layer.unregister()


def test_noalloc_t0_and_bad_args(c2_layer):
    d, layer = c2_layer
    x1 = synth.make_tokens(1, d.hidden, seed=1, device="cuda", dtype=torch.float32)
    o1 = torch.empty((1, d.hidden), dtype=torch.float32, device="cuda")
    L = _abi.load()
    assert L.colizig_cuda_moe_forward_noalloc(layer.id, x1.data_ptr(), 0, 0, o1.data_ptr(), None, None, None,
                                              None) == 0  # T == 0: nothing to do
    assert L.colizig_cuda_moe_forward_noalloc(layer.id, x1.data_ptr(), 7, 1, o1.data_ptr(), None, None, None,
                                              None) == -1
    assert L.colizig_cuda_moe_forward_noalloc(4242, x1.data_ptr(), 0, 1, o1.data_ptr(), None, None, None,
                                              None) == -6
    assert L.colizig_cuda_moe_forward_noalloc(layer.id, None, 0, 1, o1.data_ptr(), None, None, None, None) == -1
