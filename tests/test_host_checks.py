"""Host-side argument checks of the forward wrappers (no GPU needed).

The library receives raw pointers only, so a mis-shaped buffer would make the
kernel read and write past the caller's memory.  moe.check_io rejects such
calls before anything reaches the library; forward and forward_noalloc call it
first.
"""

import numpy as np
import pytest
import torch

from colizig_b200 import moe

D = moe.Dims(hidden=256, experts=16, topk=4, inter=128)


def _ok(T=3):
    return (torch.zeros((T, 256)), torch.zeros((T, 256)), torch.zeros((T, 4), dtype=torch.int32),
            torch.zeros((T, 4)))


def test_check_io_accepts_well_formed_buffers():
    x, out, idx, g = _ok()
    assert moe.check_io(D, x, out, idx, g) == 3
    assert moe.check_io(D, x.to(torch.bfloat16)) == 3
    assert moe.check_io(D, np.zeros((2, 256), np.float32), np.zeros((2, 256), np.float32),
                        np.zeros((2, 4), np.uint32), np.zeros((2, 4), np.float32)) == 2
    st = torch.zeros(1, dtype=torch.int32)
    assert moe.check_io(D, x, out, idx, g, st, device=x.device) == 3


def test_check_io_rejects_one_dimensional_tokens():
    with pytest.raises(ValueError, match="2-D"):
        moe.check_io(D, torch.zeros(256), torch.zeros((1, 256)))


def test_check_io_rejects_wrong_hidden_size():
    with pytest.raises(ValueError, match="columns"):
        moe.check_io(D, torch.zeros((2, 255)))


@pytest.mark.parametrize("bad", [
    ("out", torch.zeros((2, 256))),                      # too few rows
    ("out", torch.zeros((3, 256), dtype=torch.float64)),  # wrong dtype
    ("out", torch.zeros((3, 257))),                      # wrong width
    ("idx", torch.zeros((3, 5), dtype=torch.int32)),     # wrong top-k width
    ("idx", torch.zeros((3, 4))),                        # f32 ids
    ("gates", torch.zeros((3, 4), dtype=torch.int32)),   # integer gates
])
def test_check_io_rejects_mis_shaped_outputs(bad):
    x, out, idx, g = _ok()
    name, a = bad
    kw = {"out": out, "topk_idx": idx, "topk_gates": g}
    kw[{"out": "out", "idx": "topk_idx", "gates": "topk_gates"}[name]] = a
    with pytest.raises(ValueError):
        moe.check_io(D, x, **kw)


def test_check_io_rejects_bad_status_and_foreign_device():
    x, out, idx, g = _ok()
    with pytest.raises(ValueError, match="status"):
        moe.check_io(D, x, out, idx, g, torch.zeros(0, dtype=torch.int32))
    with pytest.raises(ValueError, match="status"):
        moe.check_io(D, x, out, idx, g, torch.zeros(1, dtype=torch.float32))
    with pytest.raises(ValueError, match="must be a tensor on"):
        moe.check_io(D, x, np.zeros((3, 256), np.float32), device=x.device)
