"""The C-ABI library loads and exports every declared symbol; host-side logic
that needs no GPU (CPU only, no compute calls)."""

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

import colizig_b200 as cz
from colizig_b200 import _abi, fp8, moe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "colizig_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(colizig_cuda_\w+)\s*\(", src)))


def test_header_declares_reference_surface():
    names = declared_functions()
    for n in _abi.REFERENCE_SYMBOLS:  # gpu.zig:84-89
        assert n in names
    assert set(names) == set(_abi.REFERENCE_SYMBOLS + _abi.MOE_SYMBOLS)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (colizig_cuda_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    L = _abi.load()
    for n in declared_functions():
        assert hasattr(L, n)


def test_build_targets_sm100a_only():
    mk = open(os.path.join(ROOT, "colizig_b200", "csrc", "Makefile")).read()
    assert re.findall(r"-gencode arch=(\S+)", mk) == ["compute_100a,code=sm_100a"]


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_an_error_not_a_fallback():
    L = _abi.load()
    assert L.colizig_cuda_device_name() == b""
    v = [ctypes.c_uint64(7) for _ in range(4)]
    L.colizig_cuda_stats(*[ctypes.byref(x) for x in v])  # null-safe, counters zero
    assert [x.value for x in v] == [0, 0, 0, 0]
    L.colizig_cuda_stats(None, None, None, None)
    x = np.zeros(4, np.float32)
    # not initialised -> -1 (colizig_cuda.cu:231), no CPU fallback
    assert L.colizig_cuda_matmul_fp8(x.ctypes.data, x.ctypes.data, x.ctypes.data, x.ctypes.data, 1, 1, 1, 0) == -1
    assert L.colizig_cuda_moe_forward(0, x.ctypes.data, 0, 1, x.ctypes.data, None, None, 0, None) == -1
    assert L.colizig_cuda_init() == -1  # no device
    with pytest.raises(cz.ColizigError) as e:
        cz.gpu.init()
    assert e.value.rc == -1
    with pytest.raises(cz.ColizigError):
        fp8.matmul_fp8(np.zeros((1, 16), np.float32), np.zeros((4, 16), np.uint8), np.ones((1, 1), np.float32))


def test_missing_library_raises(tmp_path):
    saved = _abi._lib
    _abi._lib = None
    try:
        with pytest.raises(RuntimeError, match="missing"):
            _abi.load(str(tmp_path / "libcolizig_cuda.so"))
    finally:
        _abi._lib = saved


def test_expert_key_scheme():  # moe.zig:97-99
    assert fp8.expert_key(0, 0, 0) == 1
    assert fp8.expert_key(1, 2, 2) == 1 + (1 * 512 + 2) * 4 + 2
    assert fp8.nblk(129) == 2


def test_dims_of_config():  # moe.zig:36-45
    d = moe.Dims.of({"hidden": 2048, "experts": 128, "topk": 8, "inter": 768})
    assert d == moe.Dims(2048, 128, 8, 768, 0, True) and not d.has_shared()
    c = d.c()
    assert (c.hidden, c.experts, c.topk, c.inter, c.shared_inter, c.norm_topk) == (2048, 128, 8, 768, 0, 1)


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_abi.MoeDims) == 24
    assert ctypes.sizeof(_abi.MoeExpert) == 48
