"""CPU oracle for colizig's block-FP8 MoE expert path.

TEST INFRASTRUCTURE ONLY.  This package is the parity checker and the timed CPU
baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it; the product package
``colizig_b200`` never does, and the product has no CPU fallback.

It binds ``libczref.so`` (built from ``oracle/czref.c`` by ``oracle/Makefile``),
a C restatement of the reference's Zig CPU path.  The function-by-function map
to the reference sources is in ``oracle/czref.h``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libczref.so")
_lib = None

BLOCK = 128


def nblk(x: int) -> int:
    """fp8.zig:19-21."""
    return (x + BLOCK - 1) // BLOCK


class CDims(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_size_t),
        ("experts", ctypes.c_size_t),
        ("topk", ctypes.c_size_t),
        ("inter", ctypes.c_size_t),
        ("shared_inter", ctypes.c_size_t),
        ("norm_topk", ctypes.c_int),
    ]


_PU8 = ctypes.POINTER(ctypes.c_uint8)
_PF32 = ctypes.POINTER(ctypes.c_float)


class CLayer(ctypes.Structure):
    _fields_ = [
        ("router", _PF32),
        ("gate_w", ctypes.POINTER(_PU8)),
        ("gate_s", ctypes.POINTER(_PF32)),
        ("up_w", ctypes.POINTER(_PU8)),
        ("up_s", ctypes.POINTER(_PF32)),
        ("down_w", ctypes.POINTER(_PU8)),
        ("down_s", ctypes.POINTER(_PF32)),
        ("sh_gate_w", _PU8),
        ("sh_gate_s", _PF32),
        ("sh_up_w", _PU8),
        ("sh_up_s", _PF32),
        ("sh_down_w", _PU8),
        ("sh_down_s", _PF32),
        ("sh_gate", _PF32),
        ("sh_gate_bf16", ctypes.POINTER(ctypes.c_uint16)),
        ("sh_up_bf16", ctypes.POINTER(ctypes.c_uint16)),
        ("sh_down_bf16", ctypes.POINTER(ctypes.c_uint16)),
    ]


def build() -> str:
    """Compile libczref.so with oracle/Makefile (gcc only, seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE, "libczref.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = ctypes.CDLL(_LIB_PATH)
    vp = ctypes.c_void_p
    sz = ctypes.c_size_t
    L.czref_nblk.argtypes = [sz]
    L.czref_nblk.restype = sz
    L.czref_e4m3_lut.argtypes = [vp]
    L.czref_expf.argtypes = [ctypes.c_float]
    L.czref_expf.restype = ctypes.c_float
    L.czref_expf_n.argtypes = [vp, vp, sz]
    L.czref_sigmoid.argtypes = [ctypes.c_float]
    L.czref_sigmoid.restype = ctypes.c_float
    L.czref_silu.argtypes = [ctypes.c_float]
    L.czref_silu.restype = ctypes.c_float
    L.czref_dequant_row.argtypes = [vp, vp, vp, sz]
    L.czref_dot_fp8_row.argtypes = [vp, vp, vp, sz]
    L.czref_dot_fp8_row.restype = ctypes.c_float
    L.czref_dot_f32.argtypes = [vp, vp, sz]
    L.czref_dot_f32.restype = ctypes.c_float
    L.czref_matmul_f32.argtypes = [vp, vp, vp, sz, sz, sz]
    L.czref_matmul_fp8.argtypes = [vp, vp, vp, vp, sz, sz, sz]
    L.czref_matmul_bf16.argtypes = [vp, vp, vp, sz, sz, sz]
    L.czref_rms.argtypes = [vp, vp, vp, sz, ctypes.c_float]
    L.czref_set_threads.argtypes = [ctypes.c_int]
    L.czref_get_threads.restype = ctypes.c_int
    L.czref_route.argtypes = [ctypes.POINTER(CLayer), ctypes.POINTER(CDims), vp, vp, vp]
    L.czref_moe_forward.argtypes = [ctypes.POINTER(CLayer), ctypes.POINTER(CDims), vp, sz, vp, vp, vp]
    L.czref_moe_forward.restype = ctypes.c_int
    _lib = L
    return L


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


# ---- scalar / row kernels -------------------------------------------------


def e4m3_lut() -> np.ndarray:
    out = np.empty(256, np.float32)
    lib().czref_e4m3_lut(_p(out))
    return out


def expf(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().czref_expf_n(_p(x), _p(y), x.size)
    return y


def sigmoid(x: float) -> float:
    return lib().czref_sigmoid(x)


def silu(x: float) -> float:
    return lib().czref_silu(x)


def dequant_row(w: np.ndarray, scale_row: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint8)
    scale_row = np.ascontiguousarray(scale_row, np.float32)
    out = np.empty(w.size, np.float32)
    lib().czref_dequant_row(_p(out), _p(w), _p(scale_row), w.size)
    return out


def dot_fp8_row(x: np.ndarray, w: np.ndarray, scale_row: np.ndarray) -> float:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    scale_row = np.ascontiguousarray(scale_row, np.float32)
    return lib().czref_dot_fp8_row(_p(x), _p(w), _p(scale_row), w.size)


def dot_f32(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return lib().czref_dot_f32(_p(a), _p(b), a.size)


def matmul_f32(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    S, I = x.shape
    O = w.shape[0]
    y = np.empty((S, O), np.float32)
    lib().czref_matmul_f32(_p(y), _p(x), _p(w), S, I, O)
    return y


def matmul_bf16(x: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """matmulBf16 (matmul.zig:36-48): y[S,O] = x[S,I] @ bf16(w)[O,I]^T, w as raw bf16 bits."""
    x = np.ascontiguousarray(x, np.float32)
    w_bits = np.ascontiguousarray(w_bits, np.uint16)
    S, I = x.shape
    O = w_bits.shape[0]
    y = np.empty((S, O), np.float32)
    lib().czref_matmul_bf16(_p(y), _p(x), _p(w_bits), S, I, O)
    return y


def matmul_fp8(x: np.ndarray, w: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """y[S,O] = x[S,I] @ dequant(w[O,I])^T with [nblk(O), nblk(I)] block scales."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    w = np.ascontiguousarray(w, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    S, I = x.shape
    O = w.shape[0]
    assert w.shape == (O, I) and scales.shape == (nblk(O), nblk(I))
    y = np.empty((S, O), np.float32)
    lib().czref_matmul_fp8(_p(y), _p(x), _p(w), _p(scales), S, I, O)
    return y


def rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rmsnorm.zig:32-40 over each row of x."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    xs = x.reshape(-1, x.shape[-1])
    out = np.empty_like(xs)
    for r in range(xs.shape[0]):
        lib().czref_rms(out[r].ctypes.data, xs[r].ctypes.data, _p(w), xs.shape[1], eps)
    return out.reshape(x.shape)


def set_threads(n: int) -> None:
    lib().czref_set_threads(int(n))


def get_threads() -> int:
    return lib().czref_get_threads()


# ---- MoE layer -------------------------------------------------------------


@dataclass
class Dims:
    """Mirrors moe.zig:23-30 (Dims)."""

    hidden: int
    experts: int
    topk: int
    inter: int
    shared_inter: int = 0
    norm_topk: bool = True

    def c(self) -> CDims:
        return CDims(self.hidden, self.experts, self.topk, self.inter, self.shared_inter, int(self.norm_topk))


@dataclass
class LayerWeights:
    """One MoE layer in the reference layout, stacked over experts.

    router [E,H] f32; gate_w/up_w [E,I,H] u8 (E4M3); gate_s/up_s [E,nb(I),nb(H)] f32;
    down_w [E,H,I] u8; down_s [E,nb(H),nb(I)] f32.  Optional shared expert
    (always-on FP8 expert): sh_gate_w/sh_up_w [SI,H], sh_down_w [H,SI] + scales,
    sh_gate [H] f32 (the sigmoid gate vector).  Or the reference's BF16 shared
    expert (NativeMatrix, moe.zig:297-338): sh_gate_bf16/sh_up_bf16 [SI,H] and
    sh_down_bf16 [H,SI] as raw bf16 bits (uint16), with sh_gate.
    """

    router: np.ndarray
    gate_w: np.ndarray
    gate_s: np.ndarray
    up_w: np.ndarray
    up_s: np.ndarray
    down_w: np.ndarray
    down_s: np.ndarray
    sh_gate_w: Optional[np.ndarray] = None
    sh_gate_s: Optional[np.ndarray] = None
    sh_up_w: Optional[np.ndarray] = None
    sh_up_s: Optional[np.ndarray] = None
    sh_down_w: Optional[np.ndarray] = None
    sh_down_s: Optional[np.ndarray] = None
    sh_gate: Optional[np.ndarray] = None
    sh_gate_bf16: Optional[np.ndarray] = None
    sh_up_bf16: Optional[np.ndarray] = None
    sh_down_bf16: Optional[np.ndarray] = None


LAYER_KEYS = ("router", "gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")
SHARED_KEYS = ("sh_gate_w", "sh_gate_s", "sh_up_w", "sh_up_s", "sh_down_w", "sh_down_s", "sh_gate")
SHARED_BF16_KEYS = ("sh_gate_bf16", "sh_up_bf16", "sh_down_bf16", "sh_gate")


def layer_from_dict(w: dict) -> LayerWeights:
    """LayerWeights from a mapping with the LAYER_KEYS (+ SHARED_KEYS) arrays."""
    kw = {k: np.ascontiguousarray(w[k]) for k in LAYER_KEYS}
    if "sh_gate_w" in w:
        kw.update({k: np.ascontiguousarray(w[k]) for k in SHARED_KEYS})
    elif "sh_gate_bf16" in w:
        kw.update({k: np.ascontiguousarray(w[k]) for k in SHARED_BF16_KEYS})
    return LayerWeights(**kw)


class _CLayerHolder:
    """Keeps the numpy arrays and ctypes pointer tables alive."""

    def __init__(self, lw: LayerWeights):
        self.lw = lw
        E = lw.gate_w.shape[0]

        def table(arr, ctype):
            arr = np.ascontiguousarray(arr)
            ptrs = (ctypes.POINTER(ctype) * E)()
            stride = arr[0].nbytes
            base = arr.ctypes.data
            for e in range(E):
                ptrs[e] = ctypes.cast(base + e * stride, ctypes.POINTER(ctype))
            return arr, ptrs

        self.arrays = []
        c = CLayer()
        router = np.ascontiguousarray(lw.router, np.float32)
        self.arrays.append(router)
        c.router = ctypes.cast(router.ctypes.data, _PF32)
        for name, ct in (("gate_w", ctypes.c_uint8), ("gate_s", ctypes.c_float), ("up_w", ctypes.c_uint8),
                         ("up_s", ctypes.c_float), ("down_w", ctypes.c_uint8), ("down_s", ctypes.c_float)):
            arr, ptrs = table(getattr(lw, name), ct)
            self.arrays += [arr, ptrs]
            setattr(c, name, ptrs)
        if lw.sh_gate_w is not None:
            for name, ct in (("sh_gate_w", ctypes.c_uint8), ("sh_gate_s", ctypes.c_float),
                             ("sh_up_w", ctypes.c_uint8), ("sh_up_s", ctypes.c_float),
                             ("sh_down_w", ctypes.c_uint8), ("sh_down_s", ctypes.c_float),
                             ("sh_gate", ctypes.c_float)):
                arr = np.ascontiguousarray(getattr(lw, name))
                self.arrays.append(arr)
                setattr(c, name, ctypes.cast(arr.ctypes.data, ctypes.POINTER(ct)))
        elif lw.sh_gate_bf16 is not None:
            for name, ct in (("sh_gate_bf16", ctypes.c_uint16), ("sh_up_bf16", ctypes.c_uint16),
                             ("sh_down_bf16", ctypes.c_uint16), ("sh_gate", ctypes.c_float)):
                arr = np.ascontiguousarray(getattr(lw, name))
                assert arr.dtype == (np.uint16 if ct is ctypes.c_uint16 else np.float32), name
                self.arrays.append(arr)
                setattr(c, name, ctypes.cast(arr.ctypes.data, ctypes.POINTER(ct)))
        self.c = c


def route(lw: LayerWeights, d: Dims, xs: np.ndarray):
    h = _CLayerHolder(lw)
    cd = d.c()
    xs = np.ascontiguousarray(xs, np.float32)
    idx = np.empty(d.topk, np.uint32)
    gates = np.empty(d.topk, np.float32)
    lib().czref_route(ctypes.byref(h.c), ctypes.byref(cd), _p(xs), _p(idx), _p(gates))
    return idx, gates


def moe_forward(lw: LayerWeights, d: Dims, x: np.ndarray):
    """forward() of moe.zig:409-426 on f32 x [S,H] -> (out [S,H], idx [S,K], gates [S,K])."""
    h = _CLayerHolder(lw)
    cd = d.c()
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    S = x.shape[0]
    out = np.empty_like(x)
    idx = np.empty((S, d.topk), np.uint32)
    gates = np.empty((S, d.topk), np.float32)
    rc = lib().czref_moe_forward(ctypes.byref(h.c), ctypes.byref(cd), _p(x), S, _p(out), _p(idx), _p(gates))
    if rc != 0:
        raise ValueError(f"czref_moe_forward rc={rc}")
    return out, idx, gates
