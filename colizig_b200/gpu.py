"""Host-side mirror of src/backend/gpu.zig (the runtime-loaded CUDA backend).

Same operations and meaning: ``init`` brings the backend up (gpu.zig:72-109),
``device_name``, ``set_vram_budget`` (:156-158), ``stats`` (:160-170),
``matmul_fp8`` (:175-190) and ``deinit`` (:116-122).  The one behavioural change
is the failure mode: the reference returns ``false`` so its caller can run the
CPU path; this package has no CPU path, so a failure raises ``ColizigError``.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _abi

_ready = False


def init(device: int = 0) -> None:
    global _ready
    L = _abi.load()
    rc = L.colizig_cuda_init() if device == 0 else L.colizig_cuda_init_device(device)
    _abi.check("colizig_cuda_init", rc)
    _ready = True


def available() -> bool:
    return _ready


def deinit() -> None:
    global _ready
    if _ready:
        _abi.load().colizig_cuda_shutdown()
    _ready = False


def device_name() -> str:
    return _abi.load().colizig_cuda_device_name().decode()


def set_vram_budget(nbytes: int) -> None:
    _abi.load().colizig_cuda_set_vram_budget(int(nbytes))


def stats():
    """(hits, misses, uploaded_mib, resident) of the keyed weight store."""
    v = [ctypes.c_uint64(0) for _ in range(4)]
    _abi.load().colizig_cuda_stats(*[ctypes.byref(x) for x in v])
    return tuple(int(x.value) for x in v)


def matmul_fp8(y: np.ndarray, x: np.ndarray, w: np.ndarray, scales: np.ndarray, S: int, I: int, O: int,
               key: int = 0) -> None:
    """y[S,O] = x[S,I] @ dequant(w[O,I])^T on the GPU (host arrays, synchronous)."""
    for a, dt in ((y, np.float32), (x, np.float32), (w, np.uint8), (scales, np.float32)):
        if a.dtype != dt or not a.flags["C_CONTIGUOUS"]:
            raise ValueError("matmul_fp8 wants C-contiguous f32 y/x/scales and u8 w")
    rc = _abi.load().colizig_cuda_matmul_fp8(y.ctypes.data, x.ctypes.data, w.ctypes.data, scales.ctypes.data,
                                             int(S), int(I), int(O), int(key))
    _abi.check("colizig_cuda_matmul_fp8", rc)
