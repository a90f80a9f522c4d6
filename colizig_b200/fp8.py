"""Host-side mirror of src/ops/fp8.zig's public block-FP8 operations.

``matmul_fp8_keyed(x, w, scales, key)`` is fp8.zig:165-188 matmulFp8Keyed and
``matmul_fp8`` is :192-194, computed by libcolizig_cuda.so.  Weight element
(o, i) is e4m3(w[o, i]) * scales[o // 128, i // 128] (fp8.zig:3-6).
"""

from __future__ import annotations

import numpy as np

from . import gpu

BLOCK = 128


def nblk(x: int) -> int:
    """fp8.zig:19-21."""
    return (x + BLOCK - 1) // BLOCK


def matmul_fp8_keyed(x: np.ndarray, w: np.ndarray, scales: np.ndarray, key: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    w = np.ascontiguousarray(w, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    S, I = x.shape
    O = w.shape[0]
    if w.shape != (O, I) or scales.shape != (nblk(O), nblk(I)):
        raise ValueError(f"shape mismatch: x {x.shape} w {w.shape} scales {scales.shape}")
    if not gpu.available():
        gpu.init()
    y = np.empty((S, O), np.float32)
    gpu.matmul_fp8(y, x, w, scales, S, I, O, key)
    return y


def matmul_fp8(x: np.ndarray, w: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return matmul_fp8_keyed(x, w, scales, 0)


def expert_key(layer: int, expert: int, role: int) -> int:
    """moe.zig:97-99: 1 + ((layer*512 + expert)*4 + role), role 0/1/2 = gate/up/down."""
    return 1 + (layer * 512 + expert) * 4 + role


def attn_key(layer: int, role: int) -> int:
    """src/qwen3moe/attn.zig:46-50 attnKey: the expert slot 1020 + role (0..3 = q/k/v/o)
    of the expert key scheme, so attention projections share the keyed store."""
    if not 0 <= role <= 3:
        raise ValueError("role is 0..3 (q, k, v, o)")
    return expert_key(layer, 1020 + role, 0)

