"""ctypes binding of libcolizig_cuda.so (declarations in include/colizig_cuda.h).

Mirrors src/backend/gpu.zig:72-109, which resolves the backend's symbols by name
and treats a missing symbol as "backend unavailable".  Here a missing library or
symbol is an error: this package has no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# COLIZIG_LIBRARY overrides the in-tree library (to compare builds); unset in normal use.
LIB_PATH = os.environ.get("COLIZIG_LIBRARY") or os.path.join(HERE, "libcolizig_cuda.so")

# the six symbols of the reference surface (gpu.zig:84-89) + the MoE-level ones
REFERENCE_SYMBOLS = (
    "colizig_cuda_init",
    "colizig_cuda_device_name",
    "colizig_cuda_shutdown",
    "colizig_cuda_matmul_fp8",
    "colizig_cuda_matmul_fp8_device",
    "colizig_cuda_set_vram_budget",
    "colizig_cuda_stats",
)
MOE_SYMBOLS = (
    "colizig_cuda_init_device",
    "colizig_cuda_moe_register_layer",
    "colizig_cuda_moe_unregister_layer",
    "colizig_cuda_moe_load_safetensors",
    "colizig_cuda_moe_forward",
    "colizig_cuda_moe_stack_forward",
    "colizig_cuda_moe_check",
    "colizig_cuda_debug_expf",
    "colizig_cuda_debug_hold_router",
    "colizig_cuda_debug_error_bits",
    "colizig_cuda_debug_watch_wait",
    "colizig_cuda_moe_forward_noalloc",
    "colizig_cuda_ep_unique_id",
    "colizig_cuda_ep_init",
    "colizig_cuda_ep_shutdown",
    "colizig_cuda_ep_set_timeout",
    "colizig_cuda_ep_abort",
    "colizig_cuda_ep_combine_mode",
    "colizig_cuda_moe_decode_batch",
    "colizig_cuda_ep_set_combine",
    "colizig_cuda_kernel_timer",
    "colizig_cuda_kernel_timer_read",
)

# callback types of colizig_cuda_debug_watch_wait (query / async error, abort)
WATCH_QUERY = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)
WATCH_ABORT = ctypes.CFUNCTYPE(None, ctypes.c_void_p)

COLIZIG_PTR_DEVICE = 1
COLIZIG_EP = 2
COLIZIG_EP_SHARDED = 4
COLIZIG_SHARED_BF16 = 8
COLIZIG_X_F32 = 0
COLIZIG_X_BF16 = 1

ERRORS = {
    -1: "bad arguments / not initialised",
    -2: "device allocation failed",
    -3: "host->device copy failed",
    -4: "kernel launch failed",
    -5: "device->host copy failed",
    -6: "layer not registered",
    -7: "device-side wait timed out",
    -8: "shape not supported",
    -9: "NCCL / expert-parallel error",
    -10: "checkpoint file missing, unreadable or malformed, or a tensor missing",
}


class ColizigError(RuntimeError):
    def __init__(self, fn: str, rc: int):
        super().__init__(f"{fn} returned {rc} ({ERRORS.get(rc, 'unknown')})")
        self.rc = rc


class MoeDims(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_uint32),
        ("experts", ctypes.c_uint32),
        ("topk", ctypes.c_uint32),
        ("inter", ctypes.c_uint32),
        ("shared_inter", ctypes.c_uint32),
        ("norm_topk", ctypes.c_uint32),
    ]


class MoeExpert(ctypes.Structure):
    _fields_ = [
        ("gate_w", ctypes.c_void_p),
        ("gate_s", ctypes.c_void_p),
        ("up_w", ctypes.c_void_p),
        ("up_s", ctypes.c_void_p),
        ("down_w", ctypes.c_void_p),
        ("down_s", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library and declare every exported signature.  Raises if the
    library or any declared symbol is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with __graft_entry__.build() (no CPU fallback)")
        L = ctypes.CDLL(path)
        for name in REFERENCE_SYMBOLS + MOE_SYMBOLS:
            if not hasattr(L, name):
                raise RuntimeError(f"{name} missing from {path}")
        vp, u32, u64, i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        P64 = ctypes.POINTER(ctypes.c_uint64)
        L.colizig_cuda_init.restype = i32
        L.colizig_cuda_init.argtypes = []
        L.colizig_cuda_init_device.restype = i32
        L.colizig_cuda_init_device.argtypes = [i32]
        L.colizig_cuda_device_name.restype = ctypes.c_char_p
        L.colizig_cuda_device_name.argtypes = []
        L.colizig_cuda_shutdown.restype = None
        L.colizig_cuda_shutdown.argtypes = []
        L.colizig_cuda_set_vram_budget.restype = None
        L.colizig_cuda_set_vram_budget.argtypes = [u64]
        L.colizig_cuda_stats.restype = None
        L.colizig_cuda_stats.argtypes = [P64, P64, P64, P64]
        L.colizig_cuda_matmul_fp8.restype = i32
        L.colizig_cuda_matmul_fp8.argtypes = [vp, vp, vp, vp, i32, i32, i32, u64]
        L.colizig_cuda_matmul_fp8_device.restype = i32
        L.colizig_cuda_matmul_fp8_device.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp]
        L.colizig_cuda_moe_register_layer.restype = i32
        L.colizig_cuda_moe_register_layer.argtypes = [u32, ctypes.POINTER(MoeDims), vp, ctypes.POINTER(MoeExpert),
                                                      ctypes.POINTER(MoeExpert), vp, u32]
        L.colizig_cuda_moe_unregister_layer.restype = i32
        L.colizig_cuda_moe_unregister_layer.argtypes = [u32]
        L.colizig_cuda_moe_load_safetensors.restype = i32
        L.colizig_cuda_moe_load_safetensors.argtypes = [u32, ctypes.POINTER(ctypes.c_char_p), i32, ctypes.c_char_p, u32,
                                                        ctypes.POINTER(MoeDims), u32]
        L.colizig_cuda_moe_forward.restype = i32
        L.colizig_cuda_moe_forward.argtypes = [u32, vp, i32, i32, vp, vp, vp, u32, vp]
        L.colizig_cuda_moe_stack_forward.restype = i32
        L.colizig_cuda_moe_stack_forward.argtypes = [u32, u32, vp, ctypes.c_float, vp, i32, u32, vp]
        L.colizig_cuda_moe_check.restype = i32
        L.colizig_cuda_moe_check.argtypes = [vp]
        L.colizig_cuda_moe_forward_noalloc.restype = i32
        L.colizig_cuda_moe_forward_noalloc.argtypes = [u32, vp, i32, i32, vp, vp, vp, vp, vp]
        L.colizig_cuda_ep_unique_id.restype = i32
        L.colizig_cuda_ep_unique_id.argtypes = [vp]
        L.colizig_cuda_ep_init.restype = i32
        L.colizig_cuda_ep_init.argtypes = [i32, i32, vp]
        L.colizig_cuda_ep_shutdown.restype = i32
        L.colizig_cuda_ep_shutdown.argtypes = []
        L.colizig_cuda_ep_set_timeout.restype = i32
        L.colizig_cuda_ep_set_timeout.argtypes = [i32]
        L.colizig_cuda_ep_abort.restype = i32
        L.colizig_cuda_ep_abort.argtypes = []
        L.colizig_cuda_ep_combine_mode.restype = i32
        L.colizig_cuda_ep_combine_mode.argtypes = []
        L.colizig_cuda_moe_decode_batch.restype = i32
        L.colizig_cuda_moe_decode_batch.argtypes = [u32, i32]
        L.colizig_cuda_ep_set_combine.restype = i32
        L.colizig_cuda_ep_set_combine.argtypes = [i32]
        L.colizig_cuda_kernel_timer.restype = i32
        L.colizig_cuda_kernel_timer.argtypes = [i32]
        L.colizig_cuda_kernel_timer_read.restype = i32
        L.colizig_cuda_kernel_timer_read.argtypes = [vp, vp, i32]
        L.colizig_cuda_debug_expf.restype = i32
        L.colizig_cuda_debug_expf.argtypes = [vp, vp, ctypes.c_size_t]
        L.colizig_cuda_debug_hold_router.restype = i32
        L.colizig_cuda_debug_hold_router.argtypes = [u32]
        L.colizig_cuda_debug_error_bits.restype = i32
        L.colizig_cuda_debug_error_bits.argtypes = [ctypes.c_void_p]
        L.colizig_cuda_debug_watch_wait.restype = i32
        L.colizig_cuda_debug_watch_wait.argtypes = [WATCH_QUERY, WATCH_QUERY, WATCH_ABORT, ctypes.c_void_p, i32]
        _lib = L
        return L


def check(fn: str, rc: int) -> None:
    if rc != 0:
        raise ColizigError(fn, rc)
