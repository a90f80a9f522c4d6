"""Host-side mirror of src/qwen38/moe.zig for the B200 backend.

``Dims`` is moe.zig:23-46.  ``Layer`` replaces moe.zig's ``Layer`` + the
``ExpertCache`` LRU (moe.zig:141-249, 297-338): the router and every expert's
block-FP8 weights are registered once into resident device memory.
``forward`` is moe.zig:409-426 for T tokens; ``stack_forward`` is the per-layer
caller loop of src/qwen3moe/model.zig:227-232 with attention as identity.

Arrays may be numpy (host; the call is synchronous) or torch CUDA tensors
(device; the call is stream-ordered on the current torch stream).  Weights are
stacked over experts in the reference layout:
  router [E, H] f32; gate_w / up_w [E, I, H] u8 (E4M3 bytes); gate_s / up_s
  [E, nblk(I), nblk(H)] f32; down_w [E, H, I] u8; down_s [E, nblk(H), nblk(I)] f32.
An optional always-on shared expert (``shared`` = dict of sh_gate_w, sh_gate_s,
sh_up_w, sh_up_s, sh_down_w, sh_down_s) is scaled by sigmoid(x . sh_gate).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _abi, gpu

try:
    import torch
except ImportError:  # pragma: no cover - torch is part of the image
    torch = None


@dataclass(frozen=True)
class Dims:
    hidden: int
    experts: int
    topk: int
    inter: int
    shared_inter: int = 0
    norm_topk: bool = True

    def has_shared(self) -> bool:
        return self.shared_inter != 0

    @staticmethod
    def of(cfg: dict) -> "Dims":
        """moe.zig:36-45 from a config mapping (config.zig field names)."""
        return Dims(cfg["hidden"], cfg["experts"], cfg["topk"], cfg["inter"], cfg.get("shared_inter", 0),
                    bool(cfg.get("norm_topk", True)))

    def c(self) -> _abi.MoeDims:
        return _abi.MoeDims(self.hidden, self.experts, self.topk, self.inter, self.shared_inter,
                            int(self.norm_topk))


def _is_cuda(a) -> bool:
    return torch is not None and isinstance(a, torch.Tensor) and a.is_cuda


def _ptr(a) -> int:
    if torch is not None and isinstance(a, torch.Tensor):
        if not a.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return a.data_ptr()
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("arrays must be C-contiguous")
    return a.ctypes.data


def _stream_handle(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


class Layer:
    """A registered MoE layer (resident on the device)."""

    def __init__(self, layer_id: int, dims: Dims, router, gate_w, gate_s, up_w, up_s, down_w, down_s,
                 shared: Optional[dict] = None, shared_gate=None, ep: bool = False):
        """ep=True: hold only this rank's experts (after ep.init); every forward then
        sums the ranks' outputs (inside the decode kernel, or one NCCL all-reduce)."""
        if not gpu.available():
            gpu.init()
        self.id = int(layer_id)
        self.dims = dims
        E, H, I = dims.experts, dims.hidden, dims.inter
        arrays = [router, gate_w, gate_s, up_w, up_s, down_w, down_s]
        device = _is_cuda(router)
        if any(_is_cuda(a) != device for a in arrays):
            raise ValueError("mix of host and device arrays")
        if tuple(gate_w.shape) != (E, I, H) or tuple(down_w.shape) != (E, H, I) or tuple(router.shape) != (E, H):
            raise ValueError("weight shapes do not match dims")
        keep = [a for a in arrays]
        experts = (_abi.MoeExpert * E)()
        gw, gs, uw, us, dw, ds = (_ptr(a) for a in (gate_w, gate_s, up_w, up_s, down_w, down_s))
        nbw = I * H
        nbs = ((I + 127) // 128) * ((H + 127) // 128) * 4
        for e in range(E):
            experts[e] = _abi.MoeExpert(gw + e * nbw, gs + e * nbs, uw + e * nbw, us + e * nbs, dw + e * nbw,
                                        ds + e * nbs)
        sh_ptr = None
        sg_ptr = None
        sh_bf16 = False
        if dims.has_shared():
            if shared is None or shared_gate is None:
                raise ValueError("dims.shared_inter > 0 needs shared weights and shared_gate")
            SI = dims.shared_inter
            if "sh_gate_bf16" in shared:
                # the reference's BF16 NativeMatrix shared expert (moe.zig:297-338): raw bf16
                # [SI, H] gate / up and [H, SI] down, no block scales
                sh_bf16 = True
                for k, shp in (("sh_gate_bf16", (SI, H)), ("sh_up_bf16", (SI, H)), ("sh_down_bf16", (H, SI))):
                    a = shared[k]
                    if tuple(a.shape) != shp or _dtype_name(a) not in ("bf16", "u16", "i16"):
                        raise ValueError(f"{k} must be bf16 {shp}, got {_dtype_name(a)} {tuple(a.shape)}")
                    if _is_cuda(a) != device:
                        raise ValueError("mix of host and device arrays")
                sh = _abi.MoeExpert(_ptr(shared["sh_gate_bf16"]), 0, _ptr(shared["sh_up_bf16"]), 0,
                                    _ptr(shared["sh_down_bf16"]), 0)
            else:
                sh = _abi.MoeExpert(_ptr(shared["sh_gate_w"]), _ptr(shared["sh_gate_s"]), _ptr(shared["sh_up_w"]),
                                    _ptr(shared["sh_up_s"]), _ptr(shared["sh_down_w"]), _ptr(shared["sh_down_s"]))
            keep += list(shared.values()) + [shared_gate]
            sh_ptr = ctypes.byref(sh)
            sg_ptr = _ptr(shared_gate)
        cd = dims.c()
        flags = ((_abi.COLIZIG_PTR_DEVICE if device else 0) | (_abi.COLIZIG_EP if ep else 0) |
                 (_abi.COLIZIG_SHARED_BF16 if sh_bf16 else 0))
        self.ep = bool(ep)
        if device:
            torch.cuda.synchronize()
        rc = _abi.load().colizig_cuda_moe_register_layer(self.id, ctypes.byref(cd), _ptr(router), experts, sh_ptr,
                                                         sg_ptr, flags)
        del keep
        _abi.check("colizig_cuda_moe_register_layer", rc)

    @classmethod
    def registered(cls, layer_id: int, dims: Dims, ep: bool = False) -> "Layer":
        """A handle to a layer the library already holds (registered by another
        entry point, e.g. the checkpoint loader)."""
        self = cls.__new__(cls)
        self.id = int(layer_id)
        self.dims = dims
        self.ep = bool(ep)
        return self

    @staticmethod
    def from_weights(layer_id: int, dims: Dims, w: dict, ep: bool = False) -> "Layer":
        shared = None
        if dims.has_shared():
            keys = (("sh_gate_bf16", "sh_up_bf16", "sh_down_bf16") if "sh_gate_bf16" in w else
                    ("sh_gate_w", "sh_gate_s", "sh_up_w", "sh_up_s", "sh_down_w", "sh_down_s"))
            shared = {k: w[k] for k in keys}
        return Layer(layer_id, dims, w["router"], w["gate_w"], w["gate_s"], w["up_w"], w["up_s"], w["down_w"],
                     w["down_s"], shared, w.get("sh_gate"), ep=ep)

    def unregister(self) -> None:
        _abi.check("colizig_cuda_moe_unregister_layer", _abi.load().colizig_cuda_moe_unregister_layer(self.id))

    def forward(self, x, out=None, topk_idx=None, topk_gates=None, stream=None):
        return forward(self, x, out, topk_idx, topk_gates, stream)


def _shape_of(a):
    return tuple(int(s) for s in a.shape)


def _dtype_name(a) -> str:
    if torch is not None and isinstance(a, torch.Tensor):
        return {torch.float32: "f32", torch.int32: "i32", torch.uint32: "u32", torch.bfloat16: "bf16",
                torch.int16: "i16"}.get(a.dtype, str(a.dtype))
    return {np.dtype(np.float32): "f32", np.dtype(np.int32): "i32", np.dtype(np.uint32): "u32",
            np.dtype(np.int16): "i16", np.dtype(np.uint16): "u16"}.get(np.dtype(a.dtype), str(a.dtype))


def check_io(dims: Dims, x, out=None, topk_idx=None, topk_gates=None, status=None, device=None) -> int:
    """Validates the buffers of one forward call before anything reaches the
    library, which only sees raw pointers and would read and write past a
    mis-shaped buffer.  x must be [T, hidden] (f32 or bf16; bf16 host arrays as
    16-bit integers); out f32 [T, hidden]; topk_idx 32-bit integers [T, topk];
    topk_gates f32 [T, topk]; status (device calls only) a 32-bit integer tensor
    of at least one element.  With `device` given, every tensor must live on
    it.  Returns T; raises ValueError otherwise."""
    if x is None or len(getattr(x, "shape", ())) != 2:
        raise ValueError(f"x must be 2-D [T, {dims.hidden}], got shape {None if x is None else _shape_of(x)}")
    T, H = _shape_of(x)
    if H != dims.hidden:
        raise ValueError(f"x has {H} columns, the layer's hidden size is {dims.hidden}")
    if _dtype_name(x) not in ("f32", "bf16", "i16", "u16"):
        raise ValueError(f"x must be f32 or bf16, got {_dtype_name(x)}")
    want = (("out", out, ("f32",), (T, dims.hidden)), ("topk_idx", topk_idx, ("i32", "u32"), (T, dims.topk)),
            ("topk_gates", topk_gates, ("f32",), (T, dims.topk)))
    for name, a, dts, shape in want:
        if a is None:
            continue
        if _dtype_name(a) not in dts:
            raise ValueError(f"{name} must be {'/'.join(dts)}, got {_dtype_name(a)}")
        if _shape_of(a) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {_shape_of(a)}")
    if status is not None:
        if _dtype_name(status) not in ("i32", "u32") or int(np.prod(_shape_of(status))) < 1:
            raise ValueError("status must be a 32-bit integer tensor of at least one element")
    if device is not None:
        for name, a in (("x", x), ("out", out), ("topk_idx", topk_idx), ("topk_gates", topk_gates),
                        ("status", status)):
            if a is not None and (not isinstance(a, torch.Tensor) or a.device != device):
                raise ValueError(f"{name} must be a tensor on {device}")
    return T


def forward(layer: Layer, x, out=None, topk_idx=None, topk_gates=None, stream=None, sharded: bool = False):
    """moe.zig:409-426: out[T, H] = MoE(x[T, H]).  Returns (out, topk_idx, topk_gates);
    the top-k arrays are allocated when not given.  sharded=True (a layer registered
    with ep=True): x holds this rank's own tokens and the ranks exchange rows with
    NCCL send/recv (expert-parallel prefill); every rank must make the call."""
    d = layer.dims
    L = _abi.load()
    sh = _abi.COLIZIG_EP_SHARDED if sharded else 0
    if _is_cuda(x):
        if x.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("x must be f32 or bf16")
        T = check_io(d, x, out, topk_idx, topk_gates, device=x.device)
        dt = _abi.COLIZIG_X_BF16 if x.dtype == torch.bfloat16 else _abi.COLIZIG_X_F32
        if out is None:
            out = torch.empty((T, d.hidden), dtype=torch.float32, device=x.device)
        if topk_idx is None:
            topk_idx = torch.empty((T, d.topk), dtype=torch.int32, device=x.device)
        if topk_gates is None:
            topk_gates = torch.empty((T, d.topk), dtype=torch.float32, device=x.device)
        rc = L.colizig_cuda_moe_forward(layer.id, _ptr(x), dt, T, _ptr(out), _ptr(topk_idx), _ptr(topk_gates),
                                        _abi.COLIZIG_PTR_DEVICE | sh, _stream_handle(stream))
        _abi.check("colizig_cuda_moe_forward", rc)
        return out, topk_idx, topk_gates
    # host path
    if torch is not None and isinstance(x, torch.Tensor):
        if x.dtype == torch.bfloat16:
            xa = x.contiguous().view(torch.int16).numpy()
            dt = _abi.COLIZIG_X_BF16
        else:
            xa = x.contiguous().float().numpy()
            dt = _abi.COLIZIG_X_F32
    else:
        xa = np.ascontiguousarray(x, np.float32)
        dt = _abi.COLIZIG_X_F32
    if xa.ndim == 1:
        xa = xa[None, :]  # one token
    T = check_io(d, xa, out, topk_idx, topk_gates)
    if out is None:
        out = np.empty((T, d.hidden), np.float32)
    if topk_idx is None:
        topk_idx = np.empty((T, d.topk), np.uint32)
    if topk_gates is None:
        topk_gates = np.empty((T, d.topk), np.float32)
    for name, a in (("out", out), ("topk_idx", topk_idx), ("topk_gates", topk_gates)):
        if not isinstance(a, np.ndarray):
            raise ValueError(f"{name} must be a numpy array for host tokens")
    rc = L.colizig_cuda_moe_forward(layer.id, _ptr(xa), dt, T, _ptr(out), _ptr(topk_idx), _ptr(topk_gates), sh,
                                    None)
    _abi.check("colizig_cuda_moe_forward", rc)
    return out, topk_idx, topk_gates


def forward_noalloc(layer: Layer, x, out, topk_idx=None, topk_gates=None, status=None, stream=None):
    """``forward`` for device tensors through colizig_cuda_moe_forward_noalloc:
    the library allocates nothing during the call (its scratch is a static
    device array), and neither does this wrapper, so every output tensor is
    the caller's.  ``status`` (optional int32 CUDA tensor of one element)
    receives the call's device error word (0 = ok), which is then cleared;
    without a status the word is kept for the next call that passes one.  The
    first call on a device does set-up; calls that overlap in time race on the
    shared scratch."""
    if not (_is_cuda(x) and _is_cuda(out)):
        raise ValueError("forward_noalloc takes CUDA tensors only")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("x must be f32 or bf16")
    T = check_io(layer.dims, x, out, topk_idx, topk_gates, status, device=x.device)
    dt = _abi.COLIZIG_X_BF16 if x.dtype == torch.bfloat16 else _abi.COLIZIG_X_F32
    rc = _abi.load().colizig_cuda_moe_forward_noalloc(
        layer.id, _ptr(x), dt, T, _ptr(out), None if topk_idx is None else _ptr(topk_idx),
        None if topk_gates is None else _ptr(topk_gates), None if status is None else _ptr(status),
        _stream_handle(stream))
    _abi.check("colizig_cuda_moe_forward_noalloc", rc)
    return out


def stack_forward(first_layer: int, n_layers: int, h, norm_w=None, eps: float = 1e-6, stream=None,
                  sharded: bool = False):
    """src/qwen3moe/model.zig:227-232 per layer (attention = identity):
    n = rms(h, norm_w[l]); h += moe_l(n).  Updates h ([T, H] f32) in place.
    sharded=True (layers registered with ep=True): h holds this rank's own tokens and
    every layer exchanges rows with the other ranks, as forward(..., sharded=True)."""
    L = _abi.load()
    sh = _abi.COLIZIG_EP_SHARDED if sharded else 0
    if _is_cuda(h):
        rc = L.colizig_cuda_moe_stack_forward(first_layer, n_layers, None if norm_w is None else _ptr(norm_w),
                                              float(eps), _ptr(h), h.shape[0], _abi.COLIZIG_PTR_DEVICE | sh,
                                              _stream_handle(stream))
    else:
        if not (h.dtype == np.float32 and h.flags["C_CONTIGUOUS"]):
            raise ValueError("h must be a C-contiguous f32 array")
        nwa = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
        nw = None if nwa is None else _ptr(nwa)
        rc = L.colizig_cuda_moe_stack_forward(first_layer, n_layers, nw, float(eps), _ptr(h), h.shape[0], sh, None)
    _abi.check("colizig_cuda_moe_stack_forward", rc)
    return h


def check(stream=None) -> None:
    """Raise if a device-side wait of an earlier asynchronous call gave up.  The
    error word is read in order on `stream` (default: torch's current stream, the
    one forward() launches on), so it sees every call issued there before."""
    h = _stream_handle(stream) if torch is not None else None
    _abi.check("colizig_cuda_moe_check", _abi.load().colizig_cuda_moe_check(h))


TIMER_DECODE, TIMER_PREFILL_GATE_UP, TIMER_PREFILL_DOWN, TIMER_MATMUL = 1, 2, 3, 4


def kernel_timer(capacity: int) -> None:
    """Arm (capacity > 0 launch pairs) or disarm (0) the library's kernel timer:
    CUDA event pairs around every decode kernel launch and around the two grouped
    GEMM launches of each prefill forward, captured CUDA graphs included."""
    _abi.check("colizig_cuda_kernel_timer", _abi.load().colizig_cuda_kernel_timer(int(capacity)))


def kernel_timer_read(max_n: int = 1 << 16) -> list:
    """[(kind, ms)] of the launch pairs recorded since the timer was armed (waits
    for them).  kind is TIMER_DECODE, TIMER_PREFILL_GATE_UP, TIMER_PREFILL_DOWN or
    TIMER_MATMUL (a colizig_cuda_matmul_fp8 kernel)."""
    kinds = (ctypes.c_int * max_n)()
    ms = (ctypes.c_float * max_n)()
    n = _abi.load().colizig_cuda_kernel_timer_read(ctypes.addressof(kinds), ctypes.addressof(ms), max_n)
    if n < 0:
        _abi.check("colizig_cuda_kernel_timer_read", n)
    return [(kinds[i], ms[i]) for i in range(n)]
