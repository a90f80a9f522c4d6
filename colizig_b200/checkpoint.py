"""Checkpoint -> resident registry: the host side of
colizig_cuda_moe_load_safetensors.

Mirrors src/qwen38/moe.zig:251-292 (loadExpert) and 306-329 (Layer.load) with
src/model/weights.zig:198-235 (name lookup): the library parses the safetensors
shards itself, maps them read-only and copies one MoE layer's router, experts
and shared expert into resident device memory in one call.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

from . import _abi, gpu
from .moe import Dims, Layer


def load_layer(layer_id: int, shards: Sequence[str], layer_index: int, dims: Dims, prefix: str | None = "model",
               ep: bool = False) -> Layer:
    """Register checkpoint layer `layer_index` (tensor names
    `<prefix>.layers.<layer_index>.mlp.*`, or without the prefix) as library layer
    `layer_id`.  `shards` are the safetensors files holding it (any order)."""
    if not gpu.available():
        gpu.init()
    paths = (ctypes.c_char_p * len(shards))(*[str(p).encode() for p in shards])
    cd = dims.c()
    rc = _abi.load().colizig_cuda_moe_load_safetensors(int(layer_id), paths, len(shards),
                                                      None if prefix is None else prefix.encode(), int(layer_index),
                                                      ctypes.byref(cd), _abi.COLIZIG_EP if ep else 0)
    _abi.check("colizig_cuda_moe_load_safetensors", rc)
    return Layer.registered(layer_id, dims, ep=ep)
