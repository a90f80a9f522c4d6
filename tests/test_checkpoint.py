"""The checkpoint loader's file handling, without a device: the shards are
parsed and every tensor checked before the library touches the GPU, so a
well-formed checkpoint reaches registration (which then reports -1, not
initialised, on this CPU-only host) and every defect gives -10 (unreadable,
malformed, tensor missing) or -8 (dtype / shape not matching the dims).  The
files follow the reference's safetensors layout (manifest.zig, weights.zig) and
fixture recipe (tools/gen_tiny_fixture.zig:355-416)."""

import ctypes
import os
import struct

import numpy as np
import pytest
import torch

from colizig_b200 import _abi, moe, synth
from tests.safetensors_util import layer_tensors, write_safetensors

D = synth.CONFIGS["c1"]


@pytest.fixture(scope="module")
def tensors():
    w = synth.to_numpy_layer(synth.make_layer(D, seed=3, device="cpu"))
    return layer_tensors(w, 7, prefix="model")


def _load(paths, prefix="model", layer_index=7, dims=D):
    L = _abi.load()
    arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
    cd = dims.c()
    return L.colizig_cuda_moe_load_safetensors(1, arr, len(paths), None if prefix is None else prefix.encode(),
                                               layer_index, ctypes.byref(cd), 0)


def _not_initialised_here():
    return not torch.cuda.is_available()


@pytest.mark.skipif(not _not_initialised_here(), reason="needs a host without a device")
def test_well_formed_checkpoint_reaches_registration(tmp_path, tensors):
    p = tmp_path / "model.safetensors"
    write_safetensors(p, tensors, metadata={"format": "pt"})
    assert _load([p]) == -1  # parsed and checked; registration refuses: no device here
    # the same tensors split over two shards, looked up under the bare names too
    names = list(tensors)
    a = {k: tensors[k] for k in names[::2]}
    b = {k: tensors[k] for k in names[1::2]}
    write_safetensors(tmp_path / "a.safetensors", a)
    write_safetensors(tmp_path / "b.safetensors", b)
    assert _load([tmp_path / "b.safetensors", tmp_path / "a.safetensors"]) == -1
    bare = {k[len("model."):]: v for k, v in tensors.items()}
    write_safetensors(tmp_path / "bare.safetensors", bare)
    assert _load([tmp_path / "bare.safetensors"], prefix="model") == -1
    assert _load([tmp_path / "bare.safetensors"], prefix=None) == -1


def test_missing_or_malformed_files_are_io_errors(tmp_path, tensors):
    assert _load([tmp_path / "absent.safetensors"]) == -10
    p = tmp_path / "model.safetensors"
    write_safetensors(p, tensors)
    raw = p.read_bytes()
    (tmp_path / "truncated.safetensors").write_bytes(raw[: len(raw) // 2])
    assert _load([tmp_path / "truncated.safetensors"]) == -10
    bad = bytearray(raw)
    bad[8:12] = b"}}}]"
    (tmp_path / "garbage.safetensors").write_bytes(bytes(bad))
    assert _load([tmp_path / "garbage.safetensors"]) == -10
    (tmp_path / "huge_header.safetensors").write_bytes(struct.pack("<Q", 1 << 62) + raw[8:])
    assert _load([tmp_path / "huge_header.safetensors"]) == -10
    # a tensor whose bytes do not match its shape
    t = dict(tensors)
    k = "model.layers.7.mlp.experts.3.up_proj.weight"
    t[k] = ("F8_E4M3", tensors[k][1][:, :-16])
    write_safetensors(tmp_path / "short.safetensors", t)
    assert _load([tmp_path / "short.safetensors"]) == -8
    # a missing expert scale
    t = {k: v for k, v in tensors.items() if k != "model.layers.7.mlp.experts.5.down_proj.weight_scale_inv"}
    write_safetensors(tmp_path / "missing.safetensors", t)
    assert _load([tmp_path / "missing.safetensors"]) == -10
    # another layer index is simply not there
    write_safetensors(p, tensors)
    assert _load([p], layer_index=8) == -10


def test_dtype_and_shape_mismatches_are_shape_errors(tmp_path, tensors):
    t = dict(tensors)
    k = "model.layers.7.mlp.experts.0.gate_proj.weight"
    t[k] = ("F32", tensors[k][1].astype(np.float32))
    write_safetensors(tmp_path / "f32_expert.safetensors", t)
    assert _load([tmp_path / "f32_expert.safetensors"]) == -8
    t = dict(tensors)
    t["model.layers.7.mlp.gate.weight"] = ("F32", np.zeros((D.experts, D.hidden + 16), np.float32))
    write_safetensors(tmp_path / "router_shape.safetensors", t)
    assert _load([tmp_path / "router_shape.safetensors"]) == -8
    p = tmp_path / "model.safetensors"
    write_safetensors(p, tensors)
    wrong = moe.Dims(D.hidden, D.experts, D.topk, D.inter * 2, 0, True)
    assert _load([p], dims=wrong) == -8


def test_bad_arguments(tmp_path):
    L = _abi.load()
    cd = D.c()
    assert L.colizig_cuda_moe_load_safetensors(1, None, 1, None, 0, ctypes.byref(cd), 0) == -1
    arr = (ctypes.c_char_p * 1)(b"x")
    assert L.colizig_cuda_moe_load_safetensors(1, arr, 0, None, 0, ctypes.byref(cd), 0) == -1
    assert L.colizig_cuda_moe_load_safetensors(1, arr, 1, None, 0, None, 0) == -1
    assert L.colizig_cuda_moe_load_safetensors(1, arr, 1, None, 0, ctypes.byref(cd), _abi.COLIZIG_PTR_DEVICE) == -1
