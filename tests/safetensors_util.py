"""Writes safetensors files for the checkpoint-loader tests, following the
reference's fixture recipe (tools/gen_tiny_fixture.zig:355-416: an 8-byte
little-endian header length, a JSON header of {name: {dtype, shape,
data_offsets}}, then the tensor bytes; E4M3 weights as bytes, positive f32
block scales)."""

import json
import struct

import numpy as np

NB = lambda x: (x + 127) // 128  # noqa: E731


def write_safetensors(path, tensors, metadata=None):
    """tensors: {name: (dtype, ndarray)} with dtype in F8_E4M3 / BF16 / F16 / F32
    (F8_E4M3 and BF16 arrays given as uint8 / uint16 raw values)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def bf16_bits(x):
    """f32 -> bf16 raw bits, round to nearest even (matmul.zig f32ToBf16)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def layer_tensors(w, l, prefix="model", router_bf16=False, scales_bf16=False):
    """The safetensors tensors of one MoE layer held in `w` (numpy arrays in the
    library's stacked layout, as synth.make_layer / to_numpy_layer give)."""
    t = {}
    pre = f"{prefix}.layers.{l}.mlp." if prefix else f"layers.{l}.mlp."
    r = w["router"].astype(np.float32)
    t[pre + "gate.weight"] = ("BF16", bf16_bits(r)) if router_bf16 else ("F32", r)

    def sc(a):
        return ("BF16", bf16_bits(a)) if scales_bf16 else ("F32", a.astype(np.float32))

    for e in range(w["gate_w"].shape[0]):
        for proj, wk, sk in (("gate_proj", "gate_w", "gate_s"), ("up_proj", "up_w", "up_s"),
                             ("down_proj", "down_w", "down_s")):
            t[f"{pre}experts.{e}.{proj}.weight"] = ("F8_E4M3", w[wk][e])
            t[f"{pre}experts.{e}.{proj}.weight_scale_inv"] = sc(w[sk][e])
    if "sh_gate_w" in w:
        for proj, wk, sk in (("gate_proj", "sh_gate_w", "sh_gate_s"), ("up_proj", "sh_up_w", "sh_up_s"),
                             ("down_proj", "sh_down_w", "sh_down_s")):
            t[f"{pre}shared_expert.{proj}.weight"] = ("F8_E4M3", w[wk])
            t[f"{pre}shared_expert.{proj}.weight_scale_inv"] = sc(w[sk])
        t[pre + "shared_expert_gate.weight"] = ("F32", w["sh_gate"].astype(np.float32)[None, :])
    elif "sh_gate_bf16" in w:  # the reference's BF16 shared expert: bf16 weights, no scales
        for proj, wk in (("gate_proj", "sh_gate_bf16"), ("up_proj", "sh_up_bf16"), ("down_proj", "sh_down_bf16")):
            t[f"{pre}shared_expert.{proj}.weight"] = ("BF16", np.ascontiguousarray(w[wk], np.uint16))
        t[pre + "shared_expert_gate.weight"] = ("F32", w["sh_gate"].astype(np.float32)[None, :])
    return t
