#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the reference's own code.

Runs the reference's independent NumPy implementation of the path
(``tools/reference/qwen38_ref.py``: ``e4m3_decode``, ``fp8_block_matmul``,
``Model.moe``; ``tools/reference/qwen3moe_ref.py``: ``Model.moe``) on seeded
synthetic inputs and stores inputs + outputs as ``.npz`` files.  The reference
tree is only needed to regenerate; the committed fixtures are what the tests read.

Usage:  python tests/golden/make_golden.py <reference source root> [shared_bf16]
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def e4m3_bytes(f32: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to OCP E4M3 (clipped to +-448 first), as raw bytes."""
    t = torch.from_numpy(np.clip(f32, -448.0, 448.0).astype(np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()


def nblk(x):
    return (x + 127) // 128


def layer_tensors(rng, H, E, I, SI=0):
    """C1-style distributions: E4M3 from N(0, 0.5), block scales U(1e-3, 3e-3),
    router f32 N(0, 0.02)."""
    L = {
        "router": (rng.standard_normal((E, H)) * 0.02).astype(np.float32),
        "gate_w": e4m3_bytes(rng.standard_normal((E, I, H)) * 0.5),
        "gate_s": rng.uniform(1e-3, 3e-3, (E, nblk(I), nblk(H))).astype(np.float32),
        "up_w": e4m3_bytes(rng.standard_normal((E, I, H)) * 0.5),
        "up_s": rng.uniform(1e-3, 3e-3, (E, nblk(I), nblk(H))).astype(np.float32),
        "down_w": e4m3_bytes(rng.standard_normal((E, H, I)) * 0.5),
        "down_s": rng.uniform(1e-3, 3e-3, (E, nblk(H), nblk(I))).astype(np.float32),
    }
    if SI:
        L["sh_gate_w"] = e4m3_bytes(rng.standard_normal((SI, H)) * 0.5)
        L["sh_gate_s"] = rng.uniform(1e-3, 3e-3, (nblk(SI), nblk(H))).astype(np.float32)
        L["sh_up_w"] = e4m3_bytes(rng.standard_normal((SI, H)) * 0.5)
        L["sh_up_s"] = rng.uniform(1e-3, 3e-3, (nblk(SI), nblk(H))).astype(np.float32)
        L["sh_down_w"] = e4m3_bytes(rng.standard_normal((H, SI)) * 0.5)
        L["sh_down_s"] = rng.uniform(1e-3, 3e-3, (nblk(H), nblk(SI))).astype(np.float32)
        L["sh_gate"] = (rng.standard_normal(H) * 0.02).astype(np.float32)
    return L


def dequant(ref, w, s):
    """Dense f32 weights = e4m3(w) * block scale (the reference's layout rule)."""
    wf = ref.e4m3_decode(w).astype(np.float32)
    O, I = w.shape
    return (wf * np.repeat(np.repeat(s, 128, 0), 128, 1)[:O, :I]).astype(np.float32)


def main(refroot):
    sys.path.insert(0, os.path.join(refroot, "tools", "reference"))
    import qwen38_ref as r38  # noqa: E402
    import qwen3moe_ref as r3  # noqa: E402

    # 1. every E4M3 byte (fp8.zig:355-377 covers the same set)
    allb = np.arange(256, dtype=np.uint8)
    np.save(os.path.join(HERE, "e4m3_decode_all256.npy"), r38.e4m3_decode(allb))

    # 2. block-FP8 matmul KAT shapes (fp8.zig:273-353) + a C1 projection
    rng = np.random.default_rng(0xF8)
    kat = {}
    for name, (S, I, O, allbytes) in {
        "two_blocks": (3, 200, 5, False),
        "all_finite_bytes": (1, 384, 6, True),
        "c1_gate": (2, 256, 128, False),
        "ragged": (4, 300, 131, True),
    }.items():
        x = (rng.random((S, I)) * 2 - 1).astype(np.float32)
        if allbytes:
            w = rng.integers(0, 256, (O, I), dtype=np.uint8)
            w[(w == 0x7F) | (w == 0xFF)] = 0
        else:
            w = e4m3_bytes(rng.standard_normal((O, I)) * 0.5)
        s = (0.25 + rng.random((nblk(O), nblk(I)))).astype(np.float32)
        wdec = r38.e4m3_decode(w).astype(np.float32)
        y = np.stack([r38.fp8_block_matmul(x[i], wdec, s) for i in range(S)])
        kat.update({f"{name}_x": x, f"{name}_w": w, f"{name}_s": s, f"{name}_y": y})
    np.savez_compressed(os.path.join(HERE, "fp8_matmul_kat.npz"), **kat)

    # 3. C1 tiny MoE layer (H256 E16 I128 K4, norm_topk) through qwen3moe_ref.Model.moe
    H, E, I, K = 256, 16, 128, 4
    rng = np.random.default_rng(0)
    L = layer_tensors(rng, H, E, I)
    x = rng.standard_normal((5, H)).astype(np.float32)
    m = object.__new__(r3.Model)
    m.H, m.E, m.topk, m.norm_topk = H, E, K, True
    T = {"layers.0.mlp.gate.weight": L["router"]}
    for e in range(E):
        for proj, wn, sn in (("gate_proj", "gate_w", "gate_s"), ("up_proj", "up_w", "up_s"),
                             ("down_proj", "down_w", "down_s")):
            T[f"layers.0.mlp.experts.{e}.{proj}.weight"] = r38.e4m3_decode(L[wn][e]).astype(np.float32)
            T[f"layers.0.mlp.experts.{e}.{proj}.weight_scale_inv"] = L[sn][e]
    m.T = T
    outs, idxs = [], []
    for t in range(x.shape[0]):
        n = x[t]
        logits = np.asarray(L["router"], dtype=np.float32) @ n
        idxs.append(np.argsort(-logits)[:K].astype(np.uint32))
        outs.append(m.moe(0, n))
    np.savez_compressed(os.path.join(HERE, "moe_c1.npz"), x=x, out=np.stack(outs), idx=np.stack(idxs),
                        H=H, E=E, I=I, K=K, **L)

    # 4. tiny layer with an always-on shared expert through qwen38_ref.Model.moe
    H, E, I, K, SI = 256, 16, 128, 4, 128
    rng = np.random.default_rng(1)
    L = layer_tensors(rng, H, E, I, SI)
    x = rng.standard_normal((3, H)).astype(np.float32)
    m = object.__new__(r38.Model)
    m.H, m.E, m.topk, m.norm_topk, m.prefix = H, E, K, True, "model"
    T = {
        "layers.0.mlp.gate.weight": L["router"],
        "layers.0.mlp.shared_expert.gate_proj.weight": dequant(r38, L["sh_gate_w"], L["sh_gate_s"]),
        "layers.0.mlp.shared_expert.up_proj.weight": dequant(r38, L["sh_up_w"], L["sh_up_s"]),
        "layers.0.mlp.shared_expert.down_proj.weight": dequant(r38, L["sh_down_w"], L["sh_down_s"]),
        "layers.0.mlp.shared_expert_gate.weight": L["sh_gate"],
    }
    for e in range(E):
        for proj, wn, sn in (("gate_proj", "gate_w", "gate_s"), ("up_proj", "up_w", "up_s"),
                             ("down_proj", "down_w", "down_s")):
            T[f"layers.0.mlp.experts.{e}.{proj}.weight"] = r38.e4m3_decode(L[wn][e]).astype(np.float32)
            T[f"layers.0.mlp.experts.{e}.{proj}.weight_scale_inv"] = L[sn][e]
    m.T = T
    outs, idxs = [], []
    for t in range(x.shape[0]):
        y, idx = m.moe(0, x[t])
        outs.append(np.asarray(y, np.float32))
        idxs.append(np.asarray(idx, np.uint32))
    np.savez_compressed(os.path.join(HERE, "moe_shared_tiny.npz"), x=x, out=np.stack(outs),
                        idx=np.stack(idxs), H=H, E=E, I=I, K=K, SI=SI, **L)
    shared_bf16(r38)
    print("golden fixtures written to", HERE)


def bf16_bits(f32: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, as raw 16-bit patterns."""
    t = torch.from_numpy(np.ascontiguousarray(f32, np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def shared_bf16(r38):
    """5. tiny layer whose shared expert is BF16, as the reference loads real
    Qwen4-Exp checkpoints (NativeMatrix, moe.zig:297-338): the numpy model gets
    the bf16 weights widened to f32 exactly, as its load_safetensors does."""
    H, E, I, K, SI = 256, 16, 128, 4, 256
    rng = np.random.default_rng(5)
    L = layer_tensors(rng, H, E, I)
    sh = {"sh_gate_bf16": bf16_bits(rng.standard_normal((SI, H)) * 0.05),
          "sh_up_bf16": bf16_bits(rng.standard_normal((SI, H)) * 0.05),
          "sh_down_bf16": bf16_bits(rng.standard_normal((H, SI)) * 0.05),
          "sh_gate": (rng.standard_normal(H) * 0.02).astype(np.float32)}
    widen = lambda b: (b.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    x = rng.standard_normal((3, H)).astype(np.float32)
    m = object.__new__(r38.Model)
    m.H, m.E, m.topk, m.norm_topk, m.prefix = H, E, K, True, "model"
    T = {
        "layers.0.mlp.gate.weight": L["router"],
        "layers.0.mlp.shared_expert.gate_proj.weight": widen(sh["sh_gate_bf16"]),
        "layers.0.mlp.shared_expert.up_proj.weight": widen(sh["sh_up_bf16"]),
        "layers.0.mlp.shared_expert.down_proj.weight": widen(sh["sh_down_bf16"]),
        "layers.0.mlp.shared_expert_gate.weight": sh["sh_gate"],
    }
    for e in range(E):
        for proj, wn, sn in (("gate_proj", "gate_w", "gate_s"), ("up_proj", "up_w", "up_s"),
                             ("down_proj", "down_w", "down_s")):
            T[f"layers.0.mlp.experts.{e}.{proj}.weight"] = r38.e4m3_decode(L[wn][e]).astype(np.float32)
            T[f"layers.0.mlp.experts.{e}.{proj}.weight_scale_inv"] = L[sn][e]
    m.T = T
    outs, idxs = [], []
    for t in range(x.shape[0]):
        y, idx = m.moe(0, x[t])
        outs.append(np.asarray(y, np.float32))
        idxs.append(np.asarray(idx, np.uint32))
    np.savez_compressed(os.path.join(HERE, "moe_shared_bf16_tiny.npz"), x=x, out=np.stack(outs),
                        idx=np.stack(idxs), H=H, E=E, I=I, K=K, SI=SI, **L, **sh)


if __name__ == "__main__":
    # make_golden.py <reference root> [shared_bf16]: every fixture, or only the named one
    if len(sys.argv) not in (2, 3):
        sys.exit(__doc__)
    if len(sys.argv) == 3:
        sys.path.insert(0, os.path.join(sys.argv[1], "tools", "reference"))
        import qwen38_ref  # noqa: E402

        {"shared_bf16": shared_bf16}[sys.argv[2]](qwen38_ref)
    else:
        main(sys.argv[1])
