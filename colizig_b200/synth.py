"""Seeded synthetic MoE layers and tokens with the benchmark's distributions.

No checkpoint or dataset is available, so every benchmark and parity case runs
on generated data with the configured shapes and value distributions:
  * expert weights: N(0, 0.5) (0.5 = standard deviation), clipped to +-448 and
    rounded to nearest-even OCP E4M3 (torch.float8_e4m3fn) — stored as bytes;
  * block scales ("weight_scale_inv", multiplied in): f32 U(1e-3, 3e-3) per
    128x128 block;
  * router: f32 N(0, 0.02) [experts, hidden];
  * shared-expert gate vector: f32 N(0, 0.02) [hidden];
  * tokens: bf16 (or f32) N(0, 1).
Config 3's skewed routing (Zipf(1.1) over experts): the router has no bias, so
the skew enters through a fixed unit vector u: router rows get beta_e * u and
tokens get gamma * u, with beta_e * gamma = -1.1 * ln(1 + rank_e) for a seeded
random rank order of the experts (see zipf_router / zipf_tokens).
Generation runs with torch on the requested device (CUDA for full-size layers),
in expert chunks so temporary f32 storage stays bounded.
"""

from __future__ import annotations

import numpy as np
import torch

from .moe import Dims


def nblk(x: int) -> int:
    return (x + 127) // 128


def _e4m3(shape, gen, device, std=0.5):
    w = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).mul_(std).clamp_(-448.0, 448.0)
    return w.to(torch.float8_e4m3fn).view(torch.uint8)


def _scales(shape, gen, device):
    return torch.rand(shape, generator=gen, device=device, dtype=torch.float32).mul_(2e-3).add_(1e-3)


def _stacked_e4m3(E, O, I, gen, device, chunk_bytes=1 << 30):
    out = torch.empty((E, O, I), dtype=torch.uint8, device=device)
    per = max(1, chunk_bytes // (O * I * 4))
    for e0 in range(0, E, per):
        e1 = min(E, e0 + per)
        out[e0:e1] = _e4m3((e1 - e0, O, I), gen, device)
    return out


def make_layer(d: Dims, seed: int = 0, device="cpu") -> dict:
    """One MoE layer's weights (reference layout, stacked over experts)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    E, H, I, SI = d.experts, d.hidden, d.inter, d.shared_inter
    w = {
        "router": torch.randn((E, H), generator=gen, device=device, dtype=torch.float32).mul_(0.02),
        "gate_w": _stacked_e4m3(E, I, H, gen, device),
        "gate_s": _scales((E, nblk(I), nblk(H)), gen, device),
        "up_w": _stacked_e4m3(E, I, H, gen, device),
        "up_s": _scales((E, nblk(I), nblk(H)), gen, device),
        "down_w": _stacked_e4m3(E, H, I, gen, device),
        "down_s": _scales((E, nblk(H), nblk(I)), gen, device),
    }
    if SI:
        w["sh_gate_w"] = _e4m3((SI, H), gen, device)
        w["sh_gate_s"] = _scales((nblk(SI), nblk(H)), gen, device)
        w["sh_up_w"] = _e4m3((SI, H), gen, device)
        w["sh_up_s"] = _scales((nblk(SI), nblk(H)), gen, device)
        w["sh_down_w"] = _e4m3((H, SI), gen, device)
        w["sh_down_s"] = _scales((nblk(H), nblk(SI)), gen, device)
        w["sh_gate"] = torch.randn((H,), generator=gen, device=device, dtype=torch.float32).mul_(0.02)
    return w


ZIPF_S = 1.1
ZIPF_GAMMA = 4.0


def _zipf_dir(H: int, device) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(12345)
    u = torch.randn((H,), generator=gen, device=device, dtype=torch.float32)
    return u / u.norm()


def zipf_router(w: dict, seed: int = 0) -> dict:
    """Skew a layer's routing: router row e += beta_e * u (in place)."""
    E, H = w["router"].shape
    dev = w["router"].device
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed) + 99)
    rank = torch.randperm(E, generator=gen).to(dev, torch.float32)
    beta = -ZIPF_S * torch.log1p(rank) / ZIPF_GAMMA
    w["router"] += beta[:, None] * _zipf_dir(H, dev)[None, :]
    return w


def zipf_tokens(T: int, H: int, seed: int, device="cpu", dtype=torch.bfloat16) -> torch.Tensor:
    """Tokens N(0, 1) + gamma * u (the routing skew's token side)."""
    x = torch.randn((T, H), generator=_gen(seed, device), device=device, dtype=torch.float32)
    return (x + ZIPF_GAMMA * _zipf_dir(H, x.device)[None, :]).to(dtype)


def _gen(seed: int, device):
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    return gen


def make_tokens(T: int, H: int, seed: int, device="cpu", dtype=torch.bfloat16) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    return torch.randn((T, H), generator=gen, device=device, dtype=torch.float32).to(dtype)


def bf16_shared(w: dict, d: Dims, seed: int = 0) -> dict:
    """Replace a layer's shared expert (in place) by a BF16 one as real Qwen4-Exp
    checkpoints hold it (the reference's NativeMatrix, moe.zig:297-338): gate/up
    [SI, H] and down [H, SI] bf16 from N(0, 0.02), no block scales."""
    SI, H = d.shared_inter, d.hidden
    dev = w["router"].device
    gen = torch.Generator(device=dev)
    gen.manual_seed(int(seed) + 777)
    for k in ("sh_gate_w", "sh_gate_s", "sh_up_w", "sh_up_s", "sh_down_w", "sh_down_s"):
        w.pop(k, None)
    for k, shp in (("sh_gate_bf16", (SI, H)), ("sh_up_bf16", (SI, H)), ("sh_down_bf16", (H, SI))):
        w[k] = torch.randn(shp, generator=gen, device=dev, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
    if "sh_gate" not in w:
        w["sh_gate"] = torch.randn((H,), generator=gen, device=dev, dtype=torch.float32).mul_(0.02)
    return w


def to_numpy_layer(w: dict) -> dict:
    """Host numpy copies (for the CPU oracle); bf16 tensors as their raw bits (uint16)."""
    out = {}
    for k, v in w.items():
        v = v.detach().cpu()
        out[k] = v.view(torch.int16).numpy().view(np.uint16) if v.dtype == torch.bfloat16 else v.numpy()
    return out


def tokens_f32(x: torch.Tensor) -> np.ndarray:
    """Exact f32 widening of bf16 tokens (what the reference computes on)."""
    return x.detach().float().cpu().numpy()


# Benchmark configurations 1, 2, 3 and 5 (config 4 is a 48-layer stack of config 2).
CONFIGS = {
    "c1": Dims(hidden=256, experts=16, topk=4, inter=128, shared_inter=0, norm_topk=True),
    "c2": Dims(hidden=2048, experts=128, topk=8, inter=768, shared_inter=0, norm_topk=True),
    "c3": Dims(hidden=2048, experts=128, topk=8, inter=768, shared_inter=0, norm_topk=True),  # + Zipf routing
    "c5": Dims(hidden=4096, experts=512, topk=10, inter=1024, shared_inter=1024, norm_topk=True),
}
