"""The FP8 attention projections of the Qwen3 decoder layer through the keyed
per-matrix call (src/qwen3moe/attn.zig:46-78: q/k/v/o are Fp8Matrix weights
keyed by attnKey and computed by matmulFp8Keyed, src/ops/fp8.zig:165-188), at
Qwen3-30B-A3B's shapes (hidden 2048, 32 query heads and 4 key/value heads of
128): q [4096, 2048], k and v [512, 2048], o [2048, 4096].  Against the CPU
oracle's block-FP8 matmul (within 1e-5 of ||y||_inf, the legacy call's own
tolerance), for one token and small batches, with the weights resident under
their keys (hits, no upload after the first call of each key)."""

import numpy as np
import pytest

import colizig_b200 as cz
import oracle
from tests.util import assert_close

pytestmark = pytest.mark.gpu

H, QH, KVH, HD = 2048, 32, 4, 128
SHAPES = {0: (QH * HD, H), 1: (KVH * HD, H), 2: (KVH * HD, H), 3: (H, QH * HD)}  # role -> (O, I)


def _proj(rng, O, I):
    w = rng.integers(0, 256, (O, I), dtype=np.uint8)
    w[(w == 0x7F) | (w == 0xFF)] = 0x00  # E4M3 NaN codes never occur in checkpoints
    s = rng.uniform(1e-3, 3e-3, ((O + 127) // 128, (I + 127) // 128)).astype(np.float32)
    return w, s


def test_attention_projections_keyed_match_oracle():
    rng = np.random.default_rng(31)
    layers = (0, 47)
    W = {(l, r): _proj(rng, *SHAPES[r]) for l in layers for r in range(4)}
    keys = {(l, r): cz.fp8.attn_key(l, r) for l in layers for r in range(4)}
    assert len(set(keys.values())) == len(keys)
    # attnKey sits in the expert key space (slot 1020 + role, role 0) without
    # touching the 128 routed experts of the same layer
    assert keys[(0, 0)] == cz.fp8.expert_key(0, 1020, 0) and keys[(0, 3)] - keys[(0, 0)] == 12
    cz.gpu.init()  # the budget of an uninitialised library is ignored (colizig_cuda.cu:195-202)
    cz.gpu.set_vram_budget(1 << 31)
    try:
        h0, m0, up0, _ = cz.gpu.stats()
        for S in (1, 5, 64):
            for l in layers:
                x = rng.standard_normal((S, H)).astype(np.float32)
                q = cz.fp8.matmul_fp8_keyed(x, *W[(l, 0)], key=keys[(l, 0)])
                k = cz.fp8.matmul_fp8_keyed(x, *W[(l, 1)], key=keys[(l, 1)])
                v = cz.fp8.matmul_fp8_keyed(x, *W[(l, 2)], key=keys[(l, 2)])
                assert_close(q, oracle.matmul_fp8(x, *W[(l, 0)]), 1e-5, f"q S={S}")
                assert_close(k, oracle.matmul_fp8(x, *W[(l, 1)]), 1e-5, f"k S={S}")
                assert_close(v, oracle.matmul_fp8(x, *W[(l, 2)]), 1e-5, f"v S={S}")
                a = rng.standard_normal((S, QH * HD)).astype(np.float32)  # the attention output
                o = cz.fp8.matmul_fp8_keyed(a, *W[(l, 3)], key=keys[(l, 3)])
                assert_close(o, oracle.matmul_fp8(a, *W[(l, 3)]), 1e-5, f"o S={S}")
        h1, m1, up1, res = cz.gpu.stats()
        assert m1 - m0 == len(keys)  # one upload per key ...
        assert h1 - h0 == 3 * len(keys) - len(keys)  # ... then hits
        assert res >= len(keys)
        wbytes = sum(w.nbytes + s.nbytes for w, s in W.values())
        assert (up1 - up0) <= (wbytes >> 20) + len(keys)  # MiB uploaded: the weights once
    finally:
        cz.gpu.set_vram_budget(0)


def test_decode_call_repeats_bitwise():
    """The decode-sized call (staged through page-locked buffers) repeats its result."""
    rng = np.random.default_rng(32)
    w, s = _proj(rng, *SHAPES[0])
    x = rng.standard_normal((1, H)).astype(np.float32)
    cz.gpu.init()
    cz.gpu.set_vram_budget(1 << 30)
    try:
        ys = [cz.fp8.matmul_fp8_keyed(x, w, s, key=cz.fp8.attn_key(3, 0)) for _ in range(4)]
        assert all(np.array_equal(ys[0], y) for y in ys[1:])
        assert_close(ys[0], oracle.matmul_fp8(x, w, s), 1e-5)
    finally:
        cz.gpu.set_vram_budget(0)


def test_device_pointer_call_matches_host_call():
    """colizig_cuda_matmul_fp8_device (device pointers, stream-ordered) gives the
    host-pointer call's bits for the same weights and tokens."""
    import torch

    from colizig_b200 import _abi

    rng = np.random.default_rng(33)
    for S in (1, 7):
        for O, I in SHAPES.values():
            w, s = _proj(rng, O, I)
            x = rng.standard_normal((S, I)).astype(np.float32)
            yh = cz.fp8.matmul_fp8_keyed(x, w, s, key=0)
            wd, sd, xd = (torch.from_numpy(a).cuda() for a in (w, s, x))
            yd = torch.empty((S, O), dtype=torch.float32, device="cuda")
            rc = _abi.load().colizig_cuda_matmul_fp8_device(yd.data_ptr(), xd.data_ptr(), wd.data_ptr(),
                                                            sd.data_ptr(), S, I, O,
                                                            torch.cuda.current_stream().cuda_stream)
            assert rc == 0
            torch.cuda.synchronize()
            assert np.array_equal(yd.cpu().numpy(), yh)

