"""colizig_b200 — B200 (sm_100a) backend for colizig's block-FP8 MoE expert path.

The compute lives in libcolizig_cuda.so (C ABI: include/colizig_cuda.h), a
drop-in for the reference's runtime-loaded ``colizig_cuda`` backend
(src/backend/gpu.zig) plus MoE-layer entry points.  The Python modules mirror
the reference's host-side interfaces:

  gpu   src/backend/gpu.zig   init / device_name / set_vram_budget / stats /
                              matmul_fp8 / deinit
  fp8   src/ops/fp8.zig       nblk / matmul_fp8_keyed / matmul_fp8
  moe   src/qwen38/moe.zig    Dims / Layer / forward, plus stack_forward
                              (src/qwen3moe/model.zig:227-232)
  ep    expert parallelism over the GPUs of one node (partition of moe.zig's
        experts; NCCL all-reduce inside the library)
  checkpoint  src/model/weights.zig + moe.zig Layer.load / loadExpert: one MoE
        layer from safetensors shards straight into resident device memory

There is no CPU fallback: if the library is missing or a call fails, an
exception is raised.
"""

from . import _abi, checkpoint, ep, fp8, gpu, moe  # noqa: F401
from ._abi import ColizigError  # noqa: F401

__all__ = ["gpu", "fp8", "moe", "ep", "checkpoint", "ColizigError"]
