"""Device back-ends for the optimizer: which collectives object and which math object a CUDA
run uses.  See `NvlinkCollectives` for the fused reduce-scatter / all-gather path over peer
memory; NCCL (`TorchCollectives`) stays as baseline and fallback."""
from __future__ import annotations

import os

from .collectives import TorchCollectives


def make_device_backends(model, env):
    from ..optim.cuda_math import CudaMath
    math = CudaMath(rank=env.rank)
    if env.world_size == 1 or os.environ.get("MNG_COMM", "fused") == "nccl":
        return TorchCollectives(), math
    try:
        from .nvlink_fused import NvlinkCollectives
        return NvlinkCollectives(model, env, math), math
    except Exception as e:  # noqa: BLE001
        if os.environ.get("MNG_COMM") == "fused_strict":
            raise
        if env.master:
            print(f"[nvlink] fused collectives unavailable ({e!r}); using NCCL", flush=True)
        return TorchCollectives(), math
