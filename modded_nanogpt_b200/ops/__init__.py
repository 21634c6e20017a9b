"""Op dispatch: hand-written sm_100a kernels on CUDA tensors, PyTorch oracles elsewhere.

`set_backend("reference")` forces the PyTorch restatements everywhere (A/B tests, CPU runs);
`set_backend("cuda")` (default on a GPU box) routes each op to its kernel and raises if the
native extension is missing, so a GPU run never silently falls back.
"""
from __future__ import annotations

import os

import torch

from . import reference

_BACKEND = os.environ.get("MNG_BACKEND", "auto")
_DISABLED: set[str] = set(filter(None, os.environ.get("MNG_DISABLE_KERNELS", "").split(",")))


def set_backend(name: str) -> None:
    global _BACKEND
    assert name in ("auto", "cuda", "reference")
    _BACKEND = name


def get_backend() -> str:
    return _BACKEND


def disable_kernels(*names: str) -> None:
    _DISABLED.update(names)


def enable_kernels(*names: str) -> None:
    for n in names:
        _DISABLED.discard(n)


def use_kernel(name: str, *tensors) -> bool:
    """True when op `name` should run its CUDA kernel for these tensors."""
    if _BACKEND == "reference" or name in _DISABLED:
        return False
    if not tensors or not all(t.is_cuda for t in tensors if isinstance(t, torch.Tensor)):
        return False
    from . import native
    return native.available(required=True)
