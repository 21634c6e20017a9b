"""Loader of the in-tree CUDA extension (`modded_nanogpt_b200/_C*.so`, built by `build_ext.py`).
On a machine with a GPU a missing extension is an error, never a silent fallback."""
from __future__ import annotations

import importlib
import os

import torch

_mod = None
_err = None


def load():
    global _mod, _err
    if _mod is None and _err is None:
        try:
            # MNG_NATIVE=_Cdbg runs everything on the bounds-checked build (python build_ext.py --debug)
            _mod = importlib.import_module("modded_nanogpt_b200." + os.environ.get("MNG_NATIVE", "_C"))
        except Exception as e:  # noqa: BLE001
            _err = e
    return _mod


def available(required: bool = False) -> bool:
    m = load()
    if m is None and required and torch.cuda.is_available():
        raise RuntimeError(
            "modded_nanogpt_b200._C (the sm_100a CUDA extension) is not built; run "
            "`python build_ext.py` at the repository root") from _err
    return m is not None


def lib():
    if not available(required=True):
        raise RuntimeError("CUDA extension unavailable") from _err
    return _mod
