"""Library fallbacks (counted as baseline, not product): FlashAttention-2's varlen kernel for
attention shapes the hand-written kernel does not cover."""
from __future__ import annotations

import torch
from torch import Tensor

_fa = None


def _flash():
    global _fa
    if _fa is None:
        from flash_attn import flash_attn_varlen_func
        _fa = flash_attn_varlen_func
    return _fa


def flash_attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, window: int, scale: float, max_len: int) -> Tensor:
    """q,k,v [T,H,D] bf16; keys j in [i-window, i] of the same document (`train_gpt.py:1139-1141`)."""
    return _flash()(q, k, v, cu_seqlens_q=cu_seqlens, cu_seqlens_k=cu_seqlens, max_seqlen_q=max_len, max_seqlen_k=max_len,
                    causal=True, softmax_scale=scale, window_size=(window, 0))
