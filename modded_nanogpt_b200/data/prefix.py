"""Prefix-token table for the prefix-token auxiliary loss.

For token T the table holds the id of the token whose byte string is the longest proper
prefix of T's byte string and is itself in the vocabulary, or -1 (`train_gpt.py:1175-1198`).
The algorithm is the same sort-and-stack sweep; the vocabulary source is pluggable because the
GPT-2 BPE ranks are a network download: `load_gpt2_ranks()` uses tiktoken when its cache is
populated, `synthetic_ranks()` builds a deterministic stand-in with BPE-like prefix structure.
"""
from __future__ import annotations

import numpy as np
import torch


def build_prefix_table(vocab_size: int, byte_to_id: dict | None = None) -> torch.Tensor:
    if byte_to_id is None:
        byte_to_id = load_gpt2_ranks() or synthetic_ranks(50257)
    table = [-1] * vocab_size
    stack: list = []          # (bytes, id) of the live ancestors, shortest first
    for b, tid in sorted(byte_to_id.items()):
        while stack and not b.startswith(stack[-1][0]):
            stack.pop()
        if stack and tid < vocab_size:
            table[tid] = stack[-1][1]
        stack.append((b, tid))
    return torch.tensor(table, dtype=torch.int64)


def load_gpt2_ranks():
    try:
        import tiktoken  # noqa: WPS433
        return dict(tiktoken.get_encoding("gpt2")._mergeable_ranks)
    except Exception:
        return None


def synthetic_ranks(n: int = 50257, seed: int = 0) -> dict:
    """256 single bytes, then tokens formed by appending a byte (or a short tail) to an earlier
    token, like BPE merges do, so about as many tokens have a prefix in the vocabulary as in a
    real BPE table."""
    rng = np.random.default_rng(seed)
    toks = [bytes([i]) for i in range(256)]
    seen = set(toks)
    while len(toks) < n - 1:
        base = toks[int(rng.integers(0, len(toks)))]
        tail = bytes(rng.integers(97, 123, size=int(rng.integers(1, 4))).astype(np.uint8))
        cand = base + tail
        if len(cand) <= 16 and cand not in seen:
            seen.add(cand)
            toks.append(cand)
    return {b: i for i, b in enumerate(toks)}
