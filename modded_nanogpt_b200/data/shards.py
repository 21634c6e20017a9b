"""Token-shard file IO and synthetic corpus generation.

File format (same as the reference's, `data/fineweb.py:28-52`, read at `train_gpt.py:1697-1707`):
a header of 256 little-endian int32 (magic 20240520, version 1, token count) followed by the
tokens as uint16.  Every document starts with the end-of-text id 50256.

The synthetic generator makes streams of the same statistics the benchmarks prescribe:
token ids Zipf(s) over 0..50255, documents delimited by 50256 with lognormal or geometric
lengths.  It is deterministic in (seed, shard index).
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import torch

MAGIC = 20240520
VERSION = 1
HEADER_INTS = 256
BOS_ID = 50256


def write_shard(path, tokens: np.ndarray) -> None:
    tokens = np.ascontiguousarray(tokens, dtype=np.uint16)
    assert tokens.size < 2 ** 31
    header = np.zeros(HEADER_INTS, dtype=np.int32)
    header[0], header[1], header[2] = MAGIC, VERSION, tokens.size
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with open(tmp, "wb") as f:
        f.write(header.tobytes())
        f.write(tokens.tobytes())
    os.replace(tmp, path)


def read_shard(path, pin: bool | None = None) -> torch.Tensor:
    """Read a shard straight into (optionally pinned) host memory as a uint16 tensor."""
    path = Path(path)
    with open(path, "rb", buffering=0) as f:
        header = np.frombuffer(f.read(HEADER_INTS * 4), dtype=np.int32)
        if header.size != HEADER_INTS or header[0] != MAGIC:
            raise ValueError(f"{path}: bad magic in shard header")
        if header[1] != VERSION:
            raise ValueError(f"{path}: unsupported shard version {header[1]}")
        n = int(header[2])
        if pin is None:
            pin = torch.cuda.is_available()
        tokens = torch.empty(n, dtype=torch.uint16, pin_memory=pin)
        got = f.readinto(tokens.numpy())
        if got != 2 * n:
            raise ValueError(f"{path}: header claims {n} tokens, file holds {got // 2}")
    return tokens


class ZipfSampler:
    """Bounded Zipf(s) over `n` symbols by inverse-CDF lookup."""

    def __init__(self, n: int = 50256, s: float = 1.1):
        w = 1.0 / np.arange(1, n + 1, dtype=np.float64) ** s
        self.cdf = np.cumsum(w / w.sum())
        self.cdf[-1] = 1.0
        self.n = n

    def sample(self, rng: np.random.Generator, count: int) -> np.ndarray:
        return np.minimum(np.searchsorted(self.cdf, rng.random(count), side="right"), self.n - 1).astype(np.uint16)


def synth_tokens(num_tokens: int, seed: int = 0, *, doc_len: str = "lognormal", median_len: float = 600.0,
                 sigma: float = 1.0, mean_len: float = 200.0, max_doc_len: int = 4096, zipf_s: float = 1.1,
                 vocab: int = 50256) -> np.ndarray:
    """A stream of exactly `num_tokens` uint16 ids that starts with BOS.  Document lengths
    (BOS included) are lognormal(median, sigma) capped at `max_doc_len`, or geometric(mean)."""
    rng = np.random.default_rng(seed)
    out = ZipfSampler(vocab, zipf_s).sample(rng, num_tokens)
    est = int(num_tokens / max(8.0, min(median_len, mean_len) if doc_len == "geometric" else median_len * 0.5)) + 16
    pos, starts = 0, []
    while pos < num_tokens:
        if doc_len == "lognormal":
            lens = np.exp(rng.normal(np.log(median_len), sigma, est))
        elif doc_len == "geometric":
            lens = rng.geometric(1.0 / mean_len, est).astype(np.float64)
        else:
            raise ValueError(doc_len)
        lens = np.clip(lens.astype(np.int64), 2, max_doc_len)
        s = pos + np.concatenate([[0], np.cumsum(lens)[:-1]])
        s = s[s < num_tokens]
        starts.append(s)
        pos = int(s[-1] + lens[len(s) - 1]) if len(s) else num_tokens
    out[np.concatenate(starts)] = BOS_ID
    return out


def write_synthetic_corpus(root, *, train_tokens: int, val_tokens: int, shard_tokens: int = 100_000_000, seed: int = 0,
                           **kw) -> tuple[str, str]:
    """Write `fineweb_val_000000.bin` and `fineweb_train_00000N.bin` under
    `root/data/fineweb10B/` (the directory layout `train_gpt.py:1884-1885` globs).  Returns the
    two glob patterns.  Existing shards of the right size are kept."""
    d = Path(root) / "data" / "fineweb10B"
    d.mkdir(parents=True, exist_ok=True)

    def ensure(path, n, sd):
        if path.exists() and path.stat().st_size == HEADER_INTS * 4 + 2 * n:
            return
        write_shard(path, synth_tokens(n, sd, **kw))

    ensure(d / "fineweb_val_000000.bin", val_tokens, seed + 7919)
    left, i = train_tokens, 1
    while left > 0:
        n = min(left, shard_tokens)
        ensure(d / f"fineweb_train_{i:06d}.bin", n, seed + i)
        left -= n
        i += 1
    return str(d / "fineweb_train_*.bin"), str(d / "fineweb_val_*.bin")
