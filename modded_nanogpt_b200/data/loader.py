"""BOS-aligned distributed batch loader.

Semantics follow `train_gpt.py:1712-1875`: every rank derives the document assignment of ALL
ranks from the shard's BOS index and keeps its own (deterministic, no communication); each
rank gets exactly `num_tokens_local + 1` tokens made of whole documents that start at a BOS,
truncated at `max_seq_len` and at the rank's remaining budget; `cum_seqlens` is padded to a
fixed `max_num_docs` so device shapes are static per batch size.  Validation batches are
contiguous slices with documents delimited by BOS positions.

Design differences: the loader is an object with an explicit cursor (`state_dict()` /
`load_state_dict()` make it resumable), host staging buffers are pinned once per batch shape
and reused, and the next shard is prefetched by one background thread.
"""
from __future__ import annotations

import glob
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from ..config import max_num_docs as _max_num_docs
from .shards import BOS_ID, read_shard

BIGRAM_MUL_CUR = 36313
BIGRAM_MUL_PREV = 27191


def bigram_hash(tokens: torch.Tensor, bigram_vocab_size: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """h[0] = mod, h[i] = (36313*x[i] XOR 27191*x[i-1]) % mod with mod = bigram_vocab_size-1,
    int32 (`train_gpt.py:1779-1794`).  The previous token is taken across document boundaries."""
    mod = bigram_vocab_size - 1
    x = tokens.to(torch.int32)
    if out is None:
        out = torch.empty_like(x)
    out.copy_(x)
    if x.numel() == 0:
        return out
    cur = BIGRAM_MUL_CUR * x[1:]
    prev = BIGRAM_MUL_PREV * x[:-1]
    out[0] = mod
    out[1:] = torch.bitwise_xor(cur, prev) % mod
    return out


@dataclass
class Batch:
    inputs: torch.Tensor         # int32 [T]
    targets: torch.Tensor        # int64 [T]
    cum_seqlens: torch.Tensor    # int32 [max_num_docs], padded with T
    bigram_inputs: torch.Tensor  # int32 [T]
    bigram_cpu: np.ndarray       # host copy of bigram_inputs (for the sparse-row bookkeeping)
    h2d_bytes: int = 0

    def __iter__(self):
        return iter((self.inputs, self.targets, self.cum_seqlens, self.bigram_inputs, self.bigram_cpu))


class Shard:
    """One token shard plus its BOS index.  The first 6M tokens are indexed synchronously and
    the rest by a background thread, so the first batch is not delayed by a full scan."""

    def __init__(self, tokens: torch.Tensor, world_size: int = 1, partial: int = 6_000_000):
        self.tokens = tokens
        self.np_tokens = tokens.numpy()
        self.size = tokens.numel()
        self.world_size = world_size
        self.i = 0
        self.bos_idx = np.flatnonzero(self.np_tokens[:partial] == BOS_ID).astype(np.int64)
        self._full = None
        self._ready = threading.Event()
        if self.size > partial:
            self._thread = threading.Thread(target=self._scan, daemon=True)
            self._thread.start()
        else:
            self._full = self.bos_idx
            self._thread = None
            self._ready.set()

    def _scan(self):
        self._full = np.flatnonzero(self.np_tokens == BOS_ID).astype(np.int64)
        self._ready.set()

    def _maybe_switch(self):
        if self.bos_idx is not self._full and self._ready.is_set():
            if self._thread is not None:
                self._thread.join()
            self.bos_idx = self._full

    def next_batch(self, num_tokens_local: int, max_seq_len: int):
        """Per-rank lists of document (start, end) offsets; raises StopIteration at the tail."""
        self._maybe_switch()
        bos, n = self.bos_idx, len(self.bos_idx)
        starts = [[] for _ in range(self.world_size)]
        ends = [[] for _ in range(self.world_size)]
        idx = self.i
        for r in range(self.world_size):
            cur_len = 0
            while cur_len <= num_tokens_local:
                if idx >= n:
                    if not self._ready.is_set():       # tail of the partial index: wait for the full one
                        self._ready.wait()
                        self._maybe_switch()
                        bos, n = self.bos_idx, len(self.bos_idx)
                        if idx < n:
                            continue
                    raise StopIteration("hit tail of shard")
                cur = int(bos[idx])
                idx += 1
                nxt = int(bos[idx]) if idx < n else self.size
                end = min(nxt, cur + max_seq_len, cur + num_tokens_local - cur_len + 1)
                starts[r].append(cur)
                ends[r].append(end)
                cur_len += end - cur
            assert cur_len == num_tokens_local + 1
        self.i = idx
        return starts, ends


def _prefetch(path, world_size):
    box, ready = {}, threading.Event()

    def work():
        try:
            box["shard"] = Shard(read_shard(path), world_size)
        except BaseException as e:  # surfaced on get()
            box["err"] = e
        ready.set()

    t = threading.Thread(target=work, daemon=True)
    t.start()

    def get():
        ready.wait()
        t.join()
        if "err" in box:
            raise box["err"]
        return box["shard"]
    return get


class TokenLoader:
    """Yields `Batch` objects.  `next_batch(new_params)` plays the role of the reference
    generator's `.send((num_tokens, max_seq_len, grad_accum_steps))`."""

    def __init__(self, filename_pattern: str, num_tokens: int, max_seq_len: int, grad_accum_steps: int = 1,
                 align_to_bos: bool = True, rank: int = 0, world_size: int = 1, device="cpu",
                 bigram_vocab_size: int = 0, cycle: bool = False):
        self.files = [Path(p) for p in sorted(glob.glob(filename_pattern))]
        if not self.files:
            raise FileNotFoundError(f"No files found for pattern: {filename_pattern}")
        assert num_tokens % (world_size * grad_accum_steps) == 0, "batch size must divide by world_size*grad_accum"
        self.rank, self.world_size = rank, world_size
        self.device = torch.device(device)
        self.align_to_bos = align_to_bos
        self.num_tokens = num_tokens // grad_accum_steps
        self.max_seq_len = max_seq_len
        self.bigram_vocab_size = bigram_vocab_size
        self.cycle = cycle
        self.file_idx = 0
        self.pos = 0
        self._pin = self.device.type == "cuda"
        self._stage = {}
        self.count_bytes = False
        self.bytes_copied = 0
        tokens = read_shard(self.files[0], pin=self._pin)
        if align_to_bos:
            self.shard = Shard(tokens, world_size)
            self._next = self._start_prefetch()
        else:
            self.tokens = tokens

    # -- shard rotation -----------------------------------------------------------------
    def _start_prefetch(self):
        nxt = self.file_idx + 1
        if nxt >= len(self.files):
            if not self.cycle:
                return None
            nxt = 0
        self._next_idx = nxt
        return _prefetch(self.files[nxt], self.world_size)

    def _advance_shard(self):
        if self._next is None:
            raise StopIteration("training data exhausted")
        self.shard = self._next()
        self.file_idx = self._next_idx
        self._next = self._start_prefetch()

    # -- staging ------------------------------------------------------------------------
    def _buffers(self, T: int, ndocs: int):
        """A pinned staging set that no copy still reads: the sets rotate, and each carries the event recorded after
        its last host-to-device copies, which is waited for before the host overwrites the set (the host can run
        several micro-batches ahead of the device, so rotation alone would not protect a pending copy)."""
        key = (T, ndocs)
        if key not in self._stage:
            mk = lambda n, dt: torch.empty(n, dtype=dt, pin_memory=self._pin)
            self._stage[key] = [dict(inp=mk(T, torch.int32), tgt=mk(T, torch.int64), cu=mk(ndocs, torch.int32),
                                     bg=mk(T, torch.int32), done=None) for _ in range(3)]
            self._flip = 0
        self._flip = (self._flip + 1) % 3
        st = self._stage[key][self._flip]
        if st["done"] is not None:
            st["done"].synchronize()
        return st

    def reparameterise(self, num_tokens: int, max_seq_len: int, grad_accum_steps: int):
        assert num_tokens % (self.world_size * grad_accum_steps) == 0
        self.num_tokens = num_tokens // grad_accum_steps
        self.max_seq_len = max_seq_len

    def next_batch(self, new_params=None) -> Batch:
        if new_params is not None:
            self.reparameterise(*new_params)
        T = self.num_tokens // self.world_size
        ndocs = _max_num_docs(T)
        if self.align_to_bos:
            while True:
                try:
                    starts, ends = self.shard.next_batch(T, self.max_seq_len)
                    break
                except StopIteration:
                    self._advance_shard()
            s = np.asarray(starts[self.rank], dtype=np.int64)
            e = np.asarray(ends[self.rank], dtype=np.int64)
            toks = self.shard.np_tokens
            buf = np.concatenate([toks[i:j] for i, j in zip(s, e)])
            e[-1] -= 1                          # the last document gives up one token to the target shift
            cum = np.cumsum(e - s)
        else:
            if self.pos + self.num_tokens + 1 >= self.tokens.numel():
                self.file_idx += 1
                if self.file_idx >= len(self.files):
                    if not self.cycle:
                        raise StopIteration("validation data exhausted")
                    self.file_idx = 0
                self.tokens, self.pos = read_shard(self.files[self.file_idx], pin=self._pin), 0
            lo = self.pos + self.rank * T
            buf = self.tokens.numpy()[lo: lo + T + 1]
            cum = np.flatnonzero(buf[:-1] == BOS_ID)
            self.pos += self.num_tokens
        assert buf.shape[0] == T + 1
        st = self._buffers(T, ndocs)
        st["inp"].numpy()[:] = buf[:-1]
        st["tgt"].numpy()[:] = buf[1:]
        cu = st["cu"].numpy()
        cu[:] = T
        cu[0] = 0
        k = min(len(cum), ndocs - 1)
        cu[1:k + 1] = cum[:k]
        if self.bigram_vocab_size:
            bigram_hash(st["inp"], self.bigram_vocab_size, out=st["bg"])
        else:
            st["bg"].zero_()
        dev = self.device
        to = (lambda t: t.to(dev, non_blocking=True)) if dev.type == "cuda" else (lambda t: t.clone())
        nbytes = sum(st[k].numel() * st[k].element_size() for k in ("inp", "tgt", "cu", "bg"))
        if self.count_bytes and dev.type == "cuda":
            self.bytes_copied += nbytes
        batch = Batch(to(st["inp"]), to(st["tgt"]), to(st["cu"]), to(st["bg"]), st["bg"].numpy().copy(), nbytes)
        if dev.type == "cuda":
            if st["done"] is None:
                st["done"] = torch.cuda.Event()
            st["done"].record()
        return batch

    __next__ = next_batch

    def __iter__(self):
        return self

    # -- resume -------------------------------------------------------------------------
    def state_dict(self):
        d = dict(file_idx=self.file_idx, num_tokens=self.num_tokens, max_seq_len=self.max_seq_len)
        if self.align_to_bos:
            d["cursor"] = int(self.shard.i)
        else:
            d["pos"] = int(self.pos)
        return d

    def load_state_dict(self, d):
        self.num_tokens, self.max_seq_len = d["num_tokens"], d["max_seq_len"]
        if d["file_idx"] != self.file_idx:
            self.file_idx = d["file_idx"]
            tokens = read_shard(self.files[self.file_idx], pin=self._pin)
            if self.align_to_bos:
                self.shard = Shard(tokens, self.world_size)
                self._next = self._start_prefetch()
            else:
                self.tokens = tokens
        if self.align_to_bos:
            self.shard._ready.wait()
            self.shard._maybe_switch()
            self.shard.i = d["cursor"]
        else:
            self.pos = d["pos"]


def distributed_data_generator(filename_pattern: str, num_tokens: int, max_seq_len: int, grad_accum_steps: int = 1,
                               align_to_bos: bool = True, **kw):
    """Generator facade with the reference's calling convention (`train_gpt.py:1796`): yields
    5-tuples and accepts `.send((num_tokens, max_seq_len, grad_accum_steps))`."""
    loader = TokenLoader(filename_pattern, num_tokens, max_seq_len, grad_accum_steps, align_to_bos, **kw)
    params = None
    while True:
        try:
            batch = loader.next_batch(params)
        except StopIteration:
            return
        params = yield tuple(batch)
