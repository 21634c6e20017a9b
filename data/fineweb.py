"""Tokenise a text corpus into the `.bin` shards the loaders read (same product as the reference's
`data/fineweb.py:28-126`): GPT-2 BPE ids as uint16, every document preceded by the end-of-text id
50256, fixed-size shards, shard 0 is the validation split.

    python data/fineweb.py --version 10B --shard-size 100000000            # HuggingFace FineWeb sample
    python data/fineweb.py --text-files corpus/*.txt --out data/mycorpus    # any local text, one document per file

Needs `tiktoken` (and `datasets` for the FineWeb download); neither is required by training itself."""
from __future__ import annotations

import argparse
import glob
import os
import sys
from concurrent.futures import ProcessPoolExecutor

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from modded_nanogpt_b200.data.shards import write_shard  # noqa: E402

EOT = 50256


class ShardWriter:
    """Accumulates token arrays and cuts shards of exactly `shard_size` tokens; a document may straddle two
    shards, as in the reference.  File names: `<prefix>_val_000000.bin`, then `<prefix>_train_00000N.bin`."""

    def __init__(self, out_dir: str, prefix: str, shard_size: int):
        self.out_dir, self.prefix, self.shard_size = out_dir, prefix, shard_size
        os.makedirs(out_dir, exist_ok=True)
        self.buf = np.empty(shard_size, dtype=np.uint16)
        self.fill, self.index, self.paths = 0, 0, []

    def _flush(self, n: int):
        split = "val" if self.index == 0 else "train"
        path = os.path.join(self.out_dir, f"{self.prefix}_{split}_{self.index:06d}.bin")
        write_shard(path, self.buf[:n])
        self.paths.append(path)
        self.index += 1
        self.fill = 0

    def add(self, toks: np.ndarray):
        toks = np.asarray(toks, dtype=np.uint16)
        while len(toks):
            take = min(len(toks), self.shard_size - self.fill)
            self.buf[self.fill:self.fill + take] = toks[:take]
            self.fill += take
            toks = toks[take:]
            if self.fill == self.shard_size:
                self._flush(self.shard_size)

    def close(self):
        if self.fill:
            self._flush(self.fill)
        return self.paths


def _encoder():
    import tiktoken
    return tiktoken.get_encoding("gpt2")


def tokenize_doc(text: str, enc=None) -> np.ndarray:
    enc = enc or _encoder()
    ids = [EOT] + enc.encode_ordinary(text)
    arr = np.asarray(ids)
    assert arr.min() >= 0 and arr.max() < 2 ** 16
    return arr.astype(np.uint16)


def _tok_worker(text):
    global _ENC
    try:
        _ENC
    except NameError:
        _ENC = _encoder()
    return tokenize_doc(text, _ENC)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--version", default="10B", choices=["10B", "100B"])
    ap.add_argument("-s", "--shard-size", type=int, default=10 ** 8)
    ap.add_argument("--text-files", nargs="*", help="local text files (one document each) instead of FineWeb")
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    if a.text_files:
        docs = (open(p, encoding="utf-8", errors="replace").read() for pat in a.text_files for p in sorted(glob.glob(pat)))
        out, prefix = a.out or "data/local", "fineweb"
    else:
        from datasets import load_dataset
        name = {"10B": "sample-10BT", "100B": "sample-100BT"}[a.version]
        docs = (d["text"] for d in load_dataset("HuggingFaceFW/fineweb", name=name, split="train"))
        out, prefix = a.out or os.path.join(os.path.dirname(__file__), f"fineweb{a.version}"), "fineweb"
    w = ShardWriter(out, prefix, a.shard_size)
    with ProcessPoolExecutor(max(1, (os.cpu_count() or 2) - 2)) as pool:
        for toks in pool.map(_tok_worker, docs, chunksize=16):
            w.add(toks)
    for p in w.close():
        print(p)


if __name__ == "__main__":
    main()
