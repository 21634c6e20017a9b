"""Rank-0 run log, line-compatible with the reference (`train_gpt.py:2206-2232,2342,2369`):
the file starts with the source of the entry point and of this package's kernels, then the
software versions and `nvidia-smi`; per-step lines match the regexes the reference's tooling
uses (`step:(\\d+)/(\\d+)\\s+val_loss:([0-9.]+)\\s+train_time:(\\d+)ms`)."""
from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import torch

VAL_LINE = re.compile(r"step:(\d+)/(\d+)\s+val_loss:([0-9.]+)\s+train_time:(\d+)ms\s+step_avg:([0-9.]+)ms")
TRAIN_LINE = re.compile(r"step:(\d+)/(\d+)\s+train_time:(\d+)ms\s+step_avg:([0-9.]+)ms")


class RunLogger:
    def __init__(self, run_id: str, master: bool, log_dir: str = "logs", quiet: bool = False):
        self.master, self.quiet = master, quiet
        self.path = None
        if master:
            os.makedirs(log_dir, exist_ok=True)
            self.path = os.path.join(log_dir, f"{run_id}.txt")
            if not quiet:
                print(self.path)

    def print0(self, s, console: bool = False):
        if not self.master:
            return
        with open(self.path, "a") as f:
            if console and not self.quiet:
                print(s, flush=True)
            print(s, file=f)

    def log_sources(self, entry_file: str | None = None):
        """Dump the entry script and every source file of the package into the log."""
        if not self.master:
            return
        root = Path(__file__).resolve().parents[1]
        files = ([Path(entry_file)] if entry_file else []) + sorted(
            p for p in root.rglob("*") if p.suffix in (".py", ".cu", ".cuh", ".cpp", ".h"))
        for p in files:
            try:
                self.print0(f"\n{'-' * 40}\n# {p.name}\n{'-' * 40}\n\n{p.read_text()}")
            except OSError:
                pass
        self.print0("=" * 100)

    def log_environment(self):
        self.print0(f"Running Python {sys.version}")
        self.print0(f"Running PyTorch {torch.version.__version__} compiled for CUDA {torch.version.cuda}")
        try:
            smi = subprocess.run(["nvidia-smi"], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True).stdout
        except OSError:
            smi = "nvidia-smi unavailable"
        self.print0(smi)
        self.print0("=" * 100)


def parse_log(path: str):
    """Returns (train_points, val_points) parsed from a run log: lists of
    (step, train_time_ms[, val_loss])."""
    train, val = [], []
    for line in open(path):
        m = VAL_LINE.search(line)
        if m:
            val.append((int(m.group(1)), int(m.group(4)), float(m.group(3))))
            continue
        m = TRAIN_LINE.search(line)
        if m:
            train.append((int(m.group(1)), int(m.group(3))))
    return train, val
