"""HellaSwag evaluation by packed scoring (behaviour of `evals/hellaswag.py:50-194`).

Each task contributes four "documents" - the context followed by one candidate ending - separated
by the end-of-text token, many tasks per packed sequence; the model's per-token loss is averaged
over each ending's span and the ending with the lowest mean loss is the prediction.  Counts are
summed over ranks.

Differences in design: tokenisation and the dataset are injectable (`tokenize`, `tasks`), so the
packing and scoring logic is testable offline on synthetic tasks; span means are computed with one
cumulative sum instead of a Python loop over slices; works on CPU and without a process group.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Iterable

import torch
import torch.distributed as dist

EOT_ID = 50256


@dataclass
class PackedSequence:
    inputs: torch.Tensor          # int32 [seq_len]
    targets: torch.Tensor         # int64 [seq_len]
    doc_ends: torch.Tensor        # int32 [max_docs] cumulative document ends, padded with seq_len
    spans: torch.Tensor           # int64 [n_tasks, 4, 2] (start, end) of every ending in target coordinates
    labels: torch.Tensor          # int64 [n_tasks]


def _finalize(inputs, targets, spans, labels, seq_len) -> PackedSequence:
    max_docs = ((seq_len // 70) // 128 + 1) * 128          # documents average well above 70 tokens
    pad = seq_len - len(inputs)
    inp = torch.tensor(inputs + [0] * pad, dtype=torch.int32)
    tgt = torch.tensor(targets + [0] * pad, dtype=torch.int64)
    ends = torch.nonzero(inp == EOT_ID)[:, 0] + 1            # the separator belongs to the document before it
    doc = torch.full((max_docs,), seq_len, dtype=torch.int32)
    doc[0] = 0
    n = min(len(ends), max_docs - 1)
    doc[1:n + 1] = ends[:n].to(torch.int32)
    return PackedSequence(inp, tgt, doc, torch.tensor(spans, dtype=torch.int64).view(-1, 4, 2),
                          torch.tensor(labels, dtype=torch.int64))


def pack_tasks(tasks: Iterable[dict], seq_len: int, tokenize: Callable[[str], list] | None = None) -> list[PackedSequence]:
    """tasks: dicts with either token lists (`ctx_tokens`, `ending_tokens`) or text (`ctx`, `endings`,
    tokenised with `tokenize`; endings get a leading space) and an integer `label`."""
    seqs, inputs, targets, spans, labels = [], [], [], [], []

    def flush():
        nonlocal inputs, targets, spans, labels
        seqs.append(_finalize(inputs, targets, spans, labels, seq_len))
        inputs, targets, spans, labels = [], [], [], []

    for t in tasks:
        ctx = t["ctx_tokens"] if "ctx_tokens" in t else tokenize(t["ctx"])
        ends = t["ending_tokens"] if "ending_tokens" in t else [tokenize(" " + e) for e in t["endings"]]
        assert len(ends) == 4, f"4 endings per task, got {len(ends)}"
        if len(inputs) + sum(len(ctx) + len(e) for e in ends) >= seq_len:
            flush()
        for e in ends:
            if inputs:
                inputs.append(EOT_ID)
                targets.append(EOT_ID)
            both = list(ctx) + list(e)
            start = len(inputs) + len(ctx) - 1              # targets are shifted left by one
            spans.append((start, start + len(e)))
            inputs.extend(both[:-1])
            targets.extend(both[1:])
        labels.append(int(t["label"]))
    if inputs:
        flush()
    return seqs


def score_losses(loss_per_token: torch.Tensor, spans: torch.Tensor, labels: torch.Tensor) -> tuple[int, int]:
    """(#correct, #tasks) from per-token losses: mean loss per ending span, argmin over the four."""
    c = torch.cat([loss_per_token.new_zeros(1, dtype=torch.float64), loss_per_token.double().cumsum(0)])
    s, e = spans[..., 0].to(loss_per_token.device), spans[..., 1].to(loss_per_token.device)
    means = (c[e] - c[s]) / (e - s).clamp_min(1)
    pred = means.argmin(dim=1)
    return int((pred == labels.to(pred.device)).sum()), int(labels.numel())


def score_sequence(model, schedule_cfg, seq: PackedSequence, get_bigram_hash: Callable, device) -> tuple[int, int]:
    loss = model(seq.inputs.to(device), seq.targets.to(device), seq.doc_ends.to(device),
                 get_bigram_hash(seq.inputs).to(device), schedule_cfg)
    return score_losses(loss.float(), seq.spans, seq.labels)


def load_tasks(rank: int = 0, world_size: int = 1):
    """The 10,042 validation tasks (needs the `datasets` package and a populated cache / network)."""
    from datasets import load_dataset
    ds = load_dataset(path="Rowan/hellaswag", split="validation").shuffle(seed=42)
    return [ds[i + rank] for i in range(0, len(ds) - rank, world_size)]


def gpt2_tokenizer():
    import tiktoken
    enc = tiktoken.get_encoding("gpt2")
    return enc.encode_ordinary


def evaluate(model, schedule_cfg, seq_len: int, get_bigram_hash: Callable, print0: Callable = print, tasks=None,
             tokenize=None):
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    device = next(model.parameters()).device
    t0 = time.perf_counter()
    if tasks is None:
        tasks, tokenize = load_tasks(rank, world), (tokenize or gpt2_tokenizer())
    model.eval()
    correct = count = 0
    with torch.inference_mode():
        for seq in pack_tasks(tasks, seq_len, tokenize):
            a, b = score_sequence(model, schedule_cfg, seq, get_bigram_hash, device)
            correct, count = correct + a, count + b
    if world > 1:
        t = torch.tensor([correct, count], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        correct, count = int(t[0]), int(t[1])
    if device.type == "cuda":
        torch.cuda.synchronize()
    accuracy, seconds = correct / max(count, 1), time.perf_counter() - t0
    print0(f"HellaSwag: {accuracy=:.3%} (n_correct={correct} out of n_count={count} tasks in {seconds=:.2f})", console=True)
    return accuracy
