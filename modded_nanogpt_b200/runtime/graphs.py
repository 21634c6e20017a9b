"""CUDA-graph execution of the training micro-step (forward + backward of one micro-batch).

The reference removes launch overhead with `torch.compile` graphs (`train_gpt.py:2244`); here the
eager program - autograd Functions around hand-written kernels - is recorded once per schedule
configuration into a `torch.cuda.CUDAGraph` and replayed: roughly a thousand launches per micro-step become
one, and the host never paces the device.  A configuration is (tokens, documents, window sizes, maximum
sequence length, number of multi-token-prediction weights, tied/untied embedding).  The first
`eager_runs` micro-steps of a configuration run eagerly (they are real training work and they warm
every lazy initialisation: cuBLAS handles, kernel attributes, tensor-map cache, autograd threads);
the next one is captured.  Only the current configuration's graph is kept.

Inputs are copied into static device buffers before each replay; parameter gradients accumulate in
place in the `.grad` tensors that exist when the graph is captured, so nothing may set them to None
afterwards (the optimizers of this framework zero gradients in place)."""
from __future__ import annotations

import torch

from ..models.gpt import ForwardScheduleConfig


class _Entry:
    __slots__ = ("count", "graph", "inputs", "sc", "loss", "launches")

    def __init__(self):
        self.count, self.graph, self.inputs, self.sc, self.loss, self.launches = 0, None, None, None, None, 0


class MicroStepGraphs:
    def __init__(self, trainer, eager_runs: int = 2):
        self.trainer, self.eager_runs = trainer, eager_runs
        self.entries: dict = {}
        self.replays = 0
        self.replayed_launches = 0      # launches of this framework's own kernels executed through replays

    def _key(self, batch, sc):
        opt = self.trainer.manager.optimizer
        return (batch.inputs.numel(), batch.cum_seqlens.numel(), sc.ws_short, sc.ws_long, sc.train_max_seq_len,
                sc.mtp_weights.numel(), bool(getattr(opt, "split_embed", False)))

    def _eager(self, batch, sc):
        t = self.trainer
        losses = t.model(batch.inputs, batch.targets, batch.cum_seqlens, batch.bigram_inputs, sc)
        loss = losses.sum() * t.env.grad_scale
        loss.backward()
        return loss.detach()

    def _capture(self, ent, batch, sc):
        t = self.trainer
        for p in t.model.parameters():                       # every gradient must exist: replay accumulates in place
            if p.requires_grad and p.grad is None:
                p.grad = torch.zeros_like(p)
        ent.inputs = tuple(x.clone() for x in (batch.inputs, batch.targets, batch.cum_seqlens, batch.bigram_inputs))
        ent.sc = ForwardScheduleConfig(sc.mtp_weights.clone(), sc.prefix_weight.clone(), sc.ws_short, sc.ws_long,
                                       sc.train_max_seq_len)
        torch.cuda.synchronize()
        from ..ops import native
        g = torch.cuda.CUDAGraph()
        n0 = native.lib().launch_count()
        with torch.cuda.graph(g):
            losses = t.model(*ent.inputs, ent.sc)
            loss = losses.sum() * t.env.grad_scale
            loss.backward()
            ent.loss = loss.detach()
        ent.graph = g
        ent.launches = native.lib().launch_count() - n0     # recorded, not executed, during the capture

    def run(self, batch, sc) -> torch.Tensor:
        key = self._key(batch, sc)
        ent = self.entries.get(key)
        if ent is None:
            self.entries.clear()                             # a new configuration: drop the previous graph and its memory
            ent = self.entries[key] = _Entry()
        if ent.graph is None:
            if ent.count < self.eager_runs:
                ent.count += 1
                return self._eager(batch, sc)
            self._capture(ent, batch, sc)
        for dst, src in zip(ent.inputs, (batch.inputs, batch.targets, batch.cum_seqlens, batch.bigram_inputs)):
            dst.copy_(src, non_blocking=True)
        ent.sc.mtp_weights.copy_(sc.mtp_weights, non_blocking=True)
        ent.sc.prefix_weight.copy_(sc.prefix_weight, non_blocking=True)
        ent.graph.replay()
        self.replays += 1
        self.replayed_launches += ent.launches
        return ent.loss.clone()
