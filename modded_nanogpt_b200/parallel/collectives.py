"""Collective layer used by the optimizer.

`TorchCollectives` issues `torch.distributed` collectives (NCCL on GPU tensors, gloo on CPU
tensors) asynchronously and returns handles; it is the baseline and the CPU path, with the same
call pattern as the reference (`train_gpt.py:588-642`): reduce_scatter_tensor / all_reduce with
AVG, all_gather_into_tensor, all launched `async_op=True`.

`parallel.nvlink.NvlinkCollectives` provides the same interface with hand-written kernels that
move the data over NVLink peer pointers and fuse the neighbouring optimizer math.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class _Done:
    def wait(self):
        return None


class _Handle:
    def __init__(self, work, post=None):
        self.work, self.post = work, post

    def wait(self):
        if self.work is not None:
            self.work.wait()
            self.work = None
        if self.post is not None:
            self.post()
            self.post = None


class TorchCollectives:
    fused = False

    def __init__(self, group=None):
        self.group = group
        self.world_size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        # gloo has no AVG: sum then scale
        self._avg_native = dist.is_initialized() and dist.get_backend(group) != "gloo"

    def _avg(self, t):
        return (lambda: t.mul_(1.0 / self.world_size)) if not self._avg_native else None

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor):
        """out <- mean over ranks of this rank's 1/world leading-dim slice of inp."""
        if self.world_size == 1:
            out.copy_(inp)
            return _Done()
        cpu = not inp.is_cuda
        op = dist.ReduceOp.AVG if (self._avg_native and not cpu) else dist.ReduceOp.SUM
        if cpu and inp.dtype == torch.bfloat16:      # gloo reduces bf16 poorly: go through fp32
            tmp_in, tmp_out = inp.float(), torch.empty_like(out, dtype=torch.float32)
            w = dist.reduce_scatter_tensor(tmp_out, tmp_in.contiguous(), op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            return _Handle(w, lambda: out.copy_(tmp_out.mul_(1.0 / self.world_size)))
        w = dist.reduce_scatter_tensor(out, inp.contiguous(), op=op, group=self.group, async_op=True)
        return _Handle(w, None if op == dist.ReduceOp.AVG else (lambda: out.mul_(1.0 / self.world_size)))

    def all_reduce(self, t: torch.Tensor):
        if self.world_size == 1:
            return _Done()
        cpu = not t.is_cuda
        if cpu and t.dtype == torch.bfloat16:
            tmp = t.float()
            w = dist.all_reduce(tmp, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            return _Handle(w, lambda: t.copy_(tmp.mul_(1.0 / self.world_size)))
        op = dist.ReduceOp.AVG if (self._avg_native and not cpu) else dist.ReduceOp.SUM
        w = dist.all_reduce(t, op=op, group=self.group, async_op=True)
        return _Handle(w, None if op == dist.ReduceOp.AVG else (lambda: t.mul_(1.0 / self.world_size)))

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor):
        if self.world_size == 1:
            if out.data_ptr() != inp.data_ptr():
                out.copy_(inp.view_as(out))
            return _Done()
        w = dist.all_gather_into_tensor(out, inp.contiguous(), group=self.group, async_op=True)
        return _Handle(w)

    def all_to_all(self, out, inp, out_splits=None, in_splits=None):
        w = dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                   group=self.group, async_op=True)
        return _Handle(w)

    def barrier(self):
        if self.world_size > 1:
            dist.barrier(self.group)
