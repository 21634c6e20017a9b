"""Sparse row exchange for the bigram-embedding gradient.

Only the rows of the (377280 x 768) gradient that some token touched since the last Adam step
are non-zero, so instead of a dense reduce-scatter each rank sends every touched row to the rank
that owns it.  Protocol of `train_gpt.py:263-346`:

1. `start(rows)`      host: sorted unique touched row ids -> per-owner send counts (own rows
                      dropped), counts exchanged over the CPU group;
2. `share_indexes()`  row ids exchanged with uneven all-to-all;
3. `share_rows(grad)` rows gathered and exchanged;
4. `merge(grad)`      received rows index-added into the local dense gradient, the owned slice
                      scaled by 1/world returned.

`RowTracker` accumulates the touched-row mask across micro-batches and steps.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


class RowTracker:
    def __init__(self, num_rows: int):
        self.mask = np.zeros(num_rows, dtype=np.uint8)

    def mark(self, rows: np.ndarray):
        self.mask[rows] = 1

    def take(self) -> np.ndarray:
        idx = np.flatnonzero(self.mask).astype(np.int32)
        self.mask.fill(0)
        return idx

    def peek(self) -> np.ndarray:
        return np.flatnonzero(self.mask).astype(np.int32)


class SparseRowExchange:
    def __init__(self, num_rows: int, rank: int, world_size: int, device, cpu_group=None, group=None):
        assert num_rows % world_size == 0
        self.N, self.rank, self.world = num_rows, rank, world_size
        self.rows_per_rank = num_rows // world_size
        self.device = torch.device(device)
        self.cpu_group, self.group = cpu_group, group
        pin = self.device.type == "cuda"
        # two pinned staging buffers, each with the event recorded after its last copy to the device: the host may run
        # more than a step ahead of the device, and must not overwrite a buffer whose copy has not run yet
        self._stages = [[torch.empty(num_rows, dtype=torch.int32, pin_memory=pin), None] for _ in range(2)]
        self._flip = 0
        self._state = None

    @torch.no_grad()
    def start(self, rows_np: np.ndarray):
        n = rows_np.shape[0]
        self._flip ^= 1
        slot = self._stages[self._flip]
        if slot[1] is not None:
            slot[1].synchronize()
        stage = slot[0][:n]
        stage.copy_(torch.from_numpy(rows_np))
        send_idx = stage.to(self.device, non_blocking=True)
        if self.device.type == "cuda":
            if slot[1] is None:
                slot[1] = torch.cuda.Event()
            slot[1].record()
        bounds = np.arange(0, self.rows_per_rank * (self.world + 1), self.rows_per_rank, dtype=np.int64)
        ins = np.searchsorted(rows_np, bounds)
        send_counts = torch.from_numpy((ins[1:] - ins[:-1]).astype(np.int64))
        send_counts[self.rank] = 0
        send_idx = torch.cat([send_idx[:ins[self.rank]], send_idx[ins[self.rank + 1]:]])
        recv_counts = torch.empty_like(send_counts)
        work = dist.all_to_all_single(recv_counts, send_counts, group=self.cpu_group, async_op=True)
        self._state = dict(send_idx=send_idx, send_counts=send_counts, recv_counts=recv_counts, counts_work=work)

    @torch.no_grad()
    def share_indexes(self):
        st = self._state
        st.pop("counts_work").wait()
        st["recv_counts"] = st["recv_counts"].tolist()
        st["send_counts"] = st["send_counts"].tolist()
        st["recv_idx"] = torch.empty(sum(st["recv_counts"]), dtype=torch.int32, device=self.device)
        st["idx_work"] = dist.all_to_all_single(st["recv_idx"], st["send_idx"], output_split_sizes=st["recv_counts"],
                                                input_split_sizes=st["send_counts"], group=self.group, async_op=True)

    @property
    def ready(self) -> bool:
        return self._state is not None and "recv_idx" in self._state

    @torch.no_grad()
    def share_rows(self, grad: torch.Tensor):
        st = self._state
        d = grad.shape[1]
        send_vals = grad[st["send_idx"].long()].contiguous()
        st["recv_vals"] = torch.empty(sum(st["recv_counts"]) * d, dtype=grad.dtype, device=grad.device)
        st["val_work"] = dist.all_to_all_single(
            st["recv_vals"], send_vals.view(-1), output_split_sizes=[c * d for c in st["recv_counts"]],
            input_split_sizes=[c * d for c in st["send_counts"]], group=self.group, async_op=True)

    @torch.no_grad()
    def merge(self, grad: torch.Tensor) -> torch.Tensor:
        st, self._state = self._state, None
        st["idx_work"].wait()
        st["val_work"].wait()
        d = grad.shape[1]
        grad.index_add_(0, st["recv_idx"].long(), st["recv_vals"].view(-1, d))
        lo = self.rows_per_rank * self.rank
        return grad[lo: lo + self.rows_per_rank].mul_(1.0 / self.world)

    def bytes_sent(self, d: int, itemsize: int = 2) -> int:
        st = self._state
        return 0 if st is None else int(sum(st["send_counts"])) * d * itemsize
