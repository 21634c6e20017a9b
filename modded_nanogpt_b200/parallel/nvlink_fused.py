"""Fused collectives over NVLink peer memory.

Every parameter and its gradient live in one symmetric-memory arena (same offsets on every rank,
peer-mapped through `torch.distributed._symmetric_memory`).  The optimizer kernels then do the
communication themselves (`csrc/optim.cu`):

* gradient reduce-scatter (NorMuon banks, sharded Adam tables) and all-reduce (replicated Adam
  parameters): the update kernel reads the shard from every rank's gradient buffer with plain peer
  loads, sums in fp32 and scales by 1/world - no separate reduction pass, no staging buffer;
* parameter all-gather: the kernel that computes the new weights stores them into every rank's
  parameter tensor with peer stores;
* sparse pull for embedding-type gradients (`enable_row_masks`): every rank keeps a byte per row of the table saying
  whether its gradient row was touched since the last Adam step and copies that mask into every peer's memory before
  the barrier; the Adam kernel then skips the peer loads of untouched rows (they are exactly zero), so only touched
  rows cross NVLink - the device-side counterpart of the host-driven row exchange of `train_gpt.py:263-346`;
* from 8 ranks on (or with `MNG_MULTIMEM=1`), when the symmetric-memory handle offers an NVSwitch multicast address for
  the arena, the gradient read is a single `multimem.ld_reduce` per vector (the switch sums the ranks' copies, so
  1/world of the bytes arrive) and the weight write a single `multimem.st`; the plain peer loads/stores are the path
  below that (they measured faster at 2 GPUs, where every multicast access crosses the switch even for the rank's own
  copy, and equal at 4), with `MNG_MULTIMEM=0`, on machines without multicast and in every test that lets a rank fail;
* ordering: one `peer_barrier` kernel (release/acquire flags in the arena's signal pad, bounded
  spin that reports through the status word) after backward and one after the updates.

This replaces `reduce_scatter_tensor` / `all_reduce` / `all_gather_into_tensor` of
`train_gpt.py:588-642` for every parameter whose shard is 16-byte aligned; the small replicated parameters are updated together by one
kernel that reads all ranks' copies of their gradients, and what neither path takes falls back to NCCL through the base class.  Loads and stores are ordinary
global accesses on peer pointers: no TMA multicast, no library kernel is handed a peer pointer.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops.native import lib
from .collectives import TorchCollectives

PAD_BYTES = 4096


def _align(n: int, a: int = 256) -> int:
    return -(-n // a) * a


class NvlinkCollectives(TorchCollectives):
    fused = True

    def __init__(self, model, env, math):
        super().__init__()
        import torch.distributed._symmetric_memory as symm
        assert self.world_size <= 8
        self.math = math
        self.device = env.device
        layout, off = {}, PAD_BYTES
        params = [(getattr(p, "label", n), p) for n, p in model.named_parameters()]
        for label, p in params:
            nb = p.numel() * p.element_size()
            layout[label] = [off, 0, nb]
            off += _align(nb)
        # the gradients follow the parameters as one contiguous region, the NorMuon ones first, so that clearing
        # them after a step is one fill (NorMuon-only steps clear the first part)
        if hasattr(model, "param_table"):
            table = model.param_table()
        else:
            from ..trainer import track1_param_table
            table = track1_param_table()
        is_muon = lambda label: table.get(label, {}).get("optim") == "normuon"
        self.grad_lo = self.grad_muon_hi = off
        for label, p in sorted(params, key=lambda lp: not is_muon(lp[0])):       # stable: NorMuon parameters first
            layout[label][1] = off
            off += _align(layout[label][2])
            if is_muon(label):
                self.grad_muon_hi = off
        self.grad_hi = off
        self.arena = symm.empty(off, dtype=torch.uint8, device=env.device)
        self.handle = symm.rendezvous(self.arena, dist.group.WORLD.group_name)
        self.arena.zero_()
        self.base_ptrs = [int(x) for x in self.handle.buffer_ptrs]
        assert len(self.base_ptrs) == self.world_size
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        # measured on B200 (Adam + NorMuon step, peer loads vs multimem): 2 ranks 3.15 vs 5.15 ms, 4 ranks 3.69 vs 3.68 ms,
        # 8 ranks 4.03 vs 3.35 ms: the switch-side reduction pays once most of a shard's gradient bytes are remote
        want = os.environ.get("MNG_MULTIMEM", "auto")
        use_mc = want == "1" or (want == "auto" and self.world_size > 4)
        self.mc_base = mc if use_mc and self.world_size > 1 else 0
        self.offsets = {}
        for label, p in params:
            po, go, nb = layout[label]
            pv = self.arena[po:po + nb].view(p.dtype).view(p.shape)
            gv = self.arena[go:go + nb].view(p.dtype).view(p.shape)
            pv.copy_(p.data)
            p.data = pv
            p.grad = gv
            self.offsets[label] = (po, go)
        self.epoch = 0
        self.row_masks = {}           # label -> dict(touched, masks, peers, cols): see enable_row_masks
        torch.cuda.synchronize()
        dist.barrier()

    # -- sparse pull ---------------------------------------------------------------------------------
    def enable_row_masks(self, label: str, param) -> bool:
        """Collective.  From now on the gradient rows of `param` ([rows, cols]) that `mark_rows` was not told about since
        the last Adam step are treated as zero and not read from this rank by anybody."""
        import torch.distributed._symmetric_memory as symm
        if label not in self.offsets or param.dim() != 2 or param.shape[1] % 8 or param.shape[0] % self.world_size:
            return False
        rows, W = param.shape[0], self.world_size
        masks = symm.empty((W, rows), dtype=torch.uint8, device=self.device)
        handle = symm.rendezvous(masks, dist.group.WORLD.group_name)
        masks.fill_(1)                                        # until the first publication: read everything
        peers = [handle.get_buffer(q, (W, rows), torch.uint8) for q in range(W)]
        self.row_masks[label] = dict(touched=torch.zeros(rows, dtype=torch.uint8, device=self.device), masks=masks,
                                     peers=peers, handle=handle, cols=param.shape[1])
        torch.cuda.synchronize()
        dist.barrier()
        return True

    def mark_rows(self, label: str, rows: torch.Tensor):
        st = self.row_masks.get(label)
        if st is not None:
            st["touched"].index_fill_(0, rows.reshape(-1).long(), 1)

    def _publish_masks(self):
        # plain device-to-device copies into the peers' mask tables; ordered before the barrier on this stream
        for st in self.row_masks.values():
            for q in range(self.world_size):
                st["peers"][q][self.rank].copy_(st["touched"], non_blocking=True)

    # ------------------------------------------------------------------------------------------
    def _ptrs(self, label: str, which: int):
        off = self.offsets[label][which]
        return [b + off for b in self.base_ptrs]

    def _mc(self, label: str, which: int) -> int:
        return self.mc_base + self.offsets[label][which] if self.mc_base else 0

    def peer_barrier(self):
        self.epoch += 1
        lib().peer_barrier(self.base_ptrs, self.rank, self.epoch, self.arena)

    def handles(self, cfg) -> bool:
        if cfg.label not in self.offsets:
            return False
        if cfg.optim == "normuon":
            return self.math.kernel_shapes(cfg.reshape[-2], cfg.reshape[-1])      # tiny matrices: collective library
        po, _ = self.offsets[cfg.label]
        # shard length in elements must keep 16-byte vectors aligned
        return cfg.label in self._adam_ok

    def prepare(self, optimizer):
        """Decide per Adam parameter whether its shard can use the vectorised fused kernel."""
        self._adam_ok = set()
        for label, c in optimizer.cfgs.items():
            if c.optim != "adam" or label not in self.offsets:
                continue
            p = optimizer.params[label]
            vec = 4 if p.dtype == torch.float32 else 8
            n = p.numel() // self.world_size if c.comms.startswith("sharded") else p.numel()
            if n % vec == 0 and p.dtype in (torch.float32, torch.bfloat16):
                self._adam_ok.add(label)

    def clear_grad(self, p):
        p.grad.zero_()

    def clear_grads(self, do_adam: bool):
        """One fill over the contiguous gradient region (NorMuon-only steps: its first part)."""
        lib().fill_zero(self.arena[self.grad_lo:self.grad_hi if do_adam else self.grad_muon_hi])

    def fused_small_adam(self, labels, optimizer):
        """All small replicated Adam parameters in one launch: every rank reads all ranks' gradients straight from the
        arena and updates its own copy (the all-reduce of `train_gpt.py:597-599`, one per parameter there)."""
        items = []
        for label in labels:
            step_size, eff_wd = optimizer.adam_scalars(label)
            po, go = self.offsets[label]
            items.append((optimizer.params[label].data, None, optimizer.state[label], optimizer.cfgs[label], step_size, eff_wd, po, go))
        self.math.adam_batch(items, base_ptrs=self.base_ptrs, grad_mul=1.0 / self.world_size)

    # -- called by NorMuonAndAdam.step ---------------------------------------------------------------
    def launch_fused_reduce(self, label, grad, cfg, state):
        return (None, None)           # nothing to launch: the update kernel reads the peers directly

    def reduce_barrier(self):
        self._publish_masks()
        self.peer_barrier()           # every rank's backward (and tied-embedding transpose-add) is complete

    def gather_barrier(self):
        self.peer_barrier()           # every rank's peer stores have landed

    def fused_update_and_gather(self, label, _grad, cfg, state, optimizer, do_adam):
        W, r = self.world_size, self.rank
        gptrs, pptrs = self._ptrs(label, 1), self._ptrs(label, 0)
        p = optimizer.params[label]
        if cfg.optim == "normuon":
            per_chunk = p.numel() // W
            v = self.math.normuon_direction(None, state, cfg, grad_ptrs=gptrs, off=r * per_chunk, grad_mul=1.0 / W,
                                            grad_mc=self._mc(label, 1))
            self.math.normuon_apply(None, state, v, cfg, param_ptrs=pptrs, off=r * per_chunk, param_mc=self._mc(label, 0))
            return None
        step_size, eff_wd = optimizer.adam_scalars(label)
        if cfg.comms.startswith("sharded"):
            n = p.numel() // W
            shard = p.data.view(-1)[r * n:(r + 1) * n]
            rm = self.row_masks.get(label)
            self.math.adam(shard, None, state, cfg, step_size, eff_wd, grad_ptrs=gptrs, param_ptrs=pptrs, off=r * n,
                           grad_mul=1.0 / W, row_mask=rm["masks"] if rm else None, row_elems=rm["cols"] if rm else 0,
                           grad_mc=self._mc(label, 1), param_mc=self._mc(label, 0))
            if rm:
                rm["touched"].zero_()                         # the gradients are cleared after this step as well
        else:       # replicated: all ranks read all gradients and apply the same update to their own copy
            self.math.adam(p.data.view(-1), None, state, cfg, step_size, eff_wd, grad_ptrs=gptrs,
                           param_ptrs=[pptrs[r]], off=0, grad_mul=1.0 / W, grad_mc=self._mc(label, 1))
        return None
