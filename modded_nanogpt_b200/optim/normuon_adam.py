"""NorMuon + Adam in one optimizer with explicitly scheduled communication.

Semantics of `train_gpt.py:374-947`:

* every parameter has a `.label` and an entry in `param_table` (optim "normuon"/"adam", comms
  "replicated" / "sharded" / "sharded_sparse", betas, lr_mul, wd_mul);
* `step(do_adam)`: phase 1 launches all gradient reductions in `scatter_order`; phase 2 walks
  `work_order` (small -> large), waits for that parameter's reduction, updates this rank's shard
  and launches the all-gather of the updated shard; phase 3 waits for the gathers;
* NorMuon parameters are banks of whole matrices, `.reshape[0] / world` matrices per rank:
  fp32 Nesterov momentum -> Polar Express (bf16) -> NorMuon variance normalisation -> cautious
  weight decay applied to an exact fp32 master held as bf16 weight + uint16 mantissa;
* Adam parameters: fp32 moments on the shard, bias correction, cautious weight decay, applied
  straight to the bf16/fp32 parameter; updated only when `do_adam`;
* while `embed` is tied to `lm_head`, only `lm_head` is communicated and updated (with
  `embed.grad^T` added to its gradient) and `embed <- lm_head^T` afterwards;
  `copy_lm_state_to_embed()` re-shards lm_head's Adam moments at the untie step.

Differences in design: state is keyed by label (checkpoints are portable across processes),
collectives go through a pluggable `collectives` object (torch.distributed baseline or the
fused NVLink kernels), and the per-shard math goes through `self.math` (PyTorch oracle or the
fused CUDA kernels).
"""
from __future__ import annotations

import contextlib
import os
from dataclasses import asdict, dataclass

import torch
from torch import Tensor, nn

from ..ops import reference as ref
from ..parallel.collectives import TorchCollectives


@dataclass
class ParamConfig:
    label: str
    optim: str
    comms: str
    adam_betas: tuple | None
    lr_mul: float
    wd_mul: float
    lr: float
    initial_lr: float
    weight_decay: float
    eps: float | None = None
    reshape: tuple | None = None
    chunk_size: int | None = None
    momentum: float | None = None
    beta2: float | None = None
    per_matrix_lr_mul: list | None = None
    table_comms: str = ""       # `comms` as the parameter table states it (`comms` itself becomes "none" on one rank)


class TorchMath:
    """Per-shard update math in PyTorch (oracle / CPU path)."""

    def __init__(self, polar_dtype=torch.bfloat16):
        self.polar_dtype = polar_dtype

    def normuon_direction(self, grad_chunk: Tensor, state: dict, cfg: ParamConfig) -> Tensor:
        g = grad_chunk.float()
        g = ref.nesterov_momentum_(g, state["momentum_buffer"], cfg.momentum)
        v = ref.polar_express(g, self.polar_dtype)
        shape = grad_chunk.shape
        red_dim = -1 if shape[-2] >= shape[-1] else -2
        return ref.normuon_variance_reduction_(v, state["second_momentum_buffer"], cfg.beta2, red_dim)

    def normuon_apply(self, p_slice: Tensor, state: dict, v: Tensor, cfg: ParamConfig) -> None:
        eff_wd = cfg.wd_mul * cfg.weight_decay * cfg.lr
        if cfg.per_matrix_lr_mul is not None:
            for m, mul in enumerate(cfg.per_matrix_lr_mul):
                ref.cautious_update_mantissa_(p_slice[m], state["mantissa"][m], v[m], eff_wd, cfg.lr_mul * mul * cfg.lr)
        else:
            ref.cautious_update_mantissa_(p_slice, state["mantissa"], v, eff_wd, cfg.lr_mul * cfg.lr)

    def adam(self, p_slice: Tensor, grad: Tensor, state: dict, cfg: ParamConfig, step_size: float, eff_wd: float) -> None:
        b1, b2 = cfg.adam_betas
        ref.adam_update_(p_slice, grad, state["exp_avg"], state["exp_avg_sq"], b1, b2, cfg.eps, step_size, eff_wd)

    def transpose_add(self, src: Tensor, dst: Tensor) -> None:      # dst (N,M) += src (M,N)^T
        dst.add_(src.T)

    def transpose_copy(self, src: Tensor, dst: Tensor) -> None:     # dst (N,M) = src (M,N)^T
        dst.copy_(src.T)


class NorMuonAndAdam:
    def __init__(self, named_params, param_table: dict, scatter_order: list, work_order: list,
                 adam_defaults: dict, normuon_defaults: dict, *, collectives=None, math=None,
                 sparse_exchange=None, rank: int | None = None, world_size: int | None = None):
        self.coll = collectives or TorchCollectives()
        self.math = math or TorchMath()
        self.world_size = world_size if world_size is not None else self.coll.world_size
        self.rank = rank if rank is not None else self.coll.rank
        self.adam_defaults, self.normuon_defaults = adam_defaults, normuon_defaults
        self.param_table = param_table
        self.sparse = sparse_exchange

        self.params: dict[str, nn.Parameter] = {}
        self.cfgs: dict[str, ParamConfig] = {}
        self.state: dict[str, dict] = {}
        for name, p in named_params:
            label = getattr(p, "label", None)
            assert label is not None and label in param_table, f"parameter {name} has no entry in param_table"
            assert label not in self.params, f"duplicate label {label}"
            self.params[label] = p
            self.cfgs[label] = self._build_cfg(p, label)
        present = set(self.params)
        # labels of parameters this model does not have are dropped; every present one must be scheduled
        self.scatter_order = [l for l in scatter_order if l in present]
        self.work_order = [l for l in work_order if l in present]
        assert set(self.scatter_order) == present and set(self.work_order) == present
        for c in self.cfgs.values():
            c.table_comms = c.comms
        if self.world_size == 1:
            for c in self.cfgs.values():
                c.comms = "none"
        self._init_state()
        self._pending: dict[str, tuple] = {}
        self.split_embed = False
        self.keep_grads = False     # zero gradients in place after a step instead of dropping the tensors

    # reference-compatible views -------------------------------------------------------
    @property
    def param_cfgs(self):
        return {self.params[l]: c for l, c in self.cfgs.items()}

    @property
    def param_states(self):
        return {self.params[l]: s for l, s in self.state.items()}

    # ----------------------------------------------------------------------------------
    def _sparse_active(self) -> bool:
        return self.sparse is not None

    def _build_cfg(self, p: nn.Parameter, label: str) -> ParamConfig:
        e = self.param_table[label]
        optim, comms = e["optim"], e["comms"]
        if comms == "sharded_sparse" and not self._sparse_active():
            comms = "sharded"
        betas = tuple(e["adam_betas"]) if e.get("adam_betas") else None
        lr_mul, wd_mul = e.get("lr_mul", 1.0), e.get("wd_mul", 1.0)
        if optim == "adam":
            d = self.adam_defaults
            chunk = p.shape[0] // self.world_size if comms.startswith("sharded") else None
            if chunk is not None:
                assert p.shape[0] % self.world_size == 0, f"{label}: dim 0 must divide by world size"
            return ParamConfig(label, optim, comms, betas, lr_mul, wd_mul, d["lr"], d["lr"], d["weight_decay"],
                               eps=d["eps"], chunk_size=chunk)
        if optim == "normuon":
            d = self.normuon_defaults
            reshape = getattr(p, "reshape", None)
            if reshape is None:
                raise ValueError(f"NorMuon param {label} must have a .reshape attribute")
            if reshape[0] % self.world_size:
                raise ValueError(f"{label}: reshape[0]={reshape[0]} must be divisible by world_size")
            chunk = reshape[0] // self.world_size
            rows, cols = reshape[-2], reshape[-1]
            lr_mul = max(1.0, rows / cols) ** 0.5 * lr_mul
            per_matrix = None
            if label == "mlp_bank":     # odd matrices are the down projections: 2x learning rate
                per_matrix = [2.0 if (self.rank * chunk + i) % 2 == 1 else 1.0 for i in range(chunk)]
            return ParamConfig(label, optim, comms, betas, lr_mul, wd_mul, d["lr"], d["lr"], d["weight_decay"],
                               reshape=tuple(reshape), chunk_size=chunk, momentum=d["momentum"], beta2=d["beta2"],
                               per_matrix_lr_mul=per_matrix)
        raise ValueError(f"unknown optim type {optim}")

    def _init_state(self):
        for label, p in self.params.items():
            c = self.cfgs[label]
            if c.optim == "adam":
                like = p[:c.chunk_size] if c.chunk_size is not None else p
                m = torch.zeros_like(like, dtype=torch.float32)
                self.state[label] = dict(step=0, exp_avg=m, exp_avg_sq=torch.zeros_like(m))
            else:
                shape = (c.chunk_size, *c.reshape[1:])
                sm_shape = (*shape[:-1], 1) if shape[-2] >= shape[-1] else (*shape[:-2], 1, shape[-1])
                self.state[label] = dict(
                    momentum_buffer=torch.zeros(shape, dtype=torch.float32, device=p.device),
                    second_momentum_buffer=torch.zeros(sm_shape, dtype=torch.float32, device=p.device),
                    mantissa=torch.zeros(shape, dtype=torch.uint16, device=p.device))

    # ----------------------------------------------------------------------------------
    def reset(self):
        self.split_embed = False
        for label, c in self.cfgs.items():
            if c.optim == "normuon":
                for k in ("momentum_buffer", "second_momentum_buffer", "mantissa"):
                    self.state[label][k].zero_()

    def copy_lm_state_to_embed(self):
        """lm_head moments are sharded along model_dim, embed's along vocab: gather, transpose,
        take this rank's vocab slice (`train_gpt.py:657-694`)."""
        lm, em = self.state["lm_head"], self.state["embed"]
        em["step"] = lm["step"]
        lm_p = self.params["lm_head"]
        for key in ("exp_avg", "exp_avg_sq"):
            if self.world_size > 1:
                full = torch.empty(lm_p.shape, dtype=lm[key].dtype, device=lm[key].device)
                self.coll.all_gather(full, lm[key]).wait()
                c = self.cfgs["embed"].chunk_size
                em[key].copy_(full.T[self.rank * c:(self.rank + 1) * c])
            else:
                em[key].copy_(lm[key].T)
        self.split_embed = True

    def state_dict(self):
        out = {"split_embed": self.split_embed, "state": {}, "cfgs": {l: asdict(c) for l, c in self.cfgs.items()},
               "rank": self.rank, "world_size": self.world_size}
        for l, s in self.state.items():
            out["state"][l] = {k: (v.detach().clone() if isinstance(v, Tensor) else v) for k, v in s.items()}
        return out

    def load_state_dict(self, sd):
        states = sd.get("state")
        if states is None and "param_states" in sd:      # reference layout keyed by id(param)
            by_id = {id(p): l for l, p in self.params.items()}
            states = {by_id[i]: s for i, s in sd["param_states"].items() if i in by_id}
        for l, s in states.items():
            if l not in self.state:
                continue
            for k, v in s.items():
                cur = self.state[l].get(k)
                if isinstance(v, Tensor) and isinstance(cur, Tensor):
                    cur.copy_(v.to(cur.device, cur.dtype) if v.dtype != torch.uint16 else v.to(cur.device))
                else:
                    self.state[l][k] = v
        self.split_embed = bool(sd.get("split_embed", self.split_embed))

    # ----------------------------------------------------------------------------------
    def _launch_reduce(self, label: str, grad: Tensor):
        c, coll = self.cfgs[label], self.coll
        if c.comms == "none":
            self._pending[label] = (None, grad.view(c.reshape) if c.optim == "normuon" else grad)
        elif c.comms == "replicated":
            self._pending[label] = (coll.all_reduce(grad), grad)
        elif c.comms == "sharded":
            src = grad.view(c.reshape) if c.optim == "normuon" else grad
            chunk = torch.empty((c.chunk_size, *src.shape[1:]), dtype=grad.dtype, device=grad.device)
            self._pending[label] = (coll.reduce_scatter(chunk, src), chunk)
        elif c.comms == "sharded_sparse":
            self.sparse.share_rows(grad)
            self._pending[label] = ("sparse", grad)

    def _update_lanes(self):
        """Side streams for the independent updates of one step (CUDA parameters only; MNG_OPT_STREAMS=0: none)."""
        if not hasattr(self, "_lanes"):
            p = next(iter(self.params.values()))
            on = p.is_cuda and os.environ.get("MNG_OPT_STREAMS", "1") != "0"
            self._lanes = [torch.cuda.Stream(device=p.device) for _ in range(4)] if on else None
        return self._lanes

    def _shard_of(self, label: str) -> Tensor:
        p, c = self.params[label], self.cfgs[label]
        if c.optim == "normuon":
            view = p.data.view(c.reshape)
            return view[self.rank * c.chunk_size:(self.rank + 1) * c.chunk_size]
        if c.chunk_size is not None:
            return p.data[self.rank * c.chunk_size:(self.rank + 1) * c.chunk_size]
        return p.data

    def _full_of(self, label: str) -> Tensor:
        p, c = self.params[label], self.cfgs[label]
        return p.data.view(c.reshape) if c.optim == "normuon" else p.data

    @torch.no_grad()
    def step(self, do_adam: bool = True):
        lm_p, em_p = self.params.get("lm_head"), self.params.get("embed")
        tied = lm_p is not None and em_p is not None and not self.split_embed
        # fused path: collectives + math in one kernel per bank
        fused = getattr(self.coll, "fused", False)

        # small replicated Adam parameters (gates, scalars, MUDD matrices): one kernel launch for all of them when the
        # math object offers it and no library collective is needed (one rank, or gradients readable in peer memory)
        small = []
        can_batch = do_adam and hasattr(self.math, "adam_batch") and (self.world_size == 1 or (fused and hasattr(self.coll, "fused_small_adam")))

        # ---- phase 1: reductions -------------------------------------------------------
        for label in self.scatter_order:
            p, c = self.params[label], self.cfgs[label]
            if (c.optim == "adam" and not do_adam) or p.grad is None:
                continue
            if (can_batch and c.optim == "adam" and c.table_comms == "replicated" and p.numel() <= (1 << 20)
                    and (p.is_cuda or getattr(self.math, "batch_on_cpu", False))
                    and p.dtype in (torch.float32, torch.bfloat16) and p.grad.dtype == p.dtype and p.is_contiguous()
                    and p.grad.is_contiguous() and (self.world_size == 1 or label in self.coll.offsets)):
                small.append(label)
                continue
            if label == "lm_head" and tied and em_p.grad is not None:
                self.math.transpose_add(em_p.grad, p.grad)
            if label == "embed" and tied:
                continue
            if fused and self.coll.handles(c):
                self._pending[label] = self.coll.launch_fused_reduce(label, p.grad, c, self.state[label])
            else:
                self._launch_reduce(label, p.grad)
        if fused:
            self.coll.reduce_barrier()      # all ranks' gradients are final before any peer reads them

        # ---- phase 2: updates + gathers ------------------------------------------------
        gathers, lm_gather = [], None
        if small:
            if self.world_size == 1:
                self.math.adam_batch([(self.params[l].data, self.params[l].grad, self.state[l], self.cfgs[l],
                                       *self.adam_scalars(l), 0, 0) for l in small])
            else:
                self.coll.fused_small_adam(small, self)
        # Updates that involve no library collective (one rank, or the fused peer-memory kernels) are independent of
        # one another: the bandwidth-bound Adam kernels run on one side stream and the NorMuon banks - chains of small
        # GEMMs, latency-bound once the banks are sharded - on three others, so the step costs the longest chain
        # instead of their sum.
        lanes = self._update_lanes() if (fused or self.world_size == 1) else None
        if lanes:
            main = torch.cuda.current_stream()
            for s in lanes:
                s.wait_stream(main)
        n_muon = 0
        for label in self.work_order:
            if label not in self._pending:
                continue
            c = self.cfgs[label]
            handle, grad_chunk = self._pending[label]
            if handle == "sparse":
                grad_chunk = self.sparse.merge(grad_chunk)
            elif handle is not None:
                handle.wait()
            lane = None
            if lanes and (self.world_size == 1 or self.coll.handles(c)):
                lane = lanes[0] if c.optim == "adam" else lanes[1 + n_muon % (len(lanes) - 1)]
                n_muon += c.optim != "adam"
            with (torch.cuda.stream(lane) if lane is not None else contextlib.nullcontext()):
                if fused and self.coll.handles(c):
                    g = self.coll.fused_update_and_gather(label, grad_chunk, c, self.state[label], self, do_adam)
                else:
                    p_slice = self._shard_of(label)
                    if c.optim == "adam":
                        self._adam_update(label, p_slice, grad_chunk)
                    else:
                        v = self.math.normuon_direction(grad_chunk, self.state[label], c)
                        self.math.normuon_apply(p_slice, self.state[label], v, c)
                    g = None
                    if c.comms.startswith("sharded") and self.world_size > 1:
                        g = self.coll.all_gather(self._full_of(label), p_slice)
            if g is not None:
                if label == "lm_head":
                    lm_gather = g
                else:
                    gathers.append(g)

        if lanes:
            for s in lanes:
                main.wait_stream(s)

        # ---- phase 3 -------------------------------------------------------------------
        if fused:
            self.coll.gather_barrier()      # peer stores of the new weights have landed everywhere
        if lm_gather is not None:
            lm_gather.wait()
        if do_adam and tied:
            self.math.transpose_copy(lm_p.data, em_p.data)
        for g in gathers:
            g.wait()
        self._pending.clear()
        if fused and hasattr(self.coll, "clear_grads"):
            self.coll.clear_grads(do_adam)  # gradients live in one peer-mapped region: keep the buffers, one fill
        for label, p in self.params.items():
            if self.cfgs[label].optim == "adam" and not do_adam:
                continue
            if fused and hasattr(self.coll, "clear_grads"):
                continue
            if fused and p.grad is not None:
                self.coll.clear_grad(p)     # gradients live in peer-mapped memory: keep the buffer, zero it
            elif self.keep_grads and p.grad is not None:
                p.grad.zero_()              # a captured CUDA graph accumulates into this very tensor
            else:
                p.grad = None

    def adam_scalars(self, label: str):
        """Advance the step count and return (step_size, eff_wd) for this update."""
        c, st = self.cfgs[label], self.state[label]
        st["step"] += 1
        t = st["step"]
        b1, b2 = c.adam_betas
        lr = c.lr * c.lr_mul
        return lr * ((1 - b2 ** t) ** 0.5 / (1 - b1 ** t)), lr * lr * c.weight_decay * c.wd_mul

    def _adam_update(self, label: str, p_slice: Tensor, grad: Tensor):
        step_size, eff_wd = self.adam_scalars(label)
        self.math.adam(p_slice, grad, self.state[label], self.cfgs[label], step_size, eff_wd)
