"""Training manager and engine.

`TrainingManager` keeps the reference's contract (`train_gpt.py:2009-2198`): the parameter
table, scatter/work orders, `advance_schedule`, `get_forward_args`, `step_optimizers`,
`reset`/`get_state`, sparse-row bookkeeping.  `Trainer` is the public engine: it builds model,
loaders and manager for a preset and exposes `train_step`, `validate`, `run` (the full loop
with the reference's log lines), checkpoint save/resume and device-timed step statistics.
"""
from __future__ import annotations

import contextlib
import copy
import os
import sys
import time
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from .config import (Hyperparameters, ModelConfig, TrainingSchedule, track1_model, track1_stages)
from .data.loader import TokenLoader
from .models.gpt import GPT, ForwardScheduleConfig
from .optim.normuon_adam import NorMuonAndAdam
from .parallel.collectives import TorchCollectives
from .parallel.sparse_comms import RowTracker, SparseRowExchange
from .runtime.dist import DistEnv, broadcast_model
from .runtime.health import monitor_from_env
from .utils.logging import RunLogger


def track1_param_table() -> dict:
    """`train_gpt.py:2026-2050`."""
    A = "adam"
    t = {
        "qk_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None},
        "vo_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None},
        "mlp_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None},
        "scalars": {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": 5.0, "wd_mul": 0.0},
        "smear_gate": {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": 0.01, "wd_mul": 0.0},
        "ve_gate_bank": {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99]},
        "lm_head": {"optim": A, "comms": "sharded", "adam_betas": [0.5, 0.95], "wd_mul": 150.0},
        "bigram_embed": {"optim": A, "comms": "sharded_sparse", "adam_betas": [0.75, 0.95], "lr_mul": 75.0, "wd_mul": 5.0},
        "post_lambdas": {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.95], "lr_mul": 1.0, "wd_mul": 0.0},
        "resid_lambdas": {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.95], "lr_mul": 5.0, "wd_mul": 0.0},
        "value_embeds": {"optim": A, "comms": "sharded", "adam_betas": [0.75, 0.95], "lr_mul": 75.0, "wd_mul": 5.0},
        "embed": {"optim": A, "comms": "sharded", "adam_betas": [0.5, 0.95], "wd_mul": 150.0},
    }
    for name, lr in (("mudd", 0.25), ("mudd_gate", 0.1)):
        t[f"{name}_w1"] = {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": lr}
        t[f"{name}_w2"] = {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": lr}
        t[f"{name}_b2"] = {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": lr, "wd_mul": 0.0}
    t["_mudd_gate_scale"] = {"optim": A, "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": 0.1, "wd_mul": 0.0}
    return t


TRACK1_WORK_ORDER = [
    "scalars", "smear_gate", "ve_gate_bank", "mudd_b2", "mudd_gate_b2", "_mudd_gate_scale", "post_lambdas",
    "resid_lambdas", "mudd_w2", "mudd_gate_w2", "value_embeds", "bigram_embed", "mudd_w1", "mudd_gate_w1",
    "lm_head", "embed", "qk_bank", "vo_bank", "mlp_bank",
]


class TrainingManager:
    def __init__(self, model: GPT, schedule: TrainingSchedule, hp: Hyperparameters, env: DistEnv,
                 collectives=None, math=None, sparse_min_world: int = 8):
        self.model, self.schedule, self.hp, self.env = model, schedule, hp, env
        self.block_size = hp.block_size
        self.param_table = model.param_table() if hasattr(model, "param_table") else track1_param_table()
        self.work_order = list(getattr(model, "WORK_ORDER", TRACK1_WORK_ORDER))
        dev = next(model.parameters()).device
        self.sparse = None
        self.row_tracker = None
        # with the fused NVLink path every rank reads its bigram shard straight from the peers' dense
        # gradients, so the host-driven sparse exchange is only used on the NCCL / gloo path
        if (hasattr(model, "bigram_embed") and not getattr(collectives, "fused", False)
                and env.world_size >= sparse_min_world and env.world_size > 1
                and env.grad_accum_steps == 1):
            n = model.bigram_embed.weight.shape[0]
            self.sparse = SparseRowExchange(n, env.rank, env.world_size, dev)
            self.row_tracker = RowTracker(n)
        self.optimizer = NorMuonAndAdam(
            model.named_parameters(), self.param_table, list(self.param_table), self.work_order,
            adam_defaults=dict(lr=hp.adam_lr, eps=hp.adam_eps, weight_decay=hp.adam_wd),
            normuon_defaults=dict(lr=hp.muon_lr, momentum=hp.muon_momentum, beta2=hp.muon_beta2, weight_decay=hp.muon_wd),
            collectives=collectives or TorchCollectives(), math=math, sparse_exchange=self.sparse,
            rank=env.rank, world_size=env.world_size)
        if hasattr(self.optimizer.coll, "prepare"):
            self.optimizer.coll.prepare(self.optimizer)
        # fused NVLink path: the Adam kernel pulls only the bigram-gradient rows that a rank touched (`mark_rows` in
        # `Trainer.micro_step`); MNG_SPARSE_PULL=0 keeps the dense pull
        self.row_mask_labels = []
        coll = self.optimizer.coll
        if (getattr(coll, "fused", False) and hasattr(model, "bigram_embed") and env.world_size > 1
                and os.environ.get("MNG_SPARSE_PULL", "1") != "0"
                and self.param_table.get("bigram_embed", {}).get("comms") == "sharded_sparse"):
            if coll.enable_row_masks("bigram_embed", model.bigram_embed.weight):
                self.row_mask_labels.append("bigram_embed")
        self.split_step = schedule.split_step
        self.device = dev
        self.reset()

    # -- schedule ------------------------------------------------------------------------
    def apply_final_ws_ext(self):
        self.ws_long = self.schedule.ws_post_yarn_ext

    def get_forward_args(self) -> ForwardScheduleConfig:
        return ForwardScheduleConfig(self.mtp_weights, self.prefix_weight, self.ws_short * self.block_size,
                                     self.ws_long * self.block_size, self.train_max_seq_len)

    @staticmethod
    def is_adam_step(step: int) -> bool:
        return step % 2 == 1

    def get_transition_steps(self):
        return self.schedule.transition_steps()

    def advance_schedule(self, step: int):
        stage, _ = self.schedule.lookup(step)
        self.ws_short, new_long = stage.window_sizes
        cap = getattr(self.schedule, "yarn_max_ws", None)
        if new_long != self.ws_long and (cap is None or new_long <= cap):
            for y in {id(self.model.yarn): self.model.yarn, id(self.model.yarn_paired_head): self.model.yarn_paired_head}.values():
                y.apply(self.ws_long * self.block_size, new_long * self.block_size)
        # Idempotent: a pending re-parameterisation stays pending until the loader has consumed it (`Trainer._take_batch`
        # clears it), so calling this twice for the same step - `run()` and then `train_step()` - changes nothing.
        if stage.batch_size != self.batch_size or stage.train_max_seq_len != self.train_max_seq_len:
            self.train_loader_send_args = (stage.batch_size, stage.train_max_seq_len, self.env.grad_accum_steps)
            self.batch_size, self.train_max_seq_len = stage.batch_size, stage.train_max_seq_len
        self.ws_long = new_long
        self.mtp_weights = torch.tensor(self.schedule.mtp_weights[step], dtype=torch.float32, device=self.device)
        self.prefix_weight = torch.tensor([self.schedule.prefix_weights[step]], dtype=torch.float32, device=self.device)

    def step_optimizers(self, step: int):
        lr_mul = self.schedule.get_lr(step)
        mom = self.schedule.muon_momentum(step)
        for c in self.optimizer.cfgs.values():
            c.lr = c.initial_lr * lr_mul
            if c.optim == "normuon":
                c.momentum = mom
        self.optimizer.step(do_adam=self.is_adam_step(step))
        if step == self.split_step and "embed" in self.optimizer.params:
            self.optimizer.copy_lm_state_to_embed()

    def reset(self, state=None):
        if state is not None:
            self.optimizer.load_state_dict(state)
        self.optimizer.reset()
        stage, _ = self.schedule.lookup(0)
        self.ws_short, self.ws_long = stage.window_sizes
        self.batch_size, self.train_max_seq_len = stage.batch_size, stage.train_max_seq_len
        self.train_loader_send_args = None
        self.model.yarn.reset()
        if self.model.yarn_paired_head is not self.model.yarn:
            self.model.yarn_paired_head.reset()
        if self.row_tracker is not None:
            self.row_tracker.mask.fill(0)

    def get_state(self):
        return copy.deepcopy(self.optimizer.state_dict())

    # -- sparse bigram rows --------------------------------------------------------------
    def sparse_index_update(self, step: int, bigram_rows: np.ndarray):
        if self.sparse is None:
            return
        self.row_tracker.mark(bigram_rows)
        if self.is_adam_step(step):
            self.sparse.start(self.row_tracker.peek())

    def sparse_index_share(self, step: int):
        if self.sparse is None or not self.is_adam_step(step):
            return
        self.sparse.share_indexes()
        self.row_tracker.mask.fill(0)


@dataclass
class StepStats:
    loss: float
    device_ms: float


class Trainer:
    """Public engine.  `Trainer(model_cfg, schedule, hp, env)`; `train_step(step)` runs
    grad_accum micro-batches (H2D copy of the inputs, forward, backward), the optimizer step and
    the FP8 weight refresh; `validate()` the evaluation pass; `run()` the whole schedule."""

    def __init__(self, model_cfg: ModelConfig | None, schedule: TrainingSchedule | None, hp: Hyperparameters,
                 env: DistEnv, *, param_dtype=torch.bfloat16, collectives=None, math=None, logger=None,
                 model: GPT | None = None, sparse_min_world: int = 8, use_cuda_graphs: bool | None = None):
        self.hp, self.env = hp, env
        self.schedule = schedule or TrainingSchedule(track1_stages(), hp.num_scheduled_iterations,
                                                     hp.num_extension_iterations, cooldown_frac=hp.cooldown_frac)
        eval_seq = hp.val_batch_size // (env.grad_accum_steps * env.world_size)
        model_cfg = model_cfg or track1_model(eval_seq)
        torch.manual_seed(hp.seed)
        self.model = model or GPT(model_cfg, world_size=env.world_size, grad_scale=env.grad_scale,
                                  use_fp8=not hp.disable_fp8, eval_seq_len=eval_seq)
        self.model.to(env.device)
        if param_dtype != torch.float32:
            self.model.cast_params_(param_dtype)
        broadcast_model(self.model)
        if env.device.type == "cuda" and collectives is None and math is None:
            from .parallel.nvlink import make_device_backends
            collectives, math = make_device_backends(self.model, env)
        self.manager = TrainingManager(self.model, self.schedule, hp, env, collectives, math, sparse_min_world)
        self.model.quantize_mlp_fp8(bootstrap_down=True)
        self.log = logger or RunLogger(hp.run_id, env.master)
        self.train_loader = None
        # The first micro-batch of the next step is prepared (host work + asynchronous copy) at the end of a step,
        # while the device still runs that step's kernels; `_prefetch_state` is the loader cursor before it.
        pf = os.environ.get("MNG_PREFETCH_BATCH")           # default: on with a GPU; "1" / "0" force it
        self.prefetch_first_batch = pf == "1" or (pf is None and env.device.type == "cuda")
        self._prefetched = self._prefetch_state = None
        self.step = 0
        self.training_time_ms = 0.0
        self._status_host = self._status_event = None
        self.health = monitor_from_env(env)
        if use_cuda_graphs is None:
            use_cuda_graphs = env.device.type == "cuda" and os.environ.get("MNG_CUDA_GRAPHS", "1") != "0"
        self.graphs = None
        if use_cuda_graphs and env.device.type == "cuda":
            from .runtime.graphs import MicroStepGraphs
            self.graphs = MicroStepGraphs(self)
            self.manager.optimizer.keep_grads = True
        self._bigram_vocab = getattr(getattr(self.model, "cfg", None), "bigram_vocab_size", 0)
        self.model.train()

    # -- data ----------------------------------------------------------------------------
    def make_train_loader(self):
        st = self.schedule.stages[0]
        return TokenLoader(self.hp.train_files, st.batch_size, st.train_max_seq_len, self.env.grad_accum_steps,
                           True, self.env.rank, self.env.world_size, self.env.device, self._bigram_vocab)

    def make_val_loader(self):
        return TokenLoader(self.hp.val_files, self.hp.val_batch_size, -1, self.env.grad_accum_steps, False,
                           self.env.rank, self.env.world_size, self.env.device, self._bigram_vocab)

    # -- one optimizer step ----------------------------------------------------------------
    def micro_step(self, batch, step: int) -> torch.Tensor:
        m = self.manager
        m.sparse_index_update(step, batch.bigram_cpu)
        if m.row_mask_labels and self.model.training:
            m.optimizer.coll.mark_rows("bigram_embed", batch.bigram_inputs)
        if self.graphs is not None and self.model.training:
            m.sparse_index_share(step)
            return self.graphs.run(batch, m.get_forward_args())
        losses = self.model(batch.inputs, batch.targets, batch.cum_seqlens, batch.bigram_inputs, m.get_forward_args())
        loss = losses.sum() * self.env.grad_scale
        m.sparse_index_share(step)
        loss.backward()
        return loss.detach()

    def train_step(self, step: int | None = None) -> torch.Tensor:
        """Returns the (detached, device) sum-loss of the step's micro-batches."""
        step = self.step if step is None else step
        if self.health is not None:
            # peers that failed or stalled are noticed here, on the host, before any kernel that waits on them
            self.health.pre_step(step)
            with self.health.guard():
                self.check_device_status(sync=False)
                out = self._train_step(step)
                self._probe_status()
                return out
        self.check_device_status(sync=False)
        out = self._train_step(step)
        self._probe_status()
        return out

    # -- device status word ------------------------------------------------------------------
    # Every bounded device-side wait (peer barriers, mbarrier waits of the GEMM / attention kernels) records a code
    # in one status word when it gives up.  The word is read wherever the host synchronises anyway (validation,
    # checkpoint, end of run) and, without any synchronisation, one step late through an asynchronous copy into
    # pinned memory: replicas that diverged after a timed-out barrier stop the run instead of training on.
    def _probe_status(self):
        if self.env.device.type != "cuda":
            return
        from .ops import native
        if self._status_host is None:
            self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._status_event = torch.cuda.Event()
        elif not self._status_event.query():
            return                                            # the previous probe has not landed yet: keep it
        self._status_host.copy_(native.lib().status_tensor(torch.empty(0, device=self.env.device)).view(torch.int32),
                                non_blocking=True)
        self._status_event.record()

    def check_device_status(self, sync: bool = True):
        """Raises `DeviceWaitTimeout` if a kernel's bounded wait has expired.  `sync=False` only looks at the last
        asynchronous probe that has completed (no host-device synchronisation)."""
        if self.env.device.type != "cuda":
            return
        from .runtime.health import DeviceWaitTimeout, check_device
        if sync:
            ctx = self.health.guard() if self.health is not None else contextlib.nullcontext()
            with ctx:
                check_device(self.env.device)
            return
        if self._status_host is not None and self._status_event.query() and int(self._status_host[0]) != 0:
            code = int(self._status_host[0])
            self._status_host.zero_()
            raise DeviceWaitTimeout(f"device status word {code}: a bounded wait on a peer flag or barrier expired")

    def _train_step(self, step: int) -> torch.Tensor:
        if self.train_loader is None:
            self.train_loader = self.make_train_loader()
        m = self.manager
        m.advance_schedule(step)
        total = None
        for _ in range(self.env.grad_accum_steps):
            batch = self._take_batch()
            l = self.micro_step(batch, step)
            total = l if total is None else total + l
        m.step_optimizers(step)
        self.model.quantize_mlp_fp8(bootstrap_down=(step < 16))
        self.step = step + 1
        if self.prefetch_first_batch and step + 1 < self.schedule.total_steps:
            nxt, _ = self.schedule.lookup(step + 1)
            if nxt.batch_size == m.batch_size and nxt.train_max_seq_len == m.train_max_seq_len:
                state = self.train_loader.state_dict()
                try:
                    self._prefetched, self._prefetch_state = self.train_loader.next_batch(), state
                except StopIteration:                        # out of data: the step that needs the batch reports it
                    self.train_loader.load_state_dict(state)
                    self._prefetched = self._prefetch_state = None
        return total

    def _take_batch(self):
        m = self.manager
        if self._prefetched is not None:
            batch, self._prefetched, state = self._prefetched, None, self._prefetch_state
            if m.train_loader_send_args is None:
                return batch
            self.train_loader.load_state_dict(state)     # the batch geometry changed after all: rewind and redo
        batch = self.train_loader.next_batch(m.train_loader_send_args)
        m.train_loader_send_args = None
        return batch

    def loader_state(self):
        """Cursor of the training data for a checkpoint: the position before a prefetched, not yet used batch."""
        if self.train_loader is None:
            return None
        return self._prefetch_state if self._prefetched is not None else self.train_loader.state_dict()

    @torch.no_grad()
    def validate(self, val_tokens: int | None = None) -> torch.Tensor:
        hp, env = self.hp, self.env
        val_tokens = val_tokens or hp.val_tokens
        assert val_tokens % hp.val_batch_size == 0
        steps = env.grad_accum_steps * val_tokens // hp.val_batch_size
        self.check_device_status()                            # the caller has synchronised: the clock is stopped
        loader = self.make_val_loader()
        self.model.eval()
        tot = 0
        for _ in range(steps):
            b = loader.next_batch()
            tot = tot + self.model(b.inputs, b.targets, b.cum_seqlens, b.bigram_inputs, self.manager.get_forward_args()).mean()
        tot = tot / steps
        if dist.is_initialized() and env.world_size > 1:
            dist.all_reduce(tot, op=dist.ReduceOp.SUM)
            tot = tot / env.world_size
        self.model.train()
        return tot

    # -- checkpoint ------------------------------------------------------------------------
    def save_checkpoint(self, path: str | None = None):
        from .utils.checkpoint import save_checkpoint
        self.check_device_status()                            # never persist weights written after a timed-out wait
        return save_checkpoint(self, path)

    def load_checkpoint(self, path: str, strict: bool = True):
        from .utils.checkpoint import load_checkpoint
        return load_checkpoint(self, path, strict)

    # -- the whole run -----------------------------------------------------------------------
    def _sync(self):
        if self.env.device.type == "cuda":
            torch.cuda.synchronize()

    def warmup(self):
        """Run real steps at both ends of every stage transition so that every kernel variant
        and CUDA graph exists before the clock starts, then restore the initial state
        (`train_gpt.py:2264-2301`)."""
        m = self.manager
        init = dict(model=copy.deepcopy(self.model.state_dict()), optimizer=m.get_state())
        self._prefetched = self._prefetch_state = None
        self.train_loader = self.make_train_loader()
        val_loader = self.make_val_loader()
        trans = m.get_transition_steps()
        last = self.schedule.total_steps - 1
        steps = sorted({0, min(1, last)} | {s + o for s in trans for o in (-2, -1, 0, 1) if 2 <= s + o <= last})
        self.log.print0(f"Sampling steps {steps} for warmup", console=True)
        for step in steps:
            m.advance_schedule(step)
            self.model.eval()
            with torch.no_grad():
                b = val_loader.next_batch()
                self.model(b.inputs, b.targets, b.cum_seqlens, b.bigram_inputs, m.get_forward_args()).mean()
            self.model.train()
            for _ in range(self.env.grad_accum_steps):
                batch = self.train_loader.next_batch(m.train_loader_send_args)
                m.train_loader_send_args = None
                self.micro_step(batch, step)
            m.step_optimizers(step)
            self.model.quantize_mlp_fp8(bootstrap_down=True)
        self.log.print0("Resetting Model", console=True)
        if getattr(m.optimizer.coll, "fused", False) or m.optimizer.keep_grads:
            for p in self.model.parameters():       # gradients live in peer-mapped memory / captured graphs: keep the buffers
                if p.grad is not None:
                    p.grad.zero_()
        else:
            self.model.zero_grad(set_to_none=True)
        self.model.load_state_dict(init["model"])
        if self.graphs is not None:
            self.graphs.entries.clear()             # recapture after the reset: cheap, and immune to reallocated state
        m.reset(init["optimizer"])
        self.model.quantize_mlp_fp8(bootstrap_down=True)
        self.model.train()
        self._prefetched = self._prefetch_state = None
        self.train_loader = None
        self.step = 0

    def run(self, do_warmup: bool = True, start_step: int = 0):
        hp, env, m, log = self.hp, self.env, self.manager, self.log
        if do_warmup and start_step == 0:
            self.warmup()
        if self.train_loader is None:
            self.train_loader = self.make_train_loader()
        total = self.schedule.total_steps if not hp.max_steps else min(hp.max_steps, self.schedule.total_steps)
        from .data.prefix import build_prefix_table
        self._sync()
        t0 = time.perf_counter()
        if start_step == 0:
            self.model.prefix_table.copy_(build_prefix_table(self.model.vocab_size))
        val_loss = None
        for step in range(start_step, total + 1):
            last = step == total
            m.advance_schedule(step)
            if last or (hp.val_loss_every > 0 and step % hp.val_loss_every == 0):
                if last and total == self.schedule.total_steps:
                    m.apply_final_ws_ext()
                self._sync()
                self.training_time_ms += 1000 * (time.perf_counter() - t0)
                val_loss = float(self.validate())
                log.print0(f"step:{step}/{total} val_loss:{val_loss:.4f} train_time:{self.training_time_ms:.0f}ms "
                           f"step_avg:{self.training_time_ms / max(step, 1):.2f}ms", console=True)
                self._sync()
                t0 = time.perf_counter()
            if last:
                if hp.save_checkpoint:
                    self.save_checkpoint()
                break
            self.train_step(step)
            approx = self.training_time_ms + 1000 * (time.perf_counter() - t0)
            log.print0(f"step:{step + 1}/{total} train_time:{approx:.0f}ms step_avg:{approx / (step + 1):.2f}ms", console=True)
        self.check_device_status()
        if env.device.type == "cuda":
            log.print0(f"peak memory allocated: {torch.cuda.max_memory_allocated() // 1024 // 1024} MiB "
                       f"reserved: {torch.cuda.max_memory_reserved() // 1024 // 1024} MiB", console=True)
        return val_loss
