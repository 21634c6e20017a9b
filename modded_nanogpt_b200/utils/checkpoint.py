"""Checkpoint save / resume.

The `model` entry keeps the reference's layout (`train_gpt.py:2348-2352`): the state_dict of
the model with the same keys, shapes and dtypes; keys may carry the `_orig_mod.` prefix that a
compiled module's state_dict has, which is accepted on load and optionally written on save.
Added on top of what the reference stores: per-rank optimizer shards keyed by parameter label,
the step, the loader cursor, rotary (YaRN) state, and the schedule position, so that a run
can actually be resumed; every rank writes its own optimizer shard file.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

PREFIX = "_orig_mod."


def strip_prefix(sd: dict) -> dict:
    return {(k[len(PREFIX):] if k.startswith(PREFIX) else k): v for k, v in sd.items()}


def add_prefix(sd: dict) -> dict:
    return {PREFIX + k: v for k, v in sd.items()}


def adapt_bank(saved: torch.Tensor, want_shape) -> torch.Tensor:
    """Banks are padded to a multiple of the world size, so a checkpoint written at another world
    size differs in its leading dimension: truncate the padding or zero-extend it."""
    if tuple(saved.shape) == tuple(want_shape):
        return saved
    assert saved.shape[1:] == tuple(want_shape[1:]), f"incompatible shapes {tuple(saved.shape)} vs {tuple(want_shape)}"
    out = saved.new_zeros(want_shape)
    n = min(saved.shape[0], want_shape[0])
    out[:n] = saved[:n]
    return out


def load_model_state(model, sd: dict, strict: bool = True):
    sd = strip_prefix(sd)
    own = model.state_dict()
    fixed = {}
    for k, v in sd.items():
        if k in own and tuple(v.shape) != tuple(own[k].shape) and v.ndim == own[k].ndim and v.ndim >= 1:
            v = adapt_bank(v, own[k].shape)
        fixed[k] = v
    return model.load_state_dict(fixed, strict=strict)


def checkpoint_dir(trainer) -> str:
    return os.path.join("logs", trainer.hp.run_id)


def save_checkpoint(trainer, path: str | None = None, compiled_prefix: bool = True) -> str:
    env, step = trainer.env, trainer.step
    d = path or checkpoint_dir(trainer)
    os.makedirs(d, exist_ok=True)
    m = trainer.manager
    # Adam parameters are stepped every other step, so after an even step their gradients are still
    # pending: they are part of the training state
    pending = {l: p.grad.detach().cpu().clone() for l, p in m.optimizer.params.items()
               if p.grad is not None and bool(p.grad.ne(0).any())}
    shard = dict(step=step, optimizer=m.optimizer.state_dict(), rank=env.rank, world_size=env.world_size,
                 loader=trainer.loader_state(),
                 pending_grads=pending)
    torch.save(shard, os.path.join(d, f"optim_step{step:06d}_rank{env.rank}.pt"))
    main = os.path.join(d, f"state_step{step:06d}.pt")
    if env.master:
        msd = trainer.model.state_dict()
        log = dict(step=step, code="", model=add_prefix(msd) if compiled_prefix else msd,
                   optimizer=shard["optimizer"],
                   yarn=trainer.model.yarn.state_dict(), yarn_paired=trainer.model.yarn_paired_head.state_dict(),
                   schedule=dict(ws_short=m.ws_short, ws_long=m.ws_long, batch_size=m.batch_size,
                                 train_max_seq_len=m.train_max_seq_len),
                   training_time_ms=trainer.training_time_ms, world_size=env.world_size,
                   prefix_table=trainer.model.prefix_table.cpu())
        tmp = main + ".tmp"
        torch.save(log, tmp)
        os.replace(tmp, main)
    if dist.is_initialized():
        dist.barrier()
    return main


def load_checkpoint(trainer, main_path: str, strict: bool = True) -> int:
    """Restores model, optimizer shard of this rank, loader cursor, rotary and schedule state.
    Returns the step to continue from.

    The optimizer shards are per rank, so they only fit a job of the same world size.  When this rank's shard is
    missing or was written by a different world size, `strict=True` (default) raises instead of resuming with
    zeroed moments and a rewound data cursor; `strict=False` loads the model only and says so loudly."""
    log = torch.load(main_path, map_location="cpu", weights_only=False)
    if not isinstance(log, dict) or "model" not in log or "step" not in log:
        raise ValueError(f"{main_path}: not a checkpoint of this framework or of the reference")
    env = trainer.env
    step = int(log["step"])
    load_model_state(trainer.model, log["model"])
    m = trainer.manager
    d = os.path.dirname(main_path)
    shard_path = os.path.join(d, f"optim_step{step:06d}_rank{env.rank}.pt")
    if os.path.exists(shard_path) and log.get("world_size", env.world_size) == env.world_size:
        shard = torch.load(shard_path, map_location="cpu", weights_only=False)
        m.optimizer.load_state_dict(shard["optimizer"])
        for l, g in shard.get("pending_grads", {}).items():
            if l in getattr(m, "row_mask_labels", ()):           # restored rows count as touched: mark all of them
                m.optimizer.coll.row_masks[l]["touched"].fill_(1)
            p = m.optimizer.params[l]
            if p.grad is None:
                p.grad = g.to(p.device, p.dtype)
            else:
                p.grad.copy_(g)
        if shard.get("loader") is not None:
            if trainer.train_loader is None:
                trainer.train_loader = trainer.make_train_loader()
            trainer._prefetched = trainer._prefetch_state = None
            trainer.train_loader.load_state_dict(shard["loader"])
    elif (env.world_size == 1 and log.get("world_size", 1) == 1 and "optimizer" in log
          and "state" in log["optimizer"]):
        m.optimizer.load_state_dict(log["optimizer"])
        print(f"[checkpoint] {main_path}: no per-rank shard, optimizer state taken from the main file; "
              "the data cursor restarts at the first shard", flush=True)
    else:
        why = (f"written by world_size {log.get('world_size')}, this job has {env.world_size}"
               if log.get("world_size", env.world_size) != env.world_size else f"{shard_path} is missing")
        msg = (f"{main_path}: optimizer state, pending Adam gradients and the loader cursor cannot be restored ({why})")
        if strict:
            raise RuntimeError(msg + "; pass strict=False to resume from the model weights alone")
        print(f"[checkpoint] WARNING: {msg}; continuing from step {step} with fresh optimizer state and data from "
              "the first shard", flush=True)
    if "yarn" in log:
        trainer.model.yarn.load_state_dict(log["yarn"])
        trainer.model.yarn_paired_head.load_state_dict(log["yarn_paired"])
    if "schedule" in log:
        s = log["schedule"]
        m.ws_short, m.ws_long = s["ws_short"], s["ws_long"]
        m.batch_size, m.train_max_seq_len = s["batch_size"], s["train_max_seq_len"]
    if "prefix_table" in log:
        trainer.model.prefix_table.copy_(log["prefix_table"])
    trainer.training_time_ms = float(log.get("training_time_ms", 0.0))
    trainer.step = step
    trainer.model.quantize_mlp_fp8(bootstrap_down=True)
    return step
