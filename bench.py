"""Headline benchmark: train tokens/s and ms/step of the track-1 GPT at the stage-2 batch
(393,216 tokens per optimizer step = 8 micro-batches of 48x1024 packed tokens, split over the
ranks: grad_accum = 8 // N), bf16 with FP8 MLP forward and lm_head, synthetic Zipf/EoS token
streams, random-init weights.  Every step is a full training step: forward, backward, optimizer
(NorMuon every step, Adam on odd steps), FP8 weight refresh.

    python bench.py --gpus 1 --steps 10 --warmup 3
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29511 bench.py --gpus 8 --steps 10 --warmup 3

Two timed regions of K steps each, both bracketed by barrier + synchronize and timed with CUDA
events, max over ranks; both go through `Trainer.train_step`, which packs every micro-batch on the
host and copies it from pinned memory inside the timed region (the reference arm does the same):
  * `value`  - the step loss stays on the device;
  * `e2e`    - additionally reads the step loss back to the host after every step.
Inputs (K*393,216 tokens of ids/targets/hashes per region) are far larger than L2.

`--mlp bf16` runs the MLP forward in bf16 (the lm_head + loss path stays FP8): the precision the
reference arm runs at on this GPU, for a like-for-like pair next to the FP8 headline.
`--stage 0|1|2` times another stage of the schedule (131,072 / 262,144 / 393,216 tokens per step).
At N > 1 the line carries `params_identical`: a bitwise checksum of every parameter compared
across ranks after the warm-up and after the timed steps.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TOKENS_PER_S = None     # the reference publishes no B200 number for this config


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--stage", type=int, default=2, help="schedule stage whose batch/window settings are timed")
    ap.add_argument("--tokens-per-gpu", type=int, default=0, help="override the micro-batch size (smoke runs only)")
    ap.add_argument("--track", type=int, default=1, choices=[1, 2],
                    help="2 = track-2 model at its 524,288-token plateau batch (not the headline)")
    ap.add_argument("--mlp", default="fp8", choices=["fp8", "bf16"], help="precision of the MLP forward (own arm)")
    return ap.parse_args()


def reference_arm(args):
    from baseline.run_reference import run_reference
    try:
        out = run_reference(args)
    except Exception as e:  # noqa: BLE001 - a failed reference run is reported as a line, not as a crash
        import traceback
        traceback.print_exc()
        out = {"impl": "reference", "unavailable": f"reference run failed: {type(e).__name__}: {str(e)[:300]}"}
        if int(os.environ.get("RANK", "0")) != 0:
            out = {}
    if out:
        print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import torch.distributed as dist
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    from modded_nanogpt_b200.ops import fused, native
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    from modded_nanogpt_b200.utils.timing import ClockSampler, max_over_ranks

    assert torch.cuda.is_available(), "bench.py needs a GPU"
    env = init_distributed(accum_base=8)
    assert env.world_size == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={env.world_size}"
    native.available(required=True)

    model = None
    if args.track == 2:
        from modded_nanogpt_b200.config import track2_hyperparameters, track2_schedule
        from modded_nanogpt_b200.models.gpt_medium import GPTMedium
        hp2 = track2_hyperparameters()
        sched = track2_schedule(hp2)
        stages = sched.stages
        args.stage = next(i for i, s in enumerate(stages) if s.batch_size == 524288)
    else:
        stages = track1_stages()
    if args.tokens_per_gpu:
        for s in stages:
            s.batch_size = args.tokens_per_gpu * 8
    if args.track == 1:
        sched = TrainingSchedule(stages, 1270, 15, cooldown_frac=0.60)
    first = sched.boundaries[args.stage][0] + 1               # 848: inside stage 2, after the embed split
    stage = stages[args.stage]
    K, W = args.steps, args.warmup
    n_steps = W + 2 * K
    root = f"/tmp/mng_bench_{stage.batch_size}_{n_steps}"
    if env.master:
        write_synthetic_corpus(root, train_tokens=int(stage.batch_size * (n_steps + 2) * 1.02) + 1_000_000,
                               val_tokens=1_000_000, seed=0, max_doc_len=stage.train_max_seq_len)
    env.barrier()
    if args.track == 2:
        hp = track2_hyperparameters(data_path=root, val_loss_every=0, seed=0)
        eval_seq = hp.val_batch_size // 8
        torch.manual_seed(0)
        model = GPTMedium(max_seq_len=eval_seq, world_size=env.world_size, grad_scale=env.grad_scale, use_fp8=True,
                          eval_seq_len=eval_seq)
    else:
        hp = Hyperparameters(data_path=root, val_loss_every=0, seed=0, disable_fp8=(args.mlp == "bf16"))
    if model is not None and args.mlp == "bf16":
        model.use_fp8 = False
    tr = Trainer(None if model is not None else track1_model(hp.val_batch_size // 8), sched, hp, env, model=model,
                 logger=RunLogger(f"bench_{os.getpid()}", env.master, log_dir="/tmp/mng_logs", quiet=True))
    tr.model.fp8_head = True                                  # as the reference: the loss path is FP8 in both MLP modes
    # enter the timed stage the way a run would: windows / YaRN state of the earlier stages applied
    for b0, _ in sched.boundaries[:args.stage + 1]:
        tr.manager.advance_schedule(b0)
    tr.manager.optimizer.split_embed = first > sched.split_step
    tr.train_loader = tr.make_train_loader()
    tr.train_loader.reparameterise(stage.batch_size, stage.train_max_seq_len, env.grad_accum_steps)
    tr.manager.train_loader_send_args = None

    step = first
    for _ in range(W):
        tr.train_step(step)
        step += 1
    torch.cuda.synchronize()
    fused.check_status()

    def timed(region):
        nonlocal step
        env.barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(env.local_rank).start() if env.master else None
        replayed = lambda: tr.graphs.replayed_launches if tr.graphs is not None else 0
        launches0 = native.lib().launch_count() + replayed()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        out = region()
        e1.record()
        env.barrier()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        clocks = sampler.stop() if sampler else None
        ms = max_over_ranks(e0.elapsed_time(e1))
        return ms, max_over_ranks(wall * 1e3), native.lib().launch_count() + replayed() - launches0, clocks, out

    def params_checksum_identical():
        """Bitwise: every parameter's bytes summed as integers, compared across ranks."""
        if env.world_size == 1:
            return None
        sums = torch.stack([p.detach().contiguous().view(torch.int16 if p.element_size() == 2 else torch.int32)
                            .to(torch.int64).sum() for p in tr.model.parameters()])
        lo, hi = sums.clone(), sums.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        return bool(torch.equal(lo, hi))

    same_after_warmup = params_checksum_identical()

    # ---- region 1: the loss stays on the device ---------------------------------------------------
    def region_device():
        nonlocal step
        for _ in range(K):
            tr.train_step(step)
            step += 1

    dev_ms, _, launches, clocks, _ = timed(region_device)

    # ---- region 2: end to end through the public API -------------------------------------------
    h2d = d2h = 0

    def region_e2e():
        nonlocal step, h2d, d2h
        losses = []
        for _ in range(K):
            loss = tr.train_step(step)
            losses.append(float(loss))            # device -> host read of the step's result
            d2h += 4
            step += 1
        return losses

    tr.train_loader.count_bytes = True
    e2e_ms, e2e_wall_ms, _, clocks2, losses = timed(region_e2e)
    h2d = tr.train_loader.bytes_copied
    fused.check_status()
    same_at_end = params_checksum_identical()

    tokens = stage.batch_size * K
    value = tokens / (dev_ms / 1e3)
    e2e_value = tokens / (max(e2e_ms, e2e_wall_ms) / 1e3)
    if env.master:
        out = {
            "metric": (f"train tokens/s, track-1 GPT, stage-{args.stage} batch ({stage.batch_size} tok/step)" if args.track == 1 else
                       "train tokens/s, track-2 GPT, plateau batch (524288 tok/step)"), "value": value, "unit": "tokens/s",
            "n_gpus": env.world_size, "steps": K, "warmup": W, "ms_per_step": dev_ms / K, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": (value / BASELINE_TOKENS_PER_S) if BASELINE_TOKENS_PER_S else None,
            "dtype": ("bf16 (fp8 e4m3 MLP forward and lm_head)" if args.mlp == "fp8" else "bf16 (bf16 MLP; fp8 e4m3 lm_head)"), "data": "synthetic Zipf(1.1) ids, EoS-delimited lognormal docs; random-init weights",
            "impl": "ours",
            "config": {"model": ("track-1 GPT (11L, d768, 6x128 heads, vocab 50304)" if args.track == 1 else
                                 "track-2 GPT (16L, d1024, 8x128 heads, vocab 50304)"), "global_batch": stage.batch_size,
                       "seq_len": stage.train_max_seq_len, "tokens_per_gpu_per_microbatch": stage.batch_size // 8,
                       "grad_accum": env.grad_accum_steps, "parallelism": f"dp{env.world_size}",
                       "windows": [w * hp.block_size for w in stage.window_sizes], "first_step": first,
                       "l2_policy": "inputs larger than L2 (fresh token batches every step)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": max(e2e_ms, e2e_wall_ms) / K,
                    "h2d_bytes_per_step": h2d // K, "d2h_bytes_per_step": d2h // K, "last_loss": losses[-1]},
            "gpu_launches": launches,
            "params_identical": (None if same_at_end is None else bool(same_after_warmup and same_at_end)),
            "clocks": clocks,
            "clocks_e2e": clocks2,
        }
        print(json.dumps(out), flush=True)
    shutdown()


if __name__ == "__main__":
    main()
