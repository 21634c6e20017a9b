"""Per-kernel device-time table of the training step (torch.profiler, CUDA activities only).

    python bench/profile_step.py [--micro-steps 2] [--rows 60]

Builds the track-1 trainer at its stage-2 configuration on synthetic data, warms up (including the CUDA-graph
capture of the micro-step), then profiles `--micro-steps` micro-batches plus one optimizer step and prints the
kernels sorted by total device time.  Times under the profiler are for shares, not for absolute claims."""
import argparse
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def phases(tr, env, n_steps):
    """Device time (CUDA events, this rank) of: first input copy + bookkeeping, micro-steps, optimizer step, FP8 weight
    refresh; averaged separately over Adam steps (odd) and NorMuon-only steps (even)."""
    import json
    import torch
    m = tr.manager
    rows, step = [], 850
    for _ in range(n_steps):
        env.barrier()
        torch.cuda.synchronize()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        e[0].record()
        m.advance_schedule(step)
        b = tr.train_loader.next_batch()
        e[1].record()
        for i in range(env.grad_accum_steps):
            tr.micro_step(b, step)
            if i + 1 < env.grad_accum_steps:
                b = tr.train_loader.next_batch()
        e[2].record()
        m.step_optimizers(step)
        e[3].record()
        tr.model.quantize_mlp_fp8(bootstrap_down=False)
        e[4].record()
        torch.cuda.synchronize()
        rows.append(dict(adam=step % 2, inputs=e[0].elapsed_time(e[1]), micro_steps=e[1].elapsed_time(e[2]),
                         optimizer=e[2].elapsed_time(e[3]), fp8_refresh=e[3].elapsed_time(e[4]), total=e[0].elapsed_time(e[4])))
        step += 1
    if env.master:
        for parity, name in ((1, "adam step"), (0, "normuon-only step")):
            sel = [r for r in rows if r["adam"] == parity]
            if sel:
                print(name, json.dumps({k: round(sum(r[k] for r in sel) / len(sel), 3) for k in sel[0] if k != "adam"}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--micro-steps", type=int, default=2)
    ap.add_argument("--rows", type=int, default=60)
    ap.add_argument("--eager", action="store_true", help="profile the eager micro-step instead of the graph replay")
    ap.add_argument("--phases", type=int, default=0,
                    help="instead of the kernel table: CUDA-event time of the phases of N full steps (works under torchrun)")
    ap.add_argument("--ops", type=int, default=0,
                    help="instead of the kernel table: the N most expensive framework (aten) ops of one eager micro-step, "
                         "grouped by input shapes -- what is left outside the native kernels")
    a = ap.parse_args()
    if a.ops:
        a.eager = True
    import torch
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.runtime.dist import init_distributed
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    env = init_distributed(accum_base=8)
    sched = TrainingSchedule(track1_stages(), 1270, 15, cooldown_frac=0.6)
    root = "/tmp/mng_profile_data"
    if env.master:
        write_synthetic_corpus(root, train_tokens=12_000_000 if not a.phases else 393216 * (a.phases + 8), val_tokens=1_000_000,
                               seed=0, max_doc_len=2048)
    env.barrier()
    hp = Hyperparameters(data_path=root, val_loss_every=0)
    tr = Trainer(track1_model(262144), sched, hp, env, use_cuda_graphs=not a.eager,
                 logger=RunLogger("profile", True, log_dir="/tmp/mng_logs", quiet=True))
    for b0, _ in sched.boundaries[:3]:
        tr.manager.advance_schedule(b0)
    tr.manager.optimizer.split_embed = True
    tr.train_loader = tr.make_train_loader()
    tr.train_loader.reparameterise(393216, 2048, env.grad_accum_steps)
    m = tr.manager

    def micro(step):
        return tr.micro_step(tr.train_loader.next_batch(), step)

    for _ in range(4):
        micro(848)
    m.step_optimizers(849)
    tr.model.quantize_mlp_fp8(False)
    torch.cuda.synchronize()
    if a.phases:
        return phases(tr, env, a.phases)
    if a.ops:
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
            micro(851)
            torch.cuda.synchronize()
        evs = [e for e in prof.key_averages(group_by_input_shape=True) if e.key.startswith("aten::") and e.self_device_time_total > 0]
        evs.sort(key=lambda e: -e.self_device_time_total)
        print(f"aten ops of one eager micro-step: {sum(e.self_device_time_total for e in evs) / 1e3:.2f} ms of device time")
        for e in evs[:a.ops]:
            print(f"{e.self_device_time_total / 1e3:8.3f} ms {e.count:4d} x {e.self_device_time_total / e.count:8.1f} us  "
                  f"{e.key:28s} {str(e.input_shapes)[:110]}")
        return
    t = time.time()
    for _ in range(4):
        micro(850)
    torch.cuda.synchronize()
    print(f"micro-step wall ms (unprofiled): {(time.time() - t) / 4 * 1e3:.2f}")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.micro_steps):
            micro(851)
        m.step_optimizers(851)
        tr.model.quantize_mlp_fp8(False)
        torch.cuda.synchronize()
    ks = [e for e in prof.key_averages() if e.device_type == DeviceType.CUDA]
    ks.sort(key=lambda e: -e.self_device_time_total)
    tot = sum(e.self_device_time_total for e in ks)
    print(f"device time of {a.micro_steps} micro-steps + 1 optimizer step (Adam step): {tot / 1e3:.2f} ms")
    for e in ks[:a.rows]:
        print(f"{e.self_device_time_total / 1e3:9.3f} ms {100 * e.self_device_time_total / tot:5.1f}% {e.count:5d} x "
              f"{e.self_device_time_total / max(e.count, 1):9.1f} us  {e.key[:120]}")
    fused.check_status()


if __name__ == "__main__":
    main()
