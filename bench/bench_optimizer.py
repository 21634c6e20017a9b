"""Optimizer-step micro-benchmark: NorMuon (Polar Express) + Adam over all track-1 parameters with their
collectives, on random gradients.  Compares the fused NVLink path (update kernels that read the peers'
gradient shards and store the new weights to every peer) with the NCCL path (reduce-scatter / all-reduce /
all-gather around the same update kernels).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port 29533 \
        bench/bench_optimizer.py --steps 20

Mode `fused` uses `multimem.ld_reduce` / `multimem.st` through the NVSwitch multicast address when there is one,
`fused_p2p` plain peer loads and stores.  Mode `fused_sparse` gives the bigram table a gradient with 98,304 random touched rows and lets the fused Adam kernel pull
only those from the peers; the other modes reduce that table densely.
`--impl reference` times the unmodified reference's `NorMuonAndAdam.step` on the same parameters instead.
Prints one JSON line per communication mode: device time (CUDA events, max over ranks) of odd steps
(NorMuon + Adam) and even steps (NorMuon only)."""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--modes", default="nccl,fused")
    ap.add_argument("--trace", action="store_true",
                    help="after the timing, print rank 0's device timeline (start offset, duration, kernel) of one Adam step")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"],
                    help="reference: the unmodified reference optimizer (NCCL + its compiled update math) on the same shapes")
    a = ap.parse_args()
    if a.impl == "reference":
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        ref = os.path.join(root, "baseline", "_ref")
        if not os.path.exists(os.path.join(ref, "train_gpt.py")):
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not staged on this machine"}))
            return
        from baseline.reference_driver import reference_optimizer_step_ms
        out = reference_optimizer_step_ms(ref, a.steps)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(out), flush=True)
        return
    import torch
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    from modded_nanogpt_b200.utils.timing import max_over_ranks
    env = init_distributed(accum_base=8)
    for mode in a.modes.split(","):
        if mode != "nccl" and env.world_size == 1:
            continue
        # modes: nccl | fused (multimem when the arena has a multicast address) | fused_p2p (plain peer loads/stores) |
        #        fused_sparse / fused_p2p_sparse (row masks on the bigram table)
        os.environ["MNG_COMM"] = "nccl" if mode == "nccl" else "fused"
        os.environ["MNG_MULTIMEM"] = "0" if "p2p" in mode else "1"
        os.environ["MNG_SPARSE_PULL"] = "1" if mode.endswith("sparse") else "0"
        sched = TrainingSchedule(track1_stages(), 1270, 15, cooldown_frac=0.6)
        hp = Hyperparameters(val_loss_every=0, seed=0)
        tr = Trainer(track1_model(hp.val_batch_size // 8), sched, hp, env, use_cuda_graphs=False, sparse_min_world=1 << 30,
                     logger=RunLogger(f"optbench_{mode}", env.master, log_dir="/tmp/mng_logs", quiet=True))
        tr.manager.advance_schedule(848)
        tr.manager.optimizer.split_embed = True
        g = torch.Generator(device="cuda").manual_seed(env.rank)
        params = list(tr.model.parameters())

        bigram = tr.model.bigram_embed.weight

        def fill():
            for p in params:
                if p.grad is None:
                    p.grad = torch.empty_like(p)
                p.grad.copy_((torch.randn(p.shape, generator=g, device="cuda", dtype=torch.float32) * 1e-3).to(p.dtype))
            if mode.endswith("sparse"):
                # the bigram gradient as training leaves it: rows of the 2 x 49,152 tokens since the last Adam step
                rows = torch.randint(0, bigram.shape[0], (98304,), generator=g, device="cuda")
                keep = torch.zeros(bigram.shape[0], dtype=torch.bool, device="cuda")
                keep[rows] = True
                bigram.grad.mul_(keep[:, None])
                tr.manager.optimizer.coll.mark_rows("bigram_embed", rows)

        times = {0: [], 1: []}
        for step in range(849, 849 + a.steps + 4):
            fill()
            env.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            tr.manager.step_optimizers(step)
            e1.record()
            torch.cuda.synchronize()
            if step >= 853:
                times[step % 2].append(max_over_ranks(e0.elapsed_time(e1)))
        fused.check_status()
        n_hidden = sum(p.numel() for l, p in tr.manager.optimizer.params.items() if tr.manager.optimizer.cfgs[l].optim == "normuon")
        if env.master:
            med = lambda v: sorted(v)[len(v) // 2]
            print(json.dumps({"mode": mode, "n_gpus": env.world_size, "multicast": bool(getattr(tr.manager.optimizer.coll, "mc_base", 0)), "adam_step_ms": round(med(times[1]), 3),
                              "muon_only_step_ms": round(med(times[0]), 3), "normuon_params": n_hidden,
                              "all_params": sum(p.numel() for p in params)}), flush=True)
        if a.trace:
            from torch.profiler import ProfilerActivity, profile
            fill()
            env.barrier()
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
                tr.manager.step_optimizers(849 + a.steps + 4 + (a.steps % 2 == 1))      # an odd (Adam) step
                torch.cuda.synchronize()
            if env.master:
                evs = sorted((e for e in prof.events() if e.device_type.name == "CUDA"), key=lambda e: e.time_range.start)
                t0 = evs[0].time_range.start
                print(f"# {mode}: {len(evs)} device activities, span {(evs[-1].time_range.end - t0) / 1e3:.3f} ms, "
                      f"busy {sum(e.time_range.end - e.time_range.start for e in evs) / 1e3:.3f} ms")
                for e in evs:
                    print(f"{(e.time_range.start - t0):9.1f} us  {(e.time_range.end - e.time_range.start):8.1f} us  {e.name[:90]}")
        del tr
        torch.cuda.empty_cache()
    shutdown()


if __name__ == "__main__":
    main()
