"""Worker for the multi-GPU tests (launched with torch.distributed.run, one rank per GPU).

mode "optim": the fused NVLink optimizer path (peer-read reduce-scatter + NorMuon/Adam + peer-store
all-gather) against the NCCL path with the same per-shard kernels, on identical random gradients.
mode "train": a few real training steps with each path; losses must agree.
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def build(env, comm):
    from modded_nanogpt_b200.config import Hyperparameters, ModelConfig, TrainingSchedule, track1_stages
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    os.environ["MNG_COMM"] = comm
    cfg = ModelConfig(vocab_size=4000, max_seq_len=4096, bigram_vocab_size=8192, bigram_sign_table_rows=64)
    stages = track1_stages()
    for s in stages:
        s.batch_size = 2048 * 8
    sched = TrainingSchedule(stages, 1270, 15, cooldown_frac=0.6)
    hp = Hyperparameters(val_loss_every=0, seed=0, disable_fp8=False)
    return Trainer(cfg, sched, hp, env, logger=RunLogger(f"mg_{comm}", env.master, log_dir="/tmp/mng_logs", quiet=True))


def main():
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    mode = sys.argv[1] if len(sys.argv) > 1 else "optim"
    env = init_distributed(accum_base=8)
    results = {}
    multicast = False
    for name, comm, mm in (("nccl", "nccl", "0"), ("fused_p2p", "fused_strict", "0"), ("fused_multimem", "fused_strict", "1")):
        os.environ["MNG_MULTIMEM"] = mm        # "1": multimem.ld_reduce / multimem.st where the arena has a multicast address
        tr = build(env, comm)
        opt = tr.manager.optimizer
        if name == "fused_p2p":
            assert opt.coll.mc_base == 0
        if name == "fused_multimem":
            multicast = opt.coll.mc_base != 0
        assert getattr(opt.coll, "fused", False) == (comm != "nccl")
        assert bool(tr.manager.row_mask_labels) == (comm != "nccl" and env.world_size > 1)
        with torch.no_grad():      # away from the zero inits
            g = torch.Generator(device="cuda").manual_seed(1)
            for p in tr.model.parameters():
                if p.abs().max() == 0:
                    p.copy_(torch.randn(p.shape, generator=g, device="cuda", dtype=torch.float32) * 0.02)
        for step in (1, 2, 3):
            g = torch.Generator(device="cuda").manual_seed(100 * step + env.rank)
            for p in tr.model.parameters():
                grad = (torch.randn(p.shape, generator=g, device="cuda", dtype=torch.float32) * 1e-3).to(p.dtype)
                if p is tr.model.bigram_embed.weight:
                    # an embedding gradient: only the rows of the tokens seen are non-zero, and the fused path is
                    # told which (it pulls just those rows from the peers)
                    rows = torch.randint(0, p.shape[0], (p.shape[0] // 3,), generator=g, device="cuda")
                    keep = torch.zeros(p.shape[0], dtype=torch.bool, device="cuda")
                    keep[rows] = True
                    grad = grad * keep[:, None]
                    if tr.manager.row_mask_labels:
                        opt.coll.mark_rows("bigram_embed", rows)
                if p.grad is None:
                    p.grad = grad
                else:
                    p.grad.copy_(grad)
            tr.manager.advance_schedule(step)
            tr.manager.step_optimizers(step)
        torch.cuda.synchronize()
        fused.check_status()
        results[name] = {n: p.detach().float().clone() for n, p in tr.model.named_parameters()}
        # every rank must hold identical parameters after the gathers
        for n, p in tr.model.named_parameters():
            ref = p.detach().clone()
            dist.broadcast(ref, 0)
            assert torch.equal(ref, p.detach()), f"{name}: ranks disagree on {n}"
        del tr
    worst = 0.0
    for name in ("fused_p2p", "fused_multimem"):
        for n, a in results["nccl"].items():
            b = results[name][n]
            err = ((a - b).norm() / a.norm().clamp_min(1e-12)).item()
            worst = max(worst, err)
            assert err < 2e-2, (name, n, err)
    if env.master:
        print(f"MULTI_GPU_OK world={env.world_size} worst_rel_diff={worst:.3e} multicast={multicast}", flush=True)
    shutdown()


if __name__ == "__main__":
    main()
