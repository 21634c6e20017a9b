"""Loss-curve parity over the first optimizer steps of a track-1 run, on identical initial weights and identical
batches, one GPU (grad-accum 8, 131,072 tokens per step: the schedule's first stage).

    python baseline/loss_curve.py reference --steps 10 --dump /tmp/curve      # the unmodified reference (compiled)
    python baseline/loss_curve.py ours --steps 10 --dump /tmp/curve [--mlp bf16]

`reference` runs `baseline/_ref/train_gpt.py`'s own step (advance_schedule, 8 x forward/backward, step_optimizers,
quantize) from its seed-0 initialisation on seed-0 synthetic shards and writes the initial state_dict, the prefix
table, every micro-batch it consumed and the per-step losses to the dump directory.  `ours` loads those, replays the
same micro-batches through `Trainer.micro_step` / `TrainingManager.step_optimizers` and prints both curves and their
per-step relative difference as one JSON line."""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def run_reference(a):
    import torch
    from baseline.reference_driver import load_track1_definitions
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    root = "/tmp/mng_curve_data"
    batch = 8 * 2048 * 8
    write_synthetic_corpus(root, train_tokens=int(batch * (a.steps + 3) * 1.05) + 2_000_000, val_tokens=3_000_000, seed=0,
                           max_doc_len=896, shard_tokens=max(2_000_000, batch * (a.steps + 3) // 2))
    os.environ["DATA_PATH"] = root
    ns = load_track1_definitions(ref_dir)
    dist, nn = ns["dist"], ns["nn"]
    ga, rargs = ns["grad_accum_steps"], ns["args"]
    torch.manual_seed(0)
    model = ns["GPT"](vocab_size=50257, num_layers=11, num_heads=6, head_dim=128, model_dim=768,
                      max_seq_len=rargs.val_batch_size // ga).cuda()
    for m in model.modules():
        if isinstance(m, (nn.Embedding, nn.Linear)):
            m.weight.data = m.weight.data.bfloat16()
    for name in ("ve_gate_bank", "qk_bank", "vo_bank", "mlp_bank", "mudd_w1", "mudd_w2", "mudd_b2", "mudd_gate_w1",
                 "mudd_gate_w2", "mudd_gate_b2"):
        getattr(model, name).data = getattr(model, name).data.bfloat16()
    model.prefix_table.copy_(ns["build_prefix_table"](model.vocab_size))
    os.makedirs(a.dump, exist_ok=True)
    torch.save({k: v.detach().cpu() for k, v in model.state_dict().items()}, os.path.join(a.dump, "init.pt"))
    torch.save(model.prefix_table.cpu(), os.path.join(a.dump, "prefix.pt"))
    model.quantize_mlp_fp8(bootstrap_down=True)
    ns["model"] = model
    cmodel = torch.compile(model, dynamic=False, fullgraph=True)
    ns["model"] = cmodel
    tm = ns["TrainingManager"](cmodel)
    stage = ns["TRAINING_STAGES"][0]
    loader = ns["distributed_data_generator"](rargs.train_files, stage.batch_size, stage.train_max_seq_len, grad_accum_steps=ga)
    cmodel.train()
    grad_scale = ns["grad_scale"]
    losses, batches = [], []
    for step in range(a.steps):
        tm.advance_schedule(step)
        total = None
        for _ in range(ga):
            inputs, targets, cum_seqlens, bigram_inputs, bigram_cpu = loader.send(tm.train_loader_send_args)
            batches.append(tuple(t.cpu().clone() for t in (inputs, targets, cum_seqlens, bigram_inputs)))
            tm.sparse_index_update(step, bigram_cpu)
            loss = cmodel(inputs, targets, cum_seqlens, bigram_inputs, tm.get_forward_args()).sum() * grad_scale
            tm.sparse_index_share(step)
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
        tm.step_optimizers(step)
        cmodel.quantize_mlp_fp8(bootstrap_down=(step < 16))
        losses.append(float(total) / (stage.batch_size // ga))          # mean loss per token of the step
    torch.save(batches, os.path.join(a.dump, "batches.pt"))
    json.dump({"losses": losses}, open(os.path.join(a.dump, "reference.json"), "w"))
    print(json.dumps({"impl": "reference", "losses": losses}), flush=True)
    dist.destroy_process_group()


def run_ours(a):
    import torch
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages
    from modded_nanogpt_b200.data.loader import Batch
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.runtime.dist import init_distributed
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.checkpoint import load_model_state
    from modded_nanogpt_b200.utils.logging import RunLogger
    env = init_distributed(accum_base=8)
    hp = Hyperparameters(data_path="/tmp/mng_curve_data", val_loss_every=0, seed=0, disable_fp8=(a.mlp == "bf16"))
    sched = TrainingSchedule(track1_stages(), 1270, 15, cooldown_frac=0.60)
    tr = Trainer(track1_model(hp.val_batch_size // 8), sched, hp, env,
                 logger=RunLogger("curve", True, log_dir="/tmp/mng_logs", quiet=True))
    tr.model.fp8_head = True
    load_model_state(tr.model, torch.load(os.path.join(a.dump, "init.pt")), strict=False)
    tr.model.prefix_table.copy_(torch.load(os.path.join(a.dump, "prefix.pt")))
    tr.model.quantize_mlp_fp8(bootstrap_down=True)
    tr.manager.reset()
    batches = torch.load(os.path.join(a.dump, "batches.pt"))
    ref = json.load(open(os.path.join(a.dump, "reference.json")))["losses"]
    ga = env.grad_accum_steps
    losses = []
    dev = env.device
    for step in range(a.steps):
        tr.manager.advance_schedule(step)
        total = None
        for k in range(ga):
            i, t, c, b = batches[step * ga + k]
            batch = Batch(i.to(dev), t.to(dev), c.to(dev), b.to(dev), b.numpy())
            l = tr.micro_step(batch, step)
            total = l if total is None else total + l
        tr.manager.step_optimizers(step)
        tr.model.quantize_mlp_fp8(bootstrap_down=(step < 16))
        losses.append(float(total) / batches[step * ga][0].numel())
    torch.cuda.synchronize()
    fused.check_status()
    rel = [abs(x - y) / y for x, y in zip(losses, ref)]
    print(json.dumps({"impl": "ours", "mlp": a.mlp, "losses": losses, "reference": ref, "rel_diff": rel, "max_rel_diff": max(rel)}),
          flush=True)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("which", choices=["reference", "ours"])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--dump", default="/tmp/mng_curve")
    ap.add_argument("--mlp", default="fp8", choices=["fp8", "bf16"])
    a = ap.parse_args()
    (run_reference if a.which == "reference" else run_ours)(a)
