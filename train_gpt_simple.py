"""Track-3 baseline trainer (fewest optimizer steps to 3.28; `records/track_3_optimization/train_gpt_simple.py`):
12-layer GPT, batch 8 x 64 x 1024 tokens in rows of 1024, gradients all-reduced per parameter, AdamW for the
embedding / head / vectors and Muon for the block matrices, stable-then-linear-decay learning rate
(cooldown 0.7), validation on 20 x 524288 tokens.   torchrun --standalone --nproc_per_node=8 train_gpt_simple.py [trials]
Environment: DATA_PATH, TRAIN_STEPS (default 3250), SYNTHETIC_DATA=1."""
import os
import sys
import time
import uuid

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from modded_nanogpt_b200.data.loader import TokenLoader  # noqa: E402
from modded_nanogpt_b200.models.gpt_simple import GPTSimple  # noqa: E402
from modded_nanogpt_b200.optim.muon import Muon  # noqa: E402
from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown  # noqa: E402
from modded_nanogpt_b200.utils.logging import RunLogger  # noqa: E402


def rows(loader, seq_len=1024):
    b = loader.next_batch()
    return b.inputs.view(-1, seq_len), b.targets.view(-1, seq_len)


def run_trial(env, log, data_path, train_steps, val_tokens=20 * 524288, batch_size=8 * 64 * 1024, mbs=64, model_kw=None):
    dev = env.device
    model = GPTSimple(**(model_kw or {})).to(dev)
    model.embed.bfloat16()
    model.reset_parameters()
    if dist.is_initialized():
        for p in model.parameters():
            dist.broadcast(p.detach(), 0)
    pat = os.path.join(data_path, "data/fineweb10B/fineweb_{}_*.bin")
    val = TokenLoader(pat.format("val"), val_tokens, -1, 1, False, env.rank, env.world_size, dev)
    val_in, val_tg = rows(val)
    train = TokenLoader(pat.format("train"), batch_size, -1, 1, False, env.rank, env.world_size, dev, cycle=True)
    adam = torch.optim.AdamW([dict(params=[model.embed.weight], lr=0.7), dict(params=[model.proj.weight], lr=0.004),
                              dict(params=[p for p in model.parameters() if p.ndim < 2], lr=0.015)],
                             betas=(0.8, 0.95), eps=1e-10, weight_decay=0.001)
    muon = Muon([p for p in model.blocks.parameters() if p.ndim >= 2], lr=0.025, weight_decay=0.05,
                ns_dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32)
    opts = [adam, muon]
    for o in opts:
        for g in o.param_groups:
            g["initial_lr"] = g["lr"]
    t0, train_time, val_loss = time.perf_counter(), 0.0, None
    for step in range(train_steps + 1):
        freq = 125 if step / train_steps < 0.9 else 25
        if step == train_steps or step % freq == 0:
            train_time += time.perf_counter() - t0
            model.eval()
            tot = torch.zeros((), device=dev)
            with torch.no_grad(), torch.autocast(dev.type, dtype=torch.bfloat16, enabled=False):
                for i in range(0, len(val_in), mbs):
                    tot += model(val_in[i:i + mbs], val_tg[i:i + mbs])
            if dist.is_initialized():
                dist.all_reduce(tot)
            val_loss = float(tot) / val_tokens
            log.print0(f"step:{step}/{train_steps} val_loss:{val_loss:.5f} train_time:{train_time:.3f}s "
                       f"step_avg:{1000 * train_time / max(step, 1):.2f}ms", console=True)
            model.train()
            t0 = time.perf_counter()
        if step == train_steps:
            break
        x, y = rows(train)
        for i in range(0, len(x), mbs):
            model(x[i:i + mbs], y[i:i + mbs]).backward()
        if dist.is_initialized() and env.world_size > 1:
            for p in model.parameters():
                dist.all_reduce(p.grad)
        prog = step / train_steps
        eta = 1.0 if prog < 0.3 else (1 - prog) / 0.7
        for o in opts:
            for g in o.param_groups:
                g["lr"] = g["initial_lr"] * eta
            o.step()
        model.zero_grad(set_to_none=True)
    return val_loss


def main():
    env = init_distributed(accum_base=8)
    log = RunLogger(str(uuid.uuid4()), env.master)
    log.log_sources(__file__)
    trials = int(sys.argv[-1]) if len(sys.argv) > 1 and sys.argv[-1].isdigit() else 1
    data_path = os.environ.get("DATA_PATH", ".")
    steps = int(os.environ.get("TRAIN_STEPS", "3250"))
    if os.environ.get("SYNTHETIC_DATA") and env.master:
        from modded_nanogpt_b200.data.shards import write_synthetic_corpus
        write_synthetic_corpus(data_path, train_tokens=min(steps, 400) * 524288 + 1_000_000, val_tokens=20 * 524288 + 1_000_000)
    env.barrier()
    for _ in range(trials):
        run_trial(env, log, data_path, steps)
    shutdown()


if __name__ == "__main__":
    main()
