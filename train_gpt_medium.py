"""Track-2 (GPT-2-medium scale) entry point:  torchrun --standalone --nproc_per_node=8 train_gpt_medium.py

Same driver as `train_gpt.py` with the track-2 model, schedule (4700 + 40 steps, batch 131k -> 524k
tokens, windows 3 -> 23 blocks, cooldown 0.7) and optimizer settings of `train_gpt_medium.py`."""
import os
import sys

os.environ.setdefault("PYTORCH_ALLOC_CONF", "expandable_segments:True")
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from modded_nanogpt_b200.config import track2_hyperparameters, track2_schedule  # noqa: E402
from modded_nanogpt_b200.models.gpt_medium import GPTMedium  # noqa: E402
from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown  # noqa: E402
from modded_nanogpt_b200.trainer import Trainer  # noqa: E402
from modded_nanogpt_b200.utils.logging import RunLogger  # noqa: E402


def main():
    env = init_distributed(accum_base=8)
    hp = track2_hyperparameters(save_checkpoint=bool(os.environ.get("SAVE_CHECKPOINT")))
    log = RunLogger(hp.run_id, env.master)
    log.log_sources(__file__)
    log.log_environment()
    if hp.synthetic and env.master:
        from modded_nanogpt_b200.data.shards import write_synthetic_corpus
        need = (hp.max_steps or 4740) * 524288
        write_synthetic_corpus(hp.data_path, train_tokens=int(need * 1.05), val_tokens=hp.val_tokens + 1_000_000, max_doc_len=4096)
    env.barrier()
    eval_seq = hp.val_batch_size // (env.grad_accum_steps * env.world_size)
    model = GPTMedium(max_seq_len=eval_seq, world_size=env.world_size, grad_scale=env.grad_scale, use_fp8=not hp.disable_fp8,
                      eval_seq_len=eval_seq)
    trainer = Trainer(None, track2_schedule(hp), hp, env, logger=log, model=model)
    trainer.run(do_warmup=not os.environ.get("SKIP_WARMUP"))
    shutdown()


if __name__ == "__main__":
    main()
