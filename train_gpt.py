"""Track-1 speedrun entry point:  torchrun --standalone --nproc_per_node=8 train_gpt.py

Zero-flag behaviour of the reference script (`train_gpt.py:2203-2382`): read RANK / WORLD_SIZE /
LOCAL_RANK, log the sources and the environment to `logs/{run_id}.txt`, build the model on every
rank from rank 0's weights, warm every kernel variant up on the steps around each stage transition,
restore the initial state, then run the 1270 + 15 step schedule with validation every 250 steps.
Environment: DATA_PATH (shard directory root), DISABLE_FP8, SYNTHETIC_DATA=1 (generate Zipf/EoS
shards under $DATA_PATH if none exist), MAX_STEPS (stop early), SAVE_CHECKPOINT=1, RESUME_FROM=path,
RUN_EVALS=1 (HellaSwag after training), SKIP_WARMUP=1.
"""
import os
import sys

os.environ.setdefault("PYTORCH_ALLOC_CONF", "expandable_segments:True")
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages  # noqa: E402
from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown  # noqa: E402
from modded_nanogpt_b200.trainer import Trainer  # noqa: E402
from modded_nanogpt_b200.utils.logging import RunLogger  # noqa: E402


def main():
    env = init_distributed(accum_base=8)
    hp = Hyperparameters(save_checkpoint=bool(os.environ.get("SAVE_CHECKPOINT")), run_evals=bool(os.environ.get("RUN_EVALS")),
                         resume_from=os.environ.get("RESUME_FROM", ""))
    log = RunLogger(hp.run_id, env.master)
    log.log_sources(__file__)
    log.log_environment()
    if hp.synthetic and env.master:
        from modded_nanogpt_b200.data.shards import write_synthetic_corpus
        total = sum((b - a) * s.batch_size for (a, b), s in zip(TrainingSchedule(track1_stages(), 1270, 15).boundaries, track1_stages()))
        need = total if not hp.max_steps else hp.max_steps * 393216
        write_synthetic_corpus(hp.data_path, train_tokens=int(need * 1.1) + 50_000_000, val_tokens=hp.val_tokens + 1_000_000,
                               max_doc_len=2048)
    env.barrier()
    sched = TrainingSchedule(track1_stages(), hp.num_scheduled_iterations, hp.num_extension_iterations,
                             cooldown_frac=hp.cooldown_frac)
    trainer = Trainer(track1_model(hp.val_batch_size // (env.grad_accum_steps * env.world_size)), sched, hp, env, logger=log)
    start = 0
    if hp.resume_from:
        start = trainer.load_checkpoint(hp.resume_from)
    log.print0("Compiling nothing: kernels are prebuilt; warming up CUDA graphs and caches", console=True)
    trainer.run(do_warmup=not os.environ.get("SKIP_WARMUP"), start_step=start)
    if hp.run_evals:
        from modded_nanogpt_b200.eval import hellaswag
        trainer.model.eval()
        hellaswag.evaluate(model=trainer.model, schedule_cfg=trainer.manager.get_forward_args(),
                           seq_len=hp.val_batch_size // (env.grad_accum_steps * env.world_size),
                           get_bigram_hash=lambda x: __import__("modded_nanogpt_b200.data.loader", fromlist=["bigram_hash"]).bigram_hash(
                               x, trainer.model.cfg.bigram_vocab_size), print0=log.print0)
    shutdown()


if __name__ == "__main__":
    main()
