"""Track-2 (medium) and track-3 (simple) trainers on the GPU: a few real optimizer steps each."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_track2_trains_on_gpu(tmp_path):
    from modded_nanogpt_b200.config import track2_hyperparameters, track2_schedule
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    from modded_nanogpt_b200.models.gpt_medium import GPTMedium
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    root = str(tmp_path / "data")
    write_synthetic_corpus(root, train_tokens=800_000, val_tokens=70_000, seed=0, max_doc_len=600)
    hp = track2_hyperparameters(data_path=root, val_loss_every=0)
    sched = track2_schedule(hp)
    for s in sched.stages:
        s.batch_size = 8192 * 2
    env = DistEnv(0, 1, 0, torch.device("cuda", 0), 2, 0.5, True)
    torch.manual_seed(0)
    model = GPTMedium(max_seq_len=8192, world_size=1, grad_scale=0.5, use_fp8=True, eval_seq_len=8192)
    tr = Trainer(None, sched, hp, env, model=model, logger=RunLogger("t2", True, log_dir=str(tmp_path), quiet=True))
    losses = [float(tr.train_step(s)) for s in range(6)]
    torch.cuda.synchronize()
    fused.check_status()
    assert all(torch.isfinite(torch.tensor(losses))) and losses[-1] < losses[0], losses


def test_track3_trains_on_gpu(tmp_path, monkeypatch):
    import train_gpt_simple as t3
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.utils.logging import RunLogger
    root = str(tmp_path / "data")
    write_synthetic_corpus(root, train_tokens=600_000, val_tokens=70_000, seed=0, max_doc_len=600)
    monkeypatch.chdir(tmp_path)
    env = DistEnv(0, 1, 0, torch.device("cuda", 0), 1, 1.0, True)
    log = RunLogger("t3", True, log_dir=str(tmp_path), quiet=True)
    torch.manual_seed(0)
    final = t3.run_trial(env, log, root, train_steps=8, val_tokens=32768, batch_size=32768, mbs=16,
                         model_kw=dict(vocab_size=50304, num_layers=4, model_dim=256, head_dim=128))
    first = float(open(log.path).read().split("val_loss:")[1].split()[0])
    assert final < first
