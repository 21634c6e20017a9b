"""CUDA-graph replay of the training micro-step against the eager program: same data, same weights."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _trainer(tmp_path, graphs: bool, tag: str):
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, track1_model, track1_stages
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    root = str(tmp_path / "data")
    write_synthetic_corpus(root, train_tokens=600_000, val_tokens=70_000, seed=0, max_doc_len=600)
    cfg = track1_model(4096)
    stages = track1_stages()
    for s in stages:
        s.batch_size = 4096 * 2
    sched = TrainingSchedule(stages, 1270, 15, cooldown_frac=0.6)
    hp = Hyperparameters(data_path=root, val_loss_every=0, seed=0, disable_fp8=False)
    env = DistEnv(0, 1, 0, torch.device("cuda", 0), 2, 0.5, True)
    return Trainer(cfg, sched, hp, env, use_cuda_graphs=graphs,
                   logger=RunLogger(tag, True, log_dir=str(tmp_path), quiet=True))


def test_graph_replay_matches_eager(tmp_path):
    from modded_nanogpt_b200.ops import fused
    losses = {}
    for graphs in (False, True):
        tr = _trainer(tmp_path, graphs, f"g{int(graphs)}")
        out = [float(tr.train_step(step)) for step in range(8)]
        torch.cuda.synchronize()
        fused.check_status()
        losses[graphs] = out
        if graphs:
            assert tr.graphs.replays >= 10              # 16 micro-steps: 2 eager, 1 capture+replay, then replays
    a, b = torch.tensor(losses[False]), torch.tensor(losses[True])
    assert torch.isfinite(b).all()
    assert ((a - b).abs() / a.abs()).max() < 2e-2, (losses[False], losses[True])
    assert b[-1] < b[0]
