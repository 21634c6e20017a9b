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


def test_fp8_refresh_graph_matches_eager(tmp_path, monkeypatch):
    """The graph-replayed FP8 weight refresh leaves the same e4m3 copies and scales as a fresh eager quantisation."""
    from modded_nanogpt_b200.ops import fused
    monkeypatch.setenv("MNG_FP8_GRAPH", "1")
    tr = _trainer(tmp_path, False, "fp8g")
    model = tr.model
    for it in range(5):
        with torch.no_grad():
            model.mlp_bank.mul_(1.0 + 0.05 * (it + 1)).add_(torch.randn_like(model.mlp_bank) * 1e-3)
        model.quantize_mlp_fp8(bootstrap_down=False)
        st = model._fp8_state
        ref = fused.quantize_mlp_weights(model.mlp_bank, None, model._mlp_down_proj_scales.clone(),
                                         model._mlp_down_proj_next_scales.clone(), False)
        for name in ("fc8", "fc_scale", "projT8", "projT_scale"):
            a, b = getattr(st, name), getattr(ref, name)
            assert torch.equal(a.view(torch.uint8) if a.dtype != torch.float32 else a,
                               b.view(torch.uint8) if b.dtype != torch.float32 else b), (it, name)
    assert model._fp8_graph["graph"] is not None
    torch.cuda.synchronize()
    fused.check_status()
