"""Track-3 baseline: Newton-Schulz orthogonalisation, Muon step, a short CPU training run."""
import os

import torch

from modded_nanogpt_b200.models.gpt_simple import GPTSimple
from modded_nanogpt_b200.optim.muon import Muon, newton_schulz


def test_newton_schulz_and_muon_step():
    torch.manual_seed(0)
    for shape in ((64, 192), (192, 64)):
        x = newton_schulz(torch.randn(*shape), dtype=torch.float32)
        s = torch.linalg.svdvals(x)
        assert s.max() < 1.3 and s.min() > 0.3
    p = torch.nn.Parameter(torch.randn(32, 16))
    p.grad = torch.randn(32, 16)
    p0 = p.detach().clone()
    Muon([p], lr=0.1, weight_decay=0.5, ns_dtype=torch.float32).step()
    step = (p0 * (1 - 0.05) - p.detach())
    s = torch.linalg.svdvals(step / (0.1 * 2 ** 0.5))      # lr * sqrt(rows/cols)
    assert 0.3 < s.min() and s.max() < 1.3


def test_simple_trainer_learns(tiny_corpus, tmp_path, monkeypatch):
    import train_gpt_simple as t3
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.utils.logging import RunLogger
    monkeypatch.chdir(tmp_path)
    env = DistEnv(0, 1, 0, torch.device("cpu"), 1, 1.0, True)
    log = RunLogger("t3", True, log_dir=str(tmp_path), quiet=True)
    torch.manual_seed(0)
    kw = dict(vocab_size=50304, num_layers=2, model_dim=64, head_dim=32)
    final = t3.run_trial(env, log, tiny_corpus, train_steps=6, val_tokens=4096, batch_size=4096, mbs=2, model_kw=kw)
    text = open(log.path).read()
    first = float(text.split("val_loss:")[1].split()[0])
    assert final < first and "step:6/6 val_loss:" in text
    m = GPTSimple(**kw)
    m.reset_parameters()
    assert m.proj.weight.abs().max() == 0 and m.blocks[0].attn.proj.weight.abs().max() == 0
