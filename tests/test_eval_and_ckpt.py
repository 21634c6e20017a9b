"""HellaSwag packing/scoring on synthetic tasks, checkpoint layout and resume parity, log format."""
import os

import numpy as np
import pytest
import torch

from modded_nanogpt_b200.eval import hellaswag as hs


def _tasks(n, rng):
    out = []
    for _ in range(n):
        ctx = rng.integers(0, 1000, rng.integers(5, 30)).tolist()
        ends = [rng.integers(0, 1000, rng.integers(2, 12)).tolist() for _ in range(4)]
        out.append(dict(ctx_tokens=ctx, ending_tokens=ends, label=int(rng.integers(0, 4))))
    return out


def test_hellaswag_packing_layout():
    rng = np.random.default_rng(0)
    tasks = _tasks(40, rng)
    seqs = hs.pack_tasks(tasks, seq_len=1024)
    assert len(seqs) > 1 and sum(len(s.labels) for s in seqs) == 40
    ti = 0
    for s in seqs:
        assert s.inputs.shape == (1024,) and s.doc_ends[0] == 0 and s.doc_ends[-1] == 1024 and s.doc_ends.numel() % 128 == 0
        for k in range(len(s.labels)):
            t = tasks[ti]
            for e in range(4):
                a, b = s.spans[k, e].tolist()
                assert s.targets[a:b].tolist() == t["ending_tokens"][e]               # span covers exactly the ending
                assert s.inputs[a + 1 - len(t["ctx_tokens"]):a + 1].tolist() == t["ctx_tokens"]
            ti += 1
        eot = torch.nonzero(s.inputs == hs.EOT_ID)[:, 0]
        assert torch.equal(s.doc_ends[1:len(eot) + 1].long(), eot + 1)


def test_hellaswag_scoring_picks_lowest_mean_loss():
    rng = np.random.default_rng(1)
    tasks = _tasks(10, rng)
    (seq,) = hs.pack_tasks(tasks, seq_len=4096)
    loss = torch.rand(4096) + 1.0
    want = 0
    for k in range(10):
        best = int(rng.integers(0, 4))
        a, b = seq.spans[k, best].tolist()
        loss[a:b] = 0.01
        want += int(best == tasks[k]["label"])
    assert hs.score_losses(loss, seq.spans, seq.labels) == (want, 10)

    class Fake(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))

        def forward(self, inp, tgt, ends, bg, cfg):
            return loss

    lines = []
    acc = hs.evaluate(Fake(), None, 4096, lambda x: x, print0=lambda s, console=False: lines.append(s), tasks=tasks)
    assert acc == want / 10 and lines[0].startswith("HellaSwag: accuracy=")


def _trainer(root, run_id, steps=6):
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, tiny_model, tiny_stages
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    env = DistEnv(0, 1, 0, torch.device("cpu"), 1, 1.0, True)
    hp = Hyperparameters(data_path=root, num_scheduled_iterations=steps, num_extension_iterations=0, val_batch_size=2048,
                         val_tokens=4096, val_loss_every=3, run_id=run_id)
    sched = TrainingSchedule(tiny_stages(batch_tokens=1024, seq_len=256), steps, 0)
    return Trainer(tiny_model(2048), sched, hp, env, param_dtype=torch.float32,
                   logger=RunLogger(run_id, True, log_dir=os.path.join(root, "logs"), quiet=True))


@pytest.mark.parametrize("prefetch", ["0", "1"])
def test_checkpoint_resume_is_bitwise(tiny_corpus, tmp_path, monkeypatch, prefetch):
    """Also with the next step's first batch prefetched: the checkpoint stores the cursor before that batch."""
    monkeypatch.chdir(tmp_path)
    monkeypatch.setenv("MNG_PREFETCH_BATCH", prefetch)
    a = _trainer(tiny_corpus, "full")
    for s in range(6):
        a.train_step(s)
    b = _trainer(tiny_corpus, "half")
    for s in range(3):
        b.train_step(s)
    path = b.save_checkpoint()
    assert os.path.basename(path) == "state_step000003.pt"
    blob = torch.load(path, weights_only=False)
    assert set(blob) >= {"step", "code", "model", "optimizer"} and all(k.startswith("_orig_mod.") for k in blob["model"])
    c = _trainer(tiny_corpus, "resumed")
    with torch.no_grad():
        for p in c.model.parameters():
            p.add_(1.0)                       # make sure the load really restores everything
    assert c.load_checkpoint(path) == 3
    for s in range(3, 6):
        c.train_step(s)
    for (n, pa), (_, pc) in zip(a.model.state_dict().items(), c.model.state_dict().items()):
        assert torch.equal(pa, pc), n
    for l, st in a.manager.optimizer.state.items():
        for k, v in st.items():
            w = c.manager.optimizer.state[l][k]
            assert torch.equal(v, w) if isinstance(v, torch.Tensor) else v == w, (l, k)


def test_checkpoint_rejects_garbage_and_adapts_bank_padding(tmp_path):
    from modded_nanogpt_b200.utils import checkpoint as ck
    p = tmp_path / "x.pt"
    torch.save({"foo": 1}, p)

    class T:
        pass
    with pytest.raises(ValueError):
        ck.load_checkpoint(T(), str(p))
    saved = torch.arange(60 * 4, dtype=torch.float32).view(60, 2, 2)
    up = ck.adapt_bank(saved, (64, 2, 2))
    assert up.shape == (64, 2, 2) and torch.equal(up[:60], saved) and up[60:].abs().sum() == 0
    assert torch.equal(ck.adapt_bank(up, (60, 2, 2)), saved)
    assert ck.strip_prefix({"_orig_mod.a": 1, "b": 2}) == {"a": 1, "b": 2}


def test_full_run_log_lines(tiny_corpus, tmp_path, monkeypatch):
    from modded_nanogpt_b200.utils.logging import TRAIN_LINE, VAL_LINE, parse_log
    monkeypatch.chdir(tmp_path)
    t = _trainer(tiny_corpus, "runlog")
    t.log.log_environment()
    val = t.run(do_warmup=True)
    assert val is not None and val < 11.0
    text = open(t.log.path).read()
    train, vals = parse_log(t.log.path)
    assert [s for s, _ in train] == [1, 2, 3, 4, 5, 6] and [s for s, *_ in vals] == [0, 3, 6]
    assert "Sampling steps" in text and "Resetting Model" in text and "Running PyTorch" in text
    for line in text.splitlines():
        if line.startswith("step:"):
            assert VAL_LINE.fullmatch(line) or TRAIN_LINE.fullmatch(line), line


def _staged_trainer(root, run_id, steps=6):
    """Three scheduled stages with different batch sizes and document caps (as tracks 1 and 2 have)."""
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, TrainingStage, tiny_model
    from modded_nanogpt_b200.runtime.dist import DistEnv
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    env = DistEnv(0, 1, 0, torch.device("cpu"), 1, 1.0, True)
    hp = Hyperparameters(data_path=root, num_scheduled_iterations=steps, num_extension_iterations=0, val_batch_size=2048,
                         val_tokens=2048, val_loss_every=0, run_id=run_id)
    stages = [TrainingStage(duration=1 / 3, train_max_seq_len=s, batch_size=b, window_sizes=(1, 2), lr_mul=1.0,
                            mtp_weights_start=[1.0], mtp_weights_end=[1.0])
              for b, s in ((1024, 128), (2048, 256), (3072, 256))]
    stages.append(TrainingStage(train_max_seq_len=256, batch_size=3072, window_sizes=(1, 2), lr_mul=1.0,
                                mtp_weights_start=[1.0], mtp_weights_end=[1.0]))
    return Trainer(tiny_model(2048), TrainingSchedule(stages, steps, 0), hp, env, param_dtype=torch.float32,
                   logger=RunLogger(run_id, True, log_dir=os.path.join(root, "logs"), quiet=True))


@pytest.mark.parametrize("prefetch", ["0", "1"])
@pytest.mark.parametrize("drive", ["run", "train_step"])
def test_stage_transitions_reparameterise_the_loader(tiny_corpus, tmp_path, monkeypatch, prefetch, drive):
    """Every step trains on its stage's batch size and document cap, whether the schedule is advanced once
    (bare `train_step`) or twice per step (`run()` advances it before validation, `train_step` again)."""
    monkeypatch.chdir(tmp_path)
    monkeypatch.setenv("MNG_PREFETCH_BATCH", prefetch)
    t = _staged_trainer(tiny_corpus, f"stages_{drive}_{prefetch}")
    seen = []
    orig = t.micro_step

    def spy(batch, step):
        doc_lens = torch.diff(batch.cum_seqlens.long())
        seen.append((step, batch.inputs.numel(), int(doc_lens.max())))
        return orig(batch, step)

    t.micro_step = spy
    if drive == "run":
        t.run(do_warmup=False)
    else:
        for s in range(6):
            t.train_step(s)
    assert [(s, n) for s, n, _ in seen] == [(0, 1024), (1, 1024), (2, 2048), (3, 2048), (4, 3072), (5, 3072)]
    assert all(d <= 128 for s, _, d in seen if s < 2) and all(d <= 256 for _, _, d in seen)
    assert t.manager.batch_size == 3072


def test_checkpoint_from_another_world_size_is_refused(tiny_corpus, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    a = _trainer(tiny_corpus, "ws_a")
    for s in range(2):
        a.train_step(s)
    path = a.save_checkpoint()
    blob = torch.load(path, weights_only=False)
    blob["world_size"] = 8                                      # as if an 8-rank job had written it
    torch.save(blob, path)
    b = _trainer(tiny_corpus, "ws_b")
    with pytest.raises(RuntimeError, match="world_size 8"):
        b.load_checkpoint(path)
    assert b.load_checkpoint(path, strict=False) == 2           # model only, announced on stdout
    for (n, pa), (_, pb) in zip(a.model.state_dict().items(), b.model.state_dict().items()):
        assert torch.equal(pa, pb), n
    os.remove(os.path.join(os.path.dirname(path), "optim_step000002_rank0.pt"))
    blob["world_size"] = 1
    blob.pop("optimizer")
    torch.save(blob, path)
    with pytest.raises(RuntimeError, match="is missing"):
        _trainer(tiny_corpus, "ws_c").load_checkpoint(path)
