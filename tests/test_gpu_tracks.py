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


def test_track2_fused_forward_matches_op_by_op():
    """The fused CUDA path of the track-2 model against the same model run op by op (bf16) and in fp32."""
    import copy
    from modded_nanogpt_b200 import ops
    from modded_nanogpt_b200.models.gpt import ForwardScheduleConfig
    from modded_nanogpt_b200.models.gpt_medium import GPTMedium
    from modded_nanogpt_b200.ops import fused
    torch.manual_seed(0)
    m = GPTMedium(vocab_size=2000, num_layers=16, num_heads=2, head_dim=128, model_dim=256, max_seq_len=4096, use_fp8=False).cuda()
    m.cast_params_()
    with torch.no_grad():
        m.mlp_bank[:, 1].normal_(0, 0.02)
        m.attn_bank.view(-1, 256, 256)[3::4].normal_(0, 0.02)          # O projections
        for p in (m.attn_gate_bank, m.value_embed_gate_bank, m.skip_gates, m.smear_gate.weight):
            p.normal_(0, 0.3)
        m.value_embeds.normal_(0, 0.3)
        m.x0_lambdas.normal_(0, 0.2)
    T = 1024
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 2000, (T,), dtype=torch.int32, generator=g).cuda()
    tg = torch.randint(0, 2000, (T,), dtype=torch.int64, generator=g).cuda()
    cu = torch.full((64,), T, dtype=torch.int32)
    cu[:4] = torch.tensor([0, 300, 650, 800], dtype=torch.int32)
    cu = cu.cuda()
    sc = ForwardScheduleConfig(torch.tensor([1.0, 0.5], device="cuda"), torch.tensor([0.0], device="cuda"), 128, 384, 1024)
    gold_m = copy.deepcopy(m).float()

    def run(model):
        model.zero_grad(set_to_none=True)
        loss = model(ids, tg, cu, None, sc)
        loss.sum().backward()
        return loss.detach().float(), {n: p.grad.detach().float().clone() for n, p in model.named_parameters()}

    rel = lambda a, b: ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
    try:
        ops.set_backend("reference")
        gold, bf = run(gold_m), run(m)
        ops.set_backend("auto")
        fz = run(m)
    finally:
        ops.set_backend("auto")
    assert rel(fz[0], gold[0]) < max(2 * rel(bf[0], gold[0]), 1e-2)
    for n, gg in gold[1].items():
        if gg.norm() == 0:
            assert fz[1][n].norm() < 1e-3, n
            continue
        e_ref, e_f = rel(bf[1][n], gg), rel(fz[1][n], gg)
        assert e_f < max(2.5 * e_ref, 0.06), (n, e_f, e_ref)
    fused.check_status()
