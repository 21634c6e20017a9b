"""Optimizer math against closed forms, and sharded (gloo, 2 ranks) == single rank."""
import math
import os

import pytest
import torch

from modded_nanogpt_b200.ops import reference as ref
from tests.dist_utils import spawn


def test_polar_express_orthogonalises():
    torch.manual_seed(0)
    for shape in ((4, 64, 192), (2, 192, 64), (3, 96, 96)):
        g = torch.randn(*shape)
        x = ref.polar_express(g, torch.float32)
        s = torch.linalg.svdvals(x)
        assert s.max() < 1.25 and s.median() > 0.7
        if shape[-1] != shape[-2]:      # a random square matrix has near-zero singular values the 5 steps cannot lift
            assert s.min() > 0.5
            u, _, vt = torch.linalg.svd(g, full_matrices=False)
            assert (x - u @ vt).abs().max() < 0.35
        xb = ref.polar_express(g, torch.bfloat16).float()
        assert (xb - x).abs().max() < 0.05


def test_nesterov_and_variance_reduction():
    torch.manual_seed(0)
    g, buf = torch.randn(2, 8, 4), torch.randn(2, 8, 4)
    g0, b0 = g.clone(), buf.clone()
    out = ref.nesterov_momentum_(g, buf, 0.9)
    b1 = 0.9 * b0 + 0.1 * g0
    assert torch.allclose(buf, b1, atol=1e-6) and torch.allclose(out, 0.1 * g0 + 0.9 * b1, atol=1e-6)
    v = torch.randn(2, 8, 4)
    s = torch.zeros(2, 8, 1)
    n0 = v.norm(dim=(-2, -1))
    out = ref.normuon_variance_reduction_(v.clone(), s, 0.9, -1)
    assert torch.allclose(out.norm(dim=(-2, -1)), n0, rtol=1e-4)          # Frobenius norm kept
    assert torch.allclose(s, 0.1 * v.square().mean(-1, keepdim=True), atol=1e-6)
    row = out.square().mean(-1)
    assert (row.max(dim=-1).values / row.min(dim=-1).values < 1.001).all()    # first step: rows equalised


def test_mantissa_update_is_exact_fp32():
    torch.manual_seed(0)
    p32 = torch.randn(64, 32) * 0.05
    bits = p32.view(torch.int32)
    p_bf = (bits >> 16).to(torch.int16).view(torch.bfloat16).clone()
    mant = (bits & 0xFFFF).to(torch.int16).view(torch.uint16).clone()
    want = p32.clone()
    for _ in range(5):
        upd = torch.randn(64, 32).bfloat16()
        ref.cautious_update_mantissa_(p_bf, mant, upd, eff_wd=0.03, eff_lr=0.02)
        g = upd.float()
        mask = (g * want) >= 0
        want = want - want * mask * torch.tensor(0.03) * torch.tensor(0.02) - g * torch.tensor(0.02)
        got = ((p_bf.view(torch.int16).to(torch.int32) << 16) | (mant.view(torch.int16).to(torch.int32) & 0xFFFF)).view(torch.float32)
        assert torch.equal(got, want)


def test_adam_update_closed_form():
    torch.manual_seed(0)
    p, g = torch.randn(10, 4), torch.randn(10, 4)
    m, v = torch.zeros(10, 4), torch.zeros(10, 4)
    p0 = p.clone()
    lr, b1, b2 = 0.01, 0.9, 0.99
    step_size = lr * math.sqrt(1 - b2) / (1 - b1)
    ref.adam_update_(p, g, m, v, b1, b2, 1e-10, step_size, eff_wd=lr * lr * 0.5)
    u = step_size * (0.1 * g) / ((0.01 * g * g).sqrt() + 1e-10)
    u = u + (lr * lr * 0.5) * p0 * ((u * p0) > 0)
    assert torch.allclose(p, p0 - u, atol=1e-6)


# ---------------------------------------------------------------------------------------------
def _train(rank, world, root, out, steps, polar64, cfg_name):
    import torch
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, small_track1_model, tiny_model, tiny_stages
    from modded_nanogpt_b200.optim.normuon_adam import TorchMath
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger
    env = init_distributed(accum_base=2)
    hp = Hyperparameters(data_path=root, num_scheduled_iterations=steps, num_extension_iterations=0,
                         val_batch_size=2048, val_tokens=4096, val_loss_every=0)
    bt = 4 * 256 * 2 if cfg_name == 'tiny' else 512
    sched = TrainingSchedule(tiny_stages(batch_tokens=bt, seq_len=256), steps, 0, split_embed_stage=0)
    sched.split_step = 5 if cfg_name == 'tiny' else 1
    cfg = tiny_model(1024) if cfg_name == "tiny" else small_track1_model(1024)
    tr = Trainer(cfg, sched, hp, env, param_dtype=torch.float32,
                 math=TorchMath(torch.float64 if polar64 else torch.bfloat16),
                 logger=RunLogger("t", env.master, log_dir=os.path.join(root, "logs"), quiet=True),
                 sparse_min_world=2 if cfg_name == "sparse" else 8)
    losses = [float(tr.train_step(s)) for s in range(steps)]
    if rank == 0:
        torch.save(dict(model={k: v.clone() for k, v in tr.model.state_dict().items()}, losses=losses,
                        split=tr.manager.optimizer.split_embed), out)
    shutdown()


@pytest.mark.parametrize("cfg_name", ["tiny", "track1"])
def test_two_ranks_match_one_rank(tiny_corpus, tmp_path, cfg_name):
    """10 NorMuon(Polar Express, 5 iters)+Adam steps, tiny GPT, fp32: reduce-scatter/all-gather
    sharding over 2 gloo ranks reproduces the single-rank run (through the embed untie at step 5)."""
    steps = 10 if cfg_name == "tiny" else 4
    spawn(_train, 1, tiny_corpus, str(tmp_path / "a.pt"), steps, True, cfg_name)
    spawn(_train, 2, tiny_corpus, str(tmp_path / "b.pt"), steps, True, cfg_name)
    a, b = torch.load(tmp_path / "a.pt"), torch.load(tmp_path / "b.pt")
    assert a["split"] and b["split"]
    assert a["losses"][-1] < a["losses"][0]
    worst = 0.0
    for k, va in a["model"].items():
        vb = b["model"][k]
        if k in ("value_embeds", "bigram_embed.weight"):
            # Adam with eps=1e-10 turns rows whose gradient is rounding noise into +-lr sign steps, so
            # these tables depend on the summation order; they are compared loosely
            assert (va.float() - vb.float()).abs().max() < 2e-2
            continue
        if va.shape != vb.shape:      # banks are padded per world size
            n = min(va.shape[0], vb.shape[0])
            va, vb = va[:n], vb[:n]
        worst = max(worst, (va.float() - vb.float()).abs().max().item())
    assert worst < 5e-4, worst
    assert not torch.equal(a["model"]["embed.weight"], a["model"]["lm_head.weight"].T)   # untied after split


def _train_batched(rank, world, root, out, steps, batched):
    import torch
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, small_track1_model, tiny_stages
    from modded_nanogpt_b200.optim.normuon_adam import TorchMath
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger

    class BatchingMath(TorchMath):
        """The interface of the kernel-backed math object for small parameters, stated as a loop over `adam`."""
        batch_on_cpu = True
        calls = []

        def adam_batch(self, items, base_ptrs=None, grad_mul=1.0):
            assert base_ptrs is None and grad_mul == 1.0
            BatchingMath.calls.append([cfg.label for _, _, _, cfg, _, _, _, _ in items])
            for p, grad, state, cfg, step_size, eff_wd, _, _ in items:
                self.adam(p, grad, state, cfg, step_size, eff_wd)

    env = init_distributed(accum_base=2)
    hp = Hyperparameters(data_path=root, num_scheduled_iterations=steps, num_extension_iterations=0,
                         val_batch_size=2048, val_tokens=4096, val_loss_every=0)
    sched = TrainingSchedule(tiny_stages(batch_tokens=512, seq_len=256), steps, 0, split_embed_stage=0)
    sched.split_step = 1
    math_obj = BatchingMath(torch.float64) if batched else TorchMath(torch.float64)
    tr = Trainer(small_track1_model(1024), sched, hp, env, param_dtype=torch.float32, math=math_obj,
                 logger=RunLogger("t", env.master, log_dir=os.path.join(root, "logs"), quiet=True))
    for s in range(steps):
        tr.train_step(s)
    torch.save(dict(model={k: v.clone() for k, v in tr.model.state_dict().items()}, calls=BatchingMath.calls), out)
    shutdown()


def test_small_parameters_update_in_one_batch(tiny_corpus, tmp_path):
    """A math object that offers `adam_batch` receives all small replicated Adam parameters of a step in one call (never a
    NorMuon bank or a sharded table), on Adam steps only, and the result equals the one-by-one path bit for bit."""
    spawn(_train_batched, 1, tiny_corpus, str(tmp_path / "a.pt"), 4, False)
    spawn(_train_batched, 1, tiny_corpus, str(tmp_path / "b.pt"), 4, True)
    a, b = torch.load(tmp_path / "a.pt"), torch.load(tmp_path / "b.pt")
    assert a["calls"] == [] and len(b["calls"]) >= 1
    for labels in b["calls"]:
        assert len(labels) >= 8 and len(set(labels)) == len(labels)
        assert {"scalars", "smear_gate", "post_lambdas", "resid_lambdas"} <= set(labels)
        assert not {"lm_head", "embed", "value_embeds", "bigram_embed", "qk_bank", "vo_bank", "mlp_bank"} & set(labels)
    for k, va in a["model"].items():
        assert torch.equal(va, b["model"][k]), k


def _train_fused_pattern(rank, world, root, out, steps, fused_pattern):
    import torch
    import torch.distributed as dist
    from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, small_track1_model, tiny_stages
    from modded_nanogpt_b200.optim.normuon_adam import TorchMath
    from modded_nanogpt_b200.parallel.collectives import TorchCollectives
    from modded_nanogpt_b200.runtime.dist import init_distributed, shutdown
    from modded_nanogpt_b200.trainer import Trainer
    from modded_nanogpt_b200.utils.logging import RunLogger

    class BatchingMath(TorchMath):
        batch_on_cpu = True

        def adam_batch(self, items, base_ptrs=None, grad_mul=1.0):
            raise AssertionError("with several ranks the collectives object updates the small parameters")

    class FusedPattern(TorchCollectives):
        """The call pattern of the peer-memory collectives on gloo tensors: gradients stay where they are, nothing is
        launched in phase 1, one call per parameter does reduction + update + gather, the small replicated parameters
        go through one call, and gradients are cleared in place."""
        fused = True

        def __init__(self, math):
            super().__init__()
            self.math, self.offsets, self.log, self.opt = math, {}, [], None

        def prepare(self, optimizer):
            self.opt = optimizer
            self.offsets = {label: (0, 0) for label in optimizer.params}

        def enable_row_masks(self, label, param):
            return False

        def handles(self, cfg):
            return cfg.label != "ve_gate_bank"                 # one parameter stays on the library path

        def launch_fused_reduce(self, label, grad, cfg, state):
            return (None, None)

        def reduce_barrier(self):
            self.log.append("reduce_barrier")
            dist.barrier()

        def gather_barrier(self):
            self.log.append("gather_barrier")
            dist.barrier()

        def clear_grad(self, p):
            raise AssertionError("clear_grads replaces the per-parameter clears")

        def clear_grads(self, do_adam):
            self.log.append(("clear", do_adam))
            for label, p in self.opt.params.items():
                if p.grad is not None and (do_adam or self.opt.cfgs[label].optim == "normuon"):
                    p.grad.zero_()

        def fused_small_adam(self, labels, optimizer):
            self.log.append(("small", tuple(labels)))
            for label in labels:
                g = optimizer.params[label].grad.clone()
                self.all_reduce(g).wait()
                step_size, eff_wd = optimizer.adam_scalars(label)
                self.math.adam(optimizer.params[label].data, g, optimizer.state[label], optimizer.cfgs[label], step_size, eff_wd)

        def fused_update_and_gather(self, label, _grad, cfg, state, optimizer, do_adam):
            assert _grad is None
            p = optimizer.params[label]
            if cfg.comms.startswith("sharded"):
                src = p.grad.view(cfg.reshape) if cfg.optim == "normuon" else p.grad
                chunk = torch.empty((cfg.chunk_size, *src.shape[1:]), dtype=src.dtype)
                self.reduce_scatter(chunk, src).wait()
                shard = optimizer._shard_of(label)
                if cfg.optim == "normuon":
                    self.math.normuon_apply(shard, state, self.math.normuon_direction(chunk, state, cfg), cfg)
                else:
                    optimizer._adam_update(label, shard, chunk)
                self.all_gather(optimizer._full_of(label), shard).wait()
            else:
                g = p.grad.clone()
                self.all_reduce(g).wait()
                optimizer._adam_update(label, p.data, g)
            return None

    env = init_distributed(accum_base=2)
    hp = Hyperparameters(data_path=root, num_scheduled_iterations=steps, num_extension_iterations=0,
                         val_batch_size=2048, val_tokens=4096, val_loss_every=0)
    sched = TrainingSchedule(tiny_stages(batch_tokens=512, seq_len=256), steps, 0, split_embed_stage=0)
    sched.split_step = 2
    math_obj = BatchingMath(torch.float64) if fused_pattern else TorchMath(torch.float64)
    coll = FusedPattern(math_obj) if fused_pattern else None
    tr = Trainer(small_track1_model(1024), sched, hp, env, param_dtype=torch.float32, math=math_obj, collectives=coll,
                 logger=RunLogger("t", env.master, log_dir=os.path.join(root, "logs"), quiet=True))
    for s in range(steps):
        tr.train_step(s)
    if rank == 0:
        torch.save(dict(model={k: v.clone() for k, v in tr.model.state_dict().items()}, log=coll.log if coll else []), out)
    shutdown()


def test_fused_collectives_call_pattern_matches_library_path(tiny_corpus, tmp_path):
    """Two gloo ranks drive `NorMuonAndAdam.step` through the interface of the peer-memory collectives (stated with
    library collectives): same parameters as the plain library path, through the embed untie; barriers bracket the
    updates, the small replicated parameters go through one call on Adam steps only, gradients are cleared in one call."""
    steps = 5
    spawn(_train_fused_pattern, 2, tiny_corpus, str(tmp_path / "a.pt"), steps, False)
    spawn(_train_fused_pattern, 2, tiny_corpus, str(tmp_path / "b.pt"), steps, True)
    a, b = torch.load(tmp_path / "a.pt"), torch.load(tmp_path / "b.pt")
    for k, va in a["model"].items():
        tol = 2e-2 if k in ("value_embeds", "bigram_embed.weight") else 1e-5
        assert (va.float() - b["model"][k].float()).abs().max() < tol, k
    log = b["log"]
    assert log.count("reduce_barrier") == steps and log.count("gather_barrier") == steps
    smalls = [e for e in log if isinstance(e, tuple) and e[0] == "small"]
    clears = [e for e in log if isinstance(e, tuple) and e[0] == "clear"]
    assert len(clears) == steps and 0 < len(smalls) == sum(1 for c in clears if c[1])
    for e in smalls:
        assert "ve_gate_bank" in e[1] and "lm_head" not in e[1] and "qk_bank" not in e[1]
    i = 0
    for step in range(steps):                                  # per step: barrier, [small], barrier, clear
        assert log[i] == "reduce_barrier"
        i += 2 if (isinstance(log[i + 1], tuple) and log[i + 1][0] == "small") else 1
        assert log[i] == "gather_barrier" and log[i + 1][0] == "clear"
        i += 2
    assert i == len(log)
