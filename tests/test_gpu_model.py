"""Fused glue kernels, the GEMM-based DC path and the fused model forward/backward against the
op-by-op PyTorch restatement (fp32 where it matters)."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_lincomb_fwd_bwd():
    from modded_nanogpt_b200.ops.glue import Term, lincomb
    torch.manual_seed(0)
    T, D = 777, 768
    xs = [torch.randn(T, D, device="cuda").to(BF).requires_grad_(True) for _ in range(4)]
    gate = (torch.randn(T, 9, device="cuda") * 0.5).to(BF).requires_grad_(True)
    s1 = torch.tensor(1.3, device="cuda", requires_grad=True)
    lam = torch.tensor([[0.7, -0.4]], device="cuda", requires_grad=True)
    out = lincomb([Term(xs[0], scalar=s1), Term(xs[1], gate=gate, col=3), Term(xs[2], scalar=lam[0, 1], gate=gate, col=7, addc=1.0),
                   Term(xs[3]), Term(xs[0], scalar=lam[0, 0])])
    g = torch.randn_like(out)
    out.backward(g)
    got = [x.grad.clone() for x in xs] + [gate.grad.clone(), s1.grad.clone(), lam.grad.clone()]
    xr = [x.detach().float().requires_grad_(True) for x in xs]
    gr = gate.detach().float().requires_grad_(True)
    s1r, lamr = s1.detach().clone().requires_grad_(True), lam.detach().clone().requires_grad_(True)
    ref = s1r * xr[0] + gr[:, 3:4] * xr[1] + (1.0 + lamr[0, 1] * gr[:, 7:8]) * xr[2] + xr[3] + lamr[0, 0] * xr[0]
    assert _rel(out, ref) < 4e-3
    ref.backward(g.float())
    want = [x.grad for x in xr] + [gr.grad, s1r.grad, lamr.grad]
    for a, b in zip(got, want):
        assert _rel(a, b) < 1e-2, (a.shape, _rel(a, b))


def test_lincomb_grad_sinks_and_norm_fork():
    """Shared gradient buffers (x and gate sinks) and the forked norm give the gradients autograd's own sums give."""
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.ops.glue import Term, grad_sink, lincomb
    torch.manual_seed(1)
    T, D = 515, 768
    base = torch.randn(T, D, device="cuda").to(BF).requires_grad_(True)         # consumed by three lincombs
    gate = (torch.randn(T, 8, device="cuda") * 0.5).to(BF).requires_grad_(True)
    x_in = torch.randn(T, D, device="cuda").to(BF).requires_grad_(True)

    def run(shared: bool):
        for t in (base, gate, x_in):
            t.grad = None
        if shared:
            b, bs = grad_sink(base)
            g, gs = grad_sink(gate)
            bt = lambda **kw: Term(b, sink=bs, **kw)
            gk = lambda: dict(gate=g, gate_sink=gs)
            fork = fused.rms_norm_fork
        else:
            bt = lambda **kw: Term(base, **kw)
            gk = lambda: dict(gate=gate)
            fork = lambda t: (fused.rms_norm(t), t)
        x = x_in * 1.0
        for layer in range(3):
            y, x = fork(x)
            x = lincomb([Term(x), Term(y, col=2 * layer, **gk()), bt(col=2 * layer + 1, **gk()), bt(addc=0.25)])
        x = x + gate[:, 7:8] * 0.5                                               # a consumer outside the sink
        (x.float() ** 2).mean().backward()
        return x.detach(), base.grad.clone(), gate.grad.clone(), x_in.grad.clone()

    want = run(False)
    for _ in range(2):                                                           # twice: the sinks reset between backward passes
        got = run(True)
        for a, b in zip(got, want):
            assert _rel(a, b) < 1e-2, (a.shape, _rel(a, b))


@pytest.mark.parametrize("paired,key_offset,with_ve", [(False, False, False), (False, True, True), (True, False, True)])
def test_qkv_post(paired, key_offset, with_ve):
    from modded_nanogpt_b200.models.gpt_fused import _rope_tables
    from modded_nanogpt_b200.models.yarn import Yarn
    from modded_nanogpt_b200.ops.glue import qkv_post
    torch.manual_seed(1)
    T, H, Dh = 300, 6, 128
    qkv = torch.randn(T, 3 * H * Dh, device="cuda").to(BF).requires_grad_(True)
    ve = torch.randn(T, H * Dh, device="cuda").to(BF).requires_grad_(True) if with_ve else None
    vg = torch.rand(T, H, device="cuda").to(BF).requires_grad_(True) if with_ve else None
    va = torch.randn(T, H * Dh, device="cuda").to(BF).requires_grad_(True) if with_ve else None
    yarn = Yarn(Dh, 1024, paired=paired, device="cuda")
    yarn.apply(384, 896)
    cos, sin = _rope_tables(yarn, 2 * T, qkv.device)
    q, k, v = qkv_post(qkv, cos, sin, ve, vg, va, H, paired, key_offset)
    gq, gk, gv = (torch.randn_like(t) for t in (q, k, v))
    torch.autograd.backward([q, k, v], [gq, gk, gv])

    # fp32 restatement of train_gpt.py:1103-1136
    f = lambda t: None if t is None else t.detach().float().requires_grad_(True)
    qkv_r, ve_r, vg_r, va_r = f(qkv), f(ve), f(vg), f(va)
    y32 = Yarn(Dh, 1024, paired=paired, device="cuda")
    y32.apply(384, 896)
    qq, kk, vv = qkv_r.view(T, 3 * H, Dh).split(H, dim=1)
    eps = torch.finfo(torch.float32).eps
    nrm = lambda t: t * torch.rsqrt(t.square().mean(-1, keepdim=True) + eps)
    qq, kk = nrm(qq), nrm(kk)
    if not paired:
        qq, kk = y32.rotary(qq), y32.rotary(kk)
        if key_offset:
            kk = torch.cat([kk[..., :64], torch.cat([kk[:1, :, 64:], kk[:-1, :, 64:]], 0)], -1)
    else:
        qq = y32.rotary(qq.reshape(T, H // 2, 2 * Dh)).reshape(T, H, Dh)
        kk = y32.rotary(kk.reshape(T, H // 2, 2 * Dh)).reshape(T, H, Dh)
    if with_ve:
        vv = vv + vg_r[:, :, None] * ve_r.view(T, H, Dh) + va_r.view(T, H, Dh)
    assert _rel(q, qq) < 6e-3 and _rel(k, kk) < 6e-3 and _rel(v, vv) < 6e-3
    torch.autograd.backward([qq, kk, vv], [gq.float(), gk.float(), gv.float()])
    assert _rel(qkv.grad, qkv_r.grad) < 1.2e-2
    if with_ve:
        assert _rel(ve.grad, ve_r.grad) < 1e-2 and _rel(vg.grad, vg_r.grad) < 1e-2 and _rel(va.grad, va_r.grad) < 1e-2


def test_xsa_gate():
    from modded_nanogpt_b200.ops.glue import xsa_gate
    torch.manual_seed(2)
    T, H, Dh = 500, 6, 128
    y = torch.randn(T, H, Dh, device="cuda").to(BF).requires_grad_(True)
    v = torch.randn(T, H, Dh, device="cuda").to(BF).requires_grad_(True)
    gates = (torch.randn(T, 20, device="cuda") * 0.7).to(BF).requires_grad_(True)
    out = xsa_gate(y, v, gates[:, 2:8], gates[:, 11:17])
    g = torch.randn_like(out)
    out.backward(g)
    yr, vr, gr = (t.detach().float().requires_grad_(True) for t in (y, v, gates))
    dot = (yr * vr).sum(-1, keepdim=True)
    den = vr.square().sum(-1, keepdim=True).clamp_min(1e-8)
    ref = (yr - torch.tanh(gr[:, 2:8]).unsqueeze(-1) * (dot / den) * vr) * gr[:, 11:17].unsqueeze(-1)
    ref.backward(g.float())
    assert _rel(out, ref) < 5e-3
    assert _rel(y.grad, yr.grad) < 1e-2 and _rel(v.grad, vr.grad) < 1e-2 and _rel(gates.grad, gr.grad) < 1.5e-2
    only_gate = xsa_gate(y.detach(), v.detach(), None, gates.detach()[:, 11:17])
    assert _rel(only_gate, y.detach().float() * gates.detach().float()[:, 11:17].unsqueeze(-1)) < 5e-3


def test_dc_fold_kernel_matches_torch_fold():
    from modded_nanogpt_b200.ops import dc
    from modded_nanogpt_b200.ops.native import lib
    torch.manual_seed(3)
    H, nblk = 6, 5
    part = torch.randn(H, nblk, 256, 128, device="cuda").to(BF)
    want = dc._fold(part, nblk * 128, H, 128)
    got = lib().dc_fold(part)
    assert got.shape == want.shape and torch.equal(got, want)


def test_dc_gemm_path_matches_reference():
    from modded_nanogpt_b200.ops import dc, fused, reference as ref
    torch.manual_seed(3)
    T, H, Dh = 1024, 6, 128
    mk = lambda *s: (torch.randn(*s, device="cuda")).to(BF).requires_grad_(True)
    base, q, k, v = mk(T, H, Dh), mk(T, H, Dh), mk(T, H, Dh), mk(T, H, Dh)
    w1, w2 = mk(T, H), mk(T, H)
    cu = torch.full((16,), T, dtype=torch.int32, device="cuda")
    cu[:5] = torch.tensor([0, 100, 130, 517, 900], dtype=torch.int32)
    out = dc.dc_correction(base, q, k, v, w1, w2, cu, 0.1, 112)
    g = torch.randn_like(out)
    grads = torch.autograd.grad(out, (base, q, k, v, w1, w2), g)
    rs = [t.detach().float().requires_grad_(True) for t in (base, q, k, v, w1, w2)]
    outr = ref.dc_correction(*rs, cu, 0.1, 112)
    gr = torch.autograd.grad(outr, rs, g.float())
    assert _rel(out, outr) < 1e-2
    for a, b, name in zip(grads, gr, "base q k v w1 w2".split()):
        assert _rel(a, b) < 3e-2, (name, _rel(a, b))
    fused.check_status()


def _model_and_batch(T=1024):
    from modded_nanogpt_b200.config import ModelConfig
    from modded_nanogpt_b200.data.loader import bigram_hash
    from modded_nanogpt_b200.models.gpt import GPT, ForwardScheduleConfig
    torch.manual_seed(0)
    cfg = ModelConfig(vocab_size=2000, max_seq_len=4096, bigram_vocab_size=4096, bigram_sign_table_rows=64)
    m = GPT(cfg, use_fp8=False).cuda().cast_params_()
    with torch.no_grad():      # move away from the zero inits so every path carries signal
        m.mlp_bank[:, 1].normal_(0, 0.02)
        m.mudd_w2.normal_(0, 0.3)
        m.mudd_gate_w2.normal_(0, 0.3)
        m.ve_gate_bank.normal_(0, 0.3)
        m.bigram_embed.weight.normal_(0, 0.3)
        m.smear_gate.weight.normal_(0, 0.3)
        m.scalars[22] = 0.3
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 2000, (T,), dtype=torch.int32, generator=g)
    tg = torch.randint(0, 2000, (T,), dtype=torch.int64, generator=g)
    cu = torch.full((128,), T, dtype=torch.int32)
    cu[:4] = torch.tensor([0, 300, 650, 800], dtype=torch.int32)
    bg = bigram_hash(ids, cfg.bigram_vocab_size)
    sc = ForwardScheduleConfig(torch.tensor([1.0, 0.5], device="cuda"), torch.tensor([0.0], device="cuda"), 128, 384, 1024)
    return m, [t.cuda() for t in (ids, tg, cu, bg)], sc


def _run(m, batch, sc, training):
    m.zero_grad(set_to_none=True)
    if training:
        loss = m(*batch, sc)
        loss.sum().backward()
        return loss.detach().float(), {n: p.grad.detach().float().clone() for n, p in m.named_parameters()}
    with torch.no_grad():
        return m(*batch, sc).float(), {}


@pytest.mark.parametrize("training", [True, False])
def test_fused_model_matches_op_by_op(training):
    """Gold = the same model in fp32 run op by op.  The fused bf16 path must be about as close to
    it as the op-by-op bf16 path is (bf16 chains make the two bf16 runs differ from each other by
    more than either differs from fp32 on the reduction-heavy scalar gradients)."""
    import copy
    from modded_nanogpt_b200 import ops
    from modded_nanogpt_b200.ops import fused
    m, batch, sc = _model_and_batch()
    m.train(training)
    gold_m = copy.deepcopy(m).float()
    gold_m.bigram_sign_table = gold_m.bigram_sign_table.float()
    gold_m.train(training)
    res = {}
    try:
        ops.set_backend("reference")
        res["gold"] = _run(gold_m, batch, sc, training)
        res["bf16"] = _run(m, batch, sc, training)
        ops.set_backend("auto")
        res["fused"] = _run(m, batch, sc, training)
    finally:
        ops.set_backend("auto")
    lg = res["gold"][0]
    assert _rel(res["fused"][0], lg) < max(2 * _rel(res["bf16"][0], lg), 1e-2)
    for n, gg in res["gold"][1].items():
        if gg.norm() == 0:
            assert res["fused"][1][n].norm() < 1e-3, n
            continue
        e_ref, e_fused = _rel(res["bf16"][1][n], gg), _rel(res["fused"][1][n], gg)
        # single scalars are sums with heavy cancellation: their relative error is noise-dominated
        tol = max(3.0 * e_ref, 0.2) if gg.numel() == 1 else max(2.0 * e_ref, 0.05)
        assert e_fused < tol, (n, e_fused, e_ref)
    fused.check_status()
