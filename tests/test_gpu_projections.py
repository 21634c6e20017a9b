"""Bank-backed projections, gate / MUDD MLPs and the batched FP8 weight refresh against plain PyTorch fp32
restatements of the same ops."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


@pytest.fixture(scope="module")
def fused():
    from modded_nanogpt_b200.ops import fused, native
    assert native.available(required=True)
    return fused


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,N,K,two_views", [(4096, 2304, 768, True), (2048, 768, 768, False), (49152, 2304, 768, True),
                                             (1000, 512, 256, False)])
def test_bank_linear_forward_backward(fused, T, N, K, two_views):
    """y = x (lam W)^T; dx = lam dy W; grad slices += lam dy^T x; dlam = <dy^T x, W>."""
    torch.manual_seed(0)
    x = torch.randn(T, K, device="cuda").to(BF).requires_grad_(True)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(BF)
    lam = torch.tensor(0.7, device="cuda", requires_grad=True)
    n0 = (2 * N // 3) if two_views else N
    g_init = torch.randn(N, K, device="cuda").to(BF)
    views = [g_init[:n0].clone(), g_init[n0:].clone()] if two_views else [g_init.clone()]
    y = fused.bank_linear(x, lam, w, views)
    dy = (torch.randn(T, N, device="cuda") * 0.1).to(BF)
    y.backward(dy)
    xf, wf, dyf = x.detach().float(), w.float(), dy.float()
    assert _rel(y, 0.7 * xf @ wf.T) < 6e-3
    assert _rel(x.grad, 0.7 * dyf @ wf) < 6e-3
    dw = dyf.T @ xf
    got = torch.cat([v.float() for v in views])
    assert _rel(got - g_init.float(), 0.7 * dw) < 1e-2          # bf16 accumulation into a bf16 gradient
    # a sum of N*K signed terms: compare on the scale of the terms' norm
    assert abs(lam.grad.item() - (dw * wf).sum().item()) <= 1e-3 * (dw * wf).norm().item()
    # deterministic: a second backward over the same data gives the same bits
    views2 = [g_init[:n0].clone(), g_init[n0:].clone()] if two_views else [g_init.clone()]
    x2 = x.detach().clone().requires_grad_(True)
    lam2 = torch.tensor(0.7, device="cuda", requires_grad=True)
    fused.bank_linear(x2, lam2, w, views2).backward(dy)
    assert torch.equal(lam2.grad, lam.grad) and all(torch.equal(a, b) for a, b in zip(views, views2))
    assert torch.equal(x2.grad, x.grad)
    fused.check_status()


@pytest.mark.parametrize("T,n,param_scale", [(4096, 41, True), (49152, 26, True), (2048, 14, False), (1024, 5, False)])
def test_gate_mlp_forward_backward(fused, T, n, param_scale):
    torch.manual_seed(1)
    D = 768
    x = torch.randn(T, D, device="cuda").to(BF)
    w1 = (torch.randn(64, D, device="cuda") * D ** -0.5).to(BF)
    w2 = (torch.randn(48, 64, device="cuda") * 0.2).to(BF)
    b2 = torch.randn(48, device="cuda").to(BF)
    dout = torch.randn(T, n, device="cuda").to(BF)

    def run(impl, dtype):
        xs = x.detach().clone().to(dtype).requires_grad_(True)
        a, b, c = (t.detach().clone().to(dtype).requires_grad_(True) for t in (w1, w2, b2))
        sc = torch.tensor(0.1, device="cuda", requires_grad=True) if param_scale else 0.1
        out = impl(xs, a, b[:n], c[:n], sc)
        out.backward(dout.to(out.dtype))
        return out, xs.grad, a.grad, b.grad[:n], c.grad[:n], (sc.grad if param_scale else None)

    def oracle(xs, a, b, c, sc):
        h = F.gelu(F.linear(xs, a))
        return (F.linear(h, b) + c) * sc

    got = run(fused.gate_mlp, BF)
    want = run(oracle, torch.float32)
    tol = [1.2e-2, 2e-2, 2e-2, 2e-2, 2e-2]
    for g, w, t, name in zip(got, want, tol, ("out", "dx", "dw1", "dw2", "db2")):
        assert _rel(g, w) < t, (name, _rel(g, w))
    if param_scale:
        assert abs(got[5].item() - want[5].item()) < 2e-2 * abs(want[5].item()) + 1.0
    got2 = run(fused.gate_mlp, BF)
    assert all(torch.equal(a, b) for a, b in zip(got[:5], got2[:5]))          # no atomics anywhere
    fused.check_status()


def test_batched_mlp_weight_refresh_matches_per_layer_kernels(fused):
    from modded_nanogpt_b200.ops import native
    C = native.lib()
    torch.manual_seed(2)
    Lp, hid, dim = 4, 3072, 768
    bank = (torch.randn(Lp, 2, hid, dim, device="cuda") * 0.03).to(BF)
    used, nxt = torch.full((Lp,), 7.0, device="cuda"), torch.full((Lp,), 3.0, device="cuda")
    st = fused.MlpFp8State(bank)
    st.amax_bits.copy_(torch.tensor([0.0, 2.5, 0.0, 9.0], device="cuda").view(torch.int32))
    st.act_scale.fill_(5.0)
    fused.quantize_mlp_weights(bank, st, used, nxt, bootstrap=False)
    for l in range(Lp):
        q, s = C.quant_rows(bank[l, 0].contiguous())
        assert torch.equal(q.view(torch.uint8), st.fc8[l].view(torch.uint8)) and torch.equal(s, st.fc_scale[l])
        qt = torch.empty(dim, hid, dtype=torch.float8_e4m3fn, device="cuda")
        sc = torch.empty(dim, device="cuda")
        C.quant_transpose(bank[l, 1].contiguous(), qt, sc, torch.empty(dim, dtype=torch.int32, device="cuda"))
        assert torch.equal(qt.view(torch.uint8), st.projT8[l].view(torch.uint8)) and torch.equal(sc, st.projT_scale[l])
        # and against the plain statement of the op
        assert torch.allclose(st.projT_scale[l], bank[l, 1].float().abs().amax(0) / 448, rtol=1e-6)
    assert torch.allclose(used, torch.full((Lp,), 3.0, device="cuda"))
    assert torch.allclose(nxt, st.projT_scale.amax(1) * 1.12)
    want_act = torch.tensor([5.0, 2.5 * 1.8 / 448, 5.0, 9.0 * 1.8 / 448], device="cuda")
    assert torch.allclose(st.act_scale, want_act) and int(st.amax_bits.abs().sum()) == 0
    fused.quantize_mlp_weights(bank, st, used, nxt, bootstrap=True)
    assert torch.allclose(used, st.projT_scale.amax(1))
    fused.check_status()


@pytest.mark.parametrize("T,use_fp8", [(4096, False), (4096, True), (49152, True)])
def test_mlp_with_fused_residual_mix(fused, T, use_fp8):
    """a * x + b * relu(norm(x) W1^T)^2 W2 in one autograd node against the fp32 statement; also against the unfused
    pair (MLP node + lincomb) on the same kernels, which it must match closely in every gradient."""
    from modded_nanogpt_b200.ops.glue import Term, lincomb
    torch.manual_seed(3)
    D, hid = 768, 3072
    bank = torch.empty(1, 2, hid, D, device="cuda")
    bank[0, 0].uniform_(-1, 1).mul_(3 ** 0.5 * 0.5 * D ** -0.5)
    bank[0, 1].normal_(0, 0.02)
    bank = bank.to(BF)
    x = torch.randn(T, D, device="cuda").to(BF)
    g = (torch.randn(T, D, device="cuda") * 0.05).to(BF)
    st = None
    if use_fp8:
        st = fused.quantize_mlp_weights(bank, None, torch.ones(1, device="cuda"), torch.ones(1, device="cuda"), True)
        st.act_scale.fill_(0.25)                                   # relu(.)^2 of unit-variance inputs stays well below 448 * 0.25
        st = st.layer(0)

    def run(mode):
        xs = x.clone().requires_grad_(True)
        a = torch.tensor(1.05, device="cuda", requires_grad=True)
        b = torch.tensor(0.8, device="cuda", requires_grad=True)
        gv = (torch.zeros(hid, D, dtype=BF, device="cuda"), torch.zeros(hid, D, dtype=BF, device="cuda"))
        if mode == "fused":
            y = fused.norm_relu2_mlp_mix(xs, bank[0, 0], bank[0, 1], a, b, st, gv)
        elif mode == "unfused":
            h, xr = fused.norm_relu2_mlp(xs, bank[0, 0], bank[0, 1], st, gv, fork=True)
            y = lincomb([Term(xr, scalar=a), Term(h, scalar=b)])
        else:
            xf = xs.float()
            w1, w2 = bank[0, 0].float().requires_grad_(True), bank[0, 1].float().requires_grad_(True)
            h = torch.relu(F.rms_norm(xf, (D,)) @ w1.T).square() @ w2
            y = a * xf + b * h
            y.backward(g.float())
            # scale of the signed sums behind da and db: the norm of their terms
            run.term_norm = dict(da=(g.float() * xf).norm().item(), db=(g.float() * h).norm().item())
            return y, xs.grad, a.grad, b.grad, w1.grad, w2.grad
        y.backward(g)
        return y, xs.grad, a.grad, b.grad, gv[0], gv[1]

    got, unf, ref = run("fused"), run("unfused"), run("oracle")
    tol = 6e-2 if use_fp8 else 1.5e-2                          # e4m3 activations and weights in the forward
    names = ("y", "dx", "da", "db", "dW1", "dW2")
    for name, a, b in zip(names, got, ref):
        if a.numel() == 1:
            # a sum of T * D signed terms, each off by a relative error of the order of tol
            assert abs(a.item() - b.item()) < tol * abs(b.item()) + 4 * tol * run.term_norm[name], (name, a.item(), b.item())
        else:
            assert _rel(a, b) < tol, (name, _rel(a, b))
    for name, a, b in zip(names, got, unf):                       # same kernels, mix moved into the epilogues
        if a.numel() == 1:
            # bf16: the same products in both paths.  FP8: the unfused path sums g . (e4m3(post) e4m3(W2)), the fused one
            # (g W2) . post with the bf16 operands of the backward GEMM: they differ by a quantisation error per term
            slack = 2 * tol * run.term_norm[name] if use_fp8 else 1e-2
            assert abs(a.item() - b.item()) < 5e-3 * abs(b.item()) + slack, (name, a.item(), b.item())
        else:
            assert _rel(a, b) < 8e-3, (name, _rel(a, b))
    fused.check_status()


@pytest.mark.parametrize("T,paired,key_offset,with_ve", [(2048, False, False, False), (2048, True, False, True),
                                                          (4096, False, True, False), (2048, False, True, True),
                                                          (49152, False, True, True), (49152, True, False, False)])
def test_qkv_projection_with_fused_postprocessing(fused, T, paired, key_offset, with_ve):
    """qkv_proj (norm / rotary / key offset / value add inside the GEMM epilogue, backward from the outputs) against the
    projection followed by the stand-alone post-processing kernels, and both against the fp32 statement on a slice."""
    from modded_nanogpt_b200.ops.glue import qkv_post
    torch.manual_seed(5)
    D, H = 768, 6
    x = torch.randn(T, D, device="cuda").to(BF)
    w = (torch.randn(3 * D, D, device="cuda") * D ** -0.5).to(BF)
    t = torch.arange(2 * T, device="cuda", dtype=torch.float32)
    freq = (1 / 1024) ** torch.linspace(0, 1, 32, device="cuda")
    cos, sin = torch.outer(t, freq).cos().contiguous(), torch.outer(t, freq).sin().contiguous()
    ve = torch.randn(T, D, device="cuda").to(BF) if with_ve else None
    vg = torch.rand(T, H, device="cuda").to(BF) if with_ve else None
    g = [torch.randn(T, H, 128, device="cuda").to(BF) for _ in range(3)]

    def run(fused_path):
        xs = x.clone().requires_grad_(True)
        lam = torch.tensor(0.8, device="cuda", requires_grad=True)
        ves = ve.clone().requires_grad_(True) if with_ve else None
        vgs = vg.clone().requires_grad_(True) if with_ve else None
        gv = [torch.zeros(2 * D, D, dtype=BF, device="cuda"), torch.zeros(D, D, dtype=BF, device="cuda")]
        if fused_path:
            q, k, v = fused.qkv_proj(xs, lam, w, gv, cos, sin, ves, vgs, H, paired, key_offset)
        else:
            q, k, v = qkv_post(fused.bank_linear(xs, lam, w, gv), cos, sin, ves, vgs, None, H, paired, key_offset)
        torch.autograd.backward([q, k, v], g)
        return (q, k, v, xs.grad, lam.grad, gv[0], gv[1], ves.grad if with_ve else None, vgs.grad if with_ve else None)

    a, b = run(True), run(False)
    names = ("q", "k", "v", "dx", "dlam", "dW_qk", "dW_v", "dve", "dvgate")
    for n, u, v_ in zip(names, a, b):
        if u is None:
            continue
        if u.numel() == 1:
            # <dW, W>: the q and k parts cancel almost exactly (the norm makes them scale invariant), so the sum is
            # small against its terms; compare on the scale of the Cauchy-Schwarz bound
            bound = (a[5].float().norm() * w[:2 * D].float().norm() + a[6].float().norm() * w[2 * D:].float().norm()).item()
            assert abs(u.item() - v_.item()) < 2e-2 * abs(v_.item()) + 2e-3 * bound, (n, u.item(), v_.item(), bound)
        else:
            assert _rel(u, v_) < 1.2e-2, (n, _rel(u, v_))
    # boundary rows of the key offset, exactly: row 0 keeps its own stationary half, row t takes row t-1's
    if key_offset:
        kf, kp = a[1], b[1]
        assert _rel(kf[:3], kp[:3]) < 8e-3 and _rel(kf[-3:], kp[-3:]) < 8e-3
        assert (kf[1:5, :, 64:].float() - kf[1:5, :, 64:].float()).abs().max() == 0
    # fp32 statement of the forward on the first 256 rows
    sl = slice(0, 256)
    raw = ((x[sl].float() @ w.float().T) * 0.8).to(BF).float().view(256, 3, H, 128)
    eps = torch.finfo(torch.float32).eps
    nq, nk = [(r * torch.rsqrt(r.square().mean(-1, keepdim=True) + eps)).to(BF).float() for r in (raw[:, 0], raw[:, 1])]
    pos = (2 * torch.arange(256, device="cuda")[:, None] + (torch.arange(H, device="cuda")[None, :] & 1)) if paired \
        else torch.arange(256, device="cuda")[:, None].expand(256, H)
    c, s_ = cos[pos], sin[pos]                                       # [256, H, 32]

    def rope(n):
        o = n.clone()
        o[..., 0:64:2] = c * n[..., 0:64:2] + s_ * n[..., 1:64:2]
        o[..., 1:64:2] = c * n[..., 1:64:2] - s_ * n[..., 0:64:2]
        return o

    want_q, want_k = rope(nq), rope(nk)
    if key_offset:
        want_k[1:, :, 64:] = nk[:-1, :, 64:]
    want_v = raw[:, 2] + (vg[sl].float()[:, :, None] * ve[sl].float().view(256, H, 128) if with_ve else 0)
    assert _rel(a[0][sl], want_q) < 8e-3 and _rel(a[1][sl], want_k) < 8e-3 and _rel(a[2][sl], want_v) < 8e-3
    fused.check_status()
