"""Numerics of every sm_100a kernel against a plain PyTorch fp32 restatement of the same op."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

BF, F8, F8B = torch.bfloat16, torch.float8_e4m3fn, torch.float8_e5m2


@pytest.fixture(scope="module")
def fused():
    from modded_nanogpt_b200.ops import fused, native
    assert native.available(required=True)
    return fused


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _ok(fused):
    fused.check_status()


@pytest.mark.parametrize("M,N,K,batch,bn", [(256, 512, 768, 1, 256), (128, 128, 64, 1, 128), (384, 768, 3072, 3, 128),
                                             (256, 50304, 768, 1, 256), (200, 328, 136, 2, 128)])
def test_gemm_bf16_kk(fused, M, N, K, batch, bn):
    torch.manual_seed(0)
    shp = (batch,) if batch > 1 else ()
    a = torch.randn(*shp, M, K, device="cuda").to(BF)
    b = torch.randn(*shp, N, K, device="cuda").to(BF)
    out = fused.gemm(a, b, bn=bn)
    ref = a.float() @ b.float().mT
    assert _rel(out, ref) < 5e-3
    _ok(fused)


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True)])
@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_bf16_mn_major(fused, a_mn, b_mn, bn):
    torch.manual_seed(1)
    M, N, K = 384, 512, 640
    a = torch.randn(K, M, device="cuda").to(BF) if a_mn else torch.randn(M, K, device="cuda").to(BF)
    b = torch.randn(K, N, device="cuda").to(BF) if b_mn else torch.randn(N, K, device="cuda").to(BF)
    out = fused.gemm(a, b, a_mn=a_mn, b_mn=b_mn, bn=bn, out_dtype=torch.float32)
    A = a.float().T if a_mn else a.float()
    B = b.float() if b_mn else b.float().T
    assert _rel(out, A @ B) < 1e-3
    _ok(fused)


@pytest.mark.parametrize("n,rows,batch", [(768, 3072, 2), (384, 256, 3), (1024, 1024, 1)])
def test_gemm_symmetric_products(fused, n, rows, batch):
    """Gram products and b A + c A A computed on the upper-triangular tiles and mirrored: equal to the full product on
    the same kernel, exactly symmetric, and close to the fp32 statement."""
    torch.manual_seed(7)
    X = (torch.randn(batch, rows, n, device="cuda") * rows ** -0.5).to(BF)
    full = fused.gemm(X, X, a_mn=True, b_mn=True, bn=128)                      # X^T X, both operands MN-major
    sym = fused.gemm(X, X, a_mn=True, b_mn=True, symmetric=True)
    assert torch.equal(sym, sym.transpose(-1, -2))
    assert torch.equal(torch.triu(sym), torch.triu(full))                       # the computed tiles are the same tiles
    assert _rel(sym, X.float().transpose(-1, -2) @ X.float()) < 4e-3
    Xt = X.transpose(-1, -2).contiguous()                                       # [batch, n, rows]: X X^T with K-major operands
    sym2 = fused.gemm(Xt, Xt, symmetric=True)
    assert torch.equal(sym2, sym2.transpose(-1, -2)) and _rel(sym2, Xt.float() @ Xt.float().transpose(-1, -2)) < 4e-3
    A = sym
    B = fused.gemm(A, A, b_mn=True, alpha=0.5, beta=-2.0, cin=A, symmetric=True)
    want = -2.0 * A.float() + 0.5 * (A.float() @ A.float())
    assert torch.equal(B, B.transpose(-1, -2)) and _rel(B, want) < 6e-3
    B32 = fused.gemm(A, A, b_mn=True, symmetric=True, out_dtype=torch.float32)
    assert torch.equal(B32, B32.transpose(-1, -2)) and _rel(B32, A.float() @ A.float()) < 2e-3
    _ok(fused)


def test_gemm_alpha_beta_scales(fused):
    torch.manual_seed(2)
    M, N, K = 256, 256, 256
    a = torch.randn(2, M, K, device="cuda").to(BF)
    cin = torch.randn(2, M, N, device="cuda").to(BF)
    rs = torch.rand(2 * M, device="cuda") + 0.5
    cs = torch.rand(2 * N, device="cuda") + 0.5
    at = torch.tensor([0.5], device="cuda")
    out = fused.gemm(a, a, alpha=0.7, beta=-1.3, cin=cin, alpha_t=at, row_scale=rs, col_scale=cs)
    ref = 0.35 * (a.float() @ a.float().mT) * rs.view(2, M, 1) * cs.view(2, 1, N) - 1.3 * cin.float()
    assert _rel(out, ref) < 6e-3
    _ok(fused)


def _q8(x, dt=F8):
    return x.to(dt)


def test_gemm_fp8_variants(fused):
    torch.manual_seed(3)
    M, N, K = 256, 640, 512
    a = _q8(torch.randn(M, K, device="cuda"))
    b = _q8(torch.randn(N, K, device="cuda"))
    rs, cs = torch.rand(M, device="cuda") + 0.5, torch.rand(N, device="cuda") + 0.5
    out = fused.gemm(a, b, row_scale=rs, col_scale=cs)
    ref = (a.float() @ b.float().T) * rs[:, None] * cs[None, :]
    assert _rel(out, ref) < 5e-3
    a5 = _q8(torch.randn(M, K, device="cuda"), F8B)                      # e5m2 x e4m3, K-major
    assert _rel(fused.gemm(a5, b, alpha=0.25), 0.25 * (a5.float() @ b.float().T)) < 5e-3
    bmn = _q8(torch.randn(K, N, device="cuda"))                          # e4m3 x e4m3, B MN-major
    assert _rel(fused.gemm(a, bmn, b_mn=True), a.float() @ bmn.float()) < 5e-3
    amn, b5 = _q8(torch.randn(K, M, device="cuda")), _q8(torch.randn(K, N, device="cuda"), F8B)
    out = fused.gemm(amn, b5, a_mn=True, b_mn=True, out_dtype=torch.float32)   # e4m3^T x e5m2, both MN-major
    assert _rel(out, amn.float().T @ b5.float()) < 1e-3
    _ok(fused)


def test_gemm_relu2_and_dpre_epilogues(fused):
    torch.manual_seed(4)
    T, D, H = 384, 256, 1024
    x8 = _q8(torch.randn(T, D, device="cuda"))
    w8 = _q8(torch.randn(H, D, device="cuda") * 0.3)
    rs, cs = torch.rand(T, device="cuda") * 0.1 + 0.05, torch.rand(H, device="cuda") * 0.1 + 0.05
    act = torch.tensor([0.02], device="cuda")
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    post = torch.empty(T, H, dtype=BF, device="cuda")
    post8 = torch.empty(T, H, dtype=F8, device="cuda")
    fused.gemm(x8, w8, out=post, epilogue=fused.EPI_RELU2, row_scale=rs, col_scale=cs, out8=post8, act_scale=act, amax_bits=amax)
    pre = ((x8.float() @ w8.float().T) * rs[:, None] * cs[None, :]).to(BF)
    ref = torch.relu(pre).square()
    assert _rel(post, ref) < 1e-2
    ref8 = (ref.float() / 0.02).clamp(max=448).to(F8)
    assert _rel(post8, ref8) < 3e-2
    assert abs(amax.view(torch.float32).item() - post.float().max().item()) < 1e-6
    g = torch.randn(T, D, device="cuda").to(BF)
    w2 = (torch.randn(H, D, device="cuda") * 0.1).to(BF)
    dpre = fused.gemm(g, w2, epilogue=fused.EPI_DPRE, cin=post)
    ref = 2 * (g.float() @ w2.float().T).to(BF).float() * post.float().sqrt()
    assert _rel(dpre, ref) < 1e-2
    _ok(fused)


def test_rmsnorm_fwd_bwd_and_quant(fused):
    from modded_nanogpt_b200.ops import native
    C = native.lib()
    torch.manual_seed(5)
    x = (torch.randn(1000, 768, device="cuda") * 3).to(BF).requires_grad_(True)
    y = fused.rms_norm(x)
    xr = x.detach().float().requires_grad_(True)
    eps = torch.finfo(torch.float32).eps
    yr = xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + eps)
    assert _rel(y, yr) < 4e-3
    dy = torch.randn_like(y)
    y.backward(dy)
    yr.backward(dy.float())
    assert _rel(x.grad, xr.grad) < 6e-3
    y2, y8, scale, _ = C.rmsnorm_fwd(x.detach(), True, True, False)
    assert torch.equal(y2, y.detach())
    assert torch.allclose(scale, y2.float().abs().amax(-1) / 448, rtol=1e-6)
    assert _rel(y8.float() * scale[:, None], y2) < 4e-2
    q, s = C.quant_rows(y2)
    assert torch.equal(q.view(torch.uint8), y8.view(torch.uint8)) and torch.equal(s, scale)


def test_transposes(fused):
    from modded_nanogpt_b200.ops import native
    C = native.lib()
    torch.manual_seed(6)
    src = torch.randn(300, 1000, device="cuda").to(BF)
    dst = torch.randn(1000, 300, device="cuda").to(BF)
    d0 = dst.clone()
    C.transpose(src, dst, True)
    assert torch.equal(dst, (d0.float() + src.float().T).to(BF))
    C.transpose(src, dst, False)
    assert torch.equal(dst, src.T.contiguous())
    q = torch.empty(1000, 300, dtype=F8, device="cuda")
    sc = torch.empty(1000, device="cuda")
    C.quant_transpose(src, q, sc, torch.empty(1000, dtype=torch.int32, device="cuda"))
    assert torch.allclose(sc, src.float().abs().amax(0) / 448, rtol=1e-6)
    assert _rel(q.float() * sc[:, None], src.T) < 4e-2


@pytest.mark.parametrize("e5m2", [False, True])
def test_softcap_ce_kernel(fused, e5m2):
    from modded_nanogpt_b200.ops import native, reference as ref
    C = native.lib()
    torch.manual_seed(7)
    T, V = 96, 50304
    logits = (torch.randn(T, V, device="cuda") * 4).to(BF)
    tg = torch.randint(0, V, (T,), device="cuda")
    tg[5] = tg[6]                                   # two predictions of row 5 hit the same column
    pt = torch.randint(-1, V, (T,), device="cuda")
    pt[7] = tg[7]
    mtp = torch.tensor([1.0, 0.5, 0.25], device="cuda")
    pw = torch.tensor([0.3], device="cuda")
    gm = 64.0 if e5m2 else 0.125
    losses, dl = C.softcap_ce(logits, tg, mtp, pt, pw, e5m2, 23.0, 5.0, 7.5, gm)
    lg = logits.float().requires_grad_(True)
    z = ref.softcap(lg, 23.0, 5.0, 7.5)
    want = ref.softcap_ce_loss_rows(z, tg, 0, mtp, pt, pw[0], T)
    (want.sum() * gm).backward()
    assert torch.allclose(losses, want, atol=3e-2, rtol=2e-3)
    assert _rel(dl, lg.grad) < (8e-2 if e5m2 else 1.5e-2)
    cols = torch.stack([tg, pt.clamp_min(0)], 1)
    got, exp = dl.float().gather(1, cols), lg.grad.gather(1, cols)
    assert torch.allclose(got, exp, rtol=0.15 if e5m2 else 0.03, atol=1e-4 * gm)


def test_fused_mlp_matches_reference(fused):
    from modded_nanogpt_b200.ops import reference as ref
    torch.manual_seed(8)
    T, D, H = 512, 768, 3072
    x = (torch.randn(T, D, device="cuda")).to(BF).requires_grad_(True)
    bank = torch.zeros(1, 2, H, D, device="cuda", dtype=BF)
    bank[0, 0].uniform_(-0.03, 0.03)
    bank[0, 1].uniform_(-0.03, 0.03)
    w1, w2 = bank[0, 0].clone().requires_grad_(True), bank[0, 1].clone().requires_grad_(True)
    for use_fp8 in (False, True):
        st = None
        if use_fp8:
            st = fused.quantize_mlp_weights(bank, None, torch.ones(1, device="cuda"), torch.ones(1, device="cuda"), True)
            st.act_scale.fill_(4.0 / 448)
        out = fused.norm_relu2_mlp(x, w1, w2, st.layer(0) if st else None)
        g = torch.randn_like(out)
        gx, g1, g2 = torch.autograd.grad(out, (x, w1, w2), g)
        xr, w1r, w2r = (t.detach().float().requires_grad_(True) for t in (x, w1, w2))
        eps = torch.finfo(torch.float32).eps
        yr = xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + eps)
        outr = ref.relu2_mlp(yr, w1r, w2r)
        gxr, g1r, g2r = torch.autograd.grad(outr, (xr, w1r, w2r), g.float())
        tol = 6e-2 if use_fp8 else 1.5e-2
        assert _rel(out, outr) < tol
        assert _rel(gx, gxr) < tol and _rel(g1, g1r) < tol and _rel(g2, g2r) < tol
        if use_fp8:
            assert st.amax_bits.view(torch.float32).item() > 0
    fused.check_status()


@pytest.mark.parametrize("fp8", [False, True])
def test_fused_lm_head_ce(fused, fp8):
    from modded_nanogpt_b200.ops import reference as ref
    torch.manual_seed(9)
    T, D, V = 256, 768, 50304
    x = torch.randn(T, D, device="cuda")
    x = (x * torch.rsqrt(x.square().mean(-1, keepdim=True))).to(BF).requires_grad_(True)
    w = (torch.randn(D, V, device="cuda") * 0.02).to(BF).requires_grad_(True)
    tg = torch.randint(0, V, (T,), device="cuda")
    mtp = torch.tensor([1.0, 0.5], device="cuda")
    pt = torch.randint(-1, V, (T,), device="cuda")
    pw = torch.tensor([0.25], device="cuda")
    gs = 0.125
    loss = fused.softcap_ce(x, w, tg, mtp, pt, pw, 23.0, 5.0, 7.5, grad_scale=gs, fp8=fp8)
    (loss.sum() * gs).backward()
    xr, wr = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lr = ref.softcap_ce(xr, wr, tg, mtp, pt, pw, 23.0, 5.0, 7.5)
    (lr.sum() * gs).backward()
    assert torch.allclose(loss, lr, rtol=2e-2 if fp8 else 5e-3, atol=5e-2)
    assert _rel(x.grad, xr.grad) < (0.12 if fp8 else 2e-2)
    assert _rel(w.grad, wr.grad) < (0.12 if fp8 else 2e-2)
    fused.check_status()


def test_eval_loss_on_own_kernels(fused):
    """The evaluation loss (bf16 logits GEMM + streaming loss kernel, chunked) against the PyTorch statement."""
    from modded_nanogpt_b200.ops import functional, reference as ref
    torch.manual_seed(21)
    T, D, V = 1000 * 8, 768, 50304
    x = torch.randn(T, D, device="cuda").to(BF)
    w = (torch.randn(D, V, device="cuda") * 0.03).to(BF)
    tg = torch.randint(0, V, (T,), device="cuda")
    got = fused.softcap_ce_eval(x, w, tg, 23.0, 5.0, 7.5, chunk=3000)          # chunks of uneven size
    want = ref.softcap_ce_eval(x, w, tg, 23.0, 5.0, 7.5)
    exact = F.cross_entropy(23.0 * torch.sigmoid(((x.float() @ w.float()) + 5.0) / 7.5), tg, reduction="none")
    assert got.shape == want.shape and torch.isfinite(got).all()
    assert (got - exact).abs().max() < 6e-2 and abs(got.mean().item() - exact.mean().item()) < 2e-3
    assert (got - exact).abs().mean() <= (want - exact).abs().mean() * 1.5 + 1e-3   # at least as close as the bf16 softcap
    assert torch.equal(functional.softcap_ce_eval(x, w, tg, 23.0, 5.0, 7.5), fused.softcap_ce_eval(x, w, tg, 23.0, 5.0, 7.5))
    _ok(fused)


def test_fp8_linear_t(fused):
    torch.manual_seed(7)
    T, D, V = 512, 256, 1024
    x = (torch.randn(T, D, device="cuda") * 2).to(BF).requires_grad_(True)
    w = (torch.randn(D, V, device="cuda") * 0.05).to(BF).requires_grad_(True)
    x_s, w_s, g_s = 8 / 448, 0.25 / 448, 4 / 448
    y = fused.fp8_linear_t(x, w, x_s, w_s, g_s)
    g = torch.randn(T, V, device="cuda").to(BF)
    y.backward(g)
    xq = (x.float() / x_s).clamp(-448, 448).to(F8).float() * x_s
    wq = (w.float() / w_s).clamp(-448, 448).to(F8).float() * w_s
    gq = (g.float() / g_s).to(F8B).float() * g_s
    assert _rel(y, xq @ wq) < 5e-3
    assert _rel(x.grad, gq @ wq.T) < 5e-3
    assert _rel(w.grad, xq.T @ gq) < 8e-3        # fp32 from the GEMM, cast to the parameter dtype by autograd
    _ok(fused)


def test_adam_kernel(fused):
    from modded_nanogpt_b200.ops import native, reference as ref
    C = native.lib()
    torch.manual_seed(10)
    for dt, n in ((BF, 4096 * 3), (torch.float32, 4096 * 3), (BF, 8 * 1237), (torch.float32, 4 * 1237), (BF, 8), (BF, 3 * 10**6 + 8)):
        p = (torch.randn(n, device="cuda") * 0.1).to(dt)
        g = (torch.randn(n, device="cuda") * 0.01).to(dt)
        m, v = torch.rand(n, device="cuda") * 0.01, torch.rand(n, device="cuda") * 1e-4
        pr, mr, vr = p.clone(), m.clone(), v.clone()
        C.adam([g.data_ptr()], [p.data_ptr()], 0, 0, m, v, n, dt == torch.float32, 0.9, 0.99, 1e-10, 3e-3, 2e-4, 1.0, None, 0, 0, 0)
        ref.adam_update_(pr, g, mr, vr, 0.9, 0.99, 1e-10, 3e-3, 2e-4)
        assert torch.allclose(m, mr, rtol=1e-5, atol=1e-8) and torch.allclose(v, vr, rtol=1e-5, atol=1e-10)
        assert (p.float() - pr.float()).abs().max() < (2e-3 if dt == BF else 1e-6)


def test_adam_small_batch(fused):
    """One launch updates a batch of small parameters of any size and of either dtype; two "ranks" are two gradient
    buffers at the same offset from two bases in this GPU's memory."""
    from modded_nanogpt_b200.ops import native, reference as ref
    C = native.lib()
    torch.manual_seed(13)
    specs = [(22, torch.float32), (1, torch.float32), (82, BF), (98304, BF), (5248, torch.float32), (12, BF)] * 3   # 18 > one table
    arenas = [torch.zeros(4 << 20, dtype=torch.uint8, device="cuda") for _ in range(2)]
    off, entries, refs = 0, [], []
    for n, dt in specs:
        nb = n * (4 if dt == torch.float32 else 2)
        views = []
        for a in arenas:
            pv = a[off:off + nb].view(dt)
            gv = a[off + (1 << 21):off + (1 << 21) + nb].view(dt)
            views.append((pv, gv))
        p0 = (torch.randn(n, device="cuda") * 0.1).to(dt)
        gs = [(torch.randn(n, device="cuda") * 0.01).to(dt) for _ in arenas]
        for (pv, gv), g in zip(views, gs):
            pv.copy_(p0)
            gv.copy_(g)
        m, v = torch.rand(n, device="cuda") * 0.01, torch.rand(n, device="cuda") * 1e-4
        hyper = [0.9, 0.99, 1e-10, 3e-3 * (1 + len(entries)), 2e-4]
        pr, mr, vr = p0.clone(), m.clone(), v.clone()
        gavg = ((gs[0].float() + gs[1].float()) * 0.5).to(dt)
        ref.adam_update_(pr, gavg, mr, vr, *hyper)
        entries.append((off, off + (1 << 21), m, v, n, int(dt == torch.float32), hyper))
        refs.append((views[0][0], pr, m, mr, v, vr, dt))
        off += -(-nb // 256) * 256
    assert off < (1 << 21)
    C.adam_small([a.data_ptr() for a in arenas], 0, [e[0] for e in entries], [e[1] for e in entries], [e[2] for e in entries],
                 [e[3] for e in entries], [e[4] for e in entries], [e[5] for e in entries], [h for e in entries for h in e[6]], 0.5)
    for pv, pr, m, mr, v, vr, dt in refs:
        assert torch.allclose(m, mr, rtol=1e-5, atol=1e-8) and torch.allclose(v, vr, rtol=1e-5, atol=1e-10)
        assert (pv.float() - pr.float()).abs().max() < (2e-3 if dt == BF else 1e-6)
    _ok(fused)


def test_adam_kernel_row_mask(fused):
    """Rows whose mask byte is 0 are not read: the update equals Adam on the gradient with those rows zeroed, even
    when the skipped rows hold garbage.  Two "ranks" are two gradient buffers of this GPU."""
    from modded_nanogpt_b200.ops import native
    C = native.lib()
    torch.manual_seed(12)
    rows, cols = 96, 768
    n = rows * cols
    p = (torch.randn(n, device="cuda") * 0.1).to(BF)
    gs = [(torch.randn(rows, cols, device="cuda") * 0.01).to(BF) for _ in range(2)]
    mask = (torch.rand(2, rows, device="cuda") < 0.4).to(torch.uint8)
    clean = [g * mask[i][:, None].to(BF) for i, g in enumerate(gs)]                 # what the ranks "really" hold
    dirty = [torch.where(mask[i][:, None].bool(), g, torch.full_like(g, 7.0)) for i, g in enumerate(gs)]
    off, cnt = 16 * cols, 64 * cols                                                  # update rows 16..79 only
    outs = []
    for grads, mk in ((clean, None), (dirty, mask)):
        pp = p.clone()
        m, v = torch.zeros(cnt, device="cuda"), torch.zeros(cnt, device="cuda")
        C.adam([g.data_ptr() for g in grads], [pp.data_ptr(), pp.data_ptr()], 0, off, m, v, cnt, False, 0.9, 0.99, 1e-10,
               3e-3, 2e-4, 0.5, mk, cols if mk is not None else 0, 0, 0)
        outs.append((pp, m, v))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert not torch.equal(outs[0][0], p)


def test_normuon_kernels(fused):
    from modded_nanogpt_b200.ops import native, reference as ref
    C = native.lib()
    torch.manual_seed(11)
    for (mats, rows, cols) in ((3, 256, 768), (2, 3072, 768), (2, 768, 768), (2, 768, 3072)):
        g = (torch.randn(mats, rows, cols, device="cuda") * 1e-3).to(BF)
        buf = torch.randn(mats, rows, cols, device="cuda") * 1e-3
        bufr = buf.clone()
        out = torch.empty_like(g)
        ss = torch.empty(mats, device="cuda")
        C.nesterov([g.data_ptr()], 0, 0, buf, out, ss, 0.9, 1.0, 0)
        ur = ref.nesterov_momentum_(g.float(), bufr, 0.9)
        assert torch.allclose(buf, bufr, rtol=1e-5, atol=1e-9) and _rel(out, ur) < 4e-3
        assert torch.allclose(ss, out.float().square().sum((-2, -1)), rtol=1e-4)
        x = out.clone()
        C.scale_by_norm(x, ss)
        xr = out / (out.norm(dim=(-2, -1), keepdim=True) * (1 + 2e-2) + 1e-6)
        assert _rel(x, xr) < 8e-3
        # variance reduction + cautious update with mantissa
        v = torch.randn(mats, rows, cols, device="cuda").to(BF) * 0.05
        red_rows = rows >= cols
        sm_shape = (mats, rows, 1) if red_rows else (mats, 1, cols)
        sm = torch.rand(sm_shape, device="cuda") * 1e-3
        smr = sm.clone()
        p = (torch.randn(mats, rows, cols, device="cuda") * 0.05).to(BF)
        mant = torch.randint(0, 65536, (mats, rows, cols), device="cuda").to(torch.uint16)
        pr, mantr = p.clone(), mant.clone()
        muls = torch.tensor([1.0 + i for i in range(mats)], device="cuda")
        lrs = 0.02 * muls
        scratch = torch.zeros(mats * (max(rows, cols) + 65), device="cuda")
        C.normuon_apply([p.data_ptr()], 0, 0, mant, v, sm, scratch, red_rows, 0.9, 0.03, 0.02, muls, 0)
        assert int(scratch[-mats:].view(torch.int32).abs().sum()) == 0          # the per-matrix counters are left at zero
        vr = ref.normuon_variance_reduction_(v.clone(), smr, 0.9, -1 if red_rows else -2)
        for i in range(mats):
            ref.cautious_update_mantissa_(pr[i], mantr[i], vr[i], 0.03, float(lrs[i]))
        assert torch.allclose(sm, smr, rtol=1e-4, atol=1e-9)
        full = lambda a, b: ((a.view(torch.int16).to(torch.int32) << 16) | (b.view(torch.int16).to(torch.int32) & 0xFFFF)).view(torch.float32)
        assert (full(p, mant) - full(pr, mantr)).abs().max() < 2e-4


@pytest.mark.parametrize("shape", [(2, 3072, 768), (3, 768, 768), (4, 256, 768), (2, 768, 3072)])
def test_polar_express_on_the_gemm_kernels(fused, shape, monkeypatch):
    """Polar Express on the batched tcgen05 GEMMs (symmetric products on mirrored upper-triangular tiles where the
    shape allows) against the fp32 statement: same result with and without the symmetric path, singular values near 1."""
    from modded_nanogpt_b200.ops import reference as ref
    from modded_nanogpt_b200.optim import cuda_math
    torch.manual_seed(9)
    g = torch.randn(*shape, device="cuda")
    x0 = (g / (g.norm(dim=(-2, -1), keepdim=True) * 1.02 + 1e-6)).to(BF)
    outs = {}
    for sym in (True, False):
        monkeypatch.setattr(cuda_math, "SYMMETRIC_PE", sym)
        outs[sym] = cuda_math.CudaMath().polar_express(x0.clone()).float()
    assert _rel(outs[True], outs[False]) < 2e-2
    want = ref.polar_express(g, torch.float32)
    assert _rel(outs[True], want) < 8e-2                                          # bf16 iterations against fp32 ones
    if shape[-1] != shape[-2]:
        sv = torch.linalg.svdvals(outs[True])
        assert sv.max() < 1.35 and sv.min() > 0.45, (sv.min().item(), sv.max().item())
    _ok(fused)


def test_normuon_kernels_with_two_rank_buffers(fused):
    """The reduce-scatter and all-gather sides of the NorMuon kernels with two "ranks" that are two buffers of this GPU:
    the Nesterov kernel sums both gradient buffers at an offset, the update kernel reads rank 1's weights and stores the
    new ones into both."""
    from modded_nanogpt_b200.ops import native, reference as ref
    C = native.lib()
    torch.manual_seed(14)
    mats, rows, cols = 2, 768, 768
    full = 3                                                                   # matrices in the whole bank; this "rank" owns 1..2
    gs = [(torch.randn(full, rows, cols, device="cuda") * 1e-3).to(BF) for _ in range(2)]
    off = rows * cols
    buf = torch.randn(mats, rows, cols, device="cuda") * 1e-3
    bufr = buf.clone()
    out, ss = torch.empty(mats, rows, cols, dtype=BF, device="cuda"), torch.empty(mats, device="cuda")
    C.nesterov([g.data_ptr() for g in gs], 1, off, buf, out, ss, 0.9, 0.5, 0)
    gavg = ((gs[0][1:].float() + gs[1][1:].float()) * 0.5).to(BF)
    ur = ref.nesterov_momentum_(gavg.float(), bufr, 0.9)
    assert torch.allclose(buf, bufr, rtol=1e-5, atol=1e-9) and _rel(out, ur) < 4e-3
    v = torch.randn(mats, rows, cols, device="cuda").to(BF) * 0.05
    sm = torch.rand(mats, rows, 1, device="cuda") * 1e-3
    smr = sm.clone()
    ps = [(torch.randn(full, rows, cols, device="cuda") * 0.05).to(BF) for _ in range(2)]
    ps[0][1:] = ps[1][1:]                                                      # replicas agree before the step
    untouched = [p[0].clone() for p in ps]
    mant = torch.randint(0, 65536, (mats, rows, cols), device="cuda").to(torch.uint16)
    pr, mantr = ps[1][1:].clone(), mant.clone()
    muls = torch.ones(mats, device="cuda")
    scratch = torch.zeros(mats * (max(rows, cols) + 65), device="cuda")
    C.normuon_apply([p.data_ptr() for p in ps], 1, off, mant, v, sm, scratch, True, 0.9, 0.03, 0.02, muls, 0)
    vr = ref.normuon_variance_reduction_(v.clone(), smr, 0.9, -1)
    for i in range(mats):
        ref.cautious_update_mantissa_(pr[i], mantr[i], vr[i], 0.03, 0.02)
    assert torch.equal(ps[0][1:], ps[1][1:]) and (ps[1][1:].float() - pr.float()).abs().max() < 2e-3
    assert torch.equal(ps[0][0], untouched[0]) and torch.equal(ps[1][0], untouched[1])      # outside the shard: not written
    _ok(fused)


def test_embed_bwd_accumulates_in_place(fused):
    from modded_nanogpt_b200.ops import native
    C = native.lib()
    torch.manual_seed(12)
    V, D, n = 5000, 768, 20000
    ids = torch.randint(0, V, (n,), device="cuda")
    ids[:6000] = 7                                   # a heavy hitter that spans many chunks
    ids[6000:6100] = 4999
    g = torch.randn(n, D, device="cuda").to(BF)
    grad = torch.randn(V, D, device="cuda").to(BF)
    want = grad.float().index_add(0, ids, g.float())
    s, perm = torch.sort(ids)
    C.embed_bwd(g, s, perm, grad)
    touched = torch.zeros(V, dtype=torch.bool, device="cuda")
    touched[ids] = True
    assert torch.equal(grad[~touched].float(), want[~touched])          # untouched rows stay bit-identical
    assert _rel(grad[touched], want[touched]) < 6e-3
    assert _rel(grad[7], want[7]) < 2e-2
