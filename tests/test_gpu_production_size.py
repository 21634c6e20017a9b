"""The kernels at the sizes of a training step (49,152 tokens per micro-batch) and of the final validation
(262,144 tokens, window 2,560): thousands of work items for the persistent attention backward, and the rows next
to document starts and window edges checked value by value against the dense fp32 oracle.  Outputs sit between
canary rows that no kernel may touch."""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _packed(T, seed=0, mean=600, cap=2048, slots=128):
    g = torch.Generator().manual_seed(seed)
    lens = torch.exp(torch.randn(4 * T // mean, generator=g) * 0.8 + 6.0).clamp(2, cap).long()
    starts = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)])
    starts = starts[starts < T][:slots - 1]
    cu = torch.full((slots,), T, dtype=torch.int32)
    cu[:len(starts)] = starts.int()
    return cu.cuda(), starts.cuda()


def _dense_rows(q, k, v, rows, doc_start, window, scale):
    """fp32 attention output for the given query rows only: out[r] = softmax(scale q_r k_j) v_j over
    max(doc_start[r], r - window) <= j <= r."""
    outs = []
    for r in rows.tolist():
        lo = max(int(doc_start[r]), r - window)
        s = torch.einsum("hd,khd->hk", q[r].float(), k[lo:r + 1].float()) * scale
        outs.append(torch.einsum("hk,khd->hd", torch.softmax(s, -1), v[lo:r + 1].float()))
    return torch.stack(outs)


@pytest.mark.parametrize("T,H,window", [(49152, 6, 640), (49152, 6, 1408), (98304, 3, 1280)])
def test_attention_at_training_size(T, H, window):
    from flash_attn import flash_attn_varlen_func
    from modded_nanogpt_b200.ops import fused
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn(T, H, 128, device="cuda", generator=g).to(BF) for _ in range(3))
    cu, starts = _packed(T, seed=T + window, cap=4096 if T > 49152 else 2048, slots=256 if T > 49152 else 128)
    scale, max_len = 0.11, 4096
    bounds = fused.doc_bounds(cu, T)
    w = torch.randn(T, H, 128, device="cuda", generator=g).to(BF)
    res = {}
    for name in ("ours", "fa2"):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        if name == "ours":
            o = fused.attention(qq, kk, vv, cu, window, scale, max_len, bounds)
        else:
            o = flash_attn_varlen_func(qq, kk, vv, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max_len, max_seqlen_k=max_len,
                                       causal=True, softmax_scale=scale, window_size=(window, 0))
        (o.float() * w.float()).sum().backward()
        res[name] = (o.detach(), qq.grad, kk.grad, vv.grad)
    fused.check_status()
    for a, b, n in zip(res["ours"], res["fa2"], ("out", "dq", "dk", "dv")):
        assert _rel(a, b) < 1.5e-2, (n, _rel(a, b))
        assert (a.float() - b.float()).abs().max() < 0.08 * b.float().abs().max() + 2e-2, n
    # rows where a wrong boundary block would show: first rows of documents, the rows before them, rows whose window
    # starts exactly at a tile edge or one off, the first and last rows of the batch
    ds = bounds[0].long()
    st = starts[1:40]
    cand = torch.cat([st, st - 1, st + 1, st + window, st + window + 1, st + window - 1,
                      torch.tensor([0, 1, 127, 128, 129, window, window + 1, T - 1, T - 2, T - 129], device="cuda")])
    rows = cand[(cand >= 0) & (cand < T)].unique()
    want = _dense_rows(q, k, v, rows, ds, window, scale)
    got = res["ours"][0][rows].float()
    assert (got - want).abs().max() < 2e-2, (got - want).abs().max().item()


def test_attention_at_validation_size():
    """T = 262,144 tokens, window 2,560 (the final validation pass): forward only, spot rows against the dense oracle."""
    from modded_nanogpt_b200.ops import fused
    T, H, window, scale = 262144, 6, 2560, 0.09
    g = torch.Generator(device="cuda").manual_seed(2)
    q, k, v = (torch.randn(T, H, 128, device="cuda", generator=g).to(BF) for _ in range(3))
    cu, starts = _packed(T, seed=7, mean=700, cap=100000, slots=1024)
    bounds = fused.doc_bounds(cu, T)
    with torch.no_grad():
        out = fused.attention(q, k, v, cu, window, scale, T, bounds)
    fused.check_status()
    st = starts[1:20]
    cand = torch.cat([st, st - 1, st + window, st + window + 1, torch.tensor([0, 2560, 2561, 200000, T - 1], device="cuda")])
    rows = cand[(cand >= 0) & (cand < T)].unique()
    want = _dense_rows(q, k, v, rows, bounds[0].long(), window, scale)
    assert (out[rows].float() - want).abs().max() < 2e-2
    assert torch.isfinite(out.float()).all()


def test_gemm_outputs_stay_inside_their_rows():
    """Canary rows before and after the output of the pair and single-CTA GEMMs (ragged M and N included)."""
    from modded_nanogpt_b200.ops import fused
    torch.manual_seed(0)
    for M, N, K, bn in ((49152, 768, 768, None), (1000, 328, 136, 128), (4096, 2304, 768, 512), (300, 50304, 768, 256)):
        a = torch.randn(M, K, device="cuda").to(BF)
        b = torch.randn(N, K, device="cuda").to(BF)
        pad = 8
        buf = torch.full((M + 2 * pad, N), 7.0, dtype=BF, device="cuda")
        out = buf[pad:pad + M]
        fused.gemm(a, b, out=out, bn=bn)
        assert _rel(out, a.float() @ b.float().T) < 6e-3
        assert (buf[:pad] == 7.0).all() and (buf[pad + M:] == 7.0).all(), (M, N, K, bn)
    fused.check_status()


def test_glue_kernels_at_training_size():
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.ops.glue import Term, lincomb, qkv_post
    T, D, H = 49152, 768, 6
    g = torch.Generator(device="cuda").manual_seed(4)
    xs = [torch.randn(T, D, device="cuda", generator=g).to(BF).requires_grad_(True) for _ in range(3)]
    gate = torch.randn(T, 8, device="cuda", generator=g).to(BF).requires_grad_(True)
    sc = torch.tensor([0.7], device="cuda", requires_grad=True)
    y = lincomb([Term(xs[0], scalar=sc), Term(xs[1], gate=gate, col=3), Term(xs[2], addc=1.0, gate=gate, col=5)])
    w = torch.randn(T, D, device="cuda", generator=g).to(BF)
    y.backward(w)
    xf = [x.detach().float().requires_grad_(True) for x in xs]
    gf, sf = gate.detach().float().requires_grad_(True), sc.detach().clone().requires_grad_(True)
    yr = sf * xf[0] + gf[:, 3:4] * xf[1] + (1.0 + gf[:, 5:6]) * xf[2]
    yr.backward(w.float())
    assert _rel(y, yr) < 6e-3
    for a, b in zip(xs, xf):
        assert _rel(a.grad, b.grad) < 8e-3
    assert _rel(gate.grad, gf.grad) < 1.5e-2 and abs(sc.grad.item() - sf.grad.item()) < 2e-3 * abs(sf.grad.item()) + 0.5
    # QK-norm + rotary + key offset + value add at full size against the plain formulas on a slice
    qkv = torch.randn(T, 3 * D, device="cuda", generator=g).to(BF)
    t = torch.arange(T, device="cuda", dtype=torch.float32)
    freq = (1 / 1024) ** torch.linspace(0, 1, 32, device="cuda")
    cos, sin = torch.outer(t, freq).cos().contiguous(), torch.outer(t, freq).sin().contiguous()
    q, k, v = qkv_post(qkv, cos, sin, None, None, None, H, False, True)
    sl = slice(T - 300, T)
    raw = qkv[T - 301:T].float().view(301, 3, H, 128)

    def normed(x):
        return (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)).to(BF).float()

    def rope(x, c, s):
        x1, x2 = x[..., 0:64:2], x[..., 1:64:2]
        out = x.clone()
        out[..., 0:64:2] = c[:, None, :] * x1 + s[:, None, :] * x2
        out[..., 1:64:2] = c[:, None, :] * x2 - s[:, None, :] * x1
        return out

    qn, kn = normed(raw[1:, 0]), normed(raw[:, 1])
    want_q = rope(qn, cos[sl], sin[sl])
    want_k = rope(kn[1:], cos[sl], sin[sl])
    want_k[..., 64:] = kn[:-1, :, 64:]                      # stationary half comes from the previous token
    assert _rel(q[sl], want_q) < 8e-3 and _rel(k[sl], want_k) < 8e-3 and torch.equal(v[sl].float(), raw[1:, 2])
    fused.check_status()
