"""lm_head GEMM fused with the soft-capped cross entropy (no logits in memory) against the fp32 statement of the
loss and against the unfused kernels (logits GEMM + stand-alone loss kernel) on the same quantised operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu

BF = torch.bfloat16
A, B, C = 23.0, 5.0, 7.5
XS, WS = 100 / 448, 1.6 / 448


@pytest.fixture(scope="module")
def fused():
    from modded_nanogpt_b200.ops import fused, native
    assert native.available(required=True)
    return fused


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _inputs(T, V, D=768, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, D, device="cuda", generator=g)
    x = (x * torch.rsqrt(x.square().mean(-1, keepdim=True))).to(BF)
    w = (torch.randn(D, V, device="cuda", generator=g) * 0.02).to(BF)
    tg = torch.randint(0, V, (T,), device="cuda", generator=g)
    pt = torch.randint(-1, V, (T,), device="cuda", generator=g)
    return x, w, tg, pt


@pytest.mark.parametrize("T,V,n_predict,prefix", [(256, 50304, 3, True), (512, 4096, 1, False), (768, 50304, 2, True)])
def test_fused_statistics_and_gradient_kernels(fused, T, V, n_predict, prefix):
    from modded_nanogpt_b200.ops import native, reference as ref
    lib = native.lib()
    x, w, tg, pt = _inputs(T, V, seed=T)
    tg[5] = tg[6]                                   # two predictions of row 5 land on one column
    pt[7] = tg[7]                                   # prefix target equal to the next-token target
    pt[9] = -1
    tg[T - 1] = V - 1                               # last column of the last (half-empty for V = 50304) tile
    tg[0] = 0
    mtp = torch.tensor([1.0, 0.5, 0.25][:n_predict], device="cuda")
    pw = torch.tensor([0.3], device="cuda") if prefix else None
    ptg = pt if prefix else None
    gm = 32.0
    x8, _ = lib.quant_static_dual(x, XS, True, False)
    w8, wT8 = lib.quant_static_dual(w, WS, True, True)
    assert torch.equal(wT8.view(torch.uint8), w8.view(torch.uint8).T.contiguous())
    assert torch.equal(x8.view(torch.uint8), fused.quant_static_e4m3(x, XS).view(torch.uint8))
    losses, dl = lib.lmhead_ce_fused(x8, wT8, XS * WS, tg, mtp, ptg, pw, A, B, C, gm)
    # oracle on the very same quantised operands, in fp32
    lg = ((x8.float() @ w8.float()) * (XS * WS)).requires_grad_(True)
    z = ref.softcap(lg, A, B, C)
    want = ref.softcap_ce_loss_rows(z, tg, 0, mtp, ptg, pw[0] if prefix else 0.0, T)
    (want.sum() * gm).backward()
    # the sigmoid is evaluated in bf16 pairs (the reference stores it as bf16): same tolerance as the stand-alone kernel
    assert torch.allclose(losses, want, atol=3e-2, rtol=2e-3), (losses - want).abs().max().item()
    assert _rel(dl, lg.grad) < 9e-2                                     # e5m2 output: two mantissa bits, rms rounding error 7 %
    cols = torch.stack([tg, torch.roll(tg, -1), pt.clamp_min(0)], 1)   # the columns that got a fix-up
    got, exp = dl.float().gather(1, cols), lg.grad.gather(1, cols)
    assert torch.allclose(got, exp, rtol=0.13, atol=2e-5 * gm), (got - exp).abs().max().item()
    # every byte that is not a target column equals what the stand-alone loss kernel writes from fp32-accurate logits
    # within one e5m2 step: compare magnitudes through the dequantised values
    far = (dl.float() - lg.grad).abs() <= 0.13 * lg.grad.abs() + 2e-5 * gm
    assert far.float().mean().item() > 0.9995
    # deterministic
    l2, d2 = lib.lmhead_ce_fused(x8, wT8, XS * WS, tg, mtp, ptg, pw, A, B, C, gm)
    assert torch.equal(l2, losses) and torch.equal(d2.view(torch.uint8), dl.view(torch.uint8))
    fused.check_status()


def test_fused_path_matches_unfused_path_at_training_size(fused, monkeypatch):
    """T = 49,152 rows x 50,304 columns: loss, dx and dW of the fused path against the unfused kernels."""
    T, V = 49152, 50304
    x, w, tg, pt = _inputs(T, V, seed=3)
    mtp = torch.tensor([1.0, 0.5, 0.25], device="cuda")
    pw = torch.tensor([0.25], device="cuda")

    def run(flag):
        monkeypatch.setattr(fused, "CE_FUSED", flag)
        xs, ws = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        loss = fused.softcap_ce(xs, ws, tg, mtp, pt, pw, A, B, C, grad_scale=0.125, fp8=True)
        peak = torch.cuda.max_memory_allocated() - base
        (loss.sum() * 0.125).backward()
        return loss.detach(), xs.grad, ws.grad, peak

    l1, dx1, dw1, peak1 = run(True)
    l0, dx0, dw0, peak0 = run(False)
    assert torch.allclose(l1, l0, rtol=3e-3, atol=5e-2), (l1 - l0).abs().max().item()
    assert _rel(dx1, dx0) < 3e-2 and _rel(dw1, dw0) < 3e-2, (_rel(dx1, dx0), _rel(dw1, dw0))
    assert peak0 - peak1 > 4.5e9, (peak0, peak1)                       # the 4.9 GB of bf16 logits are gone
    fused.check_status()
