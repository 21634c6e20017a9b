"""CTA-pair (cta_group::2) tcgen05 GEMM against fp32 PyTorch references: every operand layout and
epilogue the framework launches on it, plus ragged shapes that exercise the out-of-range tile edges."""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF, F8, F8B = torch.bfloat16, torch.float8_e4m3fn, torch.float8_e5m2
PAIR = 512


@pytest.fixture(scope="module")
def fused():
    from modded_nanogpt_b200.ops import fused as f
    return f


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K,batch", [(256, 256, 64, 1), (512, 768, 768, 1), (2048, 3072, 768, 1), (300, 328, 136, 2),
                                         (128, 50304, 768, 1), (9728, 1024, 256, 1)])
def test_pair_bf16_kk(fused, M, N, K, batch):
    torch.manual_seed(0)
    shp = (batch,) if batch > 1 else ()
    a = torch.randn(*shp, M, K, device="cuda").to(BF)
    b = torch.randn(*shp, N, K, device="cuda").to(BF)
    out = fused.gemm(a, b, bn=PAIR)
    fused.check_status()
    assert _rel(out, a.float() @ b.float().mT) < 5e-3
    assert torch.equal(out, fused.gemm(a, b, bn=PAIR))           # run-to-run determinism


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True)])
def test_pair_bf16_mn_major(fused, a_mn, b_mn):
    torch.manual_seed(1)
    M, N, K = 768, 1280, 640
    a = torch.randn(K, M, device="cuda").to(BF) if a_mn else torch.randn(M, K, device="cuda").to(BF)
    b = torch.randn(K, N, device="cuda").to(BF) if b_mn else torch.randn(N, K, device="cuda").to(BF)
    out = fused.gemm(a, b, a_mn=a_mn, b_mn=b_mn, bn=PAIR)
    fused.check_status()
    A = a.float().T if a_mn else a.float()
    B = b.float() if b_mn else b.float().T
    assert _rel(out, A @ B) < 5e-3


def test_pair_fp8_variants(fused):
    torch.manual_seed(3)
    M, N, K = 512, 896, 512
    a, b = torch.randn(M, K, device="cuda").to(F8), torch.randn(N, K, device="cuda").to(F8)
    rs, cs = torch.rand(M, device="cuda") + 0.5, torch.rand(N, device="cuda") + 0.5
    out = fused.gemm(a, b, row_scale=rs, col_scale=cs, bn=PAIR)
    assert _rel(out, (a.float() @ b.float().T) * rs[:, None] * cs[None, :]) < 5e-3
    a5 = torch.randn(M, K, device="cuda").to(F8B)
    assert _rel(fused.gemm(a5, b, alpha=0.25, bn=PAIR), 0.25 * (a5.float() @ b.float().T)) < 5e-3
    bmn = torch.randn(K, N, device="cuda").to(F8)
    assert _rel(fused.gemm(a, bmn, b_mn=True, bn=PAIR), a.float() @ bmn.float()) < 5e-3
    amn, b5 = torch.randn(K, M, device="cuda").to(F8), torch.randn(K, N, device="cuda").to(F8B)
    out = fused.gemm(amn, b5, a_mn=True, b_mn=True, bn=PAIR)
    assert _rel(out, amn.float().T @ b5.float()) < 5e-3
    fused.check_status()


def test_pair_relu2_dpre_and_accumulate(fused):
    torch.manual_seed(4)
    T, D, H = 640, 256, 1024
    x8 = torch.randn(T, D, device="cuda").to(F8)
    w8 = (torch.randn(H, D, device="cuda") * 0.3).to(F8)
    rs, cs = torch.rand(T, device="cuda") * 0.1 + 0.05, torch.rand(H, device="cuda") * 0.1 + 0.05
    act = torch.tensor([0.02], device="cuda")
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    post = torch.empty(T, H, dtype=BF, device="cuda")
    post8 = torch.empty(T, H, dtype=F8, device="cuda")
    fused.gemm(x8, w8, out=post, epilogue=fused.EPI_RELU2, row_scale=rs, col_scale=cs, out8=post8, act_scale=act,
               amax_bits=amax, bn=PAIR)
    pre = ((x8.float() @ w8.float().T) * rs[:, None] * cs[None, :]).to(BF)
    ref = torch.relu(pre).square()
    assert _rel(post, ref) < 1e-2
    assert _rel(post8, (ref.float() / 0.02).clamp(max=448).to(F8)) < 3e-2
    assert abs(amax.view(torch.float32).item() - post.float().max().item()) < 1e-6
    g = torch.randn(T, D, device="cuda").to(BF)
    w2 = (torch.randn(H, D, device="cuda") * 0.1).to(BF)
    dpre = fused.gemm(g, w2, epilogue=fused.EPI_DPRE, cin=post, bn=PAIR)
    assert _rel(dpre, 2 * (g.float() @ w2.float().T).to(BF).float() * post.float().sqrt()) < 1e-2
    acc = torch.randn(T, H, device="cuda").to(BF)
    want = acc.float() + 0.5 * (g.float() @ w2.float().T)
    fused.gemm(g, w2, out=acc, cin=acc, alpha=0.5, beta=1.0, bn=PAIR)      # accumulation in place
    assert _rel(acc, want) < 5e-3
    post_b = torch.empty(T, H, dtype=BF, device="cuda")          # bf16 operands, no fp8 copy
    fused.gemm(g, w2, out=post_b, epilogue=fused.EPI_RELU2, bn=PAIR)
    assert _rel(post_b, torch.relu((g.float() @ w2.float().T).to(BF)).square()) < 1e-2
    fused.check_status()
