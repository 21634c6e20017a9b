"""tcgen05 attention forward against the fp32 dense reference (documents, windows, ragged tails) and its
log-sum-exp / backward hand-off to the FlashAttention-2 backward."""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _case(T, H, docs, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(T, H, 128, device="cuda", generator=g).to(BF) for _ in range(3))
    cu = torch.full((64,), T, dtype=torch.int32, device="cuda")
    cu[:len(docs)] = torch.tensor(docs, dtype=torch.int32)
    return q, k, v, cu


@pytest.mark.parametrize("T,H,docs,window", [(256, 2, [0], 1024), (1024, 6, [0, 300, 650, 800], 384), (1152, 3, [0, 1, 130, 1000], 128),
                                             (2048, 6, [0, 5, 700, 1500, 2047], 640), (1000, 2, [0, 444], 200)])
def test_attention_forward_matches_reference(T, H, docs, window):
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.ops import reference as ref
    q, k, v, cu = _case(T, H, docs)
    scale = 0.12
    out = fused.attention(q, k, v, cu, window, scale, 2048)
    fused.check_status()
    want = ref.attention_varlen(q, k, v, cu, window, scale)
    assert _rel(out, want) < 1e-2, _rel(out, want)
    assert torch.equal(out, fused.attention(q, k, v, cu, window, scale, 2048))


@pytest.mark.parametrize("T,H,docs,window", [(256, 1, [0], 1024), (1024, 6, [0, 300, 650, 800], 384), (1152, 3, [0, 1, 130, 1000], 128),
                                             (2048, 2, [0, 5, 700, 1500, 2047], 640)])
def test_attention_backward_matches_reference(T, H, docs, window):
    from modded_nanogpt_b200.ops import fused
    from modded_nanogpt_b200.ops import reference as ref
    q, k, v, cu = _case(T, H, docs, seed=5)
    w = torch.randn(T, H, 128, device="cuda")
    got, want = [], []
    for impl, dst in ((fused.attention, got), (ref.attention_varlen, want)):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = impl(qq, kk, vv, cu, window, 0.12, 2048) if impl is fused.attention else impl(qq, kk, vv, cu, window, 0.12)
        (o.float() * w).sum().backward()
        dst.extend([qq.grad, kk.grad, vv.grad])
    fused.check_status()
    for a, b, n in zip(got, want, ("dq", "dk", "dv")):
        assert _rel(a, b) < 2e-2, (n, _rel(a, b))


def test_attention_lse_and_backward_match_flash_attn():
    from flash_attn import flash_attn_varlen_func
    from modded_nanogpt_b200.ops import fused
    T, H, window, scale = 2048, 6, 384, 0.1
    q, k, v, cu = _case(T, H, [0, 300, 650, 1800], seed=3)
    ds = fused.doc_starts(cu, T)
    assert torch.equal(fused.doc_bounds(cu, T)[1], torch.tensor([300, 650, 1800, T], device="cuda", dtype=torch.int32)[
        torch.bucketize(torch.arange(T, device="cuda"), torch.tensor([300, 650, 1800], device="cuda"), right=True)])
    out, lse = fused._C().attn_fwd(q, k, v, ds, window, scale)
    qf, kf, vf = q.float(), k.float(), v.float()
    i = torch.arange(T, device="cuda")
    mask = (i[None, :] <= i[:, None]) & (i[None, :] >= i[:, None] - window) & (ds[:, None].long() <= i[None, :])
    s = torch.einsum("qhd,khd->hqk", qf, kf) * scale
    want_lse = torch.logsumexp(s.masked_fill(~mask[None], float("-inf")), dim=-1)
    assert (lse - want_lse).abs().max() < 2e-2
    grads = {}
    for name in ("ours", "fa2"):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        if name == "ours":
            o = fused.attention(qq, kk, vv, cu, window, scale, 2048)
        else:
            o = flash_attn_varlen_func(qq, kk, vv, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=2048, max_seqlen_k=2048,
                                       causal=True, softmax_scale=scale, window_size=(window, 0))
        (o.float() * torch.linspace(-1, 1, 128, device="cuda")).sum().backward()
        grads[name] = (o.detach(), qq.grad, kk.grad, vv.grad)
    for a, b, n in zip(grads["ours"], grads["fa2"], ("out", "dq", "dk", "dv")):
        assert _rel(a, b) < 2e-2, (n, _rel(a, b))
    fused.check_status()
