"""Plain-PyTorch restatement of every fused op.

These functions are (a) the oracle that the CUDA kernels are tested against, (b) the CPU/gloo
execution path, and (c) the fallback for shapes a kernel does not cover.  They follow the
reference's rounding points where those matter for parity (bf16 storage of the softcap
sigmoid, bf16 ReLU^2, bf16 Polar Express operands); citations are to the reference files.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor


def rms_norm(x: Tensor) -> Tensor:
    """Parameter-free RMSNorm over the last dim (`train_gpt.py:952-953`)."""
    return F.rms_norm(x, (x.size(-1),))


# --------------------------------------------------------------------------------------
# attention


def doc_ids_from_cu(cu_seqlens: Tensor, T: int) -> Tensor:
    """Document index of every position given padded cumulative lengths [0, e1, ..., T, T, ...]."""
    pos = torch.arange(T, device=cu_seqlens.device)
    return torch.searchsorted(cu_seqlens[1:].to(torch.int64).contiguous(), pos, right=True)


def attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, window: int, scale: float,
                     chunk: int = 2048) -> Tensor:
    """Causal sliding-window attention over packed documents.  q,k,v: [T,H,D].  Query i sees
    keys j with i-window <= j <= i in the same document (flash-attn `window_size=(W,0)`,
    `train_gpt.py:1139-1141`).  Dense math in fp32, chunked over queries."""
    T, H, D = q.shape
    doc = doc_ids_from_cu(cu_seqlens, T)
    out = torch.empty_like(q)
    qf, kf, vf = q.float(), k.float(), v.float()
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        lo = max(0, s - window)
        qi = torch.arange(s, e, device=q.device)[:, None]
        kj = torch.arange(lo, e, device=q.device)[None, :]
        mask = (kj <= qi) & (kj >= qi - window) & (doc[s:e, None] == doc[None, lo:e])
        sc = torch.einsum("qhd,khd->hqk", qf[s:e], kf[lo:e]) * scale
        sc = sc.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s:e] = torch.einsum("hqk,khd->qhd", p, vf[lo:e]).to(q.dtype)
    return out


def dc_correction(base: Tensor, q: Tensor, k: Tensor, v: Tensor, w1: Tensor, w2: Tensor, cu_seqlens: Tensor,
                  scale: float, window: int = 112, chunk: int = 1024) -> Tensor:
    """Dynamically-composable-MHA correction (`dc_triton_kernels.py:252-440`).
    P_h[t,:] = softmax over the last `window` same-document keys (self included) of scale*q_h.k_h;
    a[t,:] = sum_h w1[t,h] P_h[t,:];  out_h[t] = base_h[t] + w2[t,h] * (a[t,:] @ V_h).
    base,q,k,v: [T,H,D]; w1,w2: [T,H]."""
    T, H, D = q.shape
    doc = doc_ids_from_cu(cu_seqlens, T)
    out = torch.empty_like(base)
    qf, kf, vf = q.float(), k.float(), v.float()
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        lo = max(0, s - window + 1)
        qi = torch.arange(s, e, device=q.device)[:, None]
        kj = torch.arange(lo, e, device=q.device)[None, :]
        mask = (kj <= qi) & (qi - kj < window) & (doc[s:e, None] == doc[None, lo:e])
        sc = torch.einsum("qhd,khd->hqk", qf[s:e], kf[lo:e]) * scale
        p = torch.softmax(sc.masked_fill(~mask[None], float("-inf")), dim=-1)
        a = torch.einsum("hqk,qh->qk", p, w1[s:e].float())
        corr = torch.einsum("qk,khd->qhd", a, vf[lo:e]) * w2[s:e].float()[:, :, None]
        out[s:e] = (base[s:e].float() + corr).to(base.dtype)
    return out


# --------------------------------------------------------------------------------------
# MLP


def relu2_mlp(x: Tensor, w_fc: Tensor, w_proj: Tensor) -> Tensor:
    """relu(x @ w_fc.T)^2 @ w_proj with both weights stored (hidden, dim)
    (`triton_kernels.py:667-729`, bf16 branch)."""
    h = F.relu(F.linear(x, w_fc.type_as(x))).square()
    return h @ w_proj.type_as(x)


E4M3_MAX = 448.0


def quant_e4m3(x: Tensor, scale) -> Tensor:
    """Round x/scale to e4m3 (saturating) and return it de-quantised in x's dtype; emulates the
    fp8 storage the kernels use so CPU tests see the same rounding."""
    y = (x.float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()
    return y


def relu2_mlp_fp8(x: Tensor, w_fc: Tensor, w_proj: Tensor, act_scale: Tensor | float | None = None):
    """Emulation of the FP8 MLP forward (`train_gpt.py:1643-1665`, `triton_kernels.py:442-471`):
    per-tensor amax scales for x and w_fc, fp32 accumulate, round to bf16, relu, square in bf16;
    down projection on e4m3 `post` (saturating at 448) with a supplied activation scale."""
    xa = x.detach().abs().amax().clamp(min=1e-12).float()
    wa = w_fc.detach().abs().amax().clamp(min=1e-12).float()
    xq = quant_e4m3(x, xa / E4M3_MAX)
    wq = quant_e4m3(w_fc, wa / E4M3_MAX)
    pre = (xq @ wq.T) * (xa / E4M3_MAX) * (wa / E4M3_MAX)
    post = F.relu(pre.to(torch.bfloat16)).square()
    if act_scale is None:
        return post @ w_proj.to(torch.bfloat16), post
    pa = w_proj.detach().abs().amax().clamp(min=1e-12).float()
    pq = quant_e4m3(post, act_scale)
    wpq = quant_e4m3(w_proj, pa / E4M3_MAX)
    return ((pq @ wpq) * act_scale * (pa / E4M3_MAX)).to(torch.bfloat16), post


# --------------------------------------------------------------------------------------
# softcapped cross-entropy with multi-token and prefix-token terms


def softcap(logits: Tensor, a: float, b: float, c: float) -> Tensor:
    return a * torch.sigmoid((logits + b) / c)


def softcap_ce_loss_rows(z: Tensor, targets: Tensor, row0: int, mtp_weights: Tensor, prefix_targets: Tensor | None,
                         prefix_weight: Tensor | float, n_rows_total: int) -> Tensor:
    """Per-row loss  sum_k w_k (lse - z[target_{i+k}]) + w_p (lse - z[prefix_i])  for the rows
    [row0, row0+len(z)) of a batch of `n_rows_total` rows (`triton_kernels.py:1071-1090`).
    `targets`/`prefix_targets` index the whole batch; targets past its end are dropped."""
    n, V = z.shape
    lse = torch.logsumexp(z, dim=-1)
    loss = torch.zeros(n, dtype=z.dtype, device=z.device)
    rows = torch.arange(row0, row0 + n, device=z.device)
    for kk in range(mtp_weights.numel()):
        idx = rows + kk
        ok = idx < n_rows_total
        tgt = targets[idx.clamp(max=n_rows_total - 1)]
        ok = ok & (tgt >= 0) & (tgt < V)
        zt = z.gather(1, tgt.clamp(0, V - 1)[:, None])[:, 0]
        loss = loss + torch.where(ok, mtp_weights[kk] * (lse - zt), torch.zeros_like(lse))
    if prefix_targets is not None:
        pt = prefix_targets[rows]
        ok = (pt >= 0) & (pt < V)
        zt = z.gather(1, pt.clamp(0, V - 1)[:, None])[:, 0]
        loss = loss + torch.where(ok, prefix_weight * (lse - zt), torch.zeros_like(lse))
    return loss


class _SoftcapCE(torch.autograd.Function):
    """Chunked lm_head + softcap CE: logits are never held for more than `chunk` rows.
    Backward honours `grad_output` (unlike the reference's fused op, `triton_kernels.py:1256`)."""

    @staticmethod
    def forward(ctx, x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c, chunk):
        T = x.shape[0]
        losses = torch.empty(T, dtype=torch.float32, device=x.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            z = softcap((x[s:e] @ w.type_as(x)).float(), a, b, c)
            losses[s:e] = softcap_ce_loss_rows(z, targets, s, mtp_weights, prefix_targets, prefix_weight, T)
        ctx.save_for_backward(x, w, targets, mtp_weights, prefix_targets, prefix_weight)
        ctx.cfg = (a, b, c, chunk)
        return losses

    @staticmethod
    def backward(ctx, g):
        x, w, targets, mtp_weights, prefix_targets, prefix_weight = ctx.saved_tensors
        a, b, c, chunk = ctx.cfg
        T = x.shape[0]
        dx = torch.empty_like(x)
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            with torch.enable_grad():
                xs = x[s:e].detach().requires_grad_(True)
                ws = w.detach().requires_grad_(True)
                z = softcap((xs @ ws.type_as(xs)).float(), a, b, c)
                l = softcap_ce_loss_rows(z, targets, s, mtp_weights, prefix_targets, prefix_weight, T)
                gx, gw = torch.autograd.grad(l, (xs, ws), g[s:e].to(l.dtype))
            dx[s:e] = gx
            dw += gw.float()
        return dx, dw.to(w.dtype), None, None, None, None, None, None, None, None


def softcap_ce(x: Tensor, w: Tensor, targets: Tensor, mtp_weights: Tensor, prefix_targets: Tensor | None,
               prefix_weight: Tensor | None, a: float = 23.0, b: float = 5.0, c: float = 7.5, chunk: int = 4096) -> Tensor:
    """x [T,D], w [D,V] (transposed storage) -> per-token loss fp32 [T]."""
    if prefix_weight is None:
        prefix_weight = torch.zeros((), dtype=torch.float32, device=x.device)
    prefix_weight = prefix_weight.reshape(()).float()
    if prefix_targets is None:
        prefix_targets = torch.full((x.shape[0],), -1, dtype=torch.int64, device=x.device)
    return _SoftcapCE.apply(x, w, targets, mtp_weights.float(), prefix_targets, prefix_weight, a, b, c, chunk)


def softcap_ce_eval(x: Tensor, w: Tensor, targets: Tensor, a: float = 23.0, b: float = 5.0, c: float = 7.5,
                    chunk: int = 8192) -> Tensor:
    """Evaluation loss: bf16 logits, softcap in the activation dtype, fp32 cross entropy
    (`train_gpt.py:1689-1692`)."""
    T = x.shape[0]
    out = torch.empty(T, dtype=torch.float32, device=x.device)
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        z = a * torch.sigmoid(((x[s:e] @ w.type_as(x)) + b) / c)
        out[s:e] = F.cross_entropy(z.float(), targets[s:e], reduction="none")
    return out


# --------------------------------------------------------------------------------------
# Polar Express

POLAR_EXPRESS_COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]


def polar_express(g: Tensor, dtype=torch.bfloat16) -> Tensor:
    """Five fixed-coefficient Newton-Schulz-type iterations on a batch of matrices
    (`train_gpt.py:194-253`): normalise by ||X||_F*1.02+1e-6; tall matrices iterate on
    A = X^T X with right multiplication, wide ones on A = X X^T with left multiplication.
    X, A, B are held in `dtype` with higher-precision accumulation inside each product."""
    X = g.to(dtype)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * (1 + 2e-2) + 1e-6)
    tall = g.size(-2) > g.size(-1)
    for a, b, c in POLAR_EXPRESS_COEFFS:
        if tall:
            A = X.mT @ X
            B = b * A + c * (A @ A)
            X = a * X + X @ B
        else:
            A = X @ X.mT
            B = b * A + c * (A @ A)
            X = a * X + B @ X
    return X


def nesterov_momentum_(grad_fp32: Tensor, buf: Tensor, momentum: float) -> Tensor:
    """buf <- lerp(buf, g, 1-mu); g <- lerp(g, buf, mu), both fp32, in place (`train_gpt.py:190-192`)."""
    buf.lerp_(grad_fp32, 1 - momentum)
    return grad_fp32.lerp_(buf, momentum)


def normuon_variance_reduction_(v: Tensor, second_momentum: Tensor, beta2: float, red_dim: int) -> Tensor:
    """NorMuon second-moment normalisation keeping the Frobenius norm (`train_gpt.py:934-947`)."""
    v_mean = v.float().square().mean(dim=red_dim, keepdim=True)
    n = v.size(red_dim)
    v_norm = v_mean.sum(dim=(-2, -1), keepdim=True).mul_(n).sqrt_()
    second_momentum.lerp_(v_mean.to(second_momentum.dtype), 1 - beta2)
    step = second_momentum.clamp_min(1e-10).rsqrt_()
    v_norm_new = ((v_mean * n) * step.float().square()).sum(dim=(-2, -1), keepdim=True).sqrt_()
    final = step * (v_norm / v_norm_new.clamp_min_(1e-10))
    return v.mul_(final.type_as(v))


def cautious_update_mantissa_(p_bf16: Tensor, mantissa: Tensor, upd: Tensor, eff_wd: float, eff_lr: float) -> None:
    """p(fp32 = bf16 bits << 16 | mantissa) <- p - p*[upd*p >= 0]*wd*lr - upd*lr, then split back by
    truncation (`train_gpt.py:914-932`).  p_bf16: bf16 tensor, mantissa: uint16 tensor, in place."""
    if p_bf16.dtype == torch.float32:     # fp32 parameters are their own master copy
        g = upd.float()
        mask = (g * p_bf16) >= 0
        p_bf16.copy_(p_bf16 - (p_bf16 * mask * (eff_wd * eff_lr)) - g * eff_lr)
        return
    hi = p_bf16.view(torch.int16).to(torch.int32) << 16
    lo = mantissa.view(torch.int16).to(torch.int32) & 0xFFFF
    p = (hi | lo).view(torch.float32)
    g = upd.float()
    mask = (g * p) >= 0
    wd = torch.tensor(eff_wd, dtype=torch.float32, device=p.device)
    lr = torch.tensor(eff_lr, dtype=torch.float32, device=p.device)
    p_new = p - (p * mask * wd * lr) - (g * lr)
    raw = p_new.view(torch.int32)
    p_bf16.view(torch.int16).copy_((raw >> 16).to(torch.int16))
    mantissa.view(torch.int16).copy_((raw & 0xFFFF).to(torch.int16))


def adam_update_(p: Tensor, g: Tensor, exp_avg: Tensor, exp_avg_sq: Tensor, beta1: float, beta2: float, eps: float,
                 step_size: float, eff_wd: float) -> None:
    """Adam with cautious weight decay, no master copy (`train_gpt.py:854-864`)."""
    g = g.float()
    exp_avg.mul_(beta1).add_(g, alpha=1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    step_t = torch.tensor(step_size, dtype=torch.float32, device=p.device)
    wd_t = torch.tensor(eff_wd, dtype=torch.float32, device=p.device)
    update = exp_avg.div(exp_avg_sq.sqrt().add_(eps)).mul_(step_t)
    pf = p.float()
    mask = (update * pf) > 0
    update.add_(pf * mask * wd_t)
    p.add_(update, alpha=-1.0)


def gelu(x: Tensor) -> Tensor:
    return F.gelu(x)
