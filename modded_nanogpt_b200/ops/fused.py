"""Python face of the sm_100a kernels: tensor plumbing and autograd Functions.

Forward/backward pairs here mirror the reference's fused ops:
* `relu2_mlp`  <-> `FusedLinearReLUSquareFunction` (`triton_kernels.py:667-729`): FP8 forward with a
  fused ReLU^2 epilogue, bf16 backward without ever storing the pre-activation;
* `softcap_ce` <-> `FusedSoftcappedCrossEntropy` (`triton_kernels.py:1208-1292`): FP8 lm_head GEMM,
  one-pass loss + gradient kernel, FP8 backward GEMMs - here without any transpose copies, because
  the tcgen05 descriptors read MN-major operands in place;
* `rms_norm` with an optional fused row-scaled e4m3 copy (removes the global amax pass of
  `train_gpt.py:1645-1646`).
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from . import native

EPI_STORE, EPI_RELU2, EPI_DPRE = 0, 1, 2
NUM_SMS = 148
PAIR_GEMM = os.environ.get("MNG_GEMM_PAIR", "1") != "0"


def _C():
    return native.lib()


def check_status(like: Tensor | None = None) -> int:
    """Reads the device status word (0 = no kernel reported a timed-out wait); synchronises."""
    like = like if like is not None else torch.empty(1, device="cuda")
    code = int(_C().status_tensor(like).item())
    if code:
        raise RuntimeError(f"a kernel reported error status {code} (bounded wait expired or bad argument)")
    return code


# --------------------------------------------------------------------------------------------------
# GEMM


def gemm(a: Tensor, b: Tensor, *, a_mn: bool = False, b_mn: bool = False, out: Tensor | None = None,
         out_dtype=torch.bfloat16, bn: int | None = None, alpha: float = 1.0, beta: float = 0.0, cin: Tensor | None = None,
         alpha_t: Tensor | None = None, row_scale: Tensor | None = None, col_scale: Tensor | None = None,
         epilogue: int = EPI_STORE, out8: Tensor | None = None, act_scale: Tensor | None = None,
         amax_bits: Tensor | None = None, max_ctas: int = 0, alpha2_t: Tensor | None = None,
         beta_t: Tensor | None = None, dot_out: Tensor | None = None, symmetric: bool = False) -> Tensor:
    """out = epilogue(A @ B^T) on the tcgen05 kernel.  A is [.., M, K] (or [.., K, M] with a_mn),
    B is [.., N, K] (or [.., K, N] with b_mn); fp32 accumulation.  `alpha_t`, `alpha2_t`, `beta_t`: one-element fp32
    device tensors multiplied into alpha / beta (`beta_t` alone means beta = 1 * beta_t); `dot_out` (EPI_DPRE):
    one-element fp32 accumulator that receives sum(acc * cin).  `symmetric`: the caller knows the product (and `cin`)
    to be symmetric; only the upper-triangular 128 x 128 tiles are computed and mirrored (M == N, a multiple of 128)."""
    if beta_t is not None and beta == 0.0:
        beta = 1.0
    M = a.shape[-1] if a_mn else a.shape[-2]
    N = b.shape[-1] if b_mn else b.shape[-2]
    if out is None:
        out = torch.empty((*a.shape[:-2], M, N), dtype=out_dtype, device=a.device)
    if symmetric:
        bn = 128
    if bn is None:
        batch = a.shape[0] if a.dim() == 3 else 1
        tiles256 = -(-M // 128) * -(-N // 256) * batch
        bn = 256 if (tiles256 >= NUM_SMS or N > 4096) and epilogue == EPI_STORE else 128
        if epilogue != EPI_STORE:
            bn = 256
        # CTA pairs (256 x 256 tiles, TMA output path) once there is at least one tile per pair of SMs;
        # the C side falls back to the 128 x 256 kernel for outputs it cannot describe by a tensor map
        if PAIR_GEMM and out.dtype == torch.bfloat16 and -(-M // 256) * -(-N // 256) * batch >= NUM_SMS // 2:
            bn = 512
    _C().gemm(a, b, out, a_mn, b_mn, epilogue, bn, alpha, beta, cin, alpha_t, row_scale, col_scale, out8, act_scale,
              amax_bits, max_ctas, alpha2_t, beta_t, dot_out, symmetric)
    return out


# --------------------------------------------------------------------------------------------------
# RMSNorm


class _RmsNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        y, _, _, rstd = _C().rmsnorm_fwd(xc, True, False, True)
        ctx.save_for_backward(xc, rstd)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x, rstd = ctx.saved_tensors
        return _C().rmsnorm_bwd(x, dy.contiguous().view(x.shape), rstd, None)


def rms_norm(x: Tensor) -> Tensor:
    if x.shape[-1] % 256 != 0 or x.shape[-1] > 4096:
        from . import reference
        return reference.rms_norm(x)
    return _RmsNorm.apply(x)


def _norm_bwd_plus(x: Tensor, dy: Tensor | None, rstd: Tensor, dres: Tensor | None) -> Tensor | None:
    """Gradient of a tensor that feeds both a norm (gradient `dy` of the normalised output) and a residual path
    (gradient `dres`), formed in the norm-backward pass itself."""
    if dy is None:
        return dres
    dy = dy.contiguous().view(x.shape)
    if dres is None:
        return _C().rmsnorm_bwd(x, dy, rstd, None)
    return _C().rmsnorm_bwd_add(x, dy, rstd, dres.contiguous().view(x.shape))


class _RmsNormFork(torch.autograd.Function):
    """(norm(x), x): the second output carries x on to the residual path, so that both gradients of x meet in this
    node and are summed inside the norm-backward kernel instead of by a separate elementwise pass."""

    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        y, _, _, rstd = _C().rmsnorm_fwd(xc, True, False, True)
        ctx.save_for_backward(xc, rstd)
        ctx.set_materialize_grads(False)
        return y.view(x.shape), x

    @staticmethod
    def backward(ctx, dy, dres):
        x, rstd = ctx.saved_tensors
        return _norm_bwd_plus(x, dy, rstd, dres)


def rms_norm_fork(x: Tensor):
    """Returns (norm(x), x'), where x' equals x and is what the residual path should consume."""
    if x.shape[-1] % 256 != 0 or x.shape[-1] > 4096 or not x.is_cuda:
        return rms_norm(x), x
    return _RmsNormFork.apply(x)


# --------------------------------------------------------------------------------------------------
# ReLU^2 MLP


class MlpFp8State:
    """e4m3 copies of the MLP bank with one scale per weight row, plus the delayed activation
    scale of every layer's hidden activations (amax of the previous step x 1.8 / 448)."""

    def __init__(self, bank: Tensor):
        Lp, _, hid, dim = bank.shape
        dev = bank.device
        self.fc8 = torch.empty(Lp, hid, dim, dtype=torch.float8_e4m3fn, device=dev)
        self.fc_scale = torch.empty(Lp, hid, dtype=torch.float32, device=dev)
        self.projT8 = torch.empty(Lp, dim, hid, dtype=torch.float8_e4m3fn, device=dev)
        self.projT_scale = torch.empty(Lp, dim, dtype=torch.float32, device=dev)
        self.act_scale = torch.ones(Lp, dtype=torch.float32, device=dev)
        self.amax_bits = torch.zeros(Lp, dtype=torch.int32, device=dev)
        self._scratch = torch.empty(Lp * max(hid, dim), dtype=torch.int32, device=dev)

    def layer(self, i: int):
        return (self.fc8[i], self.fc_scale[i], self.projT8[i], self.projT_scale[i], self.act_scale[i:i + 1],
                self.amax_bits[i:i + 1])


@torch.no_grad()
def quantize_mlp_weights(bank: Tensor, state: MlpFp8State | None, used_scales: Tensor, next_scales: Tensor,
                         bootstrap: bool) -> MlpFp8State:
    if state is None:
        state = MlpFp8State(bank)
    # one call for all layers: row-scaled e4m3 of the up projections, column-scaled transposed e4m3 of the down
    # projections, delayed activation scales from the amax seen since the last refresh (`train_gpt.py:1670-1675`)
    # and the per-layer maxima of the down-projection scales that keep the reference's state_dict buffers meaningful
    _C().mlp_weight_refresh(bank, state.fc8, state.fc_scale, state.projT8, state.projT_scale, state._scratch,
                            state.act_scale, state.amax_bits, used_scales, next_scales, bool(bootstrap))
    return state


class _NormRelu2Mlp(torch.autograd.Function):
    """out = relu(norm(x) @ W1^T)^2 @ W2 with W1, W2 stored (hidden, dim).

    With `mix = (a, b)` (one-element fp32 device tensors) the result is a * x + b * MLP(norm(x)): the residual mix
    of `train_gpt.py:1665` runs in the down-projection's epilogue (x arrives as the addend tile), and in the backward
    b scales the incoming gradient inside the two GEMMs that consume it, d b = <g, MLP> falls out of the
    pre-activation-gradient epilogue (sum of acc * post), a * g joins the norm backward as a scaled addend and
    d a = <g, x> is summed by that same kernel - no separate mix kernel and no stored MLP output in either direction."""

    @staticmethod
    def forward(ctx, x, w_fc, w_proj, fp8, g_fc=None, g_proj=None, fork=False, a_t=None, b_t=None):
        C = _C()
        T, D = x.shape
        ctx.grad_views = (g_fc, g_proj)
        ctx.fork = fork
        ctx.set_materialize_grads(False)
        hid = w_fc.shape[0]
        xc = x.contiguous()
        mix = {}
        ctx.mix_meta = None
        if a_t is not None:
            a32, b32 = a_t.detach().reshape(1).float(), b_t.detach().reshape(1).float()
            mix = dict(alpha2_t=b32, beta_t=a32, cin=xc)
            ctx.mix_meta = ((a_t.dtype, a_t.shape), (b_t.dtype, b_t.shape))
        post = torch.empty(T, hid, dtype=torch.bfloat16, device=x.device)
        if fp8 is not None:
            fc8, fc_scale, projT8, projT_scale, act_scale, amax_bits = fp8
            y, y8, y_scale, rstd = C.rmsnorm_fwd(xc, True, True, True)
            post8 = torch.empty(T, hid, dtype=torch.float8_e4m3fn, device=x.device)
            gemm(y8, fc8, out=post, epilogue=EPI_RELU2, row_scale=y_scale, col_scale=fc_scale, out8=post8,
                 act_scale=act_scale, amax_bits=amax_bits)
            out = gemm(post8, projT8, col_scale=projT_scale, alpha_t=act_scale, **mix)
        else:
            y, _, _, rstd = C.rmsnorm_fwd(xc, True, False, True)
            gemm(y, w_fc, out=post, epilogue=EPI_RELU2)
            out = gemm(post, w_proj, b_mn=True, **mix)
        if a_t is not None:
            ctx.save_for_backward(xc, rstd, y, post, w_fc, w_proj, a32, b32)
            return out
        ctx.save_for_backward(xc, rstd, y, post, w_fc, w_proj)
        return (out, x) if fork else out

    @staticmethod
    def backward(ctx, g, dres=None):
        C = _C()
        nothing = (None,) * 8
        if ctx.mix_meta is not None:
            x, rstd, y, post, w_fc, w_proj, a32, b32 = ctx.saved_tensors
            sc = dict(alpha_t=b32)
            dab = torch.zeros(2, dtype=torch.float32, device=x.device)
        else:
            x, rstd, y, post, w_fc, w_proj = ctx.saved_tensors
            sc, dab = {}, None
            if g is None:                                     # only the carried-on x was used
                return (dres,) + nothing
        g = g.contiguous()
        g_fc, g_proj = ctx.grad_views
        # weight gradients: either returned to autograd, or accumulated by the GEMM epilogue (beta = 1)
        # straight into the caller's slices of the parameter-bank gradient
        acc = dict(beta=1.0) if g_fc is not None else {}
        d_proj = gemm(post, g, a_mn=True, b_mn=True, out=g_proj, cin=g_proj, **acc, **sc)    # post^T g      (hid, dim)
        dpre = gemm(g, w_proj, epilogue=EPI_DPRE, cin=post, **sc,                            # 2 (g W2^T) sqrt(post)
                    **(dict(dot_out=dab[1:2]) if dab is not None else {}))
        d_fc = gemm(dpre, y, a_mn=True, b_mn=True, out=g_fc, cin=g_fc, **acc)                # dpre^T y      (hid, dim)
        dy = gemm(dpre, w_fc, b_mn=True)                                                     # dpre W1       (T, dim)
        if dab is not None:
            dx = C.rmsnorm_bwd_add_scaled(x, dy, rstd, g, a32, dab[0:1])
            (adt, ashp), (bdt, bshp) = ctx.mix_meta
            dmix = (dab[0].to(adt).reshape(ashp), dab[1].to(bdt).reshape(bshp))
        else:
            dx = _norm_bwd_plus(x, dy, rstd, dres)
            dmix = (None, None)
        if g_fc is not None:
            return (dx, None, None, None, None, None, None) + dmix
        return (dx, d_fc, d_proj, None, None, None, None) + dmix


def norm_relu2_mlp(x: Tensor, w_fc: Tensor, w_proj: Tensor, fp8_state=None, grad_views=None, fork: bool = False):
    """`grad_views = (g_fc, g_proj)`: slices of the bank gradient the weight gradients are accumulated
    into by the backward GEMMs (the weights then receive no autograd gradient).
    `fork`: also return x for the residual path; its gradient is then added inside the norm-backward kernel."""
    if grad_views is not None:
        return _NormRelu2Mlp.apply(x, w_fc.detach(), w_proj.detach(), fp8_state, grad_views[0], grad_views[1], fork)
    return _NormRelu2Mlp.apply(x, w_fc, w_proj, fp8_state, None, None, fork)


def _split_k(rows: int, tiles: int) -> int:
    """Number of token-dimension splits (1, 2, 4 or 8) for a weight-gradient GEMM with `tiles` 128 x 128 output
    tiles: the fewest splits whose cost - waves over the SMs, each 1/s long - is within 5 % of the best."""
    cost = {s: -(-tiles * s // NUM_SMS) / s for s in (1, 2, 4, 8) if rows % (s * 64) == 0}
    if not cost:
        return 1
    best = min(cost.values())
    return min(s for s, c in cost.items() if c <= 1.05 * best)


class _BankLinear(torch.autograd.Function):
    """y = x @ (lam * W)^T on the tcgen05 GEMM, for a weight W [N, K] whose rows belong to one or two slices of
    parameter banks (`train_gpt.py:1103`, `:1161`: the QKV and O projections).  lam is a device scalar applied in the
    GEMM epilogue, so no scaled copy of W is made.  Backward: dx = lam * dy W; the weight-gradient product dy^T x
    runs split along the tokens (a batched GEMM with fp32 outputs) and `bank_grad_acc` folds the splits, adds
    lam * dy^T x into the bank-gradient slices and returns d lam = <dy^T x, W>."""

    @staticmethod
    def forward(ctx, x, lam, w, *grad_views):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        lam32 = lam.detach().reshape(()).float() if lam.dtype != torch.float32 else lam.detach().reshape(())
        ctx.save_for_backward(x2, lam32, w)
        ctx.grad_views = grad_views
        ctx.lam_meta = (lam.dtype, lam.shape)
        y = gemm(x2, w, alpha_t=lam32)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, lam32, w = ctx.saved_tensors
        N, K = w.shape
        dy2 = dy.reshape(-1, N)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        T = dy2.shape[0]
        dx = gemm(dy2, w, b_mn=True, alpha_t=lam32)                           # [T, N] x [N, K]
        S = _split_k(T, -(-N // 128) * -(-K // 128))
        parts = torch.empty(S, N, K, dtype=torch.float32, device=dy.device)
        gemm(dy2.view(S, T // S, N), x2.view(S, T // S, K), a_mn=True, b_mn=True, out=parts, bn=128)
        gv = ctx.grad_views
        dlam = _C().bank_grad_acc(parts, w, lam32, gv[0], gv[1] if len(gv) > 1 else None)
        dtype, shape = ctx.lam_meta
        return (dx.view(*dy.shape[:-1], K), dlam.to(dtype).reshape(shape), None) + (None,) * len(gv)


class _QkvProj(torch.autograd.Function):
    """q, k, v = post(x @ (lam * W)^T): the QKV projection with QK RMSNorm, rotary, partial key offset and the gated
    value-embedding add (`train_gpt.py:1103-1116`) done in the GEMM's epilogue (csrc/epi_qkv.cuh), so the raw
    [T, 3*H*128] projection is neither written nor kept.  Backward: the post-processing is undone from its outputs
    (`qkv_post_bwd_from_out`), then the projection's backward as in `_BankLinear`."""

    @staticmethod
    def forward(ctx, x, lam, w, cos_t, sin_t, ve, vgate, H, paired, key_offset, *grad_views):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        lam32 = lam.detach().reshape(()).float() if lam.dtype != torch.float32 else lam.detach().reshape(())
        vec = None if ve is None else ve.contiguous()
        q, k, v, rq, rk, k_last = _C().qkv_proj(x2, w, lam32, cos_t, sin_t, vec, vgate, H, paired, key_offset)
        ctx.save_for_backward(x2, lam32, w, q, k, rq, rk, k_last, cos_t, sin_t, vec, vgate)
        ctx.grad_views = grad_views
        ctx.cfg = (H, paired, key_offset, lam.dtype, lam.shape, x.shape)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2, lam32, w, q, k, rq, rk, k_last, cos_t, sin_t, ve, vgate = ctx.saved_tensors
        H, paired, key_offset, ldt, lshape, xshape = ctx.cfg
        need_dve = ve is not None and ctx.needs_input_grad[5]
        need_dvg = vgate is not None and ctx.needs_input_grad[6]
        dy2, dve, dvg = _C().qkv_post_bwd_from_out(q, k, k_last, cos_t, sin_t, rq, rk, dq.contiguous(), dk.contiguous(),
                                                   dv.contiguous(), ve, vgate, H, paired, key_offset, need_dve, need_dvg)
        N, K = w.shape
        T = dy2.shape[0]
        dx = gemm(dy2, w, b_mn=True, alpha_t=lam32)
        S = _split_k(T, -(-N // 128) * -(-K // 128))
        parts = torch.empty(S, N, K, dtype=torch.float32, device=dy2.device)
        gemm(dy2.view(S, T // S, N), x2.view(S, T // S, K), a_mn=True, b_mn=True, out=parts, bn=128)
        gv = ctx.grad_views
        dlam = _C().bank_grad_acc(parts, w, lam32, gv[0], gv[1] if len(gv) > 1 else None)
        if dve is not None:
            dve = dve.view(ve.shape)
        return (dx.view(xshape), dlam.to(ldt).reshape(lshape), None, None, None, dve, dvg, None, None, None) + (None,) * len(gv)


def qkv_proj(x: Tensor, lam: Tensor, w: Tensor, grad_views: list, cos_t: Tensor, sin_t: Tensor, ve: Tensor | None,
             vgate: Tensor | None, H: int, paired: bool, key_offset: bool):
    """Returns q, k, v [T, H, 128].  `w` [3*H*128, K] contiguous (rows: q heads, k heads, v heads)."""
    return _QkvProj.apply(x, lam, w.detach(), cos_t, sin_t, ve, vgate, H, paired, key_offset, *grad_views)


def qkv_proj_supported(x: Tensor, w: Tensor, H: int) -> bool:
    T = x.numel() // x.shape[-1]
    return (QKV_FUSED and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and T >= 256 and T % 64 == 0
            and w.shape[0] == 3 * H * 128 and (3 * H * 128) % 256 == 0 and w.shape[1] % 64 == 0)


QKV_FUSED = os.environ.get("MNG_QKV_FUSED", "1") != "0"      # 0: projection, then the separate post-processing kernel


def bank_linear(x: Tensor, lam: Tensor, w: Tensor, grad_views: list) -> Tensor:
    """`w`: contiguous [N, K] bf16 weight (no autograd); `grad_views`: one or two contiguous bf16 gradient slices
    that together cover w's rows in order."""
    assert len(grad_views) in (1, 2) and w.is_contiguous()
    return _BankLinear.apply(x, lam, w.detach(), *grad_views)


def linear_scaled(x: Tensor, w: Tensor, lam: Tensor | None = None) -> Tensor:
    """Inference-side x @ (lam * w)^T on the same GEMM (no autograd)."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    y = gemm(x2, w.contiguous(), alpha_t=None if lam is None else lam.detach().reshape(()).float())
    return y.view(*x.shape[:-1], w.shape[0])


class _GateMlp(torch.autograd.Function):
    """out = (gelu(x W1^T) W2^T + b2) * scale for the 64-wide gate / MUDD MLPs (`train_gpt.py:1465-1467`,
    `:1601-1610`, `:1677-1680`).  x W1^T and the two products of its backward run on the tcgen05 GEMM (the weight
    gradient split along the tokens); the 64 -> n tail is one kernel per direction (csrc/gatemlp.cu)."""

    @staticmethod
    def forward(ctx, x, w1, w2, b2, scale_t, scale_c):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        w1c, w2c, b2c = w1.contiguous(), w2.contiguous(), b2.contiguous()
        st = None if scale_t is None else scale_t.detach().reshape(()).float()
        pre = gemm(x2, w1c, bn=128)                                              # [T, 64]
        out = _C().gate_tail_fwd(pre, w2c, b2c, st, scale_c)
        ctx.save_for_backward(x2, pre, w1c, w2c, b2c, st)
        ctx.cfg = (scale_c, x.shape, None if scale_t is None else (scale_t.dtype, scale_t.shape))
        return out.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dout):
        x2, pre, w1, w2, b2, st = ctx.saved_tensors
        scale_c, xshape, smeta = ctx.cfg
        T, K = x2.shape
        d2 = dout.reshape(T, -1)
        if d2.stride(1) != 1:
            d2 = d2.contiguous()
        dpre, dw2, db2, dscale = _C().gate_tail_bwd(pre, w2, b2, st, scale_c, d2)
        dx = gemm(dpre, w1, b_mn=True) if ctx.needs_input_grad[0] else None          # [T, 64] x [64, K]
        S = max(s for s in (1, 2, 4, 8, 16, 32) if T % (s * 64) == 0)
        parts = torch.empty(S, 64, K, dtype=torch.float32, device=x2.device)
        gemm(dpre.view(S, T // S, 64), x2.view(S, T // S, K), a_mn=True, b_mn=True, out=parts, bn=128)
        dw1 = parts.sum(0).to(w1.dtype)
        ds = None if smeta is None else dscale.to(smeta[0]).reshape(smeta[1])
        return (None if dx is None else dx.view(xshape)), dw1, dw2, db2, ds, None


def gate_mlp(x: Tensor, w1: Tensor, w2: Tensor, b2: Tensor, scale) -> Tensor:
    """`scale`: a Python number or a one-element fp32 tensor (then it receives a gradient)."""
    if isinstance(scale, Tensor):
        return _GateMlp.apply(x, w1, w2, b2, scale, 1.0)
    return _GateMlp.apply(x, w1, w2, b2, None, float(scale))


def gate_mlp_supported(x: Tensor, w1: Tensor, w2: Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and w1.shape[0] == 64
            and w2.shape[0] <= 48 and x.shape[-1] % 64 == 0 and x.numel() // x.shape[-1] >= 128)


def norm_relu2_mlp_mix(x: Tensor, w_fc: Tensor, w_proj: Tensor, a: Tensor, b: Tensor, fp8_state=None, grad_views=None):
    """a * x + b * relu(norm(x) W1^T)^2 W2 with the mix fused into the down projection (see `_NormRelu2Mlp`);
    a, b: one-element fp32 tensors (parameters or views of parameters)."""
    if grad_views is not None:
        return _NormRelu2Mlp.apply(x, w_fc.detach(), w_proj.detach(), fp8_state, grad_views[0], grad_views[1], False, a, b)
    return _NormRelu2Mlp.apply(x, w_fc, w_proj, fp8_state, None, None, False, a, b)


def relu2_mlp(x_normed: Tensor, w_fc: Tensor, w_proj: Tensor, fp8_state=None) -> Tensor:
    """MLP on an already normalised input (used when the caller needs the normed tensor too)."""
    post = gemm(x_normed.contiguous(), w_fc, epilogue=EPI_RELU2,
                out=torch.empty(x_normed.shape[0], w_fc.shape[0], dtype=torch.bfloat16, device=x_normed.device))
    return gemm(post, w_proj, b_mn=True)


# --------------------------------------------------------------------------------------------------
# lm_head + softcapped cross entropy


def quant_static_e4m3(x: Tensor, scale: float) -> Tensor:
    """Saturating e4m3 cast of x/scale (per-tensor static scale)."""
    return (x.float() * (1.0 / scale)).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)


class _Fp8LinearT(torch.autograd.Function):
    """y = x @ w for a weight stored (in, out), with static per-tensor scales: the reference's `nanogpt::mm_t`
    op (`train_gpt.py:68-162`).  Forward in e4m3 x e4m3, backward with the incoming gradient in e5m2:
    grad_x = g w^T in bf16, grad_w = x^T g accumulated and returned in fp32."""

    @staticmethod
    def forward(ctx, x, w, x_s, w_s, grad_s):
        x2 = x.reshape(-1, x.shape[-1])
        x8, w8 = quant_static_e4m3(x2, x_s), quant_static_e4m3(w, w_s)
        ctx.save_for_backward(x8, w8)
        ctx.cfg = (x_s, w_s, grad_s, x.shape)
        return gemm(x8, w8, b_mn=True, alpha=x_s * w_s).view(*x.shape[:-1], w.shape[1])

    @staticmethod
    def backward(ctx, g):
        x8, w8 = ctx.saved_tensors
        x_s, w_s, grad_s, xshape = ctx.cfg
        g2 = g.reshape(-1, g.shape[-1])
        g8 = (g2.float() * (1.0 / grad_s)).to(torch.float8_e5m2)
        gx = gemm(g8, w8, alpha=grad_s * w_s)                                         # [T, out] x [in, out]^T
        if x8.shape[0] % 64 == 0 and x8.shape[1] % 64 == 0:
            xt = _C().transpose_u8(x8)
        else:
            xt = x8.view(torch.uint8).t().contiguous().view(x8.dtype)
        gw = gemm(xt, g8, b_mn=True, alpha=x_s * grad_s, out_dtype=torch.float32)     # [in, T] x [T, out]
        return gx.view(xshape), gw, None, None, None


def fp8_linear_t(x: Tensor, w: Tensor, x_s: float, w_s: float, grad_s: float) -> Tensor:
    return _Fp8LinearT.apply(x, w, float(x_s), float(w_s), float(grad_s))


class _SoftcapCE(torch.autograd.Function):
    """x [T,D] bf16 (normed), w [D,V] bf16.  FP8 path: static per-tensor scales x_s, w_s and a
    gradient scale grad_s, as in the reference (`train_gpt.py:1225`)."""

    @staticmethod
    def forward(ctx, x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c, grad_scale, fp8, scales):
        C = _C()
        x_s, w_s, grad_s = scales
        if fp8 and CE_FUSED and _ce_fusable(x, w, mtp_weights):
            # no [T, V] logits in memory: the lm_head GEMM runs twice with the loss statistics and then the gradient
            # formed in its epilogues (csrc/epi_ce.cuh); the weight is quantised once, as stored and transposed
            x8, xT8 = C.quant_static_dual(x, x_s, True, True)
            w8, wT8 = C.quant_static_dual(w.contiguous(), w_s, True, True)
            g_s = grad_s * grad_scale
            losses, dl = C.lmhead_ce_fused(x8, wT8, x_s * w_s, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c,
                                           grad_scale / g_s)
            ctx.save_for_backward(xT8, w8, dl)
            ctx.cfg = (True, x_s, w_s, g_s)
            ctx.x_is_t = True
            return losses
        ctx.x_is_t = False
        if fp8:
            if x.shape[0] % 64 == 0 and x.shape[1] % 64 == 0 and w.shape[1] % 64 == 0:
                # one pass each: e4m3 of x as stored (logits GEMM) and transposed (weight-gradient GEMM), e4m3 of w
                x8, xs8 = C.quant_static_dual(x, x_s, True, True)
                w8, _ = C.quant_static_dual(w.contiguous(), w_s, True, False)
                ctx.x_is_t = True
            else:
                x8 = xs8 = quant_static_e4m3(x, x_s)
                w8 = quant_static_e4m3(w, w_s)
            logits = gemm(x8, w8, b_mn=True, alpha=x_s * w_s)
            g_s = grad_s * grad_scale
            losses, dl = C.softcap_ce(logits, targets, mtp_weights, prefix_targets, prefix_weight, True, a, b, c,
                                      grad_scale / g_s)
            ctx.save_for_backward(xs8, w8, dl)
            ctx.cfg = (True, x_s, w_s, g_s)
        else:
            logits = gemm(x.contiguous(), w, b_mn=True)
            losses, dl = C.softcap_ce(logits, targets, mtp_weights, prefix_targets, prefix_weight, False, a, b, c, grad_scale)
            ctx.save_for_backward(x, w, dl)
            ctx.cfg = (False, 1.0, 1.0, 1.0)
        return losses

    @staticmethod
    def backward(ctx, grad_out):
        xq, wq, dl = ctx.saved_tensors
        fp8, x_s, w_s, g_s = ctx.cfg
        # dl already carries grad_scale: the caller reduces the losses with .sum() * grad_scale
        dx = gemm(dl, wq, alpha=g_s * w_s)                                           # dl W^T          (T, D)
        if fp8:
            # 8-bit MN-major operands run at about 60 % of the K-major rate on both sides: transposing the small
            # [T, D] activation (38 MB) first makes A K-major and the GEMM 1.6x faster
            if ctx.x_is_t:
                xt = xq
            elif xq.shape[0] % 64 == 0 and xq.shape[1] % 64 == 0:
                xt = _C().transpose_u8(xq)
            else:
                xt = xq.view(torch.uint8).t().contiguous().view(xq.dtype)
            dw = gemm(xt, dl, b_mn=True, alpha=x_s * g_s)                            # x^T dl          (D, V)
        else:
            dw = gemm(xq, dl, a_mn=True, b_mn=True, alpha=x_s * g_s)
        return dx, dw, None, None, None, None, None, None, None, None, None, None


# 1: form loss and gradient in the epilogues of the lm_head GEMM (no [T, V] logits in memory: 4.9 GB less at T = 49,152).
# Off by default: the two fused passes measure 1.9 + 2.8 ms on B200 against 2.0 + 1.9 ms for the logits GEMM plus the
# stand-alone loss kernel (their epilogues are bound by instruction issue with two epilogue warps per scheduler).
CE_FUSED = os.environ.get("MNG_CE_FUSED", "0") == "1"


def _ce_fusable(x: Tensor, w: Tensor, mtp_weights: Tensor) -> bool:
    return (x.shape[0] % 64 == 0 and x.shape[1] % 64 == 0 and w.shape[1] % 64 == 0 and x.shape[0] >= 256
            and mtp_weights.numel() <= 3)


def softcap_ce(x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c, grad_scale=1.0, fp8=True,
               scales=(100 / 448, 1.6 / 448, 0.75 / 448)) -> Tensor:
    if prefix_weight is not None:
        prefix_weight = prefix_weight.reshape(1).float()
    return _SoftcapCE.apply(x.contiguous(), w, targets.contiguous(), mtp_weights.float().contiguous(), prefix_targets,
                            prefix_weight, a, b, c, grad_scale, fp8, scales)


def softcap_ce_eval(x: Tensor, w: Tensor, targets: Tensor, a: float, b: float, c: float, chunk: int = 16384) -> Tensor:
    """Evaluation loss per token (`train_gpt.py:1689-1692`): bf16 logits on the own GEMM, chunk by chunk, and the
    streaming loss kernel with a single target per row (its gradient output is scratch here)."""
    C = _C()
    T = x.shape[0]
    out = torch.empty(T, dtype=torch.float32, device=x.device)
    one = torch.ones(1, dtype=torch.float32, device=x.device)
    x, targets = x.contiguous(), targets.contiguous()
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        logits = gemm(x[s:e], w, b_mn=True)
        out[s:e] = C.softcap_ce(logits, targets[s:e], one, None, None, False, a, b, c, 1.0)[0]
    return out


# --------------------------------------------------------------------------------------------------
# attention / DC: tcgen05 kernels are selected here once available for the shape


def doc_bounds(cu_seqlens: Tensor, T: int) -> Tensor:
    """int32 [2, T]: for every token the index of the first token of its document and of the next
    document (cu_seqlens is padded with T)."""
    pos = torch.arange(T, device=cu_seqlens.device, dtype=cu_seqlens.dtype)
    nxt = torch.searchsorted(cu_seqlens, pos, right=True)
    return torch.stack([cu_seqlens[nxt - 1], cu_seqlens[nxt.clamp_(max=cu_seqlens.numel() - 1)]]).to(torch.int32)


def doc_starts(cu_seqlens: Tensor, T: int) -> Tensor:
    return doc_bounds(cu_seqlens, T)[0]


class _Attention(torch.autograd.Function):
    """Forward and backward on the tcgen05 kernels (csrc/attn_sm100.cu).  `MNG_ATTN_BWD=fa2` routes the
    backward to FlashAttention-2's varlen kernel (library call) with the forward's output and log-sum-exp."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, bounds, window, scale, max_len):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        out, lse = _C().attn_fwd(q, k, v, bounds[0], window, scale)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens, bounds)
        ctx.cfg = (window, scale, max_len)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu, bounds = ctx.saved_tensors
        window, scale, max_len = ctx.cfg
        if ATTN_BWD_KERNEL and q.shape[0] % 4 == 0:
            dq, dk, dv = _C().attn_bwd(dout.contiguous(), q, k, v, out, lse, bounds[0], bounds[1], window, scale)
        else:
            from flash_attn.flash_attn_interface import _wrapped_flash_attn_varlen_backward as fa_bwd
            dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
            fa_bwd(dout.contiguous(), q, k, v, out, lse, dq, dk, dv, cu, cu, max_len, max_len, 0.0, scale, True, window, 0,
                   0.0, None, False, rng_state=None)
        return dq, dk, dv, None, None, None, None, None


ATTN_BWD_KERNEL = os.environ.get("MNG_ATTN_BWD", "own") != "fa2"
ATTN_KERNEL = os.environ.get("MNG_ATTN", "1") != "0"


def attention_supported(q: Tensor, window: int) -> bool:
    return ATTN_KERNEL and q.dim() == 3 and q.shape[-1] == 128 and q.dtype == torch.bfloat16 and q.shape[0] >= 128


def attention(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, window: int, scale: float, max_len: int,
              bounds: Tensor | None = None) -> Tensor:
    """`bounds` = doc_bounds(cu_seqlens, T), computed here when the caller does not share one across layers."""
    if bounds is None:
        bounds = doc_bounds(cu_seqlens, q.shape[0])
    return _Attention.apply(q, k, v, cu_seqlens, bounds, int(window), float(scale), int(max_len))

