"""Dynamically-composable-MHA correction on the tcgen05 GEMM.

out_h[t] = base_h[t] + w2[t,h] * (a[t,:] @ V_h),  a[t,:] = sum_h w1[t,h] * softmax_window(q_h k_h)[t,:]
(`dc_triton_kernels.py:252-440`).  Queries are processed in blocks of 128; the keys a block can
see (window <= 128, same document) lie in the 256 rows [128*blk - 128, 128*blk + 128), so scores
and value products are batched GEMMs over overlapping 256-row windows of K and V (strided views of
buffers padded with 128 zero rows in front, no gather).  Per head:

  forward   S_h = scale * Q_blk K_win^T            (128 x 256 per block, fp32)
            [dc_mix_fwd: mask, softmax, cross-head mix -> P_h, a]
            out_h = base_h + w2_h (.) (a V_win)    (row-scaled epilogue, beta = 1)
  backward  dM_h = dOut_h V_win^T;  [dc_mix_bwd -> dS_h, g_w1, g_w2]
            dQ_h = dS_h K_win;  dK_win += dS_h^T Q_blk;  dV_win += a^T (w2_h (.) dOut_h)
The window partial gradients of K and V are folded back with one shifted add.  No atomics, so the
backward is deterministic (the reference's is not, `dc_triton_kernels.py:543-549`).
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import fused
from .native import lib
from .reference import doc_ids_from_cu

BLK, WIN = 128, 256


def _windows(xp: Tensor, h: int, nblk: int, H: int, Dh: int) -> Tensor:
    """[nblk, 256, Dh] overlapping views of head h of a front-padded [T+128, H, Dh] buffer."""
    ld = H * Dh
    return xp.as_strided((nblk, WIN, Dh), (BLK * ld, ld, 1), xp.storage_offset() + h * Dh)


def _blocks(x: Tensor, h: int, nblk: int, H: int, Dh: int) -> Tensor:
    """[nblk, 128, Dh] views of head h of a [T, H, Dh] tensor."""
    ld = H * Dh
    return x.as_strided((nblk, BLK, Dh), (BLK * ld, ld, 1), x.storage_offset() + h * Dh)


def _pad_front(x: Tensor) -> Tensor:
    T, H, Dh = x.shape
    xp = torch.empty(T + BLK, H, Dh, dtype=x.dtype, device=x.device)
    xp[:BLK].zero_()
    xp[BLK:].copy_(x)
    return xp


def _fold(part: Tensor, T: int, H: int, Dh: int) -> Tensor:
    """part [H, nblk, 256, Dh]: window row j of block b is position 128*b - 128 + j.  Returns [T, H, Dh]."""
    nblk = T // BLK
    hi = part[:, :, BLK:]                                    # rows of the block itself
    lo = part[:, 1:, :BLK]                                   # rows that belong to the previous block
    out = hi.clone()
    out[:, :nblk - 1] += lo
    return out.permute(1, 2, 0, 3).reshape(T, H, Dh)


class _DC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, base, q, k, v, w1, w2, doc_start, scale, window):
        C = lib()
        T, H, Dh = q.shape
        nblk = T // BLK
        q, base = q.contiguous(), base.contiguous()
        kp, vp = _pad_front(k), _pad_front(v)
        S = torch.empty(H, nblk, BLK, WIN, dtype=torch.float32, device=q.device)
        for h in range(H):
            fused.gemm(_blocks(q, h, nblk, H, Dh), _windows(kp, h, nblk, H, Dh), out=S[h], alpha=scale, bn=256)
        P, a = C.dc_mix_fwd(S, w1, doc_start, window)
        del S
        out = torch.empty_like(base)
        w2t = w2.float().t().contiguous()                    # [H, T]
        for h in range(H):
            fused.gemm(a, _windows(vp, h, nblk, H, Dh), b_mn=True, out=_blocks(out, h, nblk, H, Dh),
                       cin=_blocks(base, h, nblk, H, Dh), beta=1.0, row_scale=w2t[h], bn=128)
        ctx.save_for_backward(q, kp, vp, P, a, w1, w2)
        ctx.cfg = (scale, T, H, Dh)
        return out

    @staticmethod
    def backward(ctx, dout):
        C = lib()
        q, kp, vp, P, a, w1, w2 = ctx.saved_tensors
        scale, T, H, Dh = ctx.cfg
        nblk = T // BLK
        dout = dout.contiguous()
        dM = torch.empty(H, nblk, BLK, WIN, dtype=torch.float32, device=q.device)
        for h in range(H):
            fused.gemm(_blocks(dout, h, nblk, H, Dh), _windows(vp, h, nblk, H, Dh), out=dM[h], bn=256)
        dS, g_w1, g_w2 = C.dc_mix_bwd(dM, P, a, w1, w2, scale)
        del dM
        doutw = (dout * w2[:, :, None]).contiguous()
        dq = torch.empty_like(q)
        dkp = torch.empty(H, nblk, WIN, Dh, dtype=torch.bfloat16, device=q.device)
        dvp = torch.empty(H, nblk, WIN, Dh, dtype=torch.bfloat16, device=q.device)
        for h in range(H):
            fused.gemm(dS[h], _windows(kp, h, nblk, H, Dh), b_mn=True, out=_blocks(dq, h, nblk, H, Dh), bn=128)
            fused.gemm(dS[h], _blocks(q, h, nblk, H, Dh), a_mn=True, b_mn=True, out=dkp[h], bn=128)
            fused.gemm(a, _blocks(doutw, h, nblk, H, Dh), a_mn=True, b_mn=True, out=dvp[h], bn=128)
        dk, dv = C.dc_fold(dkp), C.dc_fold(dvp)             # one pass each (`_fold` is the same in torch ops)
        return dout, dq, dk, dv, g_w1.to(w1.dtype), g_w2.to(w2.dtype), None, None, None


def supported(q: Tensor, window: int) -> bool:
    T, H, Dh = q.shape
    return q.is_cuda and q.dtype == torch.bfloat16 and T % BLK == 0 and Dh == 128 and window <= BLK and H <= 8


def dc_correction(base: Tensor, q: Tensor, k: Tensor, v: Tensor, w1: Tensor, w2: Tensor, cu_seqlens: Tensor, scale: float,
                  window: int = 112) -> Tensor:
    T = q.shape[0]
    doc = doc_ids_from_cu(cu_seqlens, T)
    doc_start = cu_seqlens.to(torch.int64)[doc].to(torch.int32).contiguous()
    return _DC.apply(base, q, k, v, w1.contiguous(), w2.contiguous(), doc_start, float(scale), int(window))
