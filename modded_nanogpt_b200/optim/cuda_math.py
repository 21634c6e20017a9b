"""Per-shard optimizer math on the sm_100a kernels.

`CudaMath` has the interface of `TorchMath` (normuon_direction / normuon_apply / adam /
transpose_add / transpose_copy).  Polar Express runs as batched tcgen05 GEMMs:
tall matrices iterate on A = X^T X (both operands read MN-major in place, no transposes),
wide ones on A = X X^T; B = b*A + c*A@A and X' = a*X + X@B (or B@X) use the GEMM's fused
alpha/beta epilogue, so one iteration is three launches (`train_gpt.py:202-253` needs a
Triton kernel per product plus cuBLAS baddbmm).

When `grad_ptrs` / `param_ptrs` (peer addresses over NVLink) are given, the first kernel sums
the gradient shard straight out of every rank's gradient buffer (reduce-scatter fused into the
momentum update) and the last kernel stores the new weights into every rank's parameter tensor
(all-gather fused into the weight update).
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from ..ops import fused
from ..ops import reference as ref
from ..ops.native import lib
from .normuon_adam import ParamConfig, TorchMath


SYMMETRIC_PE = os.environ.get("MNG_PE_SYMMETRIC", "1") != "0"


class CudaMath(TorchMath):
    def __init__(self, rank: int = 0):
        super().__init__(torch.bfloat16)
        self.rank = rank
        self._scratch: dict = {}

    def _buf(self, key, shape, dtype, device, zero: bool = False):
        t = self._scratch.get(key)
        if t is None or t.shape != torch.Size(shape) or t.dtype != dtype:
            t = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=device)
            self._scratch[key] = t
        return t

    # ------------------------------------------------------------------------------------------
    def polar_express(self, X: Tensor) -> Tensor:
        """X: [mats, rows, cols] bf16, already normalised.  Returns the orthogonalised X (bf16)."""
        mats, rows, cols = X.shape
        tall = rows > cols
        n = cols if tall else rows
        A = self._buf(("A", mats, n), (mats, n, n), torch.bfloat16, X.device)
        B = self._buf(("B", mats, n), (mats, n, n), torch.bfloat16, X.device)
        Y = self._buf(("Y", mats, rows, cols), (mats, rows, cols), torch.bfloat16, X.device)
        # A = X^T X (or X X^T) and B = b A + c A A are symmetric: from 3 x 3 tiles of 128 x 128 on, computing the upper
        # triangle and mirroring it (`triton_kernels.py:51-55`) is less work than the full product on the larger tiles
        sym = SYMMETRIC_PE and n % 128 == 0 and n >= 384
        for a, b, c in ref.POLAR_EXPRESS_COEFFS:
            if tall:
                fused.gemm(X, X, a_mn=True, b_mn=True, out=A, symmetric=sym)        # A = X^T X
            else:
                fused.gemm(X, X, out=A, symmetric=sym)                              # A = X X^T
            fused.gemm(A, A, b_mn=True, out=B, alpha=c, beta=b, cin=A, symmetric=sym)   # B = b A + c A A
            if tall:
                fused.gemm(X, B, b_mn=True, out=Y, alpha=1.0, beta=a, cin=X)        # X' = a X + X B
            else:
                fused.gemm(B, X, b_mn=True, out=Y, alpha=1.0, beta=a, cin=X)        # X' = a X + B X
            X, Y = Y, X
        return X

    @staticmethod
    def kernel_shapes(rows: int, cols: int) -> bool:
        """Matrices the tcgen05 / row kernels take: at least one 128-byte operand row per side and whole 16-byte
        vectors per matrix.  Smaller ones (the (8, 16) gate matrices of track 2) use the PyTorch statement of the
        same update; their cost is negligible."""
        return min(rows, cols) >= 64 and (rows * cols) % 256 == 0

    def normuon_direction(self, grad_chunk: Tensor, state: dict, cfg: ParamConfig, grad_ptrs=None, off: int = 0,
                          grad_mul: float = 1.0, grad_mc: int = 0) -> Tensor:
        C = lib()
        buf = state["momentum_buffer"]
        shape = buf.shape
        if not self.kernel_shapes(shape[-2], shape[-1]):
            assert grad_ptrs is None, "tiny matrices are reduced by the collective library, not by the fused kernels"
            return super().normuon_direction(grad_chunk, state, cfg)
        X = self._buf(("X", cfg.label), shape, torch.bfloat16, buf.device)
        ss = self._buf(("ss", cfg.label), (shape[0],), torch.float32, buf.device)
        if grad_ptrs is None:
            grad_chunk = grad_chunk.contiguous()
            grad_ptrs, off = [grad_chunk.data_ptr()], 0
        C.nesterov(grad_ptrs, self.rank, off, buf, X, ss, float(cfg.momentum), grad_mul, grad_mc)
        C.scale_by_norm(X, ss)
        return self.polar_express(X)

    def normuon_apply(self, p_slice: Tensor, state: dict, v: Tensor, cfg: ParamConfig, param_ptrs=None, off: int = 0,
                      param_mc: int = 0) -> None:
        C = lib()
        mats, rows, cols = v.shape
        if not self.kernel_shapes(rows, cols):
            assert param_ptrs is None
            return super().normuon_apply(p_slice, state, v, cfg)
        red_rows = rows >= cols
        eff_wd = cfg.wd_mul * cfg.weight_decay * cfg.lr
        # the per-matrix multipliers never change: they stay on the device; the step's learning rate is a launch argument
        mul = cfg.per_matrix_lr_mul or [1.0] * mats
        key = ("lr_mul", cfg.label)
        muls = self._scratch.get(key)
        if muls is None or muls[0] != tuple(mul):
            muls = (tuple(mul), torch.tensor(list(mul), dtype=torch.float32, device=v.device))
            self._scratch[key] = muls
        scratch = self._buf(("sc", cfg.label), (mats * (max(rows, cols) + 65),), torch.float32, v.device, zero=True)
        if param_ptrs is None:
            assert p_slice.is_contiguous()
            param_ptrs, off = [p_slice.data_ptr()], 0
        C.normuon_apply(param_ptrs, self.rank, off, state["mantissa"], v.contiguous(), state["second_momentum_buffer"],
                        scratch, red_rows, float(cfg.beta2), float(eff_wd), float(cfg.lr_mul * cfg.lr), muls[1], param_mc)

    def adam(self, p_slice: Tensor, grad: Tensor, state: dict, cfg: ParamConfig, step_size: float, eff_wd: float,
             grad_ptrs=None, param_ptrs=None, off: int = 0, grad_mul: float = 1.0, row_mask=None, row_elems: int = 0,
             grad_mc: int = 0, param_mc: int = 0) -> None:
        """`row_mask` ([ranks, rows] uint8, local) with `row_elems`: gradient rows a rank did not touch are not loaded."""
        n = p_slice.numel()
        is_f32 = p_slice.dtype == torch.float32
        vec = 4 if is_f32 else 8
        ok = (p_slice.is_cuda and n % vec == 0 and p_slice.is_contiguous()
              and (grad_ptrs is not None or (grad.is_contiguous() and grad.dtype == p_slice.dtype))
              and p_slice.dtype in (torch.float32, torch.bfloat16) and p_slice.data_ptr() % 16 == 0)
        if not ok:
            return super().adam(p_slice, grad, state, cfg, step_size, eff_wd)
        if grad_ptrs is None:
            grad_ptrs, param_ptrs, off = [grad.data_ptr()], [p_slice.data_ptr()], 0
        b1, b2 = cfg.adam_betas
        lib().adam(grad_ptrs, param_ptrs, self.rank, off, state["exp_avg"], state["exp_avg_sq"], n, is_f32, b1, b2, cfg.eps,
                   step_size, eff_wd, grad_mul, row_mask, row_elems, grad_mc, param_mc)

    def adam_batch(self, items, base_ptrs=None, grad_mul: float = 1.0) -> None:
        """One launch for many small replicated parameters.  `items`: (param, grad_or_None, state, cfg, step_size, eff_wd,
        p_off, g_off) with byte offsets from `base_ptrs` (every rank's address of the buffer that holds them); without
        `base_ptrs` the tensors' own addresses are used.  Each rank sums all ranks' gradients and updates its own copy."""
        p_offs, g_offs, ms, vs, ns, f32, hyper = [], [], [], [], [], [], []
        for p, grad, state, cfg, step_size, eff_wd, p_off, g_off in items:
            assert p.dtype in (torch.float32, torch.bfloat16) and p.is_contiguous()
            if base_ptrs is None:
                assert grad.is_contiguous() and grad.dtype == p.dtype
                p_off, g_off = p.data_ptr(), grad.data_ptr()
            p_offs.append(p_off); g_offs.append(g_off); ms.append(state["exp_avg"]); vs.append(state["exp_avg_sq"])
            ns.append(p.numel()); f32.append(int(p.dtype == torch.float32))
            hyper += [cfg.adam_betas[0], cfg.adam_betas[1], cfg.eps, step_size, eff_wd]
        lib().adam_small(base_ptrs or [0], self.rank if base_ptrs else 0, p_offs, g_offs, ms, vs, ns, f32, hyper, grad_mul)

    def transpose_add(self, src: Tensor, dst: Tensor) -> None:
        if src.dtype == torch.bfloat16 and src.is_contiguous() and dst.is_contiguous():
            lib().transpose(src, dst, True)
        else:
            super().transpose_add(src, dst)

    def transpose_copy(self, src: Tensor, dst: Tensor) -> None:
        if src.dtype == torch.bfloat16 and src.is_contiguous() and dst.is_contiguous():
            lib().transpose(src, dst, False)
        else:
            super().transpose_copy(src, dst)
