"""User-facing functional ops.  Each chooses the sm_100a kernel (see `native.py`, `fused.py`)
or the PyTorch oracle (`reference.py`) per call via `ops.use_kernel`."""
from __future__ import annotations

import torch
from torch import Tensor

from . import reference as ref
from . import use_kernel


def rms_norm(x: Tensor) -> Tensor:
    if use_kernel("rms_norm", x) and x.dtype == torch.bfloat16:
        from . import fused
        return fused.rms_norm(x)
    return ref.rms_norm(x)


def attention(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, window: int, scale: float, max_len: int,
              doc_start: Tensor | None = None) -> Tensor:
    """Causal, document-masked sliding-window attention on packed sequences; q,k,v [T,H,D].
    `doc_start` (int32 [2, T] from `fused.doc_bounds`: first token of each token's document and of the next
    one) may be passed by callers that run several layers on the same packing."""
    if q.is_cuda and q.dtype == torch.bfloat16:
        if use_kernel("attention", q):
            from . import fused
            if fused.attention_supported(q, window):
                return fused.attention(q, k, v, cu_seqlens, window, scale, max_len, doc_start)
        from .library import flash_attention_varlen
        return flash_attention_varlen(q, k, v, cu_seqlens, window, scale, max_len)
    return ref.attention_varlen(q, k, v, cu_seqlens, window, scale)


def dc_correction(base, q, k, v, w1, w2, cu_seqlens, scale, window=112) -> Tensor:
    if use_kernel("dc", q) and q.dtype == torch.bfloat16:
        from . import dc
        if dc.supported(q, window):
            return dc.dc_correction(base, q, k, v, w1, w2, cu_seqlens, scale, window)
    return ref.dc_correction(base, q, k, v, w1, w2, cu_seqlens, scale, window)


def relu2_mlp(x: Tensor, w_fc: Tensor, w_proj: Tensor, fp8_state=None) -> Tensor:
    """relu(x w_fc^T)^2 w_proj.  With `fp8_state` (training on CUDA) the forward runs the
    row-scaled e4m3 tcgen05 kernels; backward is bf16."""
    if use_kernel("mlp", x) and x.dtype == torch.bfloat16:
        from . import fused
        return fused.relu2_mlp(x, w_fc, w_proj, fp8_state)
    return ref.relu2_mlp(x, w_fc, w_proj)


def norm_relu2_mlp(x: Tensor, w_fc: Tensor, w_proj: Tensor, fp8_state=None) -> Tensor:
    """relu(norm(x) w_fc^T)^2 w_proj with the RMSNorm (and, for FP8, the row quantisation) fused in."""
    if use_kernel("mlp", x) and x.dtype == torch.bfloat16 and x.shape[-1] % 256 == 0:
        from . import fused
        return fused.norm_relu2_mlp(x, w_fc, w_proj, fp8_state)
    return ref.relu2_mlp(ref.rms_norm(x), w_fc, w_proj)


def softcap_ce(x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c, grad_scale: float = 1.0,
               fp8: bool = True) -> Tensor:
    """Training loss per token (fp32).  The CUDA path computes the gradient w.r.t. logits in
    the forward with the factor `grad_scale` baked in, so the caller must reduce with
    `.sum() * grad_scale` (same contract as `triton_kernels.py:1208-1292`)."""
    if use_kernel("ce", x) and x.dtype == torch.bfloat16:
        from . import fused
        return fused.softcap_ce(x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c, grad_scale, fp8)
    return ref.softcap_ce(x, w, targets, mtp_weights, prefix_targets, prefix_weight, a, b, c)


def softcap_ce_eval(x, w, targets, a, b, c) -> Tensor:
    if use_kernel("ce", x) and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[0] % 8 == 0:
        from . import fused
        return fused.softcap_ce_eval(x, w, targets, a, b, c)
    return ref.softcap_ce_eval(x, w, targets, a, b, c)
