"""Autograd wrappers of the fused glue kernels (csrc/glue.cu).

`lincomb`   out = sum_j (addc_j + s_j * g_j[t]) * x_j[t, :] - every residual / skip / MUDD mix of
            `train_gpt.py:1547-1680` is one call instead of a chain of broadcast multiplies and adds;
            its backward produces all input gradients, the per-token coefficient gradients and the
            scalar-parameter gradients in one pass.
`qkv_post`  QK RMSNorm + rotary + key offset + value-embedding add (`train_gpt.py:1103-1136`).
`xsa_gate`  gated XSA and the per-head attention gate (`train_gpt.py:1150-1159`).
"""
from __future__ import annotations

import torch
from torch import Tensor

from .native import lib


class GradSink:
    """Gradient buffer shared by the fused ops that consume one tensor.  The first consumer to run in the backward pass
    creates the buffer and hands it to autograd as its gradient; the later ones add into it (or, for gate columns,
    write their own columns) and report no gradient, so autograd forms no sums of full-size tensors."""
    __slots__ = ("buf",)

    def __init__(self):
        self.buf = None


class _SinkSource(torch.autograd.Function):
    @staticmethod
    def forward(ctx, t, sink):
        ctx.sink = sink
        return t

    @staticmethod
    def backward(ctx, g):
        ctx.sink.buf = None                     # every consumer has run: the next backward starts a new buffer
        return g, None


def grad_sink(t: Tensor):
    """Returns (t', sink): t' equals t and must be consumed ONLY through `Term(..., sink=sink)` (as x) or
    `Term(..., gate_sink=sink)` (as gate) -- a consumer that returned its own gradient tensor for t' would have it
    summed with a buffer that is still being added to.  (t, None) when no gradient is needed."""
    if not (torch.is_grad_enabled() and t.requires_grad and t.is_cuda):
        return t, None
    sink = GradSink()
    return _SinkSource.apply(t, sink), sink


class _ColsTap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, t, n):
        ctx.n = n
        ctx.set_materialize_grads(False)
        return t, t[:, :n].contiguous()

    @staticmethod
    def backward(ctx, g_main, g_cols):
        if g_cols is None:
            return g_main, None
        if g_main is None:
            raise RuntimeError("cols_tap: the carried-on tensor received no gradient")
        g_main[:, :ctx.n] += g_cols             # a few columns, in place: no full-size zero fill and sum
        return g_main, None


def cols_tap(t: Tensor, n: int):
    """Returns (t', t[:, :n]) where t' equals t and goes to t's main consumer.  The gradient of the n columns is added
    in place into the gradient t' receives, which therefore must be a tensor its producer does not reuse (the fused
    ops here return freshly allocated gradients)."""
    if not (torch.is_grad_enabled() and t.requires_grad):
        return t, t[:, :n]
    return _ColsTap.apply(t, n)


class Term:
    """One summand of `lincomb`: x * (addc + scalar * gate[:, col]).  `sink` / `gate_sink`: the `GradSink` of x / gate."""
    __slots__ = ("x", "scalar", "gate", "col", "addc", "sink", "gate_sink")

    def __init__(self, x: Tensor, scalar: Tensor | None = None, gate: Tensor | None = None, col: int = 0, addc: float = 0.0,
                 sink: GradSink | None = None, gate_sink: GradSink | None = None):
        self.x, self.scalar, self.gate, self.col, self.addc = x, scalar, gate, col, addc
        self.sink, self.gate_sink = sink, gate_sink


class _LinComb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, meta, *tensors):
        k, sidx, gidx, cols, addc = meta[:5]
        xs = [t.contiguous() for t in tensors[:k]]
        scalars = [tensors[i] if i >= 0 else None for i in sidx]
        gates = [tensors[i] if i >= 0 else None for i in gidx]
        out = lib().lincomb_fwd(xs, scalars, gates, cols, addc)
        ctx.meta = meta
        ctx.save_for_backward(*xs, *tensors[k:])
        return out

    @staticmethod
    def backward(ctx, gout):
        k, sidx, gidx, cols, addc, xsinks, gsinks = ctx.meta
        tensors = ctx.saved_tensors
        xs = list(tensors[:k])
        scalars = [tensors[i] if i >= 0 else None for i in sidx]
        gates = [tensors[i] if i >= 0 else None for i in gidx]
        need = ctx.needs_input_grad[1:]
        grads: list = [None] * len(tensors)
        dgate_bufs, dscal_bufs = {}, {}
        dgates, dscalars = [], []
        dx_into, dx_acc, silent_gates = [None] * k, [False] * k, set()
        for j in range(k):
            gi, si = gidx[j], sidx[j]
            sk = xsinks[j]
            if sk is not None and need[j]:
                if sk.buf is None:
                    sk.buf = torch.empty_like(xs[j])
                    grads[j] = sk.buf                  # the one gradient autograd sees for this tensor
                else:
                    dx_acc[j] = True
                dx_into[j] = sk.buf
            if gi >= 0 and need[gi]:
                if gi not in dgate_bufs:
                    gs = gsinks[j]
                    if gs is not None:
                        if gs.buf is None:
                            gs.buf = torch.zeros_like(tensors[gi])
                        else:
                            silent_gates.add(gi)       # an earlier consumer already handed the buffer to autograd
                        dgate_bufs[gi] = gs.buf
                    else:
                        dgate_bufs[gi] = torch.zeros_like(tensors[gi], dtype=torch.bfloat16)
                dgates.append(dgate_bufs[gi])
            else:
                dgates.append(None)
            if si >= 0 and need[si]:
                if si not in dscal_bufs:
                    dscal_bufs[si] = torch.zeros(1, dtype=torch.float32, device=gout.device)
                dscalars.append(dscal_bufs[si])
            else:
                dscalars.append(None)
        dxs = lib().lincomb_bwd(xs, scalars, gates, cols, addc, gout.contiguous(), [bool(n) for n in need[:k]], dgates, dscalars,
                                dx_into, dx_acc)
        for j in range(k):
            if dx_into[j] is None:
                grads[j] = dxs[j]
        for gi, buf in dgate_bufs.items():
            if gi in silent_gates:
                continue
            grads[gi] = buf if tensors[gi].dtype == torch.bfloat16 else buf.to(tensors[gi].dtype)
        for si, buf in dscal_bufs.items():
            grads[si] = buf.view(tensors[si].shape)
        return (None, *grads)


def lincomb(terms: list[Term]) -> Tensor:
    k = len(terms)
    extra, index = [], {}

    def slot(t):
        if t is None:
            return -1
        key = id(t)
        if key not in index:
            index[key] = k + len(extra)
            extra.append(t)
        return index[key]

    sidx = [slot(t.scalar) for t in terms]
    gidx = [slot(t.gate) for t in terms]
    for t in terms:
        assert t.gate_sink is None or t.gate.dtype == torch.bfloat16, "gate sinks hold bf16 gradients"
    meta = (k, sidx, gidx, [int(t.col) for t in terms], [float(t.addc) for t in terms], [t.sink for t in terms],
            [t.gate_sink for t in terms])
    return _LinComb.apply(meta, *[t.x for t in terms], *extra)


class _QkvPost(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos_t, sin_t, ve, vgate, vadd, H, paired, key_offset, split=False):
        qkv = qkv.contiguous()
        if ve is not None:
            ve = ve.contiguous()
        if vadd is not None:
            vadd = vadd.contiguous()
        q, k, v, rq, rk = lib().qkv_post_fwd(qkv, cos_t, sin_t, ve, vgate, vadd, H, paired, key_offset, split)
        ctx.save_for_backward(qkv, cos_t, sin_t, rq, rk, ve, vgate)
        ctx.cfg = (H, paired, key_offset, vadd is not None, split)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, cos_t, sin_t, rq, rk, ve, vgate = ctx.saved_tensors
        H, paired, key_offset, has_vadd, split = ctx.cfg
        dv = dv.contiguous()
        need_dve = ve is not None and ctx.needs_input_grad[3]
        need_dvg = vgate is not None and ctx.needs_input_grad[4]
        dqkv, dve, dvg = lib().qkv_post_bwd(qkv, cos_t, sin_t, rq, rk, dq.contiguous(), dk.contiguous(), dv, ve, vgate, H,
                                            paired, key_offset, need_dve, need_dvg, split)
        dvadd = dv.view(qkv.shape[0], -1) if has_vadd else None
        return dqkv, None, None, dve, dvg, dvadd, None, None, None, None


def qkv_post(qkv: Tensor, cos_t: Tensor, sin_t: Tensor, ve: Tensor | None, vgate: Tensor | None, vadd: Tensor | None,
             H: int, paired: bool, key_offset: bool, split: bool = False):
    """qkv [T, 3*H*128] -> q, k, v [T, H, 128].  v = v + vgate[t,h]*ve[t,h,:] + vadd[t,h,:].
    `split`: rotary pairs are (d, d + 64) for d < 32 (track-2 layout) instead of interleaved (2i, 2i+1) for i < 32."""
    return _QkvPost.apply(qkv, cos_t, sin_t, ve, vgate, vadd, H, paired, key_offset, split)


class _XsaGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, v, alpha, gate):
        y, v = y.contiguous(), v.contiguous()
        out = lib().xsa_gate_fwd(y, v, alpha, gate)
        ctx.save_for_backward(y, v, alpha, gate)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, v, alpha, gate = ctx.saved_tensors
        dy, dv, da, dg = lib().xsa_gate_bwd(y, v, alpha, gate, dout.contiguous(), None, None)
        return dy, dv, da, dg


class _XsaGateCols(torch.autograd.Function):
    """`xsa_gate` with alpha / gate given as column offsets into one wide gate tensor that has a `GradSink`: the
    backward writes its [T, H] column blocks straight into the shared gradient buffer."""

    @staticmethod
    def forward(ctx, y, v, gates, sink, col_alpha, col_gate):
        y, v = y.contiguous(), v.contiguous()
        H = y.shape[1]
        alpha = gates[:, col_alpha:col_alpha + H] if col_alpha is not None else None
        gate = gates[:, col_gate:col_gate + H] if col_gate is not None else None
        out = lib().xsa_gate_fwd(y, v, alpha, gate)
        ctx.save_for_backward(y, v, gates)
        ctx.cfg = (sink, col_alpha, col_gate)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, v, gates = ctx.saved_tensors
        sink, ca, cg = ctx.cfg
        H = y.shape[1]
        first = sink.buf is None
        if first:
            sink.buf = torch.zeros_like(gates)
        sl = lambda t, c: t[:, c:c + H] if c is not None else None
        dy, dv, _, _ = lib().xsa_gate_bwd(y, v, sl(gates, ca), sl(gates, cg), dout.contiguous(), sl(sink.buf, ca), sl(sink.buf, cg))
        return dy, dv, (sink.buf if first else None), None, None, None


def xsa_gate_cols(y: Tensor, v: Tensor, gates: Tensor, sink, col_alpha: int | None, col_gate: int | None) -> Tensor:
    """`xsa_gate(y, v, gates[:, col_alpha:+H], gates[:, col_gate:+H])` for a gate tensor from `grad_sink`."""
    if col_alpha is None and col_gate is None:
        return y
    return _XsaGateCols.apply(y, v, gates, sink, col_alpha, col_gate)


def xsa_gate(y: Tensor, v: Tensor, alpha: Tensor | None, gate: Tensor | None) -> Tensor:
    """y, v [T, H, 128]; alpha, gate: bf16 [T, H] (possibly column slices of a wider gate tensor)."""
    if alpha is None and gate is None:
        return y
    return _XsaGate.apply(y, v, alpha, gate)


class _EmbedDirect(torch.autograd.Function):
    """Row gather whose backward adds the row gradients straight into `grad_buf` (the parameter's
    persistent .grad, bf16 [V, D]) with the sorted segmented-sum kernel; the weight itself receives
    no autograd gradient."""

    @staticmethod
    def forward(ctx, ids, weight, grad_buf):
        ctx.save_for_backward(ids)
        ctx.grad_buf = grad_buf
        return torch.nn.functional.embedding(ids, weight)

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        sorted_ids, perm = torch.sort(ids.reshape(-1))
        g2 = g.reshape(-1, g.shape[-1]).contiguous()
        lib().embed_bwd(g2, sorted_ids, perm, ctx.grad_buf)
        return None, None, None


def embed_direct(ids: Tensor, weight: Tensor, grad_buf: Tensor) -> Tensor:
    """weight[ids] with gradient accumulation into grad_buf.  The dummy leaf keeps the op in the graph."""
    return _EmbedDirect.apply(ids, weight.detach().requires_grad_(True), grad_buf)
