"""CUDA execution path of `GPT.forward`: the same math as the op-by-op forward in `gpt.py`, with
every residual / gate / norm / rotary step routed through the fused sm_100a kernels
(`ops.glue`, `ops.fused`).  Selected automatically for bf16 CUDA models with head_dim 128 and
model_dim a multiple of 256; `ops.set_backend("reference")` switches it off for A/B tests."""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from ..ops import functional as ops
from ..ops import fused
from ..ops.glue import Term, cols_tap, embed_direct, grad_sink, lincomb, qkv_post, xsa_gate, xsa_gate_cols


import os

MLP_MIX_FUSED = os.environ.get("MNG_MLP_MIX", "1") != "0"    # 0: separate `lincomb` after the down projection (A/B switch)


def fused_supported(model, x: Tensor) -> bool:
    from .. import ops as ops_pkg
    return (x.is_cuda and ops_pkg.get_backend() != "reference" and model.head_dim == 128 and model.model_dim % 256 == 0
            and model.model_dim <= 1024 and model.lm_head.weight.dtype == torch.bfloat16
            and (model.cfg.bigram_dim in (0, model.model_dim)) and ops_pkg.use_kernel("glue", x))


def _rope_tables(yarn, n: int, device):
    """fp32 cos/sin [n, 32] of the 32 distinct rotary frequencies, values rounded to bf16 like the
    reference's tables (`train_gpt.py:1013-1032`)."""
    cache = getattr(yarn, "_t32", None)
    if cache is None or cache[0] != yarn._version or cache[1].size(0) < n or cache[1].device != device:
        t = torch.arange(n, dtype=torch.float32, device=device)
        theta = torch.outer(t, yarn.angular_freq.to(device)[0:yarn.head_dim // 2:2])
        cache = (yarn._version, theta.cos().bfloat16().float().contiguous(), theta.sin().bfloat16().float().contiguous())
        yarn._t32 = cache
    return cache[1], cache[2]


def forward_fused(m, input_seq: Tensor, target_seq: Tensor, seqlens: Tensor, bigram_input_seq: Tensor, sc) -> Tensor:
    cfg, L, H, Dh, D, V = m.cfg, m.num_layers, m.num_heads, m.head_dim, m.model_dim, m.vocab_size
    T = input_seq.size(0)
    ws = {False: sc.ws_short, True: sc.ws_long}
    max_len = sc.train_max_seq_len if m.training else m.eval_seq_len
    training_fp8 = m.training and m.use_fp8
    track1 = m.track1

    sa_lambdas = m.scalars[:2 * L].view(L, 2)
    smear_lambda, skip_lambda = m.scalars[2 * L], m.scalars[2 * L + 1]
    qk_all, vo_all = m.attn_layer_weights()
    resid, post = m.resid_lambdas, m.post_lambdas
    # Training: the weight-gradient GEMMs accumulate straight into slices of the bank gradients (no
    # per-layer select/stack of full-bank tensors), so the bank gradients must exist up front.
    direct = m.training and torch.is_grad_enabled()
    qk_g = vo_g = None
    if direct:
        tables = [m.embed.weight] + ([m.value_embeds] if cfg.num_value_embeds else []) + (
            [m.bigram_embed.weight] if cfg.bigram_vocab_size else [])
        for p in (m.qk_bank, m.vo_bank, m.mlp_bank, *tables):
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        A = m._num_attn_layers
        qk_g = m.qk_bank.grad[:m._num_qk_groups].view(A, 2 * D, D)
        vo_g = m.vo_bank.grad[:2 * A].view(A, 2 * D, D)

    # [Wq; Wk; Wv] of every attention layer as one contiguous matrix (Q, K live in qk_bank, V in vo_bank)
    qkv_w = m.qkv_weights() if (direct or not torch.is_grad_enabled()) else None

    ids = input_seq.long()
    gather = (lambda i, w: embed_direct(i, w, w.grad)) if direct else F.embedding
    x = gather(ids, m.embed.weight)
    x0_bigram = None
    if cfg.bigram_vocab_size:
        sign_idx = torch.zeros_like(ids)
        sign_idx[1:] = (ids[:-1] ^ ids[1:]) % m.bigram_sign_table.shape[0]
        x0_bigram = gather(bigram_input_seq.long(), m.bigram_embed.weight) * m.bigram_sign_table[sign_idx]
    ve = None
    if cfg.num_value_embeds:
        # one gather over the flat table (ids offset per table): a single embedding backward into one
        # [n*V, D] gradient instead of n full-size zero-filled select_backward tensors
        n = cfg.num_value_embeds
        offs = torch.arange(n, device=ids.device)[:, None] * V
        ve = gather((ids[None, :] + offs).reshape(-1), m.value_embeds).view(n, T, D).unbind(0)

    # smear: x[t] += smear_lambda * sigmoid(W x[t, :12]) * x[t-1]
    g = torch.zeros(T, 1, dtype=x.dtype, device=x.device)
    g[1:] = smear_lambda * torch.sigmoid(F.linear(x[1:, :12], m.smear_gate.weight))
    x_prev = torch.cat([x[:1], x[:-1]])
    x = lincomb([Term(x), Term(x_prev, gate=g, col=0)])
    x = x0 = fused.rms_norm(x)

    # document starts for the attention kernel: once per forward for the plain and the doubled (paired-head) packing
    ds1 = ds2 = seq2 = None
    if fused.ATTN_KERNEL:
        ds1 = fused.doc_bounds(seqlens, T)
        if any(pl.paired for pl in m.plan):
            seq2 = 2 * seqlens
            ds2 = fused.doc_bounds(seq2, 2 * T)
    cos_t, sin_t = _rope_tables(m.yarn, 2 * T, x.device)
    cos_p, sin_p = _rope_tables(m.yarn_paired_head, 2 * T, x.device)

    # Tensors that many lincombs consume get one shared gradient buffer each (x0, the bigram embedding, cached layer
    # outputs, the gate matrices): their consumers add into it instead of autograd summing full-size gradients.
    # The `*_s` aliases go to lincomb terms only; every other consumer keeps the plain tensor.
    sinks: dict = {}

    def sunk(name, t):
        if t is None:
            return None
        if name not in sinks:
            sinks[name] = grad_sink(t)
        return sinks[name][0]

    def X(name, t, **kw):                                    # lincomb term over a shared-gradient tensor
        ts = sunk(name, t)
        return Term(ts, sink=sinks[name][1], **kw)

    def G(name, gate):                                       # gate= / gate_sink= keywords for a shared-gradient gate
        if gate is None:
            return {}
        if gate.dtype != torch.bfloat16:                     # shared gate gradients are bf16 buffers
            return dict(gate=gate)
        gs = sunk(name, gate)
        return dict(gate=gs, gate_sink=sinks[name][1])

    pre = pg = None
    lay0 = lay1 = None
    if track1:
        pre = m._gate_mlp(x0, 0)
        lay0, lay1 = m.gate_layouts
        x = lincomb([X("x0", x0), X("x0b", x0_bigram, col=lay0["inject"][0] + 1, **G("pre", pre))])
    cache = {0: x}
    normed7 = None

    def gate_of(i):
        return (pre, lay0, "pre") if i < m.post_gate_layer else (pg, lay1, "pg")

    for pl in m.plan:
        i, mu = pl.index, None
        if track1 and i == m.post_gate_layer:
            pg = m._gate_mlp(x, 1)

        if not pl.has_attn:
            sk = torch.sigmoid(skip_lambda).reshape(1)
            x = lincomb([Term(x), X("c3", cache[3], scalar=sk, col=lay1["skip"], **G("pg", pg))])
        else:
            sl = pl.attn_slot
            if track1 and 7 in cache:
                if normed7 is None:
                    normed7 = fused.rms_norm(cache[7])
                attn_in = normed7
            else:
                attn_in, x = fused.rms_norm_fork(x)          # x's two gradients meet inside the norm backward
            ve_t = vgate = vadd = None
            if track1 and pl.last:
                cache[9] = x
                mu = m._mudd_raw(x, 0, 14)                                    # [T, 14]
                vadd = lincomb([X("c0", cache[0], col=0, **G("mu", mu)), X("c7", cache[7], col=1, **G("mu", mu)),
                                Term(x, col=2, **G("mu", mu))])
                x = lincomb([Term(x, col=5, addc=1.0, **G("mu", mu)), X("c0", cache[0], col=3, **G("mu", mu)),
                             X("c7", cache[7], col=4, **G("mu", mu))])
                vgate = mu[:, 6:8].repeat_interleave(H // 2, dim=-1).contiguous()
                ve_t = ve[pl.ve_slot]
            elif pl.ve_slot >= 0:
                ve_t = ve[pl.ve_slot]
                if direct:                                   # the 6-column gradients join the main ones in place
                    attn_in, a6 = cols_tap(attn_in, 6)
                    ve_t, v6 = cols_tap(ve_t, 6)
                    gate_in = torch.cat([a6, v6], dim=-1)
                else:
                    gate_in = torch.cat([attn_in[:, :6], ve_t[:, :6]], dim=-1)
                vgate = (2 * torch.sigmoid(F.linear(gate_in, m.ve_gate_bank[pl.ve_slot]))).contiguous()
            yarn = m.yarn_paired_head if pl.paired else m.yarn
            ct, st = (cos_p, sin_p) if pl.paired else (cos_t, sin_t)
            key_off = pl.long_window and not pl.paired
            if direct and vadd is None and fused.qkv_proj_supported(attn_in, qkv_w[sl], H):
                # projection with QK norm, rotary, key offset and value-embedding add in its epilogue
                q, k, v = fused.qkv_proj(attn_in, sa_lambdas[i, 0], qkv_w[sl], [qk_g[sl], vo_g[sl][:D]], ct, st, ve_t, vgate,
                                         H, pl.paired, key_off)
            else:
                if direct:
                    qkv = fused.bank_linear(attn_in, sa_lambdas[i, 0], qkv_w[sl], [qk_g[sl], vo_g[sl][:D]])
                elif not torch.is_grad_enabled():
                    qkv = fused.linear_scaled(attn_in, qkv_w[sl], sa_lambdas[i, 0])
                else:
                    qkv = F.linear(attn_in, sa_lambdas[i, 0] * torch.cat([qk_all[sl], vo_all[sl][:D]], dim=0))
                q, k, v = qkv_post(qkv, ct, st, ve_t, vgate, vadd, H, pl.paired, key_off)
            if pl.paired:
                y = ops.attention(q.view(2 * T, H // 2, Dh), k.view(2 * T, H // 2, Dh), v.view(2 * T, H // 2, Dh),
                                  seq2 if seq2 is not None else 2 * seqlens, ws[pl.long_window], yarn.attn_scale, 2 * max_len,
                                  ds2).view(T, H, Dh)
            else:
                y = ops.attention(q, k, v, seqlens, ws[pl.long_window], yarn.attn_scale, max_len, ds1)
            gt, lay, gname = gate_of(i) if track1 else (None, None, None)
            if track1 and pl.dc and not pl.paired:
                o = lay1["dc"]
                # RMS norm over H = 6 values per token, spelled out: the library's row-moments kernel takes 230 us
                # on [T, 6] rows, these elementwise ops a few microseconds each
                wf = pg[:, o:o + H].float()
                w1 = (wf * torch.rsqrt(wf.square().mean(dim=-1, keepdim=True) + 1e-6)).to(x.dtype).contiguous()
                w2 = pg[:, o + H:o + 2 * H].contiguous()
                y = ops.dc_correction(y, q, k, v, w1, w2, seqlens, yarn.attn_scale, cfg.dc_window)
            if track1:
                ca = lay["xsa"][i] if (pl.xsa and not pl.paired) else None
                cg = lay["attn"][i] if pl.attn_gate else None
                gts = sunk(gname, gt) if gt.dtype == torch.bfloat16 else None
                if gts is not None and sinks[gname][1] is not None:
                    y = xsa_gate_cols(y, v, gts, sinks[gname][1], ca, cg)
                else:
                    y = xsa_gate(y, v, gt[:, ca:ca + H] if ca is not None else None, gt[:, cg:cg + H] if cg is not None else None)
            if direct:
                attn_out = fused.bank_linear(y.reshape(T, D), sa_lambdas[i, 1], vo_all[sl][D:], [vo_g[sl][D:]])
            elif not torch.is_grad_enabled():
                attn_out = fused.linear_scaled(y.reshape(T, D), vo_all[sl][D:], sa_lambdas[i, 1])
            else:
                attn_out = F.linear(y.reshape(T, D), sa_lambdas[i, 1] * vo_all[sl][D:])
            if mu is not None:
                x = lincomb([Term(x, col=8, **G("mu", mu)), Term(attn_out, col=9, **G("mu", mu)),
                             X("c0", cache[0], col=10, **G("mu", mu)), X("x0b", x0_bigram, col=11, **G("mu", mu))])
            elif track1:
                o = lay["inject"][i]
                terms = [Term(x, scalar=resid[i, 0]), Term(attn_out, scalar=post[i, 0]), X("x0", x0, col=o, **G(gname, gt))]
                if i != 0:
                    terms.append(X("x0b", x0_bigram, col=o + 1, **G(gname, gt)))
                x = lincomb(terms)
            else:
                x = lincomb([Term(x, scalar=resid[i, 0]), Term(attn_out, scalar=post[i, 0])])

        if direct:
            st = m._fp8_state.layer(i) if (training_fp8 and m._fp8_state is not None) else None
            gviews = (m.mlp_bank.grad[i, 0], m.mlp_bank.grad[i, 1])
            if mu is None and MLP_MIX_FUSED:
                # resid * x + post * MLP(norm(x)) inside the down projection's epilogue (`train_gpt.py:1665`)
                x = fused.norm_relu2_mlp_mix(x, m.mlp_bank[i, 0], m.mlp_bank[i, 1], resid[i, 1], post[i, 1], st, gviews)
                h = None
            else:
                h, x = fused.norm_relu2_mlp(x, m.mlp_bank[i, 0], m.mlp_bank[i, 1], st, gviews, fork=True)
        else:
            h = m._mlp(i, x, training_fp8)
        if h is None:
            pass
        elif mu is not None:
            x = lincomb([Term(x, col=12, **G("mu", mu)), Term(h, col=13, **G("mu", mu))])
        else:
            x = lincomb([Term(x, scalar=resid[i, 1]), Term(h, scalar=post[i, 1])])
        if pl.cache:
            cache[i] = x

    if track1:
        mu = m._mudd_raw(x, 1, 5)
        x = lincomb([Term(x), X("c0", cache[0], col=0, **G("mu2", mu)), X("c7", cache[7], col=1, **G("mu2", mu)),
                     Term(cache[9], col=2, **G("mu2", mu)), Term(ve[0], col=3, **G("mu2", mu)),
                     X("c3", cache[3], col=4, **G("mu2", mu))])
    x = fused.rms_norm(x)

    if m.training:
        prefix_targets = m.prefix_table[target_seq]
        return ops.softcap_ce(x, m.lm_head.weight, target_seq, sc.mtp_weights, prefix_targets, sc.prefix_weight,
                              cfg.softcap_a, cfg.softcap_b, cfg.softcap_c, grad_scale=m.grad_scale, fp8=m.head_fp8)
    return ops.softcap_ce_eval(x, m.lm_head.weight, target_seq, cfg.softcap_a, cfg.softcap_b, cfg.softcap_c)
