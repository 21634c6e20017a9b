"""Track-2 (GPT-2-medium scale) model: 16 layers, d_model 1024, 8 heads x 128.

Topology of `train_gpt_medium.py:1037-1218`: attention in every layer with the window pattern
L S S S L S S S S S S L S S S L (long windows also get the partial key offset), split-half
rotary (pairs (d, d+64), upper quarter bands stationary), sigmoid attention gate on x[:16],
value embeddings on layers 0-4 and 11-15 through a 2*sigmoid gate, gated U-net skips 2/4/6 ->
11/10/9, a second input embedding `embed2`, per-layer residual / x0 / x02 mixing scalars, back-out
of the layer-11 stream before the head, smear, softcapped head with multi-token loss.

Design differences from the reference file: weights live in the same parameter-bank layout as the
track-1 model (`attn_bank` [4*L padded, D, D] = Q,K,V,O per layer; `mlp_bank` [L, 2, 4D, D]), the
head is stored transposed (D, V) and tied to `embed` through the optimizer, so the same
`NorMuonAndAdam`, fused collectives and FP8 head/MLP kernels serve both tracks.  The small (8,16) gate
matrices are NorMuon parameters as in the reference, stacked into two banks padded to the rank count.
`reference_state_dict()` / `load_reference_state_dict()` convert to and from the reference's
per-module key layout (`blocks.{i}.attn.qkvo_w`, `blocks.{i}.mlp.c_fc`, `lm_head.weight` (V, D), ...).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import next_multiple_of_n
from ..ops import functional as ops
from .gpt import ForwardScheduleConfig, _Weight
from .yarn import Yarn

LONG_LAYERS = (0, 4, 11, 15)
VE_LAYERS = {0: 0, 1: 1, 2: 2, 3: 3, 4: 4, 11: 0, 12: 1, 13: 2, 14: 3, 15: 4}
SKIP_IN, SKIP_OUT, BACKOUT_LAYER = (2, 4, 6), (9, 10, 11), 11


class SplitYarn(Yarn):
    """Half-truncated rotary with split halves: dims d < head_dim/4 rotate with d + head_dim/2."""

    def reset(self):
        hd = self.head_dim
        f = (1 / 1024) ** torch.linspace(0, 1, steps=hd // 4, dtype=torch.float32, device=self.device)
        self.angular_freq = torch.cat([f, f.new_zeros(hd // 4)])
        self.attn_scale = 0.1
        self._tables = None
        self._version = getattr(self, "_version", 0) + 1

    def tables(self, T: int):
        if self._tables is None or self._tables[0].size(0) < T:
            t = torch.arange(max(T, 1), dtype=torch.float32, device=self.angular_freq.device)
            theta = torch.outer(t, self.angular_freq)
            self._tables = (theta.cos().bfloat16().float(), theta.sin().bfloat16().float())
        return self._tables[0][:T], self._tables[1][:T]

    def rotary(self, x: Tensor) -> Tensor:
        cos, sin = self.tables(x.size(0))
        cos, sin = cos[:, None, :].to(x.dtype), sin[:, None, :].to(x.dtype)
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat((x1 * cos + x2 * sin, x2 * cos - x1 * sin), dim=-1)


class GPTMedium(nn.Module):
    def __init__(self, vocab_size: int = 50257, num_layers: int = 16, num_heads: int = 8, head_dim: int = 128,
                 model_dim: int = 1024, max_seq_len: int = 262144, *, world_size: int = 1, grad_scale: float = 1.0,
                 use_fp8: bool = True, eval_seq_len: int | None = None):
        super().__init__()
        L, H, Dh, D = num_layers, num_heads, head_dim, model_dim
        assert H * Dh == D
        self.num_layers, self.num_heads, self.head_dim, self.model_dim = L, H, Dh, D
        self.vocab_size = V = next_multiple_of_n(vocab_size, n=128)
        self.world_size, self.grad_scale, self.use_fp8 = world_size, grad_scale, use_fp8
        self.eval_seq_len = eval_seq_len or max_seq_len
        self.softcap = (23.0, 5.0, 7.5)
        self.register_buffer("prefix_table", torch.full((V,), -1, dtype=torch.int64), persistent=False)
        self.lm_head = _Weight(D, V)
        nn.init.normal_(self.lm_head.weight, mean=0, std=0.005)
        self.embed = _Weight(V, D)
        with torch.no_grad():
            self.embed.weight.copy_(self.lm_head.weight.T)
        self.embed2 = _Weight(V, D)
        nn.init.normal_(self.embed2.weight)
        self.value_embeds = nn.Parameter(torch.zeros(5 * V, D))
        n_attn = next_multiple_of_n(4 * L, n=world_size)
        self.attn_bank = nn.Parameter(torch.zeros(n_attn, D, D))
        self.attn_bank.reshape = (n_attn, D, D)
        Lp = L
        while (2 * Lp) % world_size:
            Lp += 1
        self.mlp_bank = nn.Parameter(torch.zeros(Lp, 2, 4 * D, D))
        self.mlp_bank.reshape = (2 * Lp, 4 * D, D)
        with torch.no_grad():
            b_attn = (3 ** 0.5) * D ** -0.5
            b_mlp = (3 ** 0.5) * 0.5 * D ** -0.5
            qkv = self.attn_bank[:4 * L].view(L, 4, D, D)
            qkv[:, :3].uniform_(-b_attn, b_attn)               # O projections stay zero
            self.mlp_bank[:L, 0].uniform_(-b_mlp, b_mlp)       # down projections stay zero
        # the small gate matrices are NorMuon parameters, as in the reference (`train_gpt_medium.py:1478`, groups padded
        # to a multiple of the rank count, `:524-543`): whole (H, 16) matrices are sharded over the ranks
        ag, vg = next_multiple_of_n(L, n=world_size), next_multiple_of_n(len(VE_LAYERS), n=world_size)
        self.attn_gate_bank = nn.Parameter(torch.zeros(ag, H, 16))
        self.attn_gate_bank.reshape = (ag, H, 16)
        self.value_embed_gate_bank = nn.Parameter(torch.zeros(vg, H, 16))
        self.value_embed_gate_bank.reshape = (vg, H, 16)
        self.smear_gate = _Weight(1, 16)
        self.skip_gates = nn.Parameter(torch.zeros(3, 1, 16))
        self.x0_lambdas = nn.Parameter(torch.zeros(2 * L))
        pad = (-L * 3 - 5) % world_size
        self.scalars = nn.Parameter(torch.cat([1.05 * torch.ones(L), torch.tensor([0.5, 1.0]).repeat(L), torch.zeros(1),
                                               0.5 * torch.ones(1), -1.5 * torch.ones(3), torch.ones(pad)]))
        self.yarn = SplitYarn(Dh, max_seq_len)
        self.yarn_paired_head = self.yarn          # one rotary state; the manager updates both names
        self._ve_slot = {layer: j for j, layer in enumerate(sorted(VE_LAYERS))}
        for name, p in self.named_parameters():
            p.label = name.replace(".weight", "")
        self._fp8_state = None

    # -- plumbing shared with the track-1 model ------------------------------------------------
    def cast_params_(self, dtype=torch.bfloat16):
        for _, p in self.named_parameters():
            if p.label not in ("scalars", "x0_lambdas"):
                p.data = p.data.to(dtype)
        return self

    def _apply(self, fn, *a, **k):
        out = super()._apply(fn, *a, **k)
        self.yarn.to(self.lm_head.weight.device)
        return out

    def quantize_mlp_fp8(self, bootstrap_down: bool = False):
        if not (self.use_fp8 and self.mlp_bank.is_cuda):
            return
        from ..ops import fused
        if not hasattr(self, "_scale_a"):
            self._scale_a = torch.ones(self.mlp_bank.shape[0], device=self.mlp_bank.device)
            self._scale_b = torch.ones_like(self._scale_a)
        with torch.no_grad():
            self._fp8_state = fused.quantize_mlp_weights(self.mlp_bank, self._fp8_state, self._scale_a, self._scale_b, bootstrap_down)

    @staticmethod
    def param_table() -> dict:
        """Optimizer settings of `train_gpt_medium.py:1476-1486` mapped onto the unified optimizer."""
        adam = lambda **k: dict(optim="adam", adam_betas=[0.8, 0.95], **k)
        return {
            "attn_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None},
            "mlp_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None},
            "scalars": {"optim": "adam", "comms": "replicated", "adam_betas": [0.9, 0.99], "lr_mul": 10.0, "wd_mul": 0.0},
            "attn_gate_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None, "lr_mul": 0.1},
            "value_embed_gate_bank": {"optim": "normuon", "comms": "sharded", "adam_betas": None, "lr_mul": 0.1},
            "smear_gate": adam(comms="replicated", lr_mul=0.01, wd_mul=0.0), "skip_gates": adam(comms="replicated", lr_mul=0.01, wd_mul=0.0),
            "x0_lambdas": adam(comms="replicated", lr_mul=5.0, wd_mul=0.0),
            "lm_head": adam(comms="sharded", wd_mul=150.0), "value_embeds": adam(comms="sharded", lr_mul=75.0, wd_mul=5.0),
            "embed2": adam(comms="sharded", lr_mul=75.0, wd_mul=5.0), "embed": adam(comms="sharded", wd_mul=150.0),
        }

    WORK_ORDER = ["scalars", "smear_gate", "skip_gates", "x0_lambdas", "value_embeds", "embed2", "lm_head", "embed",
                  "attn_gate_bank", "value_embed_gate_bank", "attn_bank", "mlp_bank"]

    # -- forward ---------------------------------------------------------------------------------
    def forward(self, input_seq: Tensor, target_seq: Tensor, seqlens: Tensor, bigram_input_seq: Tensor | None,
                schedule_cfg: ForwardScheduleConfig) -> Tensor:
        if self._fused_ok(input_seq):
            return self._forward_fused(input_seq, target_seq, seqlens, schedule_cfg)
        L, H, Dh, D, V = self.num_layers, self.num_heads, self.head_dim, self.model_dim, self.vocab_size
        T = input_seq.size(0)
        max_len = schedule_cfg.train_max_seq_len if self.training else self.eval_seq_len
        resid = self.scalars[:L]
        sa = self.scalars[L:3 * L].view(L, 2)
        smear_lambda, backout_lambda = self.scalars[3 * L], self.scalars[3 * L + 1]
        skip_lambdas = self.scalars[3 * L + 2:3 * L + 5]
        x0l = self.x0_lambdas.view(L, 2)
        ids = input_seq.long()
        x = F.embedding(ids, self.embed.weight)
        adt = x.dtype
        ve_all = self.value_embeds.view(5, V, D)
        g = smear_lambda * torch.sigmoid(F.linear(x[1:, :16], self.smear_gate.weight.type_as(x)))
        x = torch.cat([x[:1], x[1:] + g * x[:-1]])
        x = x0 = ops.rms_norm(x)
        x02 = ops.rms_norm(F.embedding(ids, self.embed2.weight))
        w_all = self.attn_bank[:4 * L].view(L, 4 * D, D)
        skips, x_backout, skip_idx = [], None, 0
        for i in range(L):
            if i in SKIP_OUT:
                sg = torch.sigmoid(skip_lambdas[skip_idx]) * 2 * torch.sigmoid(F.linear(x0[:, :16], self.skip_gates[skip_idx].type_as(x)))
                skip_idx += 1
                x = x + sg.to(adt) * skips.pop()
            if i == 0:
                x = (resid[0] + x0l[0, 0]).to(adt) * x + x0l[0, 1].to(adt) * x02
            else:
                x = resid[i].to(adt) * x + x0l[i, 0].to(adt) * x0 + x0l[i, 1].to(adt) * x02
            # attention
            xin = ops.rms_norm(x)
            w = w_all[i]
            qkv = F.linear(xin, sa[i, 0] * w[:3 * D].type_as(x)).view(T, 3 * H, Dh)
            q, k, v = qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:]
            q, k = self.yarn.rotary(ops.rms_norm(q)), self.yarn.rotary(ops.rms_norm(k))
            is_long = i in LONG_LAYERS
            if is_long:      # stationary quarter bands come from the previous token
                prev = torch.cat([k[:1], k[:-1]], dim=0)
                band = torch.zeros(Dh, dtype=torch.bool, device=k.device)
                band[Dh // 4:Dh // 2] = True
                band[3 * Dh // 4:] = True
                k = torch.where(band, prev, k)
            if i in VE_LAYERS:
                vg = 2 * torch.sigmoid(F.linear(xin[:, :16], self.value_embed_gate_bank[self._ve_slot[i]].type_as(x))).view(T, H, 1)
                v = v + vg * F.embedding(ids, ve_all[VE_LAYERS[i]]).view(T, H, Dh)
            window = (schedule_cfg.ws_long if is_long else schedule_cfg.ws_short)
            y = ops.attention(q.contiguous(), k.contiguous(), v.contiguous(), seqlens, window, self.yarn.attn_scale, max_len)
            y = y * torch.sigmoid(F.linear(xin[:, :16], self.attn_gate_bank[i].type_as(x))).view(T, H, 1)
            x = x + F.linear(y.reshape(T, D), sa[i, 1] * w[3 * D:].type_as(x))
            # MLP
            st = self._fp8_state.layer(i) if (self.training and self.use_fp8 and self._fp8_state is not None) else None
            x = x + ops.norm_relu2_mlp(x, self.mlp_bank[i, 0], self.mlp_bank[i, 1], st)
            if i in SKIP_IN:
                skips.append(x)
            if i == BACKOUT_LAYER:
                x_backout = x
        x = x - backout_lambda.to(adt) * x_backout
        x = ops.rms_norm(x)
        a, b, c = self.softcap
        if self.training:
            return ops.softcap_ce(x, self.lm_head.weight, target_seq, schedule_cfg.mtp_weights, None, None, a, b, c,
                                  grad_scale=self.grad_scale, fp8=self.use_fp8)
        return ops.softcap_ce_eval(x, self.lm_head.weight, target_seq, a, b, c)


    # -- CUDA execution path: the same math through the fused sm_100a kernels --------------------------
    def _fused_ok(self, x: Tensor) -> bool:
        from .. import ops as ops_pkg
        return (x.is_cuda and ops_pkg.get_backend() != "reference" and self.head_dim == 128 and self.model_dim % 256 == 0
                and self.model_dim <= 1024 and self.lm_head.weight.dtype == torch.bfloat16 and ops_pkg.use_kernel("glue", x))

    def _forward_fused(self, input_seq: Tensor, target_seq: Tensor, seqlens: Tensor, sc: ForwardScheduleConfig) -> Tensor:
        """`forward` with every residual / gate / norm / rotary step on the fused kernels (`ops.glue`,
        `ops.fused`) and, in training, weight and embedding gradients accumulated straight into the
        parameters' `.grad` buffers (no full-bank temporaries from slicing the parameter banks)."""
        from ..ops import fused
        from ..ops.glue import Term, cols_tap, embed_direct, grad_sink, lincomb, qkv_post, xsa_gate
        L, H, Dh, D, V = self.num_layers, self.num_heads, self.head_dim, self.model_dim, self.vocab_size
        T = input_seq.size(0)
        max_len = sc.train_max_seq_len if self.training else self.eval_seq_len
        resid = self.scalars[:L]
        sa = self.scalars[L:3 * L].view(L, 2)
        smear_lambda, backout_lambda = self.scalars[3 * L], self.scalars[3 * L + 1]
        skip_lambdas = self.scalars[3 * L + 2:3 * L + 5]
        x0l = self.x0_lambdas.view(L, 2)
        direct = self.training and torch.is_grad_enabled()
        w_all = self.attn_bank[:4 * L].view(L, 4 * D, D)
        g_all = None
        if direct:
            for p in (self.attn_bank, self.mlp_bank, self.embed.weight, self.embed2.weight, self.value_embeds):
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
            g_all = self.attn_bank.grad[:4 * L].view(L, 4 * D, D)
        ids = input_seq.long()
        gather = (lambda i, w: embed_direct(i, w, w.grad)) if direct else F.embedding
        x = gather(ids, self.embed.weight)
        offs = torch.arange(5, device=ids.device)[:, None] * V
        ve = gather((ids[None, :] + offs).reshape(-1), self.value_embeds).view(5, T, D).unbind(0)
        g = torch.zeros(T, 1, dtype=x.dtype, device=x.device)
        g[1:] = smear_lambda * torch.sigmoid(F.linear(x[1:, :16], self.smear_gate.weight))
        x = lincomb([Term(x), Term(torch.cat([x[:1], x[:-1]]), gate=g, col=0)])
        x = x0 = fused.rms_norm(x)
        x02 = fused.rms_norm(gather(ids, self.embed2.weight))
        cos, sin = self.yarn.tables(T)
        cos_t, sin_t = cos[:, :32].contiguous(), sin[:, :32].contiguous()
        bounds = fused.doc_bounds(seqlens, T) if fused.ATTN_KERNEL else None
        skips, x_backout, skip_idx = [], None, 0
        # x0 / x02 feed every layer's mix: one shared gradient buffer each instead of a sum per layer
        x0_s, x0_sink = grad_sink(x0)
        x02_s, x02_sink = grad_sink(x02)
        for i in range(L):
            terms = []
            if i in SKIP_OUT:
                sg = (torch.sigmoid(skip_lambdas[skip_idx]) * 2 * torch.sigmoid(F.linear(x0[:, :16], self.skip_gates[skip_idx]).float())
                      ).to(x.dtype)                                                  # [T, 1]
                skip_idx += 1
                terms.append(Term(skips.pop(), scalar=resid[i].reshape(1), gate=sg, col=0))
            if i == 0:
                terms += [Term(x, scalar=(resid[0] + x0l[0, 0]).reshape(1)),
                          Term(x02_s, scalar=x0l[0, 1].reshape(1), sink=x02_sink)]
            else:
                terms += [Term(x, scalar=resid[i].reshape(1)), Term(x0_s, scalar=x0l[i, 0].reshape(1), sink=x0_sink),
                          Term(x02_s, scalar=x0l[i, 1].reshape(1), sink=x02_sink)]
            x = lincomb(terms)
            xin, x = fused.rms_norm_fork(x)                  # x's gradients meet inside the norm backward
            x16 = xin[:, :16]
            if direct:
                xin, x16 = cols_tap(xin, 16)                 # gate inputs: their gradient joins the main one in place
            is_long = i in LONG_LAYERS
            if direct:
                qkv = fused.bank_linear(xin, sa[i, 0], w_all[i][:3 * D], [g_all[i][:3 * D]])
            elif not torch.is_grad_enabled():
                qkv = fused.linear_scaled(xin, w_all[i][:3 * D], sa[i, 0])
            else:
                qkv = F.linear(xin, sa[i, 0] * w_all[i][:3 * D])
            ve_t = vgate = None
            if i in VE_LAYERS:
                ve_t = ve[VE_LAYERS[i]]
                vgate = (2 * torch.sigmoid(F.linear(x16, self.value_embed_gate_bank[self._ve_slot[i]]))).contiguous()
            q, k, v = qkv_post(qkv, cos_t, sin_t, ve_t, vgate, None, H, False, is_long, split=True)
            window = sc.ws_long if is_long else sc.ws_short
            y = ops.attention(q, k, v, seqlens, window, self.yarn.attn_scale, max_len, bounds)
            agate = torch.sigmoid(F.linear(x16, self.attn_gate_bank[i])).contiguous()
            y = xsa_gate(y, v, None, agate)
            if direct:
                attn_out = fused.bank_linear(y.reshape(T, D), sa[i, 1], w_all[i][3 * D:], [g_all[i][3 * D:]])
            elif not torch.is_grad_enabled():
                attn_out = fused.linear_scaled(y.reshape(T, D), w_all[i][3 * D:], sa[i, 1])
            else:
                attn_out = F.linear(y.reshape(T, D), sa[i, 1] * w_all[i][3 * D:])
            x = lincomb([Term(x), Term(attn_out)])
            st = self._fp8_state.layer(i) if (self.training and self.use_fp8 and self._fp8_state is not None) else None
            if direct:
                h, x = fused.norm_relu2_mlp(x, self.mlp_bank[i, 0], self.mlp_bank[i, 1], st,
                                            (self.mlp_bank.grad[i, 0], self.mlp_bank.grad[i, 1]), fork=True)
            else:
                h = ops.norm_relu2_mlp(x, self.mlp_bank[i, 0], self.mlp_bank[i, 1], st)
            x = lincomb([Term(x), Term(h)])
            if i in SKIP_IN:
                skips.append(x)
            if i == BACKOUT_LAYER:
                x_backout = x
        x = lincomb([Term(x), Term(x_backout, scalar=(-backout_lambda).reshape(1))])
        x = fused.rms_norm(x)
        a, b, c = self.softcap
        if self.training:
            return ops.softcap_ce(x, self.lm_head.weight, target_seq, sc.mtp_weights, None, None, a, b, c,
                                  grad_scale=self.grad_scale, fp8=self.use_fp8)
        return ops.softcap_ce_eval(x, self.lm_head.weight, target_seq, a, b, c)

    # -- reference key layout ----------------------------------------------------------------------
    def reference_state_dict(self) -> dict:
        L, D, V = self.num_layers, self.model_dim, self.vocab_size
        sd = {"lm_head.weight": self.lm_head.weight.detach().T.contiguous(), "embed.weight": self.embed.weight.detach(),
              "embed2.weight": self.embed2.weight.detach(), "x0_lambdas": self.x0_lambdas.detach(), "scalars": self.scalars.detach(),
              "smear_gate.weight": self.smear_gate.weight.detach()}
        for j in range(5):
            sd[f"value_embeds.{j}.weight"] = self.value_embeds.detach().view(5, V, D)[j]
        for j in range(3):
            sd[f"skip_gates.{j}.weight"] = self.skip_gates.detach()[j]
        w = self.attn_bank.detach()[:4 * L].view(L, 4 * D, D)
        for i in range(L):
            sd[f"blocks.{i}.attn.qkvo_w"] = w[i]
            sd[f"blocks.{i}.attn.attn_gate.weight"] = self.attn_gate_bank.detach()[i]
            if i in self._ve_slot:
                sd[f"blocks.{i}.attn.value_embed_gate.weight"] = self.value_embed_gate_bank.detach()[self._ve_slot[i]]
            sd[f"blocks.{i}.mlp.c_fc"] = self.mlp_bank.detach()[i, 0]
            sd[f"blocks.{i}.mlp.c_proj"] = self.mlp_bank.detach()[i, 1]
        return sd

    @torch.no_grad()
    def load_reference_state_dict(self, sd: dict):
        sd = {(k[len("_orig_mod."):] if k.startswith("_orig_mod.") else k): v for k, v in sd.items()}
        L, D, V = self.num_layers, self.model_dim, self.vocab_size
        self.lm_head.weight.copy_(sd["lm_head.weight"].T)
        for k in ("embed.weight", "embed2.weight", "smear_gate.weight"):
            self.get_parameter(k).copy_(sd[k])
        self.x0_lambdas.copy_(sd["x0_lambdas"])
        self.scalars[:sd["scalars"].numel()].copy_(sd["scalars"][:self.scalars.numel()])
        for j in range(5):
            self.value_embeds.view(5, V, D)[j].copy_(sd[f"value_embeds.{j}.weight"])
        for j in range(3):
            self.skip_gates[j].copy_(sd[f"skip_gates.{j}.weight"])
        w = self.attn_bank[:4 * L].view(L, 4 * D, D)
        for i in range(L):
            w[i].copy_(sd[f"blocks.{i}.attn.qkvo_w"])
            self.attn_gate_bank[i].copy_(sd[f"blocks.{i}.attn.attn_gate.weight"])
            if i in self._ve_slot:
                self.value_embed_gate_bank[self._ve_slot[i]].copy_(sd[f"blocks.{i}.attn.value_embed_gate.weight"])
            self.mlp_bank[i, 0].copy_(sd[f"blocks.{i}.mlp.c_fc"])
            self.mlp_bank[i, 1].copy_(sd[f"blocks.{i}.mlp.c_proj"])
