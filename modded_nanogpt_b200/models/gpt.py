"""The track-1 GPT (and its stripped "plain" topology).

Same parameters, state_dict keys, math and loss as `train_gpt.py:1208-1693`: lm_head stored
transposed and tied to `embed` at init; attention and MLP matrices held in three parameter
banks whose leading dimension is padded to a multiple of the world size; value embeddings and
a signed bigram-hash embedding; smear; a layer without attention that adds a gated skip; MUDD
coefficient MLPs that produce data-dependent residual weights and per-token gates (XSA strength,
attention gates, injection gates, DC mixing weights); softcapped head with multi-token and
prefix-token loss terms.

The wiring is data-driven here: a per-layer plan and gate layouts are derived from
`ModelConfig`, the hot ops go through `ops.functional` (sm_100a kernels on GPU, PyTorch oracle
on CPU), and rotary state lives in `Yarn` objects outside the module tree.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..config import ModelConfig, next_multiple_of_n
from ..ops import functional as ops
from .yarn import Yarn


@dataclass
class ForwardScheduleConfig:
    mtp_weights: Tensor
    prefix_weight: Tensor
    ws_short: int          # tokens
    ws_long: int           # tokens
    train_max_seq_len: int


@dataclass
class LayerPlan:
    index: int
    has_attn: bool
    attn_slot: int         # index into the attention banks, -1 if none
    paired: bool
    long_window: bool
    ve_slot: int           # value-embedding table used, -1 if none
    xsa: bool
    attn_gate: bool
    dc: bool
    cache: bool
    last: bool


class _Weight(nn.Module):
    """Holds one `weight` parameter so state_dict keys read `<name>.weight`."""

    def __init__(self, *shape):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(*shape))


def _kaiming_uniform_(t: Tensor):
    for j in range(t.shape[0]):
        nn.init.kaiming_uniform_(t[j], a=math.sqrt(5))


class GPT(nn.Module):
    def __init__(self, cfg: ModelConfig | None = None, *, world_size: int = 1, grad_scale: float = 1.0,
                 use_fp8: bool = True, eval_seq_len: int | None = None, **ref_kwargs):
        super().__init__()
        if cfg is None:     # reference-style call: GPT(vocab_size=..., num_layers=..., ...)
            cfg = ModelConfig(**ref_kwargs)
        self.cfg = cfg
        self.world_size = world_size
        self.grad_scale = grad_scale
        self.use_fp8 = use_fp8
        # The lm_head + loss path follows `use_fp8` unless set on its own: the reference's training loss quantises
        # to FP8 even with DISABLE_FP8 (`train_gpt.py:1685-1687`), which `fp8_head = True` reproduces.
        self.fp8_head = None
        self.eval_seq_len = eval_seq_len or cfg.max_seq_len
        L, H, Dh, D = cfg.num_layers, cfg.num_heads, cfg.head_dim, cfg.model_dim
        assert H * Dh == D, "num_heads * head_dim must equal model_dim"
        self.num_layers, self.num_heads, self.head_dim, self.model_dim = L, H, Dh, D
        self.vocab_size = V = cfg.padded_vocab
        self.track1 = cfg.topology == "track1"
        if self.track1:
            assert L == 11 and H == 6, "the track-1 gate layouts are defined for 11 layers x 6 heads"

        self.register_buffer("prefix_table", torch.full((V,), -1, dtype=torch.int64), persistent=False)

        self.lm_head = _Weight(D, V)
        nn.init.normal_(self.lm_head.weight, mean=0, std=0.005)
        self.embed = _Weight(V, D)
        with torch.no_grad():
            self.embed.weight.copy_(self.lm_head.weight.T)

        # ---- layer plan --------------------------------------------------------------
        self.plan: list[LayerPlan] = []
        ve_layers = self._ve_layer_map()
        slot = 0
        for i in range(L):
            has_attn = i not in cfg.skip_attn_layers
            self.plan.append(LayerPlan(
                index=i, has_attn=has_attn, attn_slot=slot if has_attn else -1,
                paired=i in cfg.paired_head_layers, long_window=i in cfg.long_window_layers,
                ve_slot=ve_layers.get(i, -1), xsa=i in cfg.xsa_layers, attn_gate=i in cfg.attn_gate_layers,
                dc=i in cfg.dc_layers, cache=i in cfg.cache_layers, last=(i == L - 1)))
            slot += int(has_attn)
        self._num_attn_layers = A = slot

        self.yarn = Yarn(Dh, cfg.max_seq_len)
        self.yarn_paired_head = Yarn(Dh, cfg.max_seq_len, paired=True)

        # ---- banks -------------------------------------------------------------------
        if cfg.num_value_embeds:
            self.value_embeds = nn.Parameter(0.01 * torch.randn(cfg.num_value_embeds * V, D))
            self.ve_gate_bank = nn.Parameter(torch.zeros(cfg.num_value_embeds, H, 12))
        self._num_qk_groups = A * 2 * (H // 2)
        qk_pad = next_multiple_of_n(self._num_qk_groups, n=world_size)
        self.qk_bank = nn.Parameter(torch.empty(qk_pad, Dh * 2, D))
        self.qk_bank.reshape = (qk_pad, Dh * 2, D)
        vo_pad = next_multiple_of_n(A * 2, n=world_size)
        self.vo_bank = nn.Parameter(torch.empty(vo_pad, D, D))
        self.vo_bank.reshape = (vo_pad, D, D)
        bound = (3 ** 0.5) * 0.5 * D ** -0.5
        with torch.no_grad():
            self.qk_bank[:self._num_qk_groups].uniform_(-bound, bound)
            self.qk_bank[self._num_qk_groups:].zero_()
            self.vo_bank[:A * 2].uniform_(-bound, bound)
            self.vo_bank[A * 2:].zero_()

        hid = cfg.mlp_mult * D
        # pad the layer count so that the 2*L matrices split evenly over 1, 2, 4 and 8 ranks
        Lp = L
        while (2 * Lp) % max(world_size, 8 if self.track1 else world_size) != 0:
            Lp += 1
        self._mlp_layers_padded = Lp
        self.mlp_bank = nn.Parameter(torch.empty(Lp, 2, hid, D))
        self.mlp_bank.reshape = (2 * Lp, hid, D)
        with torch.no_grad():
            self.mlp_bank[:, 0].uniform_(-bound, bound)
            self.mlp_bank[:, 1].zero_()
        self.register_buffer("_mlp_down_act_scales", torch.ones(Lp))
        self.register_buffer("_mlp_down_proj_scales", torch.ones(Lp))
        self.register_buffer("_mlp_down_proj_next_scales", torch.ones(Lp))

        # ---- misc --------------------------------------------------------------------
        self.smear_gate = _Weight(1, 12)
        if cfg.bigram_vocab_size:
            self.bigram_embed = _Weight(cfg.bigram_vocab_size, cfg.bigram_dim)
            sign = torch.randn(cfg.bigram_sign_table_rows, cfg.bigram_dim).sign()
            self.register_buffer("bigram_sign_table", sign)
        self.post_lambdas = nn.Parameter(torch.ones(L, 2))
        self.resid_lambdas = nn.Parameter(torch.full((L, 2), 1.1 ** 0.5))
        pad = (-L * 2 - 2) % world_size
        sa = torch.tensor([0.5, 1.0]).repeat(L)
        self.scalars = nn.Parameter(torch.cat([sa, torch.zeros(1), -1.5 * torch.ones(1), torch.ones(pad)]))

        if self.track1:
            self._init_mudd(D)
            self._init_mudd_gate(D)

        for name, p in self.named_parameters():
            p.label = name.replace(".weight", "")
        self._fp8_state = None

    # ----------------------------------------------------------------------------------
    def _ve_layer_map(self) -> dict:
        """Value-embedding tables go to layers 1, 2 and the last three (`train_gpt.py:1543`)."""
        n, L = self.cfg.num_value_embeds, self.cfg.num_layers
        if not n:
            return {}
        assert n == 5 and L >= 6
        return {1: 0, 2: 1, L - 3: 2, L - 2: 3, L - 1: 4}

    def _init_mudd(self, D: int):
        self._mudd_scale = 0.1
        self.mudd_w1 = nn.Parameter(torch.empty(2, 64, D))
        _kaiming_uniform_(self.mudd_w1.data)
        self.mudd_w2 = nn.Parameter(torch.zeros(2, 14, 64))
        b = torch.zeros(2, 14)
        s = self._mudd_scale
        b[0, 6] = b[0, 7] = 2.0 / s                       # per-pair value-embed gate baseline
        b[0, 8], b[0, 9] = 1.1 ** 0.5 / s, 1.0 / s        # resid / post attention lambdas of the last layer
        b[0, 10], b[0, 11] = 0.0, 0.05 / s                # x0 / bigram injection
        b[0, 12], b[0, 13] = 1.1 ** 0.5 / s, 1.0 / s      # resid / post MLP lambdas
        b[1, 1] = -0.5 / s                                # post-loop back-out of cache[7]
        self.mudd_b2 = nn.Parameter(b)

    def _init_mudd_gate(self, D: int):
        """Gate MLP 0 runs on x0 and serves layers before `post_gate_layer`; gate MLP 1 runs on
        the stream entering that layer and serves the rest.  Coefficient packing: XSA strengths
        (H each), attention gates (H each), (x0, bigram) injection pairs, then for the second
        gate the skip gate and DC w1/w2 (`train_gpt.py:1436-1484`)."""
        cfg, H = self.cfg, self.num_heads
        self.post_gate_layer = 4
        self._mudd_gate_scale = nn.Parameter(torch.tensor(0.1))
        layouts = []
        for gid in (0, 1):
            mine = (lambda i: i < self.post_gate_layer) if gid == 0 else (lambda i: i >= self.post_gate_layer)
            lay, off = {"xsa": {}, "attn": {}, "inject": {}}, 0
            for i in cfg.xsa_layers:
                if mine(i):
                    lay["xsa"][i] = off
                    off += H
            for i in cfg.attn_gate_layers:
                if mine(i):
                    lay["attn"][i] = off
                    off += H
            for pl in self.plan:
                if pl.has_attn and not pl.last and mine(pl.index):
                    lay["inject"][pl.index] = off
                    off += 2
            if gid == 1:
                lay["skip"] = off
                off += 1
                lay["dc"] = off
                off += 2 * H
            lay["n"] = off
            layouts.append(lay)
        self.gate_layouts = layouts
        assert layouts[0]["n"] == 26 and layouts[1]["n"] == 41
        nmax = max(l["n"] for l in layouts)
        self.mudd_gate_w1 = nn.Parameter(torch.empty(2, 64, D))
        _kaiming_uniform_(self.mudd_gate_w1.data)
        self.mudd_gate_w2 = nn.Parameter(torch.zeros(2, nmax, 64))
        b, s = torch.zeros(2, nmax), 0.1
        for gid, lay in enumerate(layouts):
            for off in lay["attn"].values():
                b[gid, off:off + H] = 0.25 / s
            for off in lay["inject"].values():
                b[gid, off + 1] = 0.05 / s
        b[1, layouts[1]["skip"]] = 0.5 / s
        b[1, layouts[1]["dc"]:layouts[1]["dc"] + H] = 1.0 / s
        self.mudd_gate_b2 = nn.Parameter(b)

    # ----------------------------------------------------------------------------------
    def cast_params_(self, dtype=torch.bfloat16):
        """Embeddings, banks, gate and MUDD weights to bf16; `scalars`, the lambda tables and
        `_mudd_gate_scale` stay fp32 (`train_gpt.py:2242-2254`)."""
        keep = {"scalars", "post_lambdas", "resid_lambdas", "_mudd_gate_scale"}
        for name, p in self.named_parameters():
            if p.label not in keep:
                p.data = p.data.to(dtype)
        if hasattr(self, "bigram_sign_table"):
            self.bigram_sign_table = self.bigram_sign_table.to(dtype)
        return self

    def _apply(self, fn, *a, **k):
        out = super()._apply(fn, *a, **k)
        dev = self.lm_head.weight.device
        self.yarn.to(dev)
        self.yarn_paired_head.to(dev)
        return out

    def attn_layer_weights(self):
        """Per attention layer the (4*D, D) stack [Wq; Wk; Wv; Wo] viewed out of the banks."""
        A, D = self._num_attn_layers, self.model_dim
        qk = self.qk_bank[:self._num_qk_groups].view(A, 2 * D, D)
        vo = self.vo_bank[:A * 2].view(A, 2 * D, D)
        return qk, vo

    def qkv_weights(self) -> Tensor:
        """[A, 3*D, D]: the QKV projection weight of every attention layer as one contiguous matrix, copied out of
        `qk_bank` and `vo_bank` into a persistent buffer (two strided copies per call, 35 MB at track-1 size), so
        that the projection and its input gradient are one GEMM each."""
        A, D = self._num_attn_layers, self.model_dim
        qk, vo = self.attn_layer_weights()
        buf = getattr(self, "_qkv_cat", None)
        if buf is None or buf.device != qk.device or buf.dtype != qk.dtype:
            buf = self._qkv_cat = torch.empty(A, 3 * D, D, dtype=qk.dtype, device=qk.device)
        with torch.no_grad():
            buf[:, :2 * D].copy_(qk)
            buf[:, 2 * D:].copy_(vo[:, :D])
        return buf

    # ----------------------------------------------------------------------------------
    # FP8 MLP weight copies (row-scaled e4m3), refreshed after every optimizer step
    @property
    def head_fp8(self) -> bool:
        return self.use_fp8 if self.fp8_head is None else bool(self.fp8_head)

    def quantize_mlp_fp8(self, bootstrap_down: bool = False):
        """Refresh the e4m3 copies of the MLP weights (`train_gpt.py:1403-1434`).  This build
        scales each weight row separately (one scale per 768- or 3072-element row, "1xK block
        scaling") instead of per tensor; the per-layer delayed-scaling buffers of the reference
        remain in the state_dict and track the per-layer maxima."""
        if not (self.use_fp8 and self.mlp_bank.is_cuda):
            return
        from ..ops import fused

        def refresh(bootstrap):
            with torch.no_grad():
                self._fp8_state = fused.quantize_mlp_weights(self.mlp_bank, self._fp8_state,
                                                             self._mlp_down_proj_scales, self._mlp_down_proj_next_scales,
                                                             bootstrap)

        # The steady-state refresh is ~70 tiny launches.  With MNG_FP8_GRAPH=1 it is replayed as one CUDA graph once the
        # state exists and the call has run eagerly twice (every tensor it touches is persistent; a changed bank
        # address or state object drops the graph).  Measured gain: 0.47 -> 0.40 ms per step, so it is off by default.
        import os
        if bootstrap_down or self._fp8_state is None or os.environ.get("MNG_FP8_GRAPH", "0") != "1":
            return refresh(bootstrap_down)
        key = (self.mlp_bank.data_ptr(), id(self._fp8_state), self._mlp_down_proj_scales.data_ptr())
        ent = getattr(self, "_fp8_graph", None)
        if ent is None or ent["key"] != key:
            ent = self._fp8_graph = dict(key=key, runs=0, graph=None)
        if ent["graph"] is None:
            if ent["runs"] < 2:
                ent["runs"] += 1
                return refresh(False)
            g = torch.cuda.CUDAGraph()
            torch.cuda.synchronize()
            with torch.cuda.graph(g):
                refresh(False)
            ent["graph"] = g
        ent["graph"].replay()

    # ----------------------------------------------------------------------------------
    def _gate_mlp(self, x: Tensor, gid: int) -> Tensor:
        n = self.gate_layouts[gid]["n"]
        w1, w2, b2 = self.mudd_gate_w1[gid], self.mudd_gate_w2[gid, :n], self.mudd_gate_b2[gid, :n]
        if ops.use_kernel("gate_mlp", x):
            from ..ops import fused
            if fused.gate_mlp_supported(x, w1, w2):
                return fused.gate_mlp(x, w1, w2, b2, self._mudd_gate_scale)
        h = F.gelu(F.linear(x, w1.type_as(x)))
        out = F.linear(h, w2.type_as(x)) + b2.type_as(x)
        return out * self._mudd_gate_scale.type_as(x)

    def _mudd_raw(self, x: Tensor, mid: int, n: int) -> Tensor:
        w1, w2, b2 = self.mudd_w1[mid], self.mudd_w2[mid, :n], self.mudd_b2[mid, :n]
        if ops.use_kernel("gate_mlp", x):
            from ..ops import fused
            if fused.gate_mlp_supported(x, w1, w2):
                return fused.gate_mlp(x, w1, w2, b2, self._mudd_scale)
        h = F.gelu(F.linear(x, w1.type_as(x)))
        return (F.linear(h, w2.type_as(x)) + b2.type_as(x)) * self._mudd_scale

    def _mudd(self, x: Tensor, mid: int, n: int):
        return self._mudd_raw(x, mid, n).split(1, dim=-1)

    def _attention(self, pl: LayerPlan, x: Tensor, w_qkvo: Tensor, sa_lambdas: Tensor, seqlens: Tensor,
                   window: int, max_len: int, aux_v, xsa_alpha, attn_gate, dc_w):
        """x: [T, D] normed input.  Returns the O-projected attention output [T, D]."""
        T, D, H, Dh = x.size(0), self.model_dim, self.num_heads, self.head_dim
        qkv = F.linear(x, sa_lambdas[0] * w_qkvo[:3 * D].type_as(x)).view(T, 3 * H, Dh)
        q, k, v = qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:]
        q, k = ops.rms_norm(q), ops.rms_norm(k)
        yarn = self.yarn_paired_head if pl.paired else self.yarn
        if not pl.paired:
            q, k = yarn.rotary(q), yarn.rotary(k)
            if pl.long_window:      # partial key offset: stationary half of k comes from the previous token
                k = torch.cat([k[:, :, :Dh // 2],
                               torch.cat([k[:1, :, Dh // 2:], k[:-1, :, Dh // 2:]], dim=0)], dim=-1)
            if aux_v is not None:
                v = v + aux_v.view_as(v)
            y = ops.attention(q.contiguous(), k.contiguous(), v.contiguous(), seqlens, window, yarn.attn_scale, max_len)
            if dc_w is not None:
                w1 = F.rms_norm(dc_w[0].float(), (H,), eps=1e-6).type_as(x)
                y = ops.dc_correction(y, q, k, v, w1.contiguous(), dc_w[1].type_as(x).contiguous(), seqlens,
                                      yarn.attn_scale, self.cfg.dc_window)
            if xsa_alpha is not None:
                dot = (y * v).sum(-1, keepdim=True)
                den = v.square().sum(-1, keepdim=True).clamp_min(1e-8)
                y = y - torch.tanh(xsa_alpha).type_as(y).view(T, H, 1) * (dot / den) * v
        else:
            # Heads (2p, 2p+1) share a 2*Dh-wide rotary row (angles of positions 2t | 2t+1); the
            # flat [T, H*Dh] buffer is then read as a 2T-long sequence of H/2 heads.
            q = yarn.rotary(q.reshape(T, H // 2, 2 * Dh)).reshape(2 * T, H // 2, Dh)
            k = yarn.rotary(k.reshape(T, H // 2, 2 * Dh)).reshape(2 * T, H // 2, Dh)
            v = v.reshape(2 * T, H // 2, Dh)
            if aux_v is not None:
                v = v + aux_v.view_as(v)
            y = ops.attention(q, k, v.contiguous(), 2 * seqlens, window, yarn.attn_scale, 2 * max_len)
            y = y.view(T, H, Dh)
        if attn_gate is not None:
            y = y * attn_gate.type_as(y).view(T, H, 1)
        y = y.reshape(T, D)
        return F.linear(y, sa_lambdas[1] * w_qkvo[3 * D:].type_as(y))

    def _mlp(self, i: int, x: Tensor, training_fp8: bool) -> Tensor:
        w_fc, w_proj = self.mlp_bank[i, 0], self.mlp_bank[i, 1]
        state = None
        if training_fp8 and self._fp8_state is not None:
            state = self._fp8_state.layer(i)
        return ops.norm_relu2_mlp(x, w_fc, w_proj, state)

    # ----------------------------------------------------------------------------------
    def forward(self, input_seq: Tensor, target_seq: Tensor, seqlens: Tensor, bigram_input_seq: Tensor,
                schedule_cfg: ForwardScheduleConfig) -> Tensor:
        assert input_seq.ndim == 1
        if input_seq.is_cuda:
            from .gpt_fused import forward_fused, fused_supported
            if fused_supported(self, input_seq):
                return forward_fused(self, input_seq, target_seq, seqlens, bigram_input_seq, schedule_cfg)
        cfg, L, H, Dh, D, V = self.cfg, self.num_layers, self.num_heads, self.head_dim, self.model_dim, self.vocab_size
        T = input_seq.size(0)
        ws = {False: schedule_cfg.ws_short, True: schedule_cfg.ws_long}
        max_len = schedule_cfg.train_max_seq_len if self.training else self.eval_seq_len
        training_fp8 = self.training and self.use_fp8

        sa_lambdas = self.scalars[:2 * L].view(L, 2)
        smear_lambda, skip_lambda = self.scalars[2 * L], self.scalars[2 * L + 1]
        qk_all, vo_all = self.attn_layer_weights()

        ids = input_seq.long()
        x = F.embedding(ids, self.embed.weight)
        adt = x.dtype
        resid = self.resid_lambdas.to(adt)
        post = self.post_lambdas.to(adt)

        x0_bigram = None
        if cfg.bigram_vocab_size:
            sign_idx = torch.zeros_like(ids)
            sign_idx[1:] = (ids[:-1] ^ ids[1:]) % self.bigram_sign_table.shape[0]
            x0_bigram = F.embedding(bigram_input_seq.long(), self.bigram_embed.weight) * self.bigram_sign_table[sign_idx].to(adt)
        ve = None
        if cfg.num_value_embeds:
            ve = self.value_embeds.view(cfg.num_value_embeds, V, D)[:, ids]

        # smear the previous token's embedding forward by one position
        g = smear_lambda * torch.sigmoid(F.linear(x[1:, :12], self.smear_gate.weight.type_as(x)))
        x = torch.cat([x[:1], x[1:] + g * x[:-1]])
        x = x0 = ops.rms_norm(x)

        def add_bigram(x, coef):
            if x0_bigram is None:
                return x
            if cfg.bigram_dim == D:
                return x + x0_bigram * coef
            return torch.cat([x[:, :cfg.bigram_dim] + x0_bigram * coef, x[:, cfg.bigram_dim:]], dim=-1)

        xsa, agate, x0g, bgg, dcw, skip_gate = {}, {}, {}, {}, {}, None
        if self.track1:
            pre = self._gate_mlp(x0, 0)
            lay = self.gate_layouts[0]
            for i, o in lay["xsa"].items():
                xsa[i] = pre[:, o:o + H]
            for i, o in lay["attn"].items():
                agate[i] = pre[:, o:o + H]
            for i, o in lay["inject"].items():
                x0g[i], bgg[i] = pre[:, o:o + 1], pre[:, o + 1:o + 2]
            x = add_bigram(x0, bgg[0])
        cache = {0: x}

        for pl in self.plan:
            i, mu = pl.index, None
            if self.track1 and i == self.post_gate_layer:
                pg = self._gate_mlp(x, 1)
                lay = self.gate_layouts[1]
                for j, o in lay["xsa"].items():
                    xsa[j] = pg[:, o:o + H]
                for j, o in lay["attn"].items():
                    agate[j] = pg[:, o:o + H]
                for j, o in lay["inject"].items():
                    x0g[j], bgg[j] = pg[:, o:o + 1], pg[:, o + 1:o + 2]
                skip_gate = pg[:, lay["skip"]:lay["skip"] + 1]
                for j in cfg.dc_layers:
                    dcw[j] = (pg[:, lay["dc"]:lay["dc"] + H], pg[:, lay["dc"] + H:lay["dc"] + 2 * H])

            if not pl.has_attn:
                x = x + (torch.sigmoid(skip_lambda) * skip_gate) * cache[3]
            else:
                w_qkvo = torch.cat([qk_all[pl.attn_slot], vo_all[pl.attn_slot]], dim=0)
                attn_in = ops.rms_norm(cache[7] if (self.track1 and 7 in cache) else x)
                aux_v = None
                if self.track1 and pl.last:
                    cache[9] = x
                    mu = self._mudd(x, 0, 14)
                    v_mudd = mu[0] * cache[0] + mu[1] * cache[7] + mu[2] * x
                    x = (1 + mu[5]) * x + mu[3] * cache[0] + mu[4] * cache[7]
                    ve_gate = torch.cat([mu[6], mu[7]], dim=-1).repeat_interleave(H // 2, dim=-1).unsqueeze(-1)
                    aux_v = (ve_gate * ve[pl.ve_slot].view(T, H, Dh)).view(T, D) + v_mudd
                elif pl.ve_slot >= 0:
                    gate_in = torch.cat([attn_in[:, :6], ve[pl.ve_slot][:, :6]], dim=-1)
                    vg = 2 * torch.sigmoid(F.linear(gate_in, self.ve_gate_bank[pl.ve_slot].type_as(x))).view(T, H, 1)
                    aux_v = (vg * ve[pl.ve_slot].view(T, H, Dh)).view(T, D)
                attn_out = self._attention(
                    pl, attn_in, w_qkvo, sa_lambdas[i], seqlens, ws[pl.long_window], max_len, aux_v,
                    xsa.get(i) if pl.xsa else None, agate.get(i) if pl.attn_gate else None,
                    dcw.get(i) if (pl.dc and not pl.paired) else None)
                if mu is not None:
                    x = add_bigram(mu[8] * x + mu[9] * attn_out + mu[10] * cache[0], mu[11])
                elif self.track1:
                    x = resid[i, 0] * x + post[i, 0] * attn_out + x0 * x0g[i]
                    if i != 0:
                        x = add_bigram(x, bgg[i])
                else:
                    x = resid[i, 0] * x + post[i, 0] * attn_out

            h = self._mlp(i, x, training_fp8)
            if mu is not None:
                x = mu[12] * x + mu[13] * h
            else:
                x = resid[i, 1] * x + post[i, 1] * h
            if pl.cache:
                cache[i] = x

        if self.track1:
            mu = self._mudd(x, 1, 5)
            x = x + mu[0] * cache[0] + mu[1] * cache[7] + mu[2] * cache[9] + mu[3] * ve[0].to(adt) + mu[4] * cache[3]
        x = ops.rms_norm(x)

        if self.training:
            prefix_targets = self.prefix_table[target_seq]
            return ops.softcap_ce(x, self.lm_head.weight, target_seq, schedule_cfg.mtp_weights, prefix_targets,
                                  schedule_cfg.prefix_weight, cfg.softcap_a, cfg.softcap_b, cfg.softcap_c,
                                  grad_scale=self.grad_scale, fp8=self.head_fp8)
        return ops.softcap_ce_eval(x, self.lm_head.weight, target_seq, cfg.softcap_a, cfg.softcap_b, cfg.softcap_c)
