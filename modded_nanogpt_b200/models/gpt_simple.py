"""Track-3 baseline model (`records/track_3_optimization/train_gpt_simple.py:56-150`): plain GPT with
learned RMSNorm gains, biased linears, split-half half-truncated rotary, causal attention over fixed
1024-token rows (scale 0.12), ReLU^2 MLP and an ISRU logit cap 15*z/sqrt(z^2+225); the loss is the sum
of token cross-entropies.  Track 3 counts optimizer steps, not wallclock, so this stays on stock ops."""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn


class RMSNormGain(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.gains = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return F.rms_norm(x, (x.size(-1),), weight=self.gains.type_as(x))


class CastLinear(nn.Linear):
    def __init__(self, i, o):
        super().__init__(i, o, bias=True)

    def forward(self, x):
        return F.linear(x, self.weight.type_as(x), self.bias.type_as(x))


def rotary_split(x: Tensor) -> Tensor:
    """x [B,T,H,D]: dims d < D/4 rotate with d + D/2, the remaining quarter pairs stay put."""
    D = x.size(-1)
    freq = (1 / 1024) ** torch.linspace(0, 1, steps=D // 4, dtype=torch.float32, device=x.device)
    freq = torch.cat([freq, freq.new_zeros(D // 4)])
    theta = torch.outer(torch.arange(x.size(1), dtype=torch.float32, device=x.device), freq)[None, :, None, :]
    cos, sin = theta.cos(), theta.sin()
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat((x1 * cos + x2 * sin, x2 * cos - x1 * sin), 3).type_as(x)


class Attention(nn.Module):
    def __init__(self, dim, head_dim=128):
        super().__init__()
        self.h, self.hd = dim // head_dim, head_dim
        self.q, self.k, self.v = CastLinear(dim, dim), CastLinear(dim, dim), CastLinear(dim, dim)
        self.proj = CastLinear(dim, dim)

    def forward(self, x):
        B, T, _ = x.shape
        q, k, v = (f(x).view(B, T, self.h, self.hd) for f in (self.q, self.k, self.v))
        q, k = rotary_split(F.rms_norm(q, (self.hd,))), rotary_split(F.rms_norm(k, (self.hd,)))
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=0.12, is_causal=True)
        return self.proj(y.transpose(1, 2).reshape(B, T, -1))


class Block(nn.Module):
    def __init__(self, dim, head_dim=128):
        super().__init__()
        self.attn = Attention(dim, head_dim)
        self.mlp_fc, self.mlp_proj = CastLinear(dim, 4 * dim), CastLinear(4 * dim, dim)
        self.norm1, self.norm2 = RMSNormGain(dim), RMSNormGain(dim)

    def forward(self, x):
        x = x + self.attn(self.norm1(x))
        return x + self.mlp_proj(self.mlp_fc(self.norm2(x)).relu().square())


class GPTSimple(nn.Module):
    def __init__(self, vocab_size=50304, num_layers=12, model_dim=768, head_dim=128):
        super().__init__()
        self.embed = nn.Embedding(vocab_size, model_dim)
        self.blocks = nn.ModuleList([Block(model_dim, head_dim) for _ in range(num_layers)])
        self.proj = CastLinear(model_dim, vocab_size)
        self.norm1, self.norm2 = RMSNormGain(model_dim), RMSNormGain(model_dim)

    @torch.no_grad()
    def reset_parameters(self):
        """`train_gpt_simple.py:268-283`: projections zero, embedding N(0,1), other matrices N(0, 0.33/fan_in)."""
        for name, p in self.named_parameters():
            if name.endswith("weight"):
                if "proj" in name:
                    p.zero_()
                elif "embed" in name:
                    p.normal_()
                else:
                    p.normal_(std=0.33 ** 0.5 / p.size(-1) ** 0.5)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)

    def forward(self, inputs: Tensor, targets: Tensor) -> Tensor:
        x = self.norm1(self.embed(inputs))
        for b in self.blocks:
            x = b(x)
        z = self.proj(self.norm2(x)).float()
        z = 15 * z * (z.square() + 225).rsqrt()
        return F.cross_entropy(z.view(targets.numel(), -1), targets.view(-1), reduction="sum")
