"""Half-truncated rotary embedding with YaRN window extension.

Behaviour of `train_gpt.py:988-1055`: head_dim/4 frequencies (1/1024)^linspace(0,1), each used
for an interleaved pair of lanes (2j, 2j+1), the second half of the head left un-rotated;
`apply(old, new)` rescales the frequencies by YaRN interpolation (alpha=1, beta=32) and the
softmax scale by 0.2*ln(new/old)+1.  "Paired" tables serve layers whose adjacent heads are
interleaved into one double-length sequence: a 2*head_dim wide row holds the angles of
positions 2t and 2t+1.

Unlike the reference the cos/sin tables are kept in fp32, sized to the longest sequence actually
seen (grown on demand) and cast at use; CUDA kernels take `angular_freq` and compute angles
on the fly.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor


class Yarn:
    def __init__(self, head_dim: int, max_seq_len: int, paired: bool = False, device="cpu"):
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.paired = paired
        self.device = torch.device(device)
        self.reset()

    # ------------------------------------------------------------------
    def reset(self):
        hd = self.head_dim
        f = (1 / 1024) ** torch.linspace(0, 1, steps=hd // 4, dtype=torch.float32, device=self.device)
        f = f.repeat_interleave(2)
        self.angular_freq = torch.cat([f, f.new_zeros(hd // 2)])
        self.attn_scale = 0.1
        self._tables = None
        self._version = getattr(self, "_version", 0) + 1

    def to(self, device):
        self.device = torch.device(device)
        self.angular_freq = self.angular_freq.to(self.device)
        self._tables = None
        return self

    def apply(self, old_window: int, new_window: int, alpha: int = 1, beta: int = 32):
        rotations = old_window * self.angular_freq / (2 * math.pi)
        s = old_window / new_window
        w = torch.clamp((rotations - alpha) / (beta - alpha), 0, 1)
        self.angular_freq = self.angular_freq * (s + w * (1 - s))
        self.attn_scale *= 0.2 * math.log(new_window / old_window) + 1
        self._tables = None
        self._version += 1

    # ------------------------------------------------------------------
    def tables(self, T: int):
        """(cos, sin_signed) of shape [T, head_dim] (or [T, 2*head_dim] when paired); the sin
        table has its odd lanes negated so that rotary(x) = cos*x + sin_signed*pairswap(x)."""
        if self._tables is None or self._tables[0].size(0) < T:
            n = max(T, 1)
            t = torch.arange(n, dtype=torch.float32, device=self.angular_freq.device)
            if not self.paired:
                theta = torch.outer(t, self.angular_freq)
                cos, sin = theta.cos(), theta.sin()
            else:
                th0 = torch.outer(2 * t, self.angular_freq)
                th1 = torch.outer(2 * t + 1, self.angular_freq)
                cos = torch.cat((th0.cos(), th1.cos()), dim=-1)
                sin = torch.cat((th0.sin(), th1.sin()), dim=-1)
            sin = sin.clone()
            sin[..., 1::2] *= -1
            self._tables = (cos.to(torch.bfloat16).float(), sin.to(torch.bfloat16).float())
        return self._tables[0][:T], self._tables[1][:T]

    def rotary(self, x: Tensor) -> Tensor:
        """x: [T, H, W] with W = head_dim (or 2*head_dim when paired)."""
        T = x.size(0)
        cos, sin = self.tables(T)
        cos, sin = cos[:, None, :].to(x.dtype), sin[:, None, :].to(x.dtype)
        x_swap = x.view(*x.shape[:-1], x.shape[-1] // 2, 2).flip(-1).reshape(x.shape)
        return cos * x + sin * x_swap

    def state_dict(self):
        return dict(angular_freq=self.angular_freq.detach().cpu().clone(), attn_scale=float(self.attn_scale))

    def load_state_dict(self, d):
        self.angular_freq = d["angular_freq"].to(self.device, torch.float32)
        self.attn_scale = float(d["attn_scale"])
        self._tables = None
        self._version += 1
