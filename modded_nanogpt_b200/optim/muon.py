"""Plain Muon for the track-3 baseline (`train_gpt_simple.py:157-214`): Nesterov momentum, 12 quintic
Newton-Schulz steps (a, b, c = 2, -1.5, 0.5) on the wide orientation in bf16, update scaled by
sqrt(max(1, rows/cols)), decoupled weight decay.  Matrices are dealt round-robin to the ranks
(largest first); each round ends with an all-gather of the updated matrices."""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def newton_schulz(G: Tensor, steps: int = 12, dtype=torch.bfloat16) -> Tensor:
    X = G.to(dtype)
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    a, b, c = 2.0, -1.5, 0.5
    for _ in range(steps):
        A = X @ X.mT
        X = a * X + (b * A + c * A @ A) @ X
    return X.mT if tall else X


class Muon(torch.optim.Optimizer):
    def __init__(self, params, lr=0.02, weight_decay=0.0, mu=0.95, ns_dtype=torch.bfloat16):
        params = sorted(list(params), key=lambda p: p.size(), reverse=True)
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, mu=mu))
        self.ns_dtype = ns_dtype

    @torch.no_grad()
    def step(self):
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        for group in self.param_groups:
            params = group["params"]
            pad = params + [torch.empty_like(params[-1])] * ((-len(params)) % world)
            for base in range(0, len(params), world):
                if base + rank < len(params):
                    p = params[base + rank]
                    st = self.state[p]
                    if not st:
                        st["momentum"] = torch.zeros_like(p)
                    st["momentum"].lerp_(p.grad, 1 - group["mu"])
                    upd = newton_schulz(p.grad.lerp_(st["momentum"], group["mu"]), dtype=self.ns_dtype).to(p.dtype)
                    upd *= max(1, p.size(-2) / p.size(-1)) ** 0.5
                    p.mul_(1 - group["lr"] * group["weight_decay"])
                    p.add_(upd, alpha=-group["lr"])
                if world > 1:
                    dist.all_gather(pad[base:base + world], pad[base + rank].contiguous())
