"""Forward / backward parity of this framework's track-1 model against the unmodified reference module on
identical weights and one identical batch.

    python baseline/parity.py --tokens 4096 [--out parity.json]

Runs in a process of its own (the reference initialises a process group at import).  The reference module is built
from `baseline/_ref/train_gpt.py` (its definitions executed unchanged, with its own DISABLE_FP8=1 and FlashAttention-2
for the Hopper-only FA3 binary), every parameter gets a small random perturbation so that no zero-initialised branch
hides a wiring difference, and its state_dict is loaded into this framework's `GPT` through `load_model_state`.
The reference evaluates its independent loss path (`train_gpt.py:1689-1692`: bf16 logits, fp32 cross entropy per
token); this framework runs its training kernels with a single prediction weight and no prefix term, which is the
same per-token loss.  Compared: per-token losses, their mean, and the gradients of the large parameters after
`loss.sum().backward()`; then the same again with this framework's FP8 MLP and FP8 head.  Prints one JSON line."""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def make_batch(T: int, vocab: int, bigram_vocab: int, seed: int = 0):
    import torch
    from modded_nanogpt_b200.data.loader import bigram_hash
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab - 1, (T + 1,), generator=g, dtype=torch.int32)
    starts = [0]
    while starts[-1] < T:
        starts.append(starts[-1] + int(torch.randint(40, 900, (1,), generator=g)))
    starts = [s for s in starts if s < T]
    ids[starts] = 50256
    cu = torch.full((128,), T, dtype=torch.int32)
    cu[:len(starts)] = torch.tensor(starts, dtype=torch.int32)
    inputs, targets = ids[:-1].contiguous(), ids[1:].long().contiguous()
    return inputs, targets, cu, bigram_hash(inputs, bigram_vocab)


def rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-20))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--out", default="")
    a = ap.parse_args()
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "train_gpt.py")):
        print(json.dumps({"unavailable": "baseline/_ref is not staged on this machine"}))
        return
    import torch
    from baseline.reference_driver import load_track1_definitions
    ns = load_track1_definitions(ref_dir)
    nn = ns["nn"]
    T = a.tokens
    torch.manual_seed(0)
    ref = ns["GPT"](vocab_size=50257, num_layers=11, num_heads=6, head_dim=128, model_dim=768, max_seq_len=max(T, 8192)).cuda()
    for m in ref.modules():
        if isinstance(m, (nn.Embedding, nn.Linear)):
            m.weight.data = m.weight.data.bfloat16()
    for name in ("ve_gate_bank", "qk_bank", "vo_bank", "mlp_bank", "mudd_w1", "mudd_w2", "mudd_b2", "mudd_gate_w1",
                 "mudd_gate_w2", "mudd_gate_b2"):
        getattr(ref, name).data = getattr(ref, name).data.bfloat16()
    gen = torch.Generator(device="cuda").manual_seed(1)
    with torch.no_grad():
        for n, p in ref.named_parameters():
            scale = 0.02 if p.dim() >= 2 else 0.05
            if n.startswith("lm_head") or n.startswith("embed") or "value_embeds" in n or "bigram" in n:
                scale = 0.01
            p.add_((torch.randn(p.shape, generator=gen, device="cuda") * scale).to(p.dtype))
    ref.prefix_table.fill_(-1)

    from modded_nanogpt_b200.config import track1_model
    from modded_nanogpt_b200.models.gpt import GPT, ForwardScheduleConfig
    from modded_nanogpt_b200.utils.checkpoint import load_model_state
    cfg = track1_model(max(T, 8192))
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}

    def ours(use_fp8: bool):
        m = GPT(cfg, world_size=1, grad_scale=1.0, use_fp8=use_fp8, eval_seq_len=max(T, 8192)).cuda()
        m.cast_params_(torch.bfloat16)
        load_model_state(m, sd, strict=False)
        m.prefix_table.fill_(-1)
        m.train()
        m.quantize_mlp_fp8(bootstrap_down=True)
        return m

    inputs, targets, cu, bg = make_batch(T, 50257, cfg.bigram_vocab_size)
    inputs, targets, cu, bg = inputs.cuda(), targets.cuda(), cu.cuda(), bg.cuda()
    one = torch.tensor([1.0], device="cuda")
    zero = torch.tensor([0.0], device="cuda")
    sc_ref = ns["ForwardScheduleConfig"](mtp_weights=one, prefix_weight=zero, ws_short=5 * 128, ws_long=11 * 128, train_max_seq_len=2048)
    sc_own = ForwardScheduleConfig(one, zero, 5 * 128, 11 * 128, 2048)

    ref.eval()
    loss_ref = ref(inputs, targets, cu, bg, sc_ref).float()
    loss_ref.sum().backward()
    gref = {n: p.grad.detach().float().clone() for n, p in ref.named_parameters() if p.grad is not None}
    out = {"tokens": T, "mean_loss_reference": float(loss_ref.mean())}
    big = ("qk_bank", "vo_bank", "mlp_bank", "lm_head.weight", "embed.weight", "value_embeds", "bigram_embed.weight", "scalars",
           "resid_lambdas", "post_lambdas", "mudd_gate_w1", "mudd_w1", "ve_gate_bank")
    for tag, fp8 in (("bf16", False), ("fp8", True)):
        m = ours(fp8)
        if fp8:
            # activation scales of the FP8 MLP are delayed by one step: one forward to measure them, refresh, then compare
            with torch.no_grad():
                m(inputs, targets, cu, bg, sc_own)
            m.quantize_mlp_fp8(bootstrap_down=True)
            for p in m.parameters():
                p.grad = None
        loss = m(inputs, targets, cu, bg, sc_own).float()
        loss.sum().backward()
        out[f"mean_loss_{tag}"] = float(loss.mean())
        out[f"mean_loss_rel_{tag}"] = abs(float(loss.mean()) - float(loss_ref.mean())) / float(loss_ref.mean())
        out[f"per_token_loss_rel_{tag}"] = rel(loss.detach(), loss_ref.detach())
        own = dict(m.named_parameters())
        grads = {}
        for n in big:
            if n in gref and n in own and own[n].grad is not None:
                g = own[n].grad.float()
                r = gref[n]
                if g.shape != r.shape:                     # bank padding
                    k = min(g.shape[0], r.shape[0])
                    g, r = g[:k], r[:k]
                grads[n] = rel(g, r)
        out[f"grad_rel_{tag}"] = grads
        del m
        torch.cuda.empty_cache()
    line = json.dumps(out)
    print(line, flush=True)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    ns["dist"].destroy_process_group()


if __name__ == "__main__":
    main()
