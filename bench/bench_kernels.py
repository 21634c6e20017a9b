"""Micro-benchmarks of the hand-written kernels, one case per invocation (CUDA-event timing after warm-up).

    python bench/bench_kernels.py --list
    python bench/bench_kernels.py --case gemm_bf16_o --rows 49152 --bn 256 --iters 10

Every case works on operands larger than the L2 cache at the default --rows.  The same command line
(with a small --iters) is what the committed profiler summaries under profiles/ were captured from."""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch

BF, F8, F8B = torch.bfloat16, torch.float8_e4m3fn, torch.float8_e5m2
V, D, H = 50304, 768, 3072


def build_case(name, T, bn, fused):
    dev = "cuda"
    r = lambda *s: torch.randn(*s, device=dev)
    fl = 2 * T * D * H
    if name == "gemm_bf16_up":          # [T,768] x [3072,768]^T
        a, b = r(T, D).to(BF), r(H, D).to(BF)
        return (lambda: fused.gemm(a, b, bn=bn)), fl, T * H * 2
    if name == "gemm_bf16_dpre":        # same product, epilogue 2*acc*sqrt(post) reading the saved activations
        a, b, post = r(T, D).to(BF), r(H, D).to(BF), r(T, H).abs().to(BF)
        return (lambda: fused.gemm(a, b, epilogue=fused.EPI_DPRE, cin=post, bn=bn)), fl, T * H * 4
    if name == "gemm_bf16_down":        # [T,3072] x [768,3072]^T
        a, b = r(T, H).to(BF), r(D, H).to(BF)
        return (lambda: fused.gemm(a, b, bn=bn)), fl, T * D * 2
    if name == "gemm_bf16_dw":          # [T,3072]^T x [T,768] -> [3072,768] fp32, both operands MN-major
        a, b = r(T, H).to(BF), r(T, D).to(BF)
        return (lambda: fused.gemm(a, b, a_mn=True, b_mn=True, bn=bn, out_dtype=torch.float32)), fl, H * D * 4
    if name == "gemm_fp8_relu2":        # fp8 up projection with relu^2, bf16 + e4m3 outputs and running max
        a, b = r(T, D).to(F8), r(H, D).to(F8)
        rs, cs = torch.ones(T, device=dev), torch.ones(H, device=dev)
        act, amax = torch.tensor([0.02], device=dev), torch.zeros(1, dtype=torch.int32, device=dev)
        o, o8 = torch.empty(T, H, dtype=BF, device=dev), torch.empty(T, H, dtype=F8, device=dev)
        return (lambda: fused.gemm(a, b, out=o, epilogue=fused.EPI_RELU2, row_scale=rs, col_scale=cs, out8=o8,
                                   act_scale=act, amax_bits=amax, bn=bn)), fl, T * H * 3
    if name == "gemm_fp8_down":
        a, b = r(T, H).to(F8), r(D, H).to(F8)
        return (lambda: fused.gemm(a, b, bn=bn)), fl, T * D * 2
    if name == "gemm_bf16_qkv":
        a, b = r(T, D).to(BF), r(3 * D, D).to(BF)
        return (lambda: fused.gemm(a, b, bn=bn)), 2 * T * D * 3 * D, T * 3 * D * 2
    if name == "gemm_bf16_o":
        a, b = r(T, D).to(BF), r(D, D).to(BF)
        return (lambda: fused.gemm(a, b, bn=bn)), 2 * T * D * D, T * D * 2
    if name == "gemm_bf16_o_null":      # same product, accumulators drained but not stored (load + MMA pipeline only)
        a, b = r(T, D).to(BF), r(D, D).to(BF)
        o = torch.empty(T, D, dtype=BF, device=dev)
        return (lambda: fused.gemm(a, b, out=o, bn=bn, epilogue=3)), 2 * T * D * D, 0
    if name == "gemm_bf16_up_null":
        a, b = r(T, D).to(BF), r(H, D).to(BF)
        o = torch.empty(T, H, dtype=BF, device=dev)
        return (lambda: fused.gemm(a, b, out=o, bn=bn, epilogue=3)), fl, 0
    if name == "gemm_fp8_logits":       # [T,768] x [768,V] (B MN-major) -> bf16 logits
        a, b = r(T, D).to(F8), r(D, V).to(F8)
        o = torch.empty(T, V, dtype=BF, device=dev)
        return (lambda: fused.gemm(a, b, b_mn=True, out=o, bn=bn)), 2 * T * D * V, T * V * 2
    if name == "gemm_fp8_logits_kk":    # same product with the weight stored [V, 768] (K-major B)
        a, b = r(T, D).to(F8), r(V, D).to(F8)
        o = torch.empty(T, V, dtype=BF, device=dev)
        return (lambda: fused.gemm(a, b, out=o, bn=bn)), 2 * T * D * V, T * V * 2
    if name == "gemm_fp8_lmhead_dw_kmajor_a":   # dW with x stored transposed [768, T] (K-major A), dl as is (MN-major B)
        a, b = r(D, T).to(F8), torch.randn(T, V, device=dev, dtype=BF).to(F8B)
        return (lambda: fused.gemm(a, b, b_mn=True, bn=bn)), 2 * T * D * V, D * V * 2
    if name == "gemm_fp8_lmhead_dx":    # e5m2 [T,V] x e4m3 [768,V]^T
        a, b = torch.randn(T, V, device=dev, dtype=BF).to(F8B), r(D, V).to(F8)
        return (lambda: fused.gemm(a, b, bn=bn)), 2 * T * D * V, T * D * 2
    if name == "gemm_fp8_lmhead_dw":    # e4m3 [T,768]^T x e5m2 [T,V] -> fp32 [768,V]
        a, b = r(T, D).to(F8), torch.randn(T, V, device=dev, dtype=BF).to(F8B)
        o = torch.empty(D, V, dtype=torch.float32, device=dev)
        return (lambda: fused.gemm(a, b, a_mn=True, b_mn=True, out=o, bn=bn)), 2 * T * D * V, D * V * 4
    if name in ("softcap_ce_e5m2", "softcap_ce_bf16"):
        from modded_nanogpt_b200.ops import native
        lib = native.lib()
        e5 = name.endswith("e5m2")
        logits = torch.randn(T, V, device=dev, dtype=BF) * 3
        tg, pt = torch.randint(0, V, (T,), device=dev), torch.randint(-1, V, (T,), device=dev)
        w, pw = torch.tensor([1.0, 0.5, 0.25], device=dev), torch.tensor([0.3], device=dev)
        return (lambda: lib.softcap_ce(logits, tg, w, pt, pw, e5, 23.0, 5.0, 7.5, 1.0)), 0, T * V * (3 if e5 else 4)
    if name == "lmhead_ce_fwdbwd":      # normed x [T,768] -> fp8 lm_head -> soft-capped CE with MTP weights -> dx, dW
        x = (r(T, D) * 0.5).to(BF).requires_grad_(True)
        w = (r(D, V) * 0.02).to(BF).requires_grad_(True)
        tg = torch.randint(0, V, (T,), device=dev)
        mtp, pw = torch.tensor([1.0, 0.5, 0.25], device=dev), torch.tensor([0.1], device=dev)
        pt = torch.randint(-1, V, (T,), device=dev)

        def run():
            x.grad = w.grad = None
            fused.softcap_ce(x, w, tg, mtp, pt, pw, 23.0, 5.0, 7.5, grad_scale=1.0, fp8=True).sum().backward()
        return run, 3 * 2 * T * D * V, T * V * 3
    if name in ("qkvproj_fused", "qkvproj_unfused"):   # QKV projection + QK norm + rotary + key offset + value add, forward + backward
        from modded_nanogpt_b200.ops.glue import qkv_post
        Hh = 6
        x = r(T, D).to(BF).requires_grad_(True)
        w = (r(3 * D, D) * D ** -0.5).to(BF)
        lam = torch.tensor(0.8, device=dev, requires_grad=True)
        t = torch.arange(T, device=dev, dtype=torch.float32)
        freq = (1 / 1024) ** torch.linspace(0, 1, 32, device=dev)
        cos, sin = torch.outer(t, freq).cos().contiguous(), torch.outer(t, freq).sin().contiguous()
        ve = r(T, D).to(BF).requires_grad_(True)
        vg = torch.rand(T, Hh, device=dev).to(BF).requires_grad_(True)
        gv = [torch.zeros(2 * D, D, dtype=BF, device=dev), torch.zeros(D, D, dtype=BF, device=dev)]
        gs = [r(T, Hh, 128).to(BF) for _ in range(3)]

        def run():
            x.grad = lam.grad = ve.grad = vg.grad = None
            if name == "qkvproj_fused":
                q, k, v = fused.qkv_proj(x, lam, w, gv, cos, sin, ve, vg, Hh, False, True)
            else:
                q, k, v = qkv_post(fused.bank_linear(x, lam, w, gv), cos, sin, ve, vg, None, Hh, False, True)
            torch.autograd.backward([q, k, v], gs)
        return run, 3 * 2 * T * D * 3 * D, T * 3 * D * 2
    if name in ("mlpmix_fused", "mlpmix_unfused"):     # a x + b relu(norm(x) W1^T)^2 W2 with FP8 forward, forward + backward
        from modded_nanogpt_b200.ops.glue import Term, lincomb
        bank = torch.empty(1, 2, H, D, device=dev)
        bank[0, 0].uniform_(-1, 1).mul_(3 ** 0.5 * 0.5 * D ** -0.5)
        bank[0, 1].normal_(0, 0.02)
        bank = bank.to(BF)
        x = r(T, D).to(BF).requires_grad_(True)
        g = (r(T, D) * 0.05).to(BF)
        st = fused.quantize_mlp_weights(bank, None, torch.ones(1, device=dev), torch.ones(1, device=dev), True)
        st.act_scale.fill_(0.25)
        st = st.layer(0)
        a_ = torch.tensor(1.05, device=dev, requires_grad=True)
        b_ = torch.tensor(0.8, device=dev, requires_grad=True)
        gv = (torch.zeros(H, D, dtype=BF, device=dev), torch.zeros(H, D, dtype=BF, device=dev))

        def run():
            x.grad = a_.grad = b_.grad = None
            if name == "mlpmix_fused":
                y = fused.norm_relu2_mlp_mix(x, bank[0, 0], bank[0, 1], a_, b_, st, gv)
            else:
                h, xr = fused.norm_relu2_mlp(x, bank[0, 0], bank[0, 1], st, gv, fork=True)
                y = lincomb([Term(xr, scalar=a_), Term(h, scalar=b_)])
            y.backward(g)
        return run, 3 * 2 * 2 * T * D * H, T * D * 2
    if name.startswith("proj_"):            # proj_{qkv|o}_{ours|lib}: bank-backed projection, forward + backward
        _, which, impl = name.split("_")
        N = 3 * D if which == "qkv" else D
        x = r(T, D).to(BF).requires_grad_(True)
        w = (r(N, D) * 0.03).to(BF)
        lam = torch.tensor(0.5, device=dev, requires_grad=True)
        gv = [torch.zeros(N, D, dtype=BF, device=dev)]
        dy = r(T, N).to(BF)

        def ours():
            x.grad = lam.grad = None
            fused.bank_linear(x, lam, w, gv).backward(dy)

        def lib():                                                              # what ran before: library GEMMs + eager glue
            x.grad = lam.grad = None
            we = (lam.detach() * w)
            y = x.detach() @ we.t()
            dx = dy @ we
            dw = dy.t() @ x.detach()
            dlam = (dw.float() * w.float()).sum()
            gv[0].addcmul_(dw, lam.detach())
            return y, dx, dlam
        return (ours if impl == "ours" else lib), 3 * 2 * T * D * N, T * (N + D) * 2
    if name.startswith("gatemlp_"):         # gatemlp_{ours|lib}: (T,768) -> 64 -> 41 gate MLP, forward + backward
        impl = name.split("_")[1]
        import torch.nn.functional as F
        x = r(T, D).to(BF).requires_grad_(True)
        w1 = (r(64, D) * D ** -0.5).to(BF).requires_grad_(True)
        w2 = (r(41, 64) * 0.1).to(BF).requires_grad_(True)
        b2 = r(41).to(BF).requires_grad_(True)
        sc = torch.tensor(0.1, device=dev, requires_grad=True)
        dout = r(T, 41).to(BF)

        def run():
            for t in (x, w1, w2, b2, sc):
                t.grad = None
            if impl == "ours":
                out = fused.gate_mlp(x, w1, w2, b2, sc)
            else:
                out = (F.linear(F.gelu(F.linear(x, w1)), w2) + b2) * sc.to(BF)
            out.backward(dout)
        return run, 3 * 2 * T * D * 64, T * D * 2
    if name == "adam_bf16":             # sharded Adam kernel on one rank: T * 1024 bf16 parameters, fp32 moments
        from modded_nanogpt_b200.ops import native
        n = T * 1024
        pw = (r(n) * 0.1).to(BF)
        gw = (r(n) * 0.01).to(BF)
        m_, v_ = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        C = native.lib()
        return (lambda: C.adam([gw.data_ptr()], [pw.data_ptr()], 0, 0, m_, v_, n, False, 0.9, 0.99, 1e-10, 3e-3, 2e-4, 1.0, None, 0,
                               0, 0)), 0, n * 22
    if name in ("dc_ours", "dc_ref"):       # DC correction of layer 10 (window 112, 6 heads), forward + backward, packed documents
        g = torch.Generator(device=dev).manual_seed(0)
        q, k, v, base = (torch.randn(T, 6, 128, device=dev, generator=g).to(BF).requires_grad_(True) for _ in range(4))
        w1 = torch.randn(T, 6, device=dev, generator=g).to(BF).requires_grad_(True)
        w2 = (torch.randn(T, 6, device=dev, generator=g) * 0.1).to(BF).requires_grad_(True)
        lens = torch.exp(torch.randn(4 * T // 600, generator=torch.Generator().manual_seed(0)) + 6.4).clamp(2, 2048).long()
        starts = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)])
        starts = starts[starts < T]
        cu = torch.full((max(len(starts) + 1, 64),), T, dtype=torch.int32)
        cu[:len(starts)] = starts.int()
        cu = cu.to(dev)
        dout = torch.randn(T, 6, 128, device=dev, generator=g).to(BF)
        if name == "dc_ours":
            from modded_nanogpt_b200.ops.dc import dc_correction
            fwd = lambda: dc_correction(base, q, k, v, w1, w2, cu, 0.12, 112)
        else:                               # the reference's Triton kernels (`dc_triton_kernels.py:1266`), unmodified
            ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
            if not os.path.exists(os.path.join(ref, "dc_triton_kernels.py")):
                raise SystemExit(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not staged on this machine"}))
            sys.path.insert(0, ref)
            from dc_triton_kernels import dc_attention_postonly_nodd_correction_add_base_triton as ref_dc
            fwd = lambda: ref_dc(base, q[None], k[None], v[None], (w1[None], w2[None]), None, scaling=0.12, window=112, seq_lens=cu)

        def run():
            for t in (q, k, v, base, w1, w2):
                t.grad = None
            fwd().backward(dout.view_as(base) if name == "dc_ours" else dout)
        # scores + PV over the 112-key window, forward, and about 2.5x that backward
        return run, int(3.5 * 4 * 128 * 6 * T * 112), 4 * T * 6 * 256
    if name.startswith("attn"):             # attn[bwd]_{ours|fa2}_{short|long|paired}: packed documents, sliding window
        op, impl, kind = name.split("_")
        Tq, Hh, window = (2 * T, 3, 2 * 640) if kind == "paired" else (T, 6, 640 if kind == "short" else 1408)
        g = torch.Generator(device=dev).manual_seed(0)
        q, k, v = (torch.randn(Tq, Hh, 128, device=dev, generator=g).to(BF) for _ in range(3))
        lens = torch.exp(torch.randn(4 * Tq // 600, generator=torch.Generator().manual_seed(0)) + 6.4).clamp(2, 2048).long()
        if kind == "paired":
            lens = lens * 2
        starts = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)])
        starts = starts[starts < Tq]
        cu = torch.full((max(len(starts) + 1, 64),), Tq, dtype=torch.int32)
        cu[:len(starts)] = starts.int()
        cu = cu.to(dev)
        pos = torch.arange(Tq, device=dev)
        bounds = fused.doc_bounds(cu, Tq)
        ds = bounds[0].contiguous()
        flops = 4 * 128 * Hh * int((pos - torch.maximum(ds.long(), pos - window) + 1).sum())
        max_len = 4096
        if op == "attnbwd":                 # 5 GEMMs of the same size as the forward's 2
            lib = fused._C()
            out, lse = lib.attn_fwd(q, k, v, ds, window, 0.12)
            dout = torch.randn_like(out)
            if impl == "ours":
                de = bounds[1].contiguous()
                return (lambda: lib.attn_bwd(dout, q, k, v, out, lse, ds, de, window, 0.12)), flops * 5 // 2, 3 * Tq * Hh * 256
            from flash_attn.flash_attn_interface import _wrapped_flash_attn_varlen_backward as fa_bwd
            dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
            return (lambda: fa_bwd(dout, q, k, v, out, lse, dq, dk, dv, cu, cu, max_len, max_len, 0.0, 0.12, True, window, 0, 0.0,
                                   None, False, rng_state=None)), flops * 5 // 2, 3 * Tq * Hh * 256
        if impl == "ours":
            lib = fused._C()
            return (lambda: lib.attn_fwd(q, k, v, ds, window, 0.12)), flops, Tq * Hh * 256
        from flash_attn import flash_attn_varlen_func
        return (lambda: flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max_len, max_seqlen_k=max_len,
                                               causal=True, softmax_scale=0.12, window_size=(window, 0))), flops, Tq * Hh * 256
    raise SystemExit(f"unknown case {name}")


CASES = ["qkvproj_fused", "qkvproj_unfused", "mlpmix_fused", "mlpmix_unfused", "proj_qkv_ours", "proj_qkv_lib", "proj_o_ours", "proj_o_lib", "gatemlp_ours", "gatemlp_lib", "gemm_bf16_up", "gemm_bf16_dpre", "gemm_bf16_down", "gemm_bf16_dw", "gemm_fp8_relu2", "gemm_fp8_down", "gemm_bf16_qkv",
         "gemm_bf16_o", "gemm_bf16_o_null", "gemm_bf16_up_null", "gemm_fp8_logits", "gemm_fp8_logits_kk", "gemm_fp8_lmhead_dw_kmajor_a", "gemm_fp8_lmhead_dx", "gemm_fp8_lmhead_dw", "softcap_ce_e5m2", "softcap_ce_bf16", "lmhead_ce_fwdbwd",
         "adam_bf16", "dc_ours", "dc_ref", "attn_ours_short", "attn_fa2_short", "attn_ours_long", "attn_fa2_long", "attn_ours_paired", "attn_fa2_paired",
         "attnbwd_ours_short", "attnbwd_fa2_short", "attnbwd_ours_long", "attnbwd_fa2_long", "attnbwd_ours_paired", "attnbwd_fa2_paired"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--rows", type=int, default=49152)
    ap.add_argument("--bn", type=int, default=0, help="GEMM tile: 128, 256, 512 (CTA pair); 0 = the wrapper's choice")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--list", action="store_true")
    a = ap.parse_args()
    if a.list:
        print("\n".join(CASES))
        return
    if a.case == "ref_lmhead_ce":          # the reference's fused lm_head + CE op at the same shape (separate process state)
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        ref = os.path.join(root, "baseline", "_ref")
        if not os.path.exists(os.path.join(ref, "triton_kernels.py")):
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not staged on this machine"}))
            return
        from baseline.reference_driver import reference_lmhead_ce_ms
        print(json.dumps(reference_lmhead_ce_ms(ref, a.rows, a.iters, a.warmup)), flush=True)
        return
    from modded_nanogpt_b200.ops import fused
    for name in (CASES if a.case == "all" else a.case.split(",")):
        torch.manual_seed(0)
        fn, flops, out_bytes = build_case(name, a.rows, a.bn or None, fused)
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / a.iters
        fused.check_status()
        print(json.dumps(dict(case=name, rows=a.rows, bn=a.bn, us=round(ms * 1e3, 1), tflops=round(flops / ms / 1e9, 1),
                              out_gbs=round(out_bytes / ms / 1e6, 1))), flush=True)
        del fn
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
