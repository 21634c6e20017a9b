"""Runs the unmodified reference trainer (`baseline/_ref/train_gpt.py` with its Triton/NVRTC kernel
files) for the benchmark config of `bench.py`: stage-2 batch (393,216 tokens per optimizer step,
grad_accum = 8 // N micro-batches of 49,152 tokens per rank), same synthetic shards, W warm-up steps
(which also absorb torch.compile), K timed steps, CUDA events, max over ranks.

The reference is a script whose training loop is module-level code, so it cannot be called as a
function.  This driver executes the script's definitions (everything above its "int main" banner:
kernels import, optimizer, model, loader, schedule, TrainingManager) unchanged, then issues the
same calls the script's own main section makes for each step (`train_gpt.py:2234-2261` model
construction, `:2357-2365` step body).  None of this repository's model, kernel or engine code is
on that path.  Compatibility shims, none of which touches the files or the math:

* `kernels.get_kernel('kernels-community/flash-attn3')` needs the network and returns a Hopper
  binary; a stub module hands out FlashAttention-2's `flash_attn_varlen_func` (same signature);
* `tiktoken.get_encoding("gpt2")` needs the network; it returns a deterministic synthetic BPE-like
  rank table (only used for the prefix-token table);
* `torch.cuda._compile_kernel(..., compute_capability="90")` builds an sm_90 cubin that cannot load
  on this GPU; the wrapper substitutes the device's own capability.
"""
from __future__ import annotations

import os
import sys
import time
import types


def _install_shims():
    import torch

    stub = types.ModuleType("kernels")

    def get_kernel(name, version=None, **kw):
        from flash_attn import flash_attn_varlen_func
        iface = types.SimpleNamespace(flash_attn_varlen_func=flash_attn_varlen_func)
        return types.SimpleNamespace(flash_attn_interface=iface)

    stub.get_kernel = get_kernel
    sys.modules["kernels"] = stub

    import tiktoken
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from modded_nanogpt_b200.data.prefix import synthetic_ranks      # data only: a vocabulary table
    ranks = synthetic_ranks(50257)
    tiktoken.get_encoding = lambda name: types.SimpleNamespace(_mergeable_ranks=ranks, eot_token=50256, n_vocab=50257)

    orig = torch.cuda._compile_kernel
    major, minor = torch.cuda.get_device_capability()

    def compile_kernel(*a, **kw):
        if kw.get("compute_capability") is not None:
            kw["compute_capability"] = f"{major}{minor}"
        return orig(*a, **kw)

    torch.cuda._compile_kernel = compile_kernel


def drive(args, ref_dir: str) -> dict:
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if world != args.gpus:
        return {"impl": "reference", "unavailable": f"--gpus {args.gpus} but WORLD_SIZE={world}"}
    K, W = args.steps, args.warmup
    stage_idx = int(getattr(args, "stage", 2))
    batch = (8, 16, 24)[stage_idx] * 2048 * 8
    root = f"/tmp/mng_bench_ref_{stage_idx}_{K}_{W}"
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus   # data generation only
    if rank == 0:
        need = int(batch * (K * 2 + W + 12) * 1.02) + 1_000_000
        # the reference loader preloads a second shard at start-up, so there must be at least two
        write_synthetic_corpus(root, train_tokens=need, val_tokens=3_000_000, seed=0, max_doc_len=(896, 2048, 2048)[stage_idx],
                               shard_tokens=max(2_000_000, need // 3 + 1))
    os.environ["DATA_PATH"] = root
    # The reference's FP8 MLP Triton kernel (linear_relu_square_kernel, TMA-descriptor persistent GEMM
    # tuned for Hopper) does not get through Triton 3.6's make_ttgir pass for sm_100, so by default the
    # reference runs with its own DISABLE_FP8 switch (bf16 MLP; its lm_head + CE path stays FP8).
    # MNG_REF_FP8=1 tries the FP8 mode.
    if not os.environ.get("MNG_REF_FP8"):
        os.environ["DISABLE_FP8"] = "1"

    import torch
    _install_shims()
    path = os.path.join(ref_dir, "train_gpt.py")
    sys.argv = [path]
    sys.path.insert(0, ref_dir)
    src = open(path).read()
    cut = src.index("# int main")
    cut = src.rindex("# ----", 0, cut)
    mod = types.ModuleType("reference_train_gpt")         # a real module: dataclasses look their module up
    mod.__file__ = path
    sys.modules[mod.__name__] = mod
    ns = mod.__dict__
    exec(compile(src[:cut], path, "exec"), ns)            # the reference's definitions, unchanged
    dist, nn = ns["dist"], ns["nn"]
    # torch 2.11 refuses to trace the lazy initialisation of this module-level cache inside an
    # autograd.Function (the reference pins torch 2.10): fill the cache eagerly with its own helper
    sys.modules["triton_kernels"]._get_dummy_f32(ns["device"])
    ga, device = ns["grad_accum_steps"], ns["device"]
    rargs, sched = ns["args"], ns["training_schedule"]

    # model construction: the calls of train_gpt.py:2234-2261
    model = ns["GPT"](vocab_size=50257, num_layers=11, num_heads=6, head_dim=128, model_dim=768,
                      max_seq_len=rargs.val_batch_size // (ga * world)).cuda()
    for m in model.modules():
        if isinstance(m, (nn.Embedding, nn.Linear)):
            m.weight.data = m.weight.data.bfloat16()
    for name in ("ve_gate_bank", "qk_bank", "vo_bank", "mlp_bank", "mudd_w1", "mudd_w2", "mudd_b2", "mudd_gate_w1",
                 "mudd_gate_w2", "mudd_gate_b2"):
        getattr(model, name).data = getattr(model, name).data.bfloat16()
    for p in model.parameters():
        dist.broadcast(p.detach(), 0)
    dist.broadcast(model.bigram_sign_table, 0)
    model.quantize_mlp_fp8(bootstrap_down=True)
    model = torch.compile(model, dynamic=False, fullgraph=True)
    ns["model"] = model
    tm = ns["TrainingManager"](model)
    ns["training_manager"] = tm
    model.prefix_table.copy_(ns["build_prefix_table"](model.vocab_size))

    for b0, _ in sched.boundaries[:stage_idx + 1]:
        tm.advance_schedule(b0)
    first = sched.boundaries[stage_idx][0] + 1
    tm.optimizer.split_embed = first > tm.split_step
    stage = ns["TRAINING_STAGES"][stage_idx]
    loader = ns["distributed_data_generator"](rargs.train_files, stage.batch_size, stage.train_max_seq_len,
                                              grad_accum_steps=ga)
    tm.train_loader_send_args = None
    model.train()
    grad_scale = ns["grad_scale"]

    def one_step(step, read_loss):
        tm.advance_schedule(step)
        total = None
        for _ in range(ga):
            inputs, targets, cum_seqlens, bigram_inputs, bigram_cpu = loader.send(tm.train_loader_send_args)
            tm.sparse_index_update(step, bigram_cpu)
            loss = model(inputs, targets, cum_seqlens, bigram_inputs, tm.get_forward_args()).sum() * grad_scale
            tm.sparse_index_share(step)
            loss.backward()
            # the step loss is summed on the device and read once per step, as the other arm does
            total = loss.detach() if total is None else total + loss.detach()
            del loss
        tm.step_optimizers(step)
        model.quantize_mlp_fp8(bootstrap_down=(step < 16))
        return float(total) if read_loss else 0.0

    from torch._dynamo.utils import counters

    def compiled_frames():
        return int(counters["frames"]["ok"]) + int(counters["stats"]["unique_graphs"])

    # Warm-up: W steps, then (untimed, to the reference's benefit) more until an odd and an even step in a row
    # compiled nothing new: the sparse-comms path that only exists at 8 ranks compiles late.
    step = first
    extra = 0
    quiet = 0
    for i in range(max(W, 2) + 8):
        before = compiled_frames()
        one_step(step, False)
        step += 1
        quiet = quiet + 1 if compiled_frames() == before else 0
        if i + 1 >= max(W, 2):
            if quiet >= 2:
                break
            extra += 1
    frames_before_timing = compiled_frames()

    from modded_nanogpt_b200.utils.timing import ClockSampler          # nvidia-smi polling thread (read-only queries)

    def timed(read_loss):
        nonlocal step
        dist.barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(int(os.environ["LOCAL_RANK"])).start() if rank == 0 else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        last = 0.0
        for _ in range(K):
            last = one_step(step, read_loss)
            step += 1
        e1.record()
        dist.barrier()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
        clocks = sampler.stop() if sampler else None
        t = torch.tensor([e0.elapsed_time(e1), wall], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]), float(t[1]), last, clocks

    dev_ms, _, _, clocks = timed(False)
    e2e_ms, e2e_wall, last, clocks_e2e = timed(True)
    recompiles_in_timed = compiled_frames() - frames_before_timing
    tokens = stage.batch_size * K
    T = stage.batch_size // 8
    max_docs = {16384: 64, 32768: 96, 49152: 128}[T]
    h2d = ga * (T * 4 + T * 8 + max_docs * 4 + T * 4)
    out = {
        "impl": "reference", "metric": f"train tokens/s, track-1 GPT, stage-{stage_idx} batch ({stage.batch_size} tok/step)",
        "value": tokens / (dev_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": dev_ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": ("bf16 (fp8 lm_head; bf16 MLP: reference run with its own DISABLE_FP8=1)" if os.environ.get("DISABLE_FP8")
                  else "bf16 (fp8 MLP forward and lm_head)"), "data": "synthetic Zipf(1.1) ids, EoS-delimited lognormal docs; random-init weights",
        "config": {"model": "track-1 GPT (reference train_gpt.py HEAD)", "global_batch": stage.batch_size,
                   "seq_len": stage.train_max_seq_len, "grad_accum": ga, "parallelism": f"dp{world}",
                   "attention": "FlashAttention-2 (FA3 is a Hopper-only binary)", "first_step": first,
                   "reference_env": {"DISABLE_FP8": os.environ.get("DISABLE_FP8", "")}},
        "e2e": {"value": tokens / (max(e2e_ms, e2e_wall) / 1e3), "unit": "tokens/s", "ms_per_step": max(e2e_ms, e2e_wall) / K,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "last_loss": last},
        "extra_warmup_steps": extra, "recompiles_in_timed_regions": recompiles_in_timed,
        "gpu_launches": None, "clocks": clocks, "clocks_e2e": clocks_e2e,
    }
    dist.barrier()
    dist.destroy_process_group()
    return out if rank == 0 else {}


# ---------------------------------------------------------------------------------------------------
# Track 2: `train_gpt_medium.py`.  Its definitions and its start-up code (process-group init, logging) are
# interleaved, so everything above its model construction is executed unchanged (from a scratch directory: it
# writes `logs/<uuid>.txt`), then the calls of its own main section are issued for the timed steps
# (`train_gpt_medium.py:1688-1699` construction, `:1792-1799` step body).
def drive_track2(args, ref_dir: str) -> dict:
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29519")
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if world != args.gpus:
        return {"impl": "reference", "unavailable": f"--gpus {args.gpus} but WORLD_SIZE={world}"}
    K, W = args.steps, args.warmup
    batch = 524288
    root = f"/tmp/mng_bench_ref2_{K}_{W}"
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus   # data generation only
    if rank == 0:
        need = int(batch * (K * 2 + W + 12) * 1.02) + 1_000_000
        write_synthetic_corpus(root, train_tokens=need, val_tokens=3_000_000, seed=0, max_doc_len=4096,
                               shard_tokens=max(2_000_000, need // 3 + 1))
    os.environ["DATA_PATH"] = root
    scratch = f"/tmp/mng_ref2_cwd_{rank}"
    os.makedirs(scratch, exist_ok=True)
    os.chdir(scratch)

    import torch
    _install_shims()
    path = os.path.join(ref_dir, "train_gpt_medium.py")
    sys.argv = [path]
    sys.path.insert(0, ref_dir)
    src = open(path).read()
    cut = src.index("model: nn.Module = GPT(")
    mod = types.ModuleType("reference_train_gpt_medium")
    mod.__file__ = path
    sys.modules[mod.__name__] = mod
    ns = mod.__dict__
    exec(compile(src[:cut], path, "exec"), ns)            # definitions + process-group init, unchanged
    dist, nn = ns["dist"], ns["nn"]
    ga, rargs = ns["grad_accum_steps"], ns["args"]
    if rank != 0:                                         # the data is written by rank 0 after its own imports
        pass
    dist.barrier()
    model = ns["GPT"](vocab_size=50257, num_layers=16, num_heads=8, head_dim=128, model_dim=1024,
                      max_seq_len=rargs.val_batch_size // (ga * world)).cuda()
    for m in model.modules():
        if isinstance(m, (nn.Embedding, nn.Linear)):
            m.weight.data = m.weight.data.bfloat16()
    for p in model.parameters():
        dist.broadcast(p.detach(), 0)
    model = torch.compile(model, dynamic=False, fullgraph=True)
    tm = ns["TrainingManager"](model)

    # enter the plateau the way a run would: window / YaRN state of every earlier transition applied
    first = 3 * rargs.num_scheduled_iterations // 12 + 1                  # 1176: batch 524,288 from step 1175 on
    for s in tm.get_transition_steps():
        if s <= first:
            tm.advance_schedule(s)
    tm.split_step = first | 1          # the embedding split (due at step 785 of a run) happens in the warm-up
    loader = ns["distributed_data_generator"](rargs.train_files, batch, rargs.train_max_seq_len, grad_accum_steps=ga)
    tm.batch_size = batch
    model.train()

    def one_step(step, read_loss):
        tm.advance_schedule(step)
        total = None
        for idx in range(ga):
            if idx == ga - 1:
                tm.activate_hooks(step)
            inputs, targets, cum_seqlens = loader.send(tm.train_loader_send_args)
            loss = model(inputs, targets, cum_seqlens, tm.get_forward_args()) / ga
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
            del loss
        tm.step_optimizers(step)
        return float(total) if read_loss else 0.0

    from torch._dynamo.utils import counters

    def compiled_frames():
        return int(counters["frames"]["ok"]) + int(counters["stats"]["unique_graphs"])

    step, extra, quiet = first, 0, 0
    for i in range(max(W, 3) + 8):
        before = compiled_frames()
        one_step(step, False)
        step += 1
        quiet = quiet + 1 if compiled_frames() == before else 0
        if i + 1 >= max(W, 3):
            if quiet >= 2:
                break
            extra += 1
    frames0 = compiled_frames()

    from modded_nanogpt_b200.utils.timing import ClockSampler          # nvidia-smi polling thread (read-only queries)

    def timed(read_loss):
        nonlocal step
        dist.barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(int(os.environ["LOCAL_RANK"])).start() if rank == 0 else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        last = 0.0
        for _ in range(K):
            last = one_step(step, read_loss)
            step += 1
        e1.record()
        dist.barrier()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
        clocks = sampler.stop() if sampler else None
        t = torch.tensor([e0.elapsed_time(e1), wall], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]), float(t[1]), last, clocks

    dev_ms, _, _, clocks = timed(False)
    e2e_ms, e2e_wall, last, clocks_e2e = timed(True)
    tokens = batch * K
    T = batch // 8
    out = {
        "impl": "reference", "metric": "train tokens/s, track-2 GPT, plateau batch (524288 tok/step)",
        "value": tokens / (dev_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": dev_ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 (the reference's track-2 trainer runs with FP8 off)",
        "data": "synthetic Zipf(1.1) ids, EoS-delimited lognormal docs; random-init weights",
        "config": {"model": "track-2 GPT (reference train_gpt_medium.py HEAD)", "global_batch": batch,
                   "seq_len": rargs.train_max_seq_len, "grad_accum": ga, "parallelism": f"dp{world}",
                   "attention": "FlashAttention-2 (FA3 is a Hopper-only binary)", "first_step": first},
        "e2e": {"value": tokens / (max(e2e_ms, e2e_wall) / 1e3), "unit": "tokens/s", "ms_per_step": max(e2e_ms, e2e_wall) / K,
                "h2d_bytes_per_step": ga * (T * 4 + T * 8 + 4 * 1024), "d2h_bytes_per_step": 4, "last_loss": last},
        "extra_warmup_steps": extra, "recompiles_in_timed_regions": compiled_frames() - frames0, "gpu_launches": None,
        "clocks": clocks, "clocks_e2e": clocks_e2e,
    }
    dist.barrier()
    dist.destroy_process_group()
    return out if rank == 0 else {}


# ---------------------------------------------------------------------------------------------------
# Micro-benchmarks of two reference components at the shapes of the training step, for `bench/bench_optimizer.py
# --impl reference` and `bench/bench_kernels.py --case ref_lmhead_ce`.
def load_track1_definitions(ref_dir: str):
    """Executes the definitions of the reference's `train_gpt.py` (everything above its main section) and returns the
    namespace.  Needs RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* in the environment (it initialises the process group)."""
    for k, v in (("RANK", "0"), ("WORLD_SIZE", "1"), ("LOCAL_RANK", "0"), ("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29521")):
        os.environ.setdefault(k, v)
    os.environ.setdefault("DATA_PATH", "/tmp")
    if not os.environ.get("MNG_REF_FP8"):
        os.environ["DISABLE_FP8"] = "1"
    _install_shims()
    path = os.path.join(ref_dir, "train_gpt.py")
    sys.argv = [path]
    sys.path.insert(0, ref_dir)
    src = open(path).read()
    cut = src.index("# int main")
    cut = src.rindex("# ----", 0, cut)
    mod = types.ModuleType("reference_train_gpt")
    mod.__file__ = path
    sys.modules[mod.__name__] = mod
    exec(compile(src[:cut], path, "exec"), mod.__dict__)
    sys.modules["triton_kernels"]._get_dummy_f32(mod.__dict__["device"])
    return mod.__dict__


def reference_optimizer_step_ms(ref_dir: str, steps: int, warmup: int = 4) -> dict:
    """The reference's `NorMuonAndAdam.step` (`train_gpt.py:723-823`, NCCL collectives, compiled update math) on all
    track-1 parameters with random bf16 gradients ~N(0, 1e-3): ms per Adam (odd) step and per NorMuon-only (even)
    step, CUDA events, max over ranks."""
    import torch
    ns = load_track1_definitions(ref_dir)
    dist, nn = ns["dist"], ns["nn"]
    ga, world, rargs = ns["grad_accum_steps"], ns["world_size"], ns["args"]
    model = ns["GPT"](vocab_size=50257, num_layers=11, num_heads=6, head_dim=128, model_dim=768,
                      max_seq_len=rargs.val_batch_size // (ga * world)).cuda()
    for m in model.modules():
        if isinstance(m, (nn.Embedding, nn.Linear)):
            m.weight.data = m.weight.data.bfloat16()
    for name in ("ve_gate_bank", "qk_bank", "vo_bank", "mlp_bank", "mudd_w1", "mudd_w2", "mudd_b2", "mudd_gate_w1",
                 "mudd_gate_w2", "mudd_gate_b2"):
        getattr(model, name).data = getattr(model, name).data.bfloat16()
    for p in model.parameters():
        dist.broadcast(p.detach(), 0)
    ns["model"] = model
    tm = ns["TrainingManager"](model)
    tm.optimizer.split_embed = True
    gen = torch.Generator(device="cuda").manual_seed(1 + int(os.environ["RANK"]))
    grads = {p: (torch.randn(p.shape, generator=gen, device="cuda", dtype=torch.float32) * 1e-3).to(p.dtype)
             for p in model.parameters()}
    # with sparse comms (8 ranks) the bigram gradient rows are exchanged by index: 49,152 random rows count as touched
    import numpy as np
    times = {0: [], 1: []}
    step = 848
    for it in range(2 * (warmup + steps)):
        for p in model.parameters():
            p.grad = grads[p].clone()
        rows = np.unique(np.random.default_rng(step).integers(0, model.bigram_embed.weight.shape[0], 49152))
        tm.sparse_index_update(step, rows)                 # both return at once unless the job has 8 ranks
        tm.sparse_index_share(step)
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tm.step_optimizers(step)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if it >= 2 * warmup:
            times[step % 2].append(float(t))
        step += 1
    out = dict(impl="reference", world=world, adam_step_ms=sum(times[1]) / len(times[1]),
               normuon_only_step_ms=sum(times[0]) / len(times[0]), steps=steps)
    dist.barrier()
    dist.destroy_process_group()
    return out


def reference_lmhead_ce_ms(ref_dir: str, rows: int, iters: int, warmup: int = 3) -> dict:
    """The reference's `FusedSoftcappedCrossEntropy` (`triton_kernels.py:1208-1292`: `torch._scaled_mm` FP8 GEMMs, its
    NVRTC loss kernel, two Triton transposes) forward + backward at [rows, 768] x [768, 50304]."""
    import torch
    ns = load_track1_definitions(ref_dir)
    F = sys.modules["triton_kernels"].FusedSoftcappedCrossEntropy
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    x = (torch.randn(rows, 768, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(768, 50304, device=dev, generator=g) * 0.02).bfloat16().requires_grad_(True)
    tg = torch.randint(0, 50304, (rows,), device=dev, generator=g)
    pt = torch.randint(-1, 50304, (rows,), device=dev, generator=g)
    mtp, pw = torch.tensor([1.0, 0.5, 0.25], device=dev), torch.tensor([0.1], device=dev)

    def run():
        x.grad = w.grad = None
        F.apply(x, tg, mtp, pt, pw, w, 100 / 448, 1.6 / 448, 0.75 / 448, 1.0).sum().backward()

    try:
        for _ in range(warmup):
            run()
    except Exception as e:  # noqa: BLE001 - the eager backward of this Function only works when traced (see its source)
        eager_err = f"{type(e).__name__}: {str(e)[:160]}"
        fn = torch.compile(lambda: F.apply(x, tg, mtp, pt, pw, w, 100 / 448, 1.6 / 448, 0.75 / 448, 1.0).sum())

        def run():                                                        # noqa: F811
            x.grad = w.grad = None
            fn().backward()
        for _ in range(warmup):
            run()
    else:
        eager_err = None
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        run()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    ns["dist"].destroy_process_group()
    return dict(impl="reference", case="lmhead_ce_fwdbwd", rows=rows, ms=ms, tflops=3 * 2 * rows * 768 * 50304 / ms / 1e9,
                traced=eager_err is not None, eager_error=eager_err)
