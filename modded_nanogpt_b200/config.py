"""Typed configuration: hyper-parameters, model topologies and training-stage tables.

The reference keeps these as module globals of a single script (`train_gpt.py:1880-1992`
for track 1, `train_gpt_medium.py:1402-1449,1610-1640` for track 2).  Here they are plain
dataclasses so the same trainer can run the track-1, track-2, track-3 and tiny-CPU presets,
with environment overrides for the few knobs the reference reads from the environment
(`DATA_PATH`, `DISABLE_FP8`).
"""
from __future__ import annotations

import os
import uuid
from dataclasses import dataclass, field, replace
from itertools import accumulate


def next_multiple_of_n(v, *, n: int) -> int:
    return -(-int(v) // n) * n


# --------------------------------------------------------------------------------------
# Model topology


@dataclass
class ModelConfig:
    """Architecture constants of one GPT.  `topology` selects the layer wiring:

    * ``"track1"`` – the 11-layer speedrun model (`train_gpt.py:1208-1693`): parameter banks,
      paired heads, value/bigram embeddings, MUDD skips and gates, XSA, DC, smear.
    * ``"plain"``  – rotary + QK-norm windowed attention and ReLU² MLP in every layer with
      learned residual scalars and a softcapped head (the tiny CPU/gloo plumbing model).
    """
    vocab_size: int = 50257
    num_layers: int = 11
    num_heads: int = 6
    head_dim: int = 128
    model_dim: int = 768
    max_seq_len: int = 262144
    topology: str = "track1"
    mlp_mult: int = 4
    # track-1 wiring (layer indices)
    paired_head_layers: tuple = (0, 2, 5, 9)
    long_window_layers: tuple = (3, 10)
    skip_attn_layers: tuple = (6,)
    cache_layers: tuple = (3, 7)
    xsa_layers: tuple = (1, 3, 4, 7)
    attn_gate_layers: tuple = (3, 10)
    dc_layers: tuple = (10,)
    dc_window: int = 112
    num_value_embeds: int = 5
    # bigram hash embedding (`train_gpt.py:1902-1904`)
    bigram_vocab_size: int = 50304 * 15 // 2
    bigram_dim: int = 768
    bigram_sign_table_rows: int = 8192
    # softcap  A*sigmoid((z+B)/C)  (`triton_kernels.py:1210`)
    softcap_a: float = 23.0
    softcap_b: float = 5.0
    softcap_c: float = 7.5
    # static fp8 scales of the head (`train_gpt.py:1225`)
    head_x_scale: float = 100 / 448
    head_w_scale: float = 1.6 / 448
    head_grad_scale: float = 0.75 / 448

    @property
    def padded_vocab(self) -> int:
        return next_multiple_of_n(self.vocab_size, n=128)


def track1_model(max_seq_len: int = 262144) -> ModelConfig:
    return ModelConfig(max_seq_len=max_seq_len)


def tiny_model(max_seq_len: int = 1024) -> ModelConfig:
    """2 layers, d_model 128, 2 heads x 64, vocab 50304: the CPU/gloo plumbing model."""
    return ModelConfig(
        vocab_size=50257, num_layers=2, num_heads=2, head_dim=64, model_dim=128,
        max_seq_len=max_seq_len, topology="plain", paired_head_layers=(), long_window_layers=(1,),
        skip_attn_layers=(), cache_layers=(), xsa_layers=(), attn_gate_layers=(), dc_layers=(),
        num_value_embeds=0, bigram_vocab_size=0, bigram_dim=0,
    )


def small_track1_model(max_seq_len: int = 2048) -> ModelConfig:
    """Full track-1 wiring at toy embedding-table sizes (used by CPU tests and smoke runs)."""
    return ModelConfig(vocab_size=50257, head_dim=32, model_dim=192, max_seq_len=max_seq_len,
                       bigram_vocab_size=1024 * 3, bigram_dim=192, bigram_sign_table_rows=64)


# --------------------------------------------------------------------------------------
# Stages and schedule


@dataclass
class TrainingStage:
    lr_mul: float
    batch_size: int                      # global tokens per optimizer step
    window_sizes: tuple                  # (short, long) in blocks of `block_size` tokens
    mtp_weights_start: list
    mtp_weights_end: list
    train_max_seq_len: int
    prefix_weight_start: float = 0.0
    prefix_weight_end: float = 0.0
    duration: float | None = None        # fraction of the scheduled iterations; None = extension


def track1_stages() -> list[TrainingStage]:
    """`train_gpt.py:1979-1989`."""
    return [
        TrainingStage(duration=1 / 3, train_max_seq_len=896, batch_size=8 * 2048 * 8, window_sizes=(1, 3),
                      lr_mul=1.0, mtp_weights_start=[1.0, 0.5, 0.25], mtp_weights_end=[1.0, 0.5, 0.0],
                      prefix_weight_start=0.25, prefix_weight_end=0.25),
        TrainingStage(duration=1 / 3, train_max_seq_len=2048, batch_size=16 * 2048 * 8, window_sizes=(3, 7),
                      lr_mul=1.52, mtp_weights_start=[1.0, 0.5], mtp_weights_end=[1.0, 0.0],
                      prefix_weight_start=0.25, prefix_weight_end=0.0),
        TrainingStage(duration=1 / 3, train_max_seq_len=2048, batch_size=24 * 2048 * 8, window_sizes=(5, 11),
                      lr_mul=1.73, mtp_weights_start=[1.0], mtp_weights_end=[1.0]),
        TrainingStage(train_max_seq_len=2048, batch_size=24 * 2048 * 8, window_sizes=(6, 13), lr_mul=1.0,
                      mtp_weights_start=[1.0], mtp_weights_end=[1.0]),
    ]


class TrainingSchedule:
    """Stage lookup, LR multiplier, MTP / prefix weights and the embed-split step
    (`train_gpt.py:1920-1976`).  Weights are plain Python lists here; the trainer turns the
    current step's entry into device tensors."""

    def __init__(self, stages, scheduled_iterations: int, extension_iterations: int,
                 cooldown_frac: float = 0.5, split_embed_stage: int = 2, ws_post_yarn_ext: int = 20,
                 final_lr_frac: float = 0.15):
        self.stages = stages
        self.scheduled_iterations = scheduled_iterations
        self.extension_iterations = extension_iterations
        self.cooldown_frac = cooldown_frac
        self.ws_post_yarn_ext = ws_post_yarn_ext
        self.final_lr_frac = final_lr_frac
        self.total_steps = scheduled_iterations + extension_iterations
        cum = accumulate(s.duration for s in stages[:-1])
        ends = [0, *[round(c * scheduled_iterations) for c in cum], self.total_steps]
        assert ends[-2] == scheduled_iterations, "stage durations must sum to 1"
        self.boundaries = list(zip(ends[:-1], ends[1:]))
        split_embed_stage = min(split_embed_stage, len(self.boundaries) - 1)
        self.split_step = self.boundaries[split_embed_stage][0] | 1   # odd, so Adam runs on it
        self.mtp_weights, self.prefix_weights = [], []
        for step in range(self.total_steps + 1):
            stage, t = self.lookup(step)
            self.mtp_weights.append([a + (b - a) * t for a, b in zip(stage.mtp_weights_start, stage.mtp_weights_end)])
            self.prefix_weights.append(stage.prefix_weight_start + (stage.prefix_weight_end - stage.prefix_weight_start) * t)

    def lookup(self, step: int):
        for i, (start, end) in enumerate(self.boundaries):
            if step < end:
                return self.stages[i], (step - start) / (end - start)
        return self.stages[-1], 1.0

    def stage_index(self, step: int) -> int:
        for i, (_, end) in enumerate(self.boundaries):
            if step < end:
                return i
        return len(self.boundaries) - 1

    def get_lr(self, step: int) -> float:
        stage, _ = self.lookup(step)
        lr = stage.lr_mul
        cd_start = int(self.scheduled_iterations * (1 - self.cooldown_frac))
        if step >= cd_start:
            t = min(1.0, (step - cd_start) / max(1, self.scheduled_iterations - cd_start))
            lr = lr * (1 - t) + self.final_lr_frac * t
        return lr

    def transition_steps(self):
        return [start for start, _ in self.boundaries[1:]]

    def muon_momentum(self, step: int, warmup_steps=300, cooldown_steps=50, lo=0.85, hi=0.95) -> float:
        """Linear 0.85->0.95 warm-up, 0.95->0.85 over the last steps (`train_gpt.py:1995-2007`)."""
        cd_start = self.total_steps - cooldown_steps
        if step < warmup_steps:
            return lo + (step / warmup_steps) * (hi - lo)
        if step > cd_start:
            return hi - ((step - cd_start) / cooldown_steps) * (hi - lo)
        return hi


# --------------------------------------------------------------------------------------
# Run-level hyper-parameters


@dataclass
class Hyperparameters:
    """`train_gpt.py:1880-1904`, plus the knobs this framework adds (synthetic data, step cap,
    kernel switches, checkpoint/resume)."""
    data_path: str = field(default_factory=lambda: os.environ.get("DATA_PATH", "."))
    train_files: str = ""
    val_files: str = ""
    val_tokens: int = 10485760
    val_batch_size: int = 4 * 64 * 1024 * 8
    num_scheduled_iterations: int = 1270
    num_extension_iterations: int = 15
    cooldown_frac: float = 0.60
    run_id: str = field(default_factory=lambda: str(uuid.uuid4()))
    val_loss_every: int = 250
    save_checkpoint: bool = False
    resume_from: str = ""
    run_evals: bool = False
    block_size: int = 128               # tokens per window block (`train_gpt.py:2021`)
    disable_fp8: bool = field(default_factory=lambda: bool(os.environ.get("DISABLE_FP8", "")))
    synthetic: bool = field(default_factory=lambda: bool(os.environ.get("SYNTHETIC_DATA", "")))
    max_steps: int = field(default_factory=lambda: int(os.environ.get("MAX_STEPS", "0")))
    seed: int = 0
    # optimizer defaults (`train_gpt.py:2065-2076`)
    adam_lr: float = 0.008
    adam_eps: float = 1e-10
    adam_wd: float = 0.005
    muon_lr: float = 0.023
    muon_momentum: float = 0.95
    muon_beta2: float = 0.9
    muon_wd: float = 1.2

    def __post_init__(self):
        if not self.train_files:
            self.train_files = os.path.join(self.data_path, "data/fineweb10B/fineweb_train_*.bin")
        if not self.val_files:
            self.val_files = os.path.join(self.data_path, "data/fineweb10B/fineweb_val_*.bin")


# max documents per batch size, padded length of cu_seqlens (`train_gpt.py:1710,1817`)
TRAIN_MAX_NUM_DOCS = {16384: 64, 32768: 96, 49152: 128}


def max_num_docs(num_tokens_local: int) -> int:
    return TRAIN_MAX_NUM_DOCS.get(num_tokens_local, next_multiple_of_n(max(num_tokens_local // 300, 1), n=128))


def track1_schedule(hp: Hyperparameters | None = None) -> TrainingSchedule:
    hp = hp or Hyperparameters()
    return TrainingSchedule(track1_stages(), hp.num_scheduled_iterations, hp.num_extension_iterations,
                            cooldown_frac=hp.cooldown_frac)


def tiny_stages(batch_tokens: int = 4 * 256 * 2, seq_len: int = 256) -> list[TrainingStage]:
    return [
        TrainingStage(duration=1.0, train_max_seq_len=seq_len, batch_size=batch_tokens, window_sizes=(1, 2),
                      lr_mul=1.0, mtp_weights_start=[1.0, 0.5], mtp_weights_end=[1.0, 0.0]),
        TrainingStage(train_max_seq_len=seq_len, batch_size=batch_tokens, window_sizes=(1, 2), lr_mul=1.0,
                      mtp_weights_start=[1.0], mtp_weights_end=[1.0]),
    ]


def scaled(hp: Hyperparameters, **kw) -> Hyperparameters:
    return replace(hp, **kw)


# --------------------------------------------------------------------------------------
# Track 2 (train_gpt_medium.py:1610-1640, 1402-1433)

TRACK2_BS = (131072, 262144, 393216, 524288) + (524288,) * 8
TRACK2_WS = (3, 7, 11, 13, 15, 17, 19, 21, 23, 23, 23, 23)


def track2_stages() -> list[TrainingStage]:
    lr = [1.0, 1.52, 1.73] + [2.0] * 9
    stages = []
    for k in range(12):
        if k == 0:
            mtp = ([1.0, 0.5, 0.25], [1.0, 0.5, 0.0])
        elif k == 1:
            mtp = ([1.0, 0.5], [1.0, 0.0])
        else:
            mtp = ([1.0], [1.0])
        stages.append(TrainingStage(duration=1 / 12, train_max_seq_len=4096, batch_size=TRACK2_BS[k],
                                    window_sizes=(min(11, TRACK2_WS[k] // 2), TRACK2_WS[k]), lr_mul=lr[k],
                                    mtp_weights_start=mtp[0], mtp_weights_end=mtp[1]))
    stages.append(TrainingStage(train_max_seq_len=4096, batch_size=32 * 2048 * 8, window_sizes=(11, 23), lr_mul=0.1,
                                mtp_weights_start=[1.0], mtp_weights_end=[1.0]))
    return stages


def track2_hyperparameters(**kw) -> Hyperparameters:
    base = dict(num_scheduled_iterations=4700, num_extension_iterations=40, cooldown_frac=0.70, adam_lr=0.004, adam_eps=1e-8,
                muon_lr=0.015, muon_beta2=0.95)
    base.update(kw)
    return Hyperparameters(**base)


def track2_schedule(hp: Hyperparameters | None = None) -> TrainingSchedule:
    hp = hp or track2_hyperparameters()
    s = TrainingSchedule(track2_stages(), hp.num_scheduled_iterations, hp.num_extension_iterations,
                         cooldown_frac=hp.cooldown_frac, ws_post_yarn_ext=27, final_lr_frac=0.1)
    import math
    s.split_step = math.ceil(2 / 3 / 4 * hp.num_scheduled_iterations) | 1
    s.yarn_max_ws = 13          # rotary rescaling only follows the first few window changes
    return s
