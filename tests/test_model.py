"""Model contract: state_dict layout, wiring, masks, loss terms (CPU, fp32 oracles)."""
import math

import pytest
import torch
import torch.nn.functional as F

from modded_nanogpt_b200.config import ModelConfig, small_track1_model, tiny_model, track1_model
from modded_nanogpt_b200.models.gpt import GPT, ForwardScheduleConfig
from modded_nanogpt_b200.models.yarn import Yarn
from modded_nanogpt_b200.ops import reference as ref
from modded_nanogpt_b200.trainer import TRACK1_WORK_ORDER, track1_param_table

TRACK1_STATE = {   # name -> (shape at world_size 8, dtype after cast_params_)
    "lm_head.weight": ((768, 50304), torch.bfloat16), "embed.weight": ((50304, 768), torch.bfloat16),
    "value_embeds": ((251520, 768), torch.bfloat16), "ve_gate_bank": ((5, 6, 12), torch.bfloat16),
    "qk_bank": ((64, 256, 768), torch.bfloat16), "vo_bank": ((24, 768, 768), torch.bfloat16),
    "mlp_bank": ((12, 2, 3072, 768), torch.bfloat16), "smear_gate.weight": ((1, 12), torch.bfloat16),
    "bigram_embed.weight": ((377280, 768), torch.bfloat16), "post_lambdas": ((11, 2), torch.float32),
    "resid_lambdas": ((11, 2), torch.float32), "scalars": ((24,), torch.float32),
    "mudd_w1": ((2, 64, 768), torch.bfloat16), "mudd_w2": ((2, 14, 64), torch.bfloat16),
    "mudd_b2": ((2, 14), torch.bfloat16), "mudd_gate_w1": ((2, 64, 768), torch.bfloat16),
    "mudd_gate_w2": ((2, 41, 64), torch.bfloat16), "mudd_gate_b2": ((2, 41), torch.bfloat16),
    "_mudd_gate_scale": ((), torch.float32), "bigram_sign_table": ((8192, 768), torch.bfloat16),
    "_mlp_down_act_scales": ((12,), torch.float32), "_mlp_down_proj_scales": ((12,), torch.float32),
    "_mlp_down_proj_next_scales": ((12,), torch.float32),
}


def test_track1_state_dict_layout():
    with torch.device("meta"):
        m = GPT(track1_model(), world_size=8).cast_params_()
    sd = m.state_dict()
    assert set(sd) == set(TRACK1_STATE)
    for k, (shape, dt) in TRACK1_STATE.items():
        assert tuple(sd[k].shape) == shape and sd[k].dtype == dt, k
    n = sum(p.numel() for p in m.parameters())
    assert 640e6 < n < 650e6
    labels = {p.label for p in m.parameters()}
    assert labels == set(track1_param_table()) == set(TRACK1_WORK_ORDER)
    with torch.device("meta"):
        m1 = GPT(track1_model(), world_size=1)
    assert m1.qk_bank.shape[0] == 60 and m1.vo_bank.shape[0] == 20 and m1.mlp_bank.shape[0] == 12


def test_reference_style_constructor():
    with torch.device("meta"):
        m = GPT(vocab_size=50257, num_layers=11, num_heads=6, head_dim=128, model_dim=768, max_seq_len=2048)
    assert m.vocab_size == 50304 and m.lm_head.weight.shape == (768, 50304)


def test_init_values():
    torch.manual_seed(0)
    m = GPT(small_track1_model())
    assert torch.equal(m.embed.weight, m.lm_head.weight.T)
    assert m.mlp_bank[:, 1].abs().max() == 0 and m.mlp_bank[:, 0].abs().max() > 0
    bound = 3 ** 0.5 * 0.5 * 192 ** -0.5
    assert m.qk_bank.abs().max() <= bound
    assert m.scalars[:22].view(11, 2)[:, 0].eq(0.5).all() and m.scalars[23] == -1.5
    assert m.mudd_b2[0, 6] == 20 and m.mudd_b2[1, 1] == -5
    b = m.mudd_gate_b2
    assert b[0, 12:18].eq(2.5).all() and b[0, 19:26:2].eq(0.5).all() and b[0, 18:26:2].eq(0).all()
    assert b[1, 12:18].eq(2.5).all() and b[1, 19:28:2].eq(0.5).all() and b[1, 28] == 5 and b[1, 29:35].eq(10).all()
    assert b[1, 35:41].eq(0).all()
    assert m.gate_layouts[0]["inject"] == {0: 18, 1: 20, 2: 22, 3: 24}
    assert m.gate_layouts[1]["inject"] == {4: 18, 5: 20, 7: 22, 8: 24, 9: 26}
    assert [p.attn_slot for p in m.plan] == [0, 1, 2, 3, 4, 5, -1, 6, 7, 8, 9]
    assert [p.ve_slot for p in m.plan] == [-1, 0, 1, -1, -1, -1, -1, -1, 2, 3, 4]


def _batch(T, vocab, docs=(0, 100, 180)):
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, vocab, (T,), dtype=torch.int32, generator=g)
    tg = torch.randint(0, vocab, (T,), dtype=torch.int64, generator=g)
    cu = torch.full((16,), T, dtype=torch.int32)
    cu[:len(docs)] = torch.tensor(docs, dtype=torch.int32)
    return ids, tg, cu


@pytest.mark.parametrize("cfg", [tiny_model(), small_track1_model()], ids=["plain", "track1"])
def test_forward_backward_all_params_get_grad(cfg):
    from modded_nanogpt_b200.data.loader import bigram_hash
    torch.manual_seed(0)
    m = GPT(cfg)
    T = 256
    ids, tg, cu = _batch(T, 900)
    bg = bigram_hash(ids, cfg.bigram_vocab_size) if cfg.bigram_vocab_size else torch.zeros_like(ids)
    sc = ForwardScheduleConfig(torch.tensor([1.0, 0.5, 0.25]), torch.tensor([0.25]), 128, 384, 256)
    loss = m(ids, tg, cu, bg, sc)
    assert loss.shape == (T,) and loss.dtype == torch.float32
    # at init the head is near uniform: loss ~ sum(w) * ln(V)
    assert loss.mean().item() == pytest.approx(1.75 * math.log(m.vocab_size), rel=0.02)
    loss.sum().backward()
    assert all(p.grad is not None for p in m.parameters())
    m.eval()
    with torch.no_grad():
        ev = m(ids, tg, cu, bg, sc)
    assert ev.mean().item() == pytest.approx(math.log(m.vocab_size), rel=0.02)


def test_documents_do_not_leak():
    """Changing tokens of document 0 must not change the loss inside document 1 beyond the
    positions that smear / bigram / key-offset couple across the boundary (first 2 tokens)."""
    torch.manual_seed(0)
    m = GPT(tiny_model())
    with torch.no_grad():
        m.mlp_bank[:, 1].normal_(0, 0.02)
        m.lm_head.weight.normal_(0, 0.02)
    T = 256
    ids, tg, cu = _batch(T, 900)
    sc = ForwardScheduleConfig(torch.tensor([1.0]), torch.tensor([0.0]), 128, 384, 256)
    bg = torch.zeros_like(ids)
    m.eval()
    with torch.no_grad():
        a = m(ids, tg, cu, bg, sc)
        ids2 = ids.clone()
        ids2[:90] = torch.randint(0, 900, (90,), dtype=torch.int32)
        b = m(ids2, tg, cu, bg, sc)
    assert not torch.allclose(a[:90], b[:90])
    assert torch.allclose(a[104:], b[104:], atol=1e-5)


def test_attention_reference_window_and_docs():
    torch.manual_seed(0)
    T, H, D = 64, 2, 16
    q, k, v = (torch.randn(T, H, D) for _ in range(3))
    cu = torch.tensor([0, 20, 50, T, T], dtype=torch.int32)
    out = ref.attention_varlen(q, k, v, cu, window=8, scale=0.3, chunk=16)
    for i in (0, 19, 20, 33, 63):
        doc_start = 0 if i < 20 else 20 if i < 50 else 50
        lo = max(doc_start, i - 8)
        s = (q[i, :, None, :] * k[lo:i + 1].transpose(0, 1)).sum(-1) * 0.3
        want = (torch.softmax(s, -1)[..., None] * v[lo:i + 1].transpose(0, 1)).sum(1)
        assert torch.allclose(out[i], want, atol=1e-5)


def test_dc_correction_reference():
    torch.manual_seed(0)
    T, H, D, W = 40, 3, 8, 5
    q, k, v, base = (torch.randn(T, H, D) for _ in range(4))
    w1, w2 = torch.randn(T, H), torch.randn(T, H)
    cu = torch.tensor([0, 17, T, T], dtype=torch.int32)
    out = ref.dc_correction(base, q, k, v, w1, w2, cu, scale=0.5, window=W, chunk=16)
    for t in (0, 3, 16, 17, 18, 39):
        ds = 0 if t < 17 else 17
        lo = max(ds, t - W + 1)
        a = torch.zeros(t + 1 - lo)
        for h in range(H):
            a += w1[t, h] * torch.softmax((k[lo:t + 1, h] @ q[t, h]) * 0.5, 0)
        for h in range(H):
            want = base[t, h] + w2[t, h] * (a @ v[lo:t + 1, h])
            assert torch.allclose(out[t, h], want, atol=1e-5)


def test_softcap_ce_matches_direct_math():
    torch.manual_seed(0)
    T, D, V = 50, 16, 128
    x = torch.randn(T, D, requires_grad=True)
    w = (torch.randn(D, V) * 0.3).requires_grad_(True)
    tg = torch.randint(0, V, (T,))
    pt = torch.randint(-1, V, (T,))
    mtp, pw = torch.tensor([1.0, 0.5, 0.25]), torch.tensor([0.3])
    loss = ref.softcap_ce(x, w, tg, mtp, pt, pw, chunk=16)
    z = 23 * torch.sigmoid((x @ w + 5) / 7.5)
    lse = torch.logsumexp(z, -1)
    want = torch.zeros(T)
    for i in range(T):
        for kk in range(3):
            if i + kk < T:
                want[i] += mtp[kk] * (lse[i] - z[i, tg[i + kk]])
        if pt[i] >= 0:
            want[i] += pw[0] * (lse[i] - z[i, pt[i]])
    assert torch.allclose(loss, want, atol=1e-4)
    gx, gw = torch.autograd.grad(loss.sum() * 0.5, (x, w))
    gx2, gw2 = torch.autograd.grad(want.sum() * 0.5, (x, w))
    assert torch.allclose(gx, gx2, atol=1e-5) and torch.allclose(gw, gw2, atol=1e-4)
    ev = ref.softcap_ce_eval(x.detach(), w.detach(), tg)
    assert torch.allclose(ev, F.cross_entropy(z.detach(), tg, reduction="none"), atol=1e-4)


def test_yarn():
    y = Yarn(128, 64)
    assert y.angular_freq.shape == (128,) and y.angular_freq[64:].eq(0).all()
    assert y.angular_freq[0] == 1.0 and y.angular_freq[0] == y.angular_freq[1]
    assert y.angular_freq[63].item() == pytest.approx(1 / 1024, rel=1e-5)
    x = torch.randn(8, 2, 128)
    r = y.rotary(x)
    assert torch.equal(r[..., 64:], x[..., 64:])                    # stationary half
    assert torch.allclose(r[0], x[0])                                # position 0: identity
    th = y.angular_freq[0] * 3
    cos, sin = torch.cos(th).bfloat16().float(), torch.sin(th).bfloat16().float()
    assert torch.allclose(r[3, 0, 0], cos * x[3, 0, 0] + sin * x[3, 0, 1], atol=1e-6)
    assert torch.allclose(r[3, 0, 1], cos * x[3, 0, 1] - sin * x[3, 0, 0], atol=1e-6)
    f0 = y.angular_freq.clone()
    y.apply(384, 896)
    assert y.attn_scale == pytest.approx(0.1 * (0.2 * math.log(896 / 384) + 1))
    rot = 384 * f0 / (2 * math.pi)
    s = 384 / 896
    want = f0 * (s + torch.clamp((rot - 1) / 31, 0, 1) * (1 - s))
    assert torch.allclose(y.angular_freq, want)
    yp = Yarn(128, 64, paired=True)
    xp = torch.randn(4, 3, 256)
    rp = yp.rotary(xp)
    even, odd = Yarn(128, 64).tables(8)
    cos_e = even[4][None, :]
    assert torch.allclose(rp[2, :, :64:2], cos_e[:, :64:2] * xp[2, :, :64:2] + Yarn(128, 64).tables(8)[1][4][None, :64:2] * xp[2, :, 1:64:2], atol=1e-6)


def test_relu2_mlp_fp8_emulation_close_to_bf16():
    torch.manual_seed(0)
    x = torch.randn(64, 128)
    w1, w2 = torch.randn(512, 128) * 0.05, torch.randn(512, 128) * 0.05
    y_ref = ref.relu2_mlp(x, w1, w2)
    y8, post = ref.relu2_mlp_fp8(x, w1, w2)
    assert (y8.float() - y_ref).abs().max() / y_ref.abs().max() < 0.08
