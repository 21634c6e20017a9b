"""Track-2 model: forward/backward on CPU, reference key layout round trip, schedule table."""
import math

import pytest
import torch

from modded_nanogpt_b200.config import track2_schedule, track2_stages
from modded_nanogpt_b200.models.gpt import ForwardScheduleConfig
from modded_nanogpt_b200.models.gpt_medium import GPTMedium


def _tiny():
    torch.manual_seed(0)
    return GPTMedium(vocab_size=500, num_layers=16, num_heads=2, head_dim=32, model_dim=64, max_seq_len=512)


def test_track2_forward_backward_and_layout():
    m = _tiny()
    T = 128
    ids = torch.randint(0, 500, (T,), dtype=torch.int32)
    tg = torch.randint(0, 500, (T,))
    cu = torch.tensor([0, 50, T, T], dtype=torch.int32)
    sc = ForwardScheduleConfig(torch.tensor([1.0, 0.5]), torch.tensor([0.0]), 32, 64, 128)
    loss = m(ids, tg, cu, None, sc)
    assert loss.shape == (T,) and loss.mean().item() == pytest.approx(1.5 * math.log(512), rel=0.03)
    loss.sum().backward()
    assert all(p.grad is not None for p in m.parameters())
    assert {p.label for p in m.parameters()} == set(m.param_table()) == set(m.WORK_ORDER)
    sd = m.reference_state_dict()
    assert sd["lm_head.weight"].shape == (512, 64) and sd["blocks.3.attn.qkvo_w"].shape == (256, 64)
    assert sd["blocks.15.mlp.c_proj"].shape == (256, 64) and "blocks.7.attn.value_embed_gate.weight" not in sd
    assert "blocks.12.attn.value_embed_gate.weight" in sd and len([k for k in sd if k.startswith("value_embeds.")]) == 5
    m2 = _tiny()
    with torch.no_grad():
        for p in m2.parameters():
            p.add_(0.5)
    m2.load_reference_state_dict({"_orig_mod." + k: v for k, v in sd.items()})
    m.eval(), m2.eval()
    with torch.no_grad():
        assert torch.allclose(m(ids, tg, cu, None, sc), m2(ids, tg, cu, None, sc), atol=1e-5)


def test_track2_schedule():
    s = track2_schedule()
    assert s.total_steps == 4740 and len(track2_stages()) == 13 and s.split_step == 785
    st, _ = s.lookup(0)
    assert (st.batch_size, st.window_sizes) == (131072, (1, 3))
    st, _ = s.lookup(1600)
    assert (st.batch_size, st.window_sizes) == (524288, (7, 15))
    st, _ = s.lookup(4700)
    assert (st.batch_size, st.window_sizes) == (524288, (11, 23))
    assert s.get_lr(0) == 1.0 and s.get_lr(1300) == 2.0 and s.get_lr(4700) == pytest.approx(0.1)
    assert s.mtp_weights[0] == [1.0, 0.5, 0.25] and s.mtp_weights[800] == [1.0]
