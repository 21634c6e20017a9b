"""Table-driven checks of the track-1 schedule at every boundary."""
import pytest

from modded_nanogpt_b200.config import Hyperparameters, TrainingSchedule, max_num_docs, track1_schedule, track1_stages


def test_boundaries_and_split():
    s = track1_schedule()
    assert s.boundaries == [(0, 423), (423, 847), (847, 1270), (1270, 1285)]
    assert s.total_steps == 1285 and s.split_step == 847
    assert s.transition_steps() == [423, 847, 1270]


@pytest.mark.parametrize("step,batch,seq,ws", [
    (0, 131072, 896, (1, 3)), (422, 131072, 896, (1, 3)), (423, 262144, 2048, (3, 7)),
    (846, 262144, 2048, (3, 7)), (847, 393216, 2048, (5, 11)), (1269, 393216, 2048, (5, 11)),
    (1270, 393216, 2048, (6, 13)), (1285, 393216, 2048, (6, 13))])
def test_stage_lookup(step, batch, seq, ws):
    st, _ = track1_schedule().lookup(step)
    assert (st.batch_size, st.train_max_seq_len, st.window_sizes) == (batch, seq, ws)


def test_lr_schedule():
    s = track1_schedule()
    assert s.get_lr(0) == 1.0 and s.get_lr(423) == 1.52
    cd = int(1270 * 0.4)
    assert cd == 508 and s.get_lr(507) == 1.52
    t = (600 - cd) / (1270 - cd)
    assert s.get_lr(600) == pytest.approx(1.52 * (1 - t) + 0.15 * t)
    assert s.get_lr(1270) == pytest.approx(0.15) and s.get_lr(1284) == pytest.approx(0.15)


def test_mtp_and_prefix_weights():
    s = track1_schedule()
    assert s.mtp_weights[0] == [1.0, 0.5, 0.25]
    assert s.mtp_weights[422][2] == pytest.approx(0.25 * (1 - 422 / 423))
    assert len(s.mtp_weights[423]) == 2 and s.mtp_weights[423] == [1.0, 0.5]
    assert s.mtp_weights[847] == [1.0] and s.mtp_weights[1285] == [1.0]
    assert s.prefix_weights[0] == 0.25 and s.prefix_weights[423] == 0.25
    assert s.prefix_weights[635] == pytest.approx(0.25 * (1 - (635 - 423) / 424))
    assert s.prefix_weights[847] == 0.0


def test_muon_momentum():
    s = track1_schedule()
    assert s.muon_momentum(0) == pytest.approx(0.85) and s.muon_momentum(150) == pytest.approx(0.90)
    assert s.muon_momentum(300) == pytest.approx(0.95) and s.muon_momentum(1235) == pytest.approx(0.95)
    assert s.muon_momentum(1260) == pytest.approx(0.90) and s.muon_momentum(1285) == pytest.approx(0.85)


def test_max_num_docs():
    assert (max_num_docs(16384), max_num_docs(32768), max_num_docs(49152)) == (64, 96, 128)
    assert max_num_docs(262144) == 896 and max_num_docs(256) == 128


def test_bad_durations():
    st = track1_stages()
    st[0].duration = 0.5
    with pytest.raises(AssertionError):
        TrainingSchedule(st, 1270, 15)


def test_env_overrides(monkeypatch):
    monkeypatch.setenv("DATA_PATH", "/data/x")
    monkeypatch.setenv("DISABLE_FP8", "1")
    hp = Hyperparameters()
    assert hp.train_files == "/data/x/data/fineweb10B/fineweb_train_*.bin" and hp.disable_fp8
