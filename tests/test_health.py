"""Failure detection on the host: a rank that raises, a rank that never joins, a rank that stalls, a
heartbeat that stops, a corrupted checkpoint shard.  All ranks are CPU processes or threads."""
import os
import threading
import time

import pytest
import torch
import torch.distributed as dist

from modded_nanogpt_b200.runtime.health import HealthMonitor, RankFailure
from tests.dist_utils import free_port, spawn


def _monitors(world, **kw):
    store = dist.HashStore()
    return [HealthMonitor(r, world, store=store, **kw) for r in range(world)]


def test_all_ranks_progress():
    ms = _monitors(3, step_timeout_s=5.0)
    errs = []

    def run(m):
        try:
            for step in range(5):
                m.pre_step(step)
        except Exception as e:
            errs.append(e)
    ts = [threading.Thread(target=run, args=(m,)) for m in ms]
    [t.start() for t in ts]
    [t.join(20) for t in ts]
    assert not errs


def test_reported_failure_is_seen_before_next_step():
    a, b = _monitors(2, step_timeout_s=5.0)
    with pytest.raises(ValueError):
        with b.guard():
            raise ValueError("loss is nan")
    t0 = time.time()
    with pytest.raises(RankFailure) as e:
        a.pre_step(0)
    assert e.value.ranks == [1] and "loss is nan" in str(e.value) and time.time() - t0 < 1.0
    with pytest.raises(RankFailure):          # sticky
        a.pre_step(1)


def test_rank_that_never_joins_and_rank_that_stalls():
    store = dist.HashStore()
    a = HealthMonitor(0, 2, store=store, step_timeout_s=0.3, beat_timeout_s=0.2)
    time.sleep(0.3)
    with pytest.raises(RankFailure) as e:     # rank 1 never created its monitor
        a.pre_step(0)
    assert e.value.ranks == [1] and "heartbeat" in e.value.reason
    a, b = _monitors(2, step_timeout_s=0.3, beat_timeout_s=10.0)
    b.beat(0)
    a.pre_step(0)
    with pytest.raises(RankFailure) as e:     # rank 1 alive but stuck at step 0
        a.pre_step(1)
    assert e.value.ranks == [1] and "did not reach step 1" in e.value.reason


def test_background_thread_keeps_beating_and_records_peer_loss():
    a, b = _monitors(2, step_timeout_s=1.0, beat_timeout_s=0.4)
    a.start(0.05), b.start(0.05)
    time.sleep(0.6)
    assert a.failure is None and b.failure is None
    b.stop()                                  # rank 1's process "dies": its heartbeat stops
    time.sleep(0.8)
    assert isinstance(a.failure, RankFailure) and a.failure.ranks == [1]
    a.stop()


def _exit_worker(rank, world, port):
    """gloo ranks with a TCPStore monitor: rank 1 leaves between steps; rank 0 must raise RankFailure
    instead of waiting inside the next all-reduce."""
    from modded_nanogpt_b200.runtime.dist import init_distributed
    from modded_nanogpt_b200.runtime.health import HealthMonitor, RankFailure
    init_distributed(accum_base=2, timeout_s=20)
    m = HealthMonitor(rank, world, port=port, step_timeout_s=3.0, beat_timeout_s=1.0).start(0.1)
    x = torch.ones(4)
    try:
        for step in range(4):
            if rank == 1 and step == 2:
                m.stop()
                os._exit(0)                   # no goodbye: the heartbeat simply stops
            m.pre_step(step)
            dist.all_reduce(x)
    except RankFailure as e:
        assert e.ranks == [1] and step == 2 and float(x[0]) == 4.0
        open(os.environ["MNG_TEST_OUT"], "w").write("detected")
        os._exit(0)
    raise AssertionError("rank 0 did not notice the missing peer")


def test_exited_rank_detected_between_steps(tmp_path):
    out = tmp_path / "r0.txt"
    os.environ["MNG_TEST_OUT"] = str(out)
    try:
        spawn(_exit_worker, 2, free_port(), timeout=90)
    except Exception:
        pass                                   # the launcher may report rank 1's early exit
    assert out.read_text() == "detected"


def test_corrupt_checkpoint_is_rejected(tmp_path):
    from modded_nanogpt_b200.utils.checkpoint import load_checkpoint
    good = tmp_path / "state_step000001.pt"
    torch.save(dict(step=1, model={}), good)
    data = good.read_bytes()
    bad = tmp_path / "state_step000002.pt"
    bad.write_bytes(data[: len(data) // 2])
    with pytest.raises(Exception):
        load_checkpoint(None, str(bad))
    other = tmp_path / "state_step000003.pt"
    torch.save([1, 2, 3], other)
    with pytest.raises(ValueError):
        load_checkpoint(None, str(other))
