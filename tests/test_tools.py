"""Corpus sharder and log statistics."""
import math
import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "data"))


def test_shard_writer_splits_and_round_trips(tmp_path):
    import fineweb
    from modded_nanogpt_b200.data.shards import read_shard
    w = fineweb.ShardWriter(str(tmp_path), "fineweb", shard_size=1000)
    rng = np.random.default_rng(0)
    docs = [np.concatenate([[fineweb.EOT], rng.integers(0, 50000, rng.integers(5, 400))]).astype(np.uint16) for _ in range(20)]
    for d in docs:
        w.add(d)
    paths = w.close()
    assert os.path.basename(paths[0]) == "fineweb_val_000000.bin" and os.path.basename(paths[1]) == "fineweb_train_000001.bin"
    got = np.concatenate([read_shard(p).numpy() for p in paths])
    assert np.array_equal(got, np.concatenate(docs))
    assert all(len(read_shard(p)) == 1000 for p in paths[:-1])


def test_log_stats(tmp_path):
    from modded_nanogpt_b200.utils import log_stats as ls
    for i, (loss, ms) in enumerate([(3.2781, 75100), (3.2795, 75300), (3.2774, 74900), (3.2790, 75250)]):
        (tmp_path / f"run{i}.txt").write_text(f"junk\nstep:100/1285 val_loss:3.9 train_time:6000ms step_avg:60ms\n"
                                              f"step:1285/1285 val_loss:{loss} train_time:{ms}ms step_avg:58.5ms\n")
    rows = ls.final_results(str(tmp_path))
    assert len(rows) == 4 and rows[0][1:] == (3.2781, 75100)
    t, p = ls.one_sample_below([r[1] for r in rows], 3.28)
    assert t < 0 and 0 < p < 0.05
    assert abs(ls.t_cdf(0.0, 7) - 0.5) < 1e-12 and abs(ls.t_cdf(2.0, 10) - 0.963306) < 1e-4 and abs(ls.t_cdf(-1.0, 3) - 0.195501) < 1e-4
    t, df, p = ls.welch([1.0, 1.1, 0.9, 1.05], [1.5, 1.6, 1.4, 1.55])
    assert t < 0 and p < 0.01 and 3 < df <= 6 and not math.isnan(p)
