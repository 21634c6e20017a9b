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


def test_loss_curve_figures(tmp_path):
    from modded_nanogpt_b200.utils import figures as fg
    for name, off in (("a", 0.0), ("b", 0.01)):
        d = tmp_path / name
        d.mkdir()
        for i in range(3):
            lines = [f"step:{s}/1285 val_loss:{10.8 - 7.5 * (s / 1285) ** 0.5 + off + 0.001 * i:.4f} train_time:{60 * s}ms step_avg:60.00ms"
                     for s in (0, 250, 500, 750, 1000, 1250, 1285)]
            (d / f"run{i}.txt").write_text("code\n" + "\n".join(lines) + "\n")
    (tmp_path / "a" / "run2.txt").write_text("step:0/1285 val_loss:10.8 train_time:0ms step_avg:0ms\n")   # a run cut short
    ca = fg.average_runs(str(tmp_path / "a"))
    assert [s for s, *_ in ca] == [0]                                   # only steps every run reached are averaged
    (tmp_path / "a" / "run2.txt").unlink()
    ca, cb = fg.average_runs(str(tmp_path / "a")), fg.average_runs(str(tmp_path / "b"))
    assert [s for s, *_ in ca] == [0, 250, 500, 750, 1000, 1250, 1285] and abs(ca[-1][1] - (3.3 + 0.0005)) < 1e-3
    assert abs(cb[-1][1] - ca[-1][1] - 0.0095) < 1e-3 and ca[-1][2] == 77.1
    assert fg._ticks(0, 1285) == [0, 250, 500, 750, 1000, 1250] and fg._ticks(3.2, 3.4, 4) == [3.2, 3.25, 3.3, 3.35, 3.4]
    svg = fg.render_svg({"run a": ca, "run b": cb}, x="time", target=3.28, y_max=6.0)
    assert svg.startswith("<svg") and svg.count("<path") == 2 and "target 3.28" in svg and "run b (final" in svg
    import xml.dom.minidom
    xml.dom.minidom.parseString(svg)                                    # well-formed
