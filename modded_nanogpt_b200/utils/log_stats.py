"""Statistics over run logs: final validation loss and training time per run, mean / standard deviation, and
one-sided t-tests without scipy (the reference's `analyze_sweep.py` does the same job for its sweep folders).

    python -m modded_nanogpt_b200.utils.log_stats logs/ [--baseline other_logs/] [--target 3.28]

Parses the `step:k/N val_loss:... train_time:...ms` lines that both this framework and the reference print."""
from __future__ import annotations

import argparse
import glob
import math
import os
import re
import statistics

VAL_LINE = re.compile(r"step:(\d+)/(\d+)\s+val_loss:([0-9.]+)\s+train_time:(\d+)ms")


def final_results(log_dir: str) -> list[tuple[str, float, int]]:
    """(file, final val_loss, train_time_ms) of every log in `log_dir` that reached a validation line."""
    rows = []
    for path in sorted(glob.glob(os.path.join(log_dir, "*.txt"))):
        hits = VAL_LINE.findall(open(path, errors="replace").read())
        if hits:
            rows.append((os.path.basename(path), float(hits[-1][2]), int(hits[-1][3])))
    return rows


def _log_beta(a: float, b: float) -> float:
    return math.lgamma(a) + math.lgamma(b) - math.lgamma(a + b)


def reg_inc_beta(a: float, b: float, x: float) -> float:
    """Regularised incomplete beta I_x(a, b) by Lentz's continued fraction."""
    if x <= 0.0:
        return 0.0
    if x >= 1.0:
        return 1.0
    if x > (a + 1) / (a + b + 2):
        return 1.0 - reg_inc_beta(b, a, 1.0 - x)
    tiny, f, c, d = 1e-300, 1.0, 1.0, 0.0
    for i in range(0, 400):
        m = i // 2
        if i == 0:
            num = 1.0
        elif i % 2 == 0:
            num = m * (b - m) * x / ((a + 2 * m - 1) * (a + 2 * m))
        else:
            num = -(a + m) * (a + b + m) * x / ((a + 2 * m) * (a + 2 * m + 1))
        d = 1.0 + num * d
        d = tiny if abs(d) < tiny else d
        d = 1.0 / d
        c = 1.0 + num / c
        c = tiny if abs(c) < tiny else c
        f *= c * d
        if abs(1.0 - c * d) < 1e-12:
            break
    return math.exp(a * math.log(x) + b * math.log1p(-x) - _log_beta(a, b)) * (f - 1.0) / a


def t_cdf(t: float, df: float) -> float:
    """P(T <= t) for Student's t with `df` degrees of freedom."""
    tail = 0.5 * reg_inc_beta(df / 2, 0.5, df / (df + t * t))
    return tail if t < 0 else 1.0 - tail


def one_sample_below(values: list[float], target: float) -> tuple[float, float]:
    """t statistic and one-sided p-value of H1: mean(values) < target (the speedrun acceptance test)."""
    n = len(values)
    if n < 2:
        return float("nan"), float("nan")
    sd = statistics.stdev(values)
    if sd == 0:
        return (-math.inf, 0.0) if values[0] < target else (math.inf, 1.0)
    t = (statistics.fmean(values) - target) / (sd / math.sqrt(n))
    return t, t_cdf(t, n - 1)


def welch(a: list[float], b: list[float]) -> tuple[float, float, float]:
    """Welch's t, degrees of freedom and one-sided p of H1: mean(a) < mean(b)."""
    va, vb = statistics.variance(a) / len(a), statistics.variance(b) / len(b)
    t = (statistics.fmean(a) - statistics.fmean(b)) / math.sqrt(va + vb)
    df = (va + vb) ** 2 / (va ** 2 / (len(a) - 1) + vb ** 2 / (len(b) - 1))
    return t, df, t_cdf(t, df)


def summarise(rows) -> str:
    if not rows:
        return "no finished runs"
    loss, ms = [r[1] for r in rows], [r[2] for r in rows]
    sd = lambda v: statistics.stdev(v) if len(v) > 1 else 0.0
    return (f"n={len(rows)}  val_loss {statistics.fmean(loss):.5f} +- {sd(loss):.5f}  "
            f"train_time {statistics.fmean(ms) / 1e3:.3f}s +- {sd(ms) / 1e3:.3f}s")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("log_dir")
    ap.add_argument("--baseline")
    ap.add_argument("--target", type=float, default=3.28)
    a = ap.parse_args()
    rows = final_results(a.log_dir)
    for name, loss, ms in rows:
        print(f"{name}  val_loss {loss:.5f}  train_time {ms / 1e3:.3f}s")
    print(summarise(rows))
    if len(rows) > 1:
        t, p = one_sample_below([r[1] for r in rows], a.target)
        print(f"H1 mean val_loss < {a.target}: t = {t:.3f}, p = {p:.4g}")
    if a.baseline:
        base = final_results(a.baseline)
        print("baseline:", summarise(base))
        if len(rows) > 1 and len(base) > 1:
            t, df, p = welch([r[2] for r in rows], [r[2] for r in base])
            print(f"H1 train_time below baseline: Welch t = {t:.3f}, df = {df:.1f}, p = {p:.4g}")


if __name__ == "__main__":
    main()
