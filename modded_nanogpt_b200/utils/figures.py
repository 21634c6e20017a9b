"""Loss-curve figures from run logs, written as stand-alone SVG files (no plotting library needed).

    python -m modded_nanogpt_b200.utils.figures out.svg LABEL=logs_dir [LABEL2=other_dir ...] [--x step|time] [--target 3.28]

Every `*.txt` log of a directory contributes its `step:k/N val_loss:... train_time:...ms` lines; the runs of one
directory are averaged point by point (validation steps shared by all of its runs) and drawn as one curve.  The
reference keeps a matplotlib script for the same job next to its track-3 results
(`records/track_3_optimization/make_figures.py`: curves averaged over the runs of an entry, a target line, a legend)."""
from __future__ import annotations

import argparse
import glob
import os
import re

VAL_LINE = re.compile(r"step:(\d+)/(\d+)\s+val_loss:([0-9.]+)\s+train_time:(\d+)ms")
PALETTE = ["#1f77b4", "#ff7f0e", "#2ca02c", "#d62728", "#9467bd", "#8c564b", "#e377c2", "#7f7f7f", "#bcbd22", "#17becf"]


def parse_curve(path: str) -> list[tuple[int, float, float]]:
    """[(step, val_loss, train_time_s)] of one log, in file order."""
    return [(int(s), float(l), int(ms) / 1e3) for s, _, l, ms in VAL_LINE.findall(open(path, errors="replace").read())]


def average_runs(log_dir: str) -> list[tuple[int, float, float]]:
    """Point-wise mean over the runs of a directory, on the validation steps every run reached."""
    runs = [parse_curve(p) for p in sorted(glob.glob(os.path.join(log_dir, "*.txt")))]
    runs = [{s: (l, t) for s, l, t in r} for r in runs if r]
    if not runs:
        return []
    steps = sorted(set.intersection(*(set(r) for r in runs)))
    n = len(runs)
    return [(s, sum(r[s][0] for r in runs) / n, sum(r[s][1] for r in runs) / n) for s in steps]


def _ticks(lo: float, hi: float, n: int = 6) -> list[float]:
    """Round tick positions (1, 2, 2.5 or 5 times a power of ten apart) covering [lo, hi]."""
    import math
    if hi <= lo:
        return [lo]
    raw = (hi - lo) / n
    p = 10.0 ** math.floor(math.log10(raw))
    step = next(b * p for b in (1, 2, 2.5, 5, 10) if b * p >= raw)
    v = math.ceil(lo / step - 1e-9) * step
    out = []
    while v <= hi + 1e-9 * step:
        out.append(round(v, 10))
        v += step
    return out


def render_svg(curves: dict[str, list[tuple[int, float, float]]], x: str = "step", target: float | None = None,
               title: str = "validation loss", y_max: float | None = None) -> str:
    W, H, L, R, T, B = 900, 520, 70, 20, 40, 55
    pts = {k: [((s if x == "step" else t), l) for s, l, t in v] for k, v in curves.items() if v}
    xs = [p[0] for v in pts.values() for p in v] or [0, 1]
    ys = [p[1] for v in pts.values() for p in v if y_max is None or p[1] <= y_max] or [0, 1]
    x0, x1 = min(xs), max(xs)
    y0, y1 = min(ys + ([target] if target is not None else [])), max(ys)
    pad = 0.05 * (y1 - y0 or 1.0)
    y0, y1 = y0 - pad, y1 + pad
    fx = lambda v: L + (v - x0) / (x1 - x0 or 1) * (W - L - R)
    fy = lambda v: T + (y1 - min(max(v, y0), y1)) / (y1 - y0) * (H - T - B)
    o = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" viewBox="0 0 {W} {H}" font-family="sans-serif" font-size="12">',
         f'<rect width="{W}" height="{H}" fill="white"/>', f'<text x="{W / 2}" y="22" text-anchor="middle" font-size="15">{title}</text>']
    for v in _ticks(x0, x1):
        o.append(f'<line x1="{fx(v):.1f}" y1="{T}" x2="{fx(v):.1f}" y2="{H - B}" stroke="#e5e5e5"/>')
        o.append(f'<text x="{fx(v):.1f}" y="{H - B + 18}" text-anchor="middle">{v:g}</text>')
    for v in _ticks(y0, y1):
        o.append(f'<line x1="{L}" y1="{fy(v):.1f}" x2="{W - R}" y2="{fy(v):.1f}" stroke="#e5e5e5"/>')
        o.append(f'<text x="{L - 8}" y="{fy(v) + 4:.1f}" text-anchor="end">{v:g}</text>')
    o.append(f'<rect x="{L}" y="{T}" width="{W - L - R}" height="{H - T - B}" fill="none" stroke="#444"/>')
    o.append(f'<text x="{(L + W - R) / 2}" y="{H - 12}" text-anchor="middle">{"optimizer step" if x == "step" else "training time (s)"}</text>')
    o.append(f'<text x="16" y="{(T + H - B) / 2}" text-anchor="middle" transform="rotate(-90 16 {(T + H - B) / 2})">validation loss</text>')
    if target is not None:
        o.append(f'<line x1="{L}" y1="{fy(target):.1f}" x2="{W - R}" y2="{fy(target):.1f}" stroke="#000" stroke-dasharray="6 4"/>')
        o.append(f'<text x="{W - R - 4}" y="{fy(target) - 5:.1f}" text-anchor="end">target {target:g}</text>')
    for i, (label, v) in enumerate(pts.items()):
        c = PALETTE[i % len(PALETTE)]
        path = " ".join(f"{'M' if j == 0 else 'L'}{fx(px):.1f},{fy(py):.1f}" for j, (px, py) in enumerate(v))
        o.append(f'<path d="{path}" fill="none" stroke="{c}" stroke-width="2"/>')
        for px, py in v:
            o.append(f'<circle cx="{fx(px):.1f}" cy="{fy(py):.1f}" r="2.5" fill="{c}"/>')
        ly = T + 16 + 18 * i
        o.append(f'<line x1="{W - R - 190}" y1="{ly - 4}" x2="{W - R - 165}" y2="{ly - 4}" stroke="{c}" stroke-width="2"/>')
        o.append(f'<text x="{W - R - 160}" y="{ly}">{label} (final {v[-1][1]:.4f})</text>')
    o.append("</svg>")
    return "\n".join(o)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("series", nargs="+", help="LABEL=log_dir")
    ap.add_argument("--x", default="step", choices=["step", "time"])
    ap.add_argument("--target", type=float, default=None)
    ap.add_argument("--y-max", type=float, default=None)
    a = ap.parse_args()
    curves = {}
    for s in a.series:
        label, _, d = s.partition("=")
        curves[label] = average_runs(d or label)
    with open(a.out, "w") as f:
        f.write(render_svg(curves, a.x, a.target, y_max=a.y_max))
    print(f"wrote {a.out}: " + ", ".join(f"{k}: {len(v)} points" for k, v in curves.items()))


if __name__ == "__main__":
    main()
