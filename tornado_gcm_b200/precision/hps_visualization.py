"""Plots of HPS results — reference ``precision/hps_visualization.py:52-277``.

Sensitivity bars (log scale, coloured by recommendation), the zone
partition, the eigengap spectrum with the chosen K, and K against spectral
resolution.  The figures are written as self-contained SVG (plain text: no
plotting library or graphics stack is needed); a requested ``.png`` path is
written with the ``.svg`` suffix.  Every function returns the path it wrote.
"""

from __future__ import annotations

import html
import math
import pathlib
from typing import Optional, Sequence

from tornado_gcm_b200.precision.sensitivity import SensitivityMap
from tornado_gcm_b200.precision.zone_discovery import DiscoveryResult

_COLORS = {"critical": "#d62728", "moderate": "#ff7f0e", "tolerant": "#2ca02c", "invalid_baseline": "#7f7f7f",
           "FP64": "#d62728", "FP32": "#ff7f0e", "TF32": "#bcbd22", "BF16": "#2ca02c"}
_W, _H, _M = 720, 420, 60


class _Svg:
    def __init__(self, title: str):
        self.parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{_W}" height="{_H}" '
                      f'font-family="sans-serif" font-size="11">',
                      f'<rect width="{_W}" height="{_H}" fill="white"/>',
                      f'<text x="{_W / 2}" y="22" text-anchor="middle" font-size="14">{html.escape(title)}</text>']

    def rect(self, x, y, w, h, fill):
        self.parts.append(f'<rect x="{x:.1f}" y="{y:.1f}" width="{max(w, 0):.1f}" height="{max(h, 0):.1f}" '
                          f'fill="{fill}"/>')

    def line(self, x0, y0, x1, y1, stroke="black", dash=None):
        d = f' stroke-dasharray="{dash}"' if dash else ""
        self.parts.append(f'<line x1="{x0:.1f}" y1="{y0:.1f}" x2="{x1:.1f}" y2="{y1:.1f}" stroke="{stroke}"{d}/>')

    def text(self, x, y, s, anchor="middle", rotate=None, size=11):
        r = f' transform="rotate({rotate} {x:.1f} {y:.1f})"' if rotate is not None else ""
        self.parts.append(f'<text x="{x:.1f}" y="{y:.1f}" text-anchor="{anchor}" font-size="{size}"{r}>'
                          f'{html.escape(str(s))}</text>')

    def circle(self, x, y, r, fill):
        self.parts.append(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="{r}" fill="{fill}"/>')

    def axes(self, xlabel: str, ylabel: str):
        self.line(_M, _H - _M, _W - 20, _H - _M)
        self.line(_M, 40, _M, _H - _M)
        self.text((_W + _M) / 2, _H - 12, xlabel)
        self.text(16, (_H - _M + 40) / 2, ylabel, rotate=-90)

    def write(self, path) -> pathlib.Path:
        p = pathlib.Path(path)
        if p.suffix.lower() != ".svg":
            p = p.with_suffix(".svg")
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text("\n".join(self.parts + ["</svg>"]), encoding="utf-8")
        return p


def _log_y(v: float, lo: float, hi: float) -> float:
    v = min(max(v, lo), hi)
    f = (math.log10(v) - math.log10(lo)) / max(math.log10(hi) - math.log10(lo), 1e-12)
    return _H - _M - f * (_H - _M - 40)


def _bars(svg: _Svg, names: Sequence[str], values: Sequence[float], colors: Sequence[str]):
    finite = [v for v in values if math.isfinite(v) and v > 0]
    lo = min(finite) / 10 if finite else 1e-12
    hi = max(finite) * 10 if finite else 1.0
    n = max(len(names), 1)
    bw = (_W - _M - 40) / n
    for i, (nm, v, c) in enumerate(zip(names, values, colors)):
        x = _M + 10 + i * bw
        y = _log_y(v if math.isfinite(v) and v > 0 else hi, lo, hi)
        svg.rect(x, y, bw * 0.7, _H - _M - y, c)
        svg.text(x + bw * 0.35, _H - _M + 12, nm[-18:], rotate=30, anchor="start", size=9)
    for e in range(int(math.floor(math.log10(lo))), int(math.ceil(math.log10(hi))) + 1):
        y = _log_y(10.0 ** e, lo, hi)
        svg.text(_M - 4, y + 3, f"1e{e}", anchor="end", size=9)
    for thr in (0.1, 1e-3):
        if lo < thr < hi:
            y = _log_y(thr, lo, hi)
            svg.line(_M, y, _W - 20, y, "#555", "4 3")


def plot_sensitivity_bar(smap: SensitivityMap, output_path, title: str = "Module Precision Sensitivity (HPS Level-1)"):
    rec = smap.get_zone_recommendation()
    ranked = smap.sensitivity_ranking
    svg = _Svg(title)
    svg.axes("module", "drift (log)")
    _bars(svg, [n for n, _ in ranked], [float(d) for _, d in ranked], [_COLORS[rec[n]] for n, _ in ranked])
    return svg.write(output_path)


def plot_zone_partition(result: DiscoveryResult, smap: SensitivityMap, output_path,
                        title: str = "Auto-Discovered Zone Partition (HPS Level-2)"):
    names, vals, cols = [], [], []
    for z in sorted(result.zones, key=lambda z: z.sensitivity_centroid, reverse=True):
        for m in z.members:
            names.append(f"Z{z.zone_id}:{m}")
            vals.append(float(smap.modules[m].drift) if m in smap.modules else float("nan"))
            cols.append(_COLORS.get(z.recommended_precision, "#1f77b4"))
    svg = _Svg(title)
    svg.axes("zone:module", "drift (log)")
    _bars(svg, names, vals, cols)
    return svg.write(output_path)


def _line_plot(svg: _Svg, xs: Sequence[float], ys: Sequence[float], mark: Optional[int] = None):
    if not xs:
        return
    x0, x1 = min(xs), max(xs)
    y0, y1 = min(ys), max(ys)
    sx = lambda x: _M + (x - x0) / max(x1 - x0, 1e-12) * (_W - _M - 40)
    sy = lambda y: _H - _M - (y - y0) / max(y1 - y0, 1e-12) * (_H - _M - 60)
    for i in range(len(xs) - 1):
        svg.line(sx(xs[i]), sy(ys[i]), sx(xs[i + 1]), sy(ys[i + 1]), "#1f77b4")
    for i, (x, y) in enumerate(zip(xs, ys)):
        svg.circle(sx(x), sy(y), 4 if i == mark else 2.5, "#d62728" if i == mark else "#1f77b4")
        svg.text(sx(x), _H - _M + 14, f"{x:g}", size=9)
    svg.text(_M - 4, sy(y0) + 3, f"{y0:.3g}", anchor="end", size=9)
    svg.text(_M - 4, sy(y1) + 3, f"{y1:.3g}", anchor="end", size=9)


def plot_eigengap(result: DiscoveryResult, output_path, title: str = "Eigengap Analysis (K Selection)"):
    svg = _Svg(title)
    svg.axes("k", "λ_k − λ_(k−1)")
    gaps = list(result.eigengaps)
    _line_plot(svg, [float(i + 1) for i in range(len(gaps))], gaps, mark=result.k - 1 if result.k >= 1 else None)
    return svg.write(output_path)


def plot_multi_resolution_scaling(resolution_data: dict, output_path,
                                  title: str = "Zone Count K vs Spectral Resolution L_max"):
    items = sorted(resolution_data.items(), key=lambda kv: kv[1][0])
    svg = _Svg(title)
    svg.axes("L_max", "K")
    _line_plot(svg, [float(v[0]) for _, v in items], [float(v[1]) for _, v in items])
    return svg.write(output_path)


def plot_hps_results(smap: SensitivityMap, result: DiscoveryResult, output_dir,
                     resolution_data: Optional[dict] = None) -> list:
    out = pathlib.Path(output_dir)
    paths = [plot_sensitivity_bar(smap, out / "hps_sensitivity.svg"),
             plot_zone_partition(result, smap, out / "hps_zones.svg"),
             plot_eigengap(result, out / "hps_eigengap.svg")]
    if resolution_data:
        paths.append(plot_multi_resolution_scaling(resolution_data, out / "hps_k_scaling.svg"))
    return paths
