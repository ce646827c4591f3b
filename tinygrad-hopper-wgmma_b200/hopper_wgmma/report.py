"""Measurement tables from the workload's output (the reference's scripts/report.py for B200).

    python -m hopper_wgmma.report sweep [--reps 30] > sweep.log        # run the shape sweep + ladders on this GPU
    python -m hopper_wgmma.report summary sweep.log [...] > summary.md  # markdown tables from TIME lines

``sweep`` runs hopper_wgmma.workload in-process for every shape of ladder.SWEEP_SHAPES with the configs of
ladder.SWEEP_CONFIGS, and the ladder (ladder.LADDER) at 4096 and 8192, each config timed interleaved with cuBLAS on
the same inputs (CUDA events, median of --reps launches, a 256 MiB L2-flush write before every timed launch, which
also keeps the host's launch submission ahead of the GPU for the microsecond-scale shapes). ``summary`` keeps, per shape, the best config (as the
reference's report does, results/summary.md) and prints TFLOPS, % of cuBLAS and % of the measured B200 peak.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import sys
from pathlib import Path


def _time_lines(text: str):
  for line in text.splitlines():
    if line.startswith("TIME "):
      yield json.loads(line[5:])


def sweep(reps: int, out) -> None:
  from . import workload
  from .ladder import LADDER, SWEEP_CONFIGS, SWEEP_SHAPES
  jobs = [((4096, 4096, 4096), list(LADDER)), ((8192, 8192, 8192), list(LADDER))]
  jobs += [(shape, SWEEP_CONFIGS) for shape in SWEEP_SHAPES]
  for (m, n, k), names in jobs:
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
      workload.main(["--shape", f"{m}x{n}x{k}", "--configs", ",".join(names), "--reps", str(reps), "--torch",
                     "--check", "--time", "--flush"])
    tag = "ladder" if names == list(LADDER) else "sweep"
    for line in buf.getvalue().splitlines():
      if line.startswith(("TIME ", "CHECK ", "SKIP ")):
        print(f"{line} " if line.startswith("TIME ") else line, file=out, flush=True)
    print(f"DONE {tag} {m}x{n}x{k}", file=out, flush=True)


def summary(texts: list[str], peak_tflops: float) -> str:
  recs = [r for t in texts for r in _time_lines(t) if r.get("label") != "cublas"]
  by_shape: dict[tuple, list] = {}
  for r in recs: by_shape.setdefault(tuple(r["shape"]), []).append(r)
  out = ["| M×N×K | best config | µs (median) | TFLOPS | cuBLAS TFLOPS | % of cuBLAS | % of peak |",
         "|---|---|---:|---:|---:|---:|---:|"]
  for shape in sorted(by_shape, key=lambda s: s[0] * s[1] * s[2]):
    best = max(by_shape[shape], key=lambda r: r.get("pct_cublas", 0.0))
    out.append(f"| {shape[0]}×{shape[1]}×{shape[2]} | {best['label']} | {best['us_median']:.1f} | {best['tflops']:.0f} | "
               f"{best['cublas_tflops']:.0f} | {best['pct_cublas']:.1f}% | {100 * best['tflops'] / peak_tflops:.1f}% |")
  out.append("")
  for shape in sorted(by_shape, key=lambda s: s[0] * s[1] * s[2]):
    rows = by_shape[shape]
    out.append(f"**{shape[0]}×{shape[1]}×{shape[2]}** — " + ", ".join(
      f"{r['label']} {r['pct_cublas']:.1f}%" for r in sorted(rows, key=lambda r: -r.get("pct_cublas", 0.0))))
    out.append("")
  return "\n".join(out)


def main(argv=None) -> int:
  ap = argparse.ArgumentParser()
  sub = ap.add_subparsers(dest="cmd", required=True)
  a = sub.add_parser("sweep")
  a.add_argument("--reps", type=int, default=30)
  b = sub.add_parser("summary")
  b.add_argument("logs", nargs="+")
  b.add_argument("--peak", type=float, default=0.0, help="TFLOPS; default: MEASURED_PEAKS.json bf16_tflops or 1590")
  args = ap.parse_args(argv)
  if args.cmd == "sweep":
    sweep(args.reps, sys.stdout)
    return 0
  peak = args.peak
  if not peak:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    peak = json.loads(p.read_text())["bf16_tflops"] if p.exists() else 1590.0
  print(summary([Path(f).read_text() for f in args.logs], peak))
  return 0


if __name__ == "__main__":
  raise SystemExit(main())
