"""Measurement tables from the workload's output (the reference's scripts/report.py for B200).

    python -m hopper_wgmma.report sweep [--reps 30] > sweep.log        # run the shape sweep + ladders on this GPU
    python -m hopper_wgmma.report ncu-sweep [--reps 5] > ncu.log        # the same, timed by Nsight Compute
    python -m hopper_wgmma.report summary sweep.log [...] > summary.md  # markdown tables from TIME lines
    python -m hopper_wgmma.report ncu-summary ncu.log [...]             # the same from an ncu-sweep's NCU lines

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
    if line.startswith(("TIME ", "NCU ")):
      rec = json.loads(line.split(" ", 1)[1])
      rec.setdefault("us_median", rec.get("us_best"))
      yield rec


def sweep(reps: int, out) -> None:
  from . import workload
  from .ladder import LADDER, SWEEP_CONFIGS, SWEEP_SHAPES
  ladder = list(LADDER) + ["pair_wide_hilbert"]   # the reference's rungs, plus B200's wide pair tiles
  jobs = [((4096, 4096, 4096), ladder), ((8192, 8192, 8192), ladder)]
  jobs += [(shape, SWEEP_CONFIGS) for shape in SWEEP_SHAPES]
  for (m, n, k), names in jobs:
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
      workload.main(["--shape", f"{m}x{n}x{k}", "--configs", ",".join(names), "--reps", str(reps), "--torch",
                     "--check", "--time", "--flush"])
    tag = "ladder" if set(LADDER) <= set(names) else "sweep"
    for line in buf.getvalue().splitlines():
      if line.startswith(("TIME ", "CHECK ", "SKIP ")):
        print(f"{line} " if line.startswith("TIME ") else line, file=out, flush=True)
    print(f"DONE {tag} {m}x{n}x{k}", file=out, flush=True)


def ncu_sweep(reps: int, out, jobs=None) -> None:
  """The reference's measurement protocol (modal_runner.py:42, 90-94; ncu_table.py:12-19): every config's kernel
  time is Nsight Compute's gpu__time_duration.sum, best of ``reps`` launches, next to cuBLAS on the same inputs.
  One workload process per shape; the plain command runs first and must exit 0, then the same command runs under
  ncu collecting only that one metric (a single pass, clocks not locked). Our launches are attributed to configs in
  launch order (each config: one checked launch, then ``reps``)."""
  import os
  import subprocess
  import tempfile

  from . import ncu_table
  from .ladder import LADDER, SWEEP_CONFIGS, SWEEP_SHAPES
  if jobs is None:
    ladder = list(LADDER) + ["pair_wide_hilbert"]   # the reference's rungs, plus B200's wide pair tiles
    jobs = [((4096, 4096, 4096), ladder), ((8192, 8192, 8192), ladder)]
    jobs += [(shape, SWEEP_CONFIGS) for shape in SWEEP_SHAPES]
  env = dict(os.environ, PYTHONPATH=str(Path(__file__).resolve().parents[1]))
  for (m, n, k), names in jobs:
    cmd = [sys.executable, "-m", "hopper_wgmma.workload", "--shape", f"{m}x{n}x{k}", "--configs", ",".join(names),
           "--reps", str(reps), "--torch"]
    plain = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if plain.returncode != 0:
      print(f"ERROR {m}x{n}x{k}: plain run exited {plain.returncode}: {plain.stderr[-300:]}", file=out, flush=True)
      continue
    ran = [ln.split()[1] for ln in plain.stdout.splitlines() if ln.startswith("KERNEL ") and ln.split()[1] != "cublas"]
    with tempfile.TemporaryDirectory() as td:
      log = Path(td) / "launches.csv"
      prof = subprocess.run(["ncu", "--metrics", "gpu__time_duration.sum", "--clock-control", "none",
                             "-k", "regex:sm100_gemm|nvjet|gemm|xmma|cutlass", "--csv", "--log-file", str(log), *cmd],
                            capture_output=True, text=True, env=env)
      text = log.read_text() if log.exists() else ""
    if prof.returncode != 0 or not text:
      tail = " | ".join((prof.stdout + prof.stderr).strip().splitlines()[-4:])
      print(f"ERROR {m}x{n}x{k}: ncu exited {prof.returncode}: {tail[-400:]}", file=out, flush=True)
      continue
    rows = list(ncu_table._rows(text))
    ours = [us for name, us in rows if "sm100_gemm" in name]
    cub = [us for name, us in rows if "sm100_gemm" not in name]
    per = reps + 1
    cub_best = min(cub) if cub else None
    for i, label in enumerate(ran):
      g = ours[i * per:(i + 1) * per]
      if len(g) != per: break
      best = min(g)
      rec = {"label": label, "shape": [m, n, k], "us_best": round(best, 2), "tflops": round(2 * m * n * k / best / 1e6, 1)}
      if cub_best:
        rec.update(cublas_us_best=round(cub_best, 2), cublas_tflops=round(2 * m * n * k / cub_best / 1e6, 1),
                   pct_cublas=round(100.0 * cub_best / best, 1))
      print("NCU " + json.dumps(rec), file=out, flush=True)


def _ncu_lines(text: str):
  for line in text.splitlines():
    if line.startswith("NCU "): yield json.loads(line[4:])


def ncu_summary(texts: list[str], peak_tflops: float) -> str:
  """Markdown table of an ``ncu-sweep`` log: per shape the config with the best ratio to cuBLAS (kernel time =
  best-of-reps gpu__time_duration), then every config's ratio, best first."""
  by_shape: dict[tuple, list] = {}
  for t in texts:
    for r in _ncu_lines(t): by_shape.setdefault(tuple(r["shape"]), []).append(r)
  out = ["| M×N×K | best config | µs | TFLOPS | cuBLAS TFLOPS | % of cuBLAS | % of peak |",
         "|---|---|---:|---:|---:|---:|---:|"]
  order = sorted(by_shape, key=lambda s: s[0] * s[1] * s[2])
  for shape in order:
    best = max(by_shape[shape], key=lambda r: r.get("pct_cublas", 0.0))
    out.append(f"| {shape[0]}×{shape[1]}×{shape[2]} | {best['label']} | {best['us_best']:.1f} | {best['tflops']:.0f} | "
               f"{best['cublas_tflops']:.0f} | {best['pct_cublas']:.1f}% | {100 * best['tflops'] / peak_tflops:.1f}% |")
  out.append("")
  for shape in order:
    rows = sorted(by_shape[shape], key=lambda r: -r.get("pct_cublas", 0.0))
    out.append(f"**{shape[0]}×{shape[1]}×{shape[2]}** — " + ", ".join(f"{r['label']} {r['pct_cublas']:.1f}%" for r in rows))
    out.append("")
  return "\n".join(out)


def summary(texts: list[str], peak_tflops: float) -> str:
  recs = [r for t in texts for r in _time_lines(t) if r.get("label") != "cublas"]
  by_shape: dict[tuple, list] = {}
  for r in recs: by_shape.setdefault(tuple(r["shape"]), []).append(r)
  out = ["| M×N×K | best config | µs | TFLOPS | cuBLAS TFLOPS | % of cuBLAS | % of peak |",
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
  c = sub.add_parser("ncu-sweep")
  c.add_argument("--reps", type=int, default=5)
  c.add_argument("--shapes", default="", help="comma-separated MxNxK list (default: ladder shapes + the sweep)")
  c.add_argument("--configs", default="", help="comma-separated config names (default: per-shape defaults)")
  b = sub.add_parser("summary")
  b.add_argument("logs", nargs="+")
  b.add_argument("--peak", type=float, default=0.0, help="TFLOPS; default: MEASURED_PEAKS.json bf16_tflops or 1590")
  d = sub.add_parser("ncu-summary")
  d.add_argument("logs", nargs="+")
  d.add_argument("--peak", type=float, default=0.0, help="TFLOPS; default: MEASURED_PEAKS.json bf16_tflops or 1590")
  args = ap.parse_args(argv)
  if args.cmd == "sweep":
    sweep(args.reps, sys.stdout)
    return 0
  if args.cmd == "ncu-sweep":
    jobs = None
    if args.shapes:
      from .ladder import SWEEP_CONFIGS
      names = args.configs.split(",") if args.configs else SWEEP_CONFIGS
      jobs = [(tuple(int(x) for x in sh.split("x")), names) for sh in args.shapes.split(",")]
    ncu_sweep(args.reps, sys.stdout, jobs)
    return 0
  peak = args.peak
  if not peak:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    peak = json.loads(p.read_text())["bf16_tflops"] if p.exists() else 1590.0
  fn = ncu_summary if args.cmd == "ncu-summary" else summary
  print(fn([Path(f).read_text() for f in args.logs], peak))
  return 0


if __name__ == "__main__":
  raise SystemExit(main())
