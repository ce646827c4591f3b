"""Nsight Compute CSV -> kernel times, TFLOPS and launch-list shares (the reference's scripts/ncu_table.py).

    python -m hopper_wgmma.ncu_table LAUNCHES.csv [--flops F] [--labels WORKLOAD.log]

As a library: ``best(csv_text)`` -> {kernel: best microseconds} (best of repeated launches, ncu_table.py:12-19),
``launch_list(csv_text)`` -> [(kernel, launches, total microseconds, share)], ``labels(log_text)`` maps the
``KERNEL <label> <name>`` lines of hopper_wgmma.workload to labels (ncu_table.py:22-29), ``tflops(us, m, n, k)`` =
2mnk / t (ncu_table.py:32-33).
"""
from __future__ import annotations

import argparse
import csv
import io
import re

UNIT_US = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3, "second": 1e6, "s": 1e6}


def _rows(text: str):
  """Rows of an ncu --csv metrics dump that carry gpu__time_duration, as (kernel name, microseconds)."""
  start = text.find('"ID"')
  if start < 0: return
  for r in csv.DictReader(io.StringIO(text[start:])):
    if r.get("Metric Name") != "gpu__time_duration.sum": continue
    name = r["Kernel Name"].split("(")[0].strip()
    if name.startswith("void "): name = name[5:]
    yield name, float(r["Metric Value"].replace(",", "")) * UNIT_US[r["Metric Unit"]]


def best(text: str) -> dict[str, float]:
  out: dict[str, float] = {}
  for name, us in _rows(text):
    out[name] = min(out.get(name, us), us)
  return out


def launch_list(text: str) -> list[tuple[str, int, float, float]]:
  count: dict[str, int] = {}
  total: dict[str, float] = {}
  for name, us in _rows(text):
    count[name] = count.get(name, 0) + 1
    total[name] = total.get(name, 0.0) + us
  all_us = sum(total.values()) or 1.0
  return sorted(((k, count[k], total[k], total[k] / all_us) for k in total), key=lambda r: -r[2])


def labels(text: str) -> dict[str, str]:
  out = {}
  for line in text.splitlines():
    if line.startswith("KERNEL "):
      parts = line.split(maxsplit=2)
      if len(parts) == 3: out[parts[2].strip()] = parts[1]
  return out


def tflops(us: float, m: int, n: int, k: int) -> float:
  return 2 * m * n * k / us / 1e6


def main(argv=None) -> int:
  ap = argparse.ArgumentParser()
  ap.add_argument("csv")
  ap.add_argument("--shape", default="", help="MxNxK to print TFLOPS of each GEMM kernel's best launch")
  ap.add_argument("--match", default="sm100_gemm|nvjet|gemm", help="regex selecting the GEMM kernels for --shape")
  args = ap.parse_args(argv)
  text = open(args.csv).read()
  print(f"{'kernel':70s} {'launches':>8s} {'total us':>12s} {'share':>7s} {'best us':>10s}")
  b = best(text)
  for name, n, tot, share in launch_list(text):
    print(f"{name[:70]:70s} {n:8d} {tot:12.1f} {100 * share:6.1f}% {b[name]:10.2f}")
  if args.shape:
    m, n, k = (int(x) for x in args.shape.split("x"))
    for name, us in sorted(b.items(), key=lambda kv: kv[1]):
      if not re.search(args.match, name): continue
      print(f"TFLOPS {name[:70]:70s} {tflops(us, m, n, k):8.1f}")
  return 0


if __name__ == "__main__":
  raise SystemExit(main())
