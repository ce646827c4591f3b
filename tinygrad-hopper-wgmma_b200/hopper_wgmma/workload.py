"""Launch (and optionally time) GEMM configs on one shape: the reference's measurement workload
(scripts/ncu_workload.py) for B200.

    python -m hopper_wgmma.workload --shape 4096 --configs tma_store,hilbert --reps 5 --torch --check [--time]

  --shape MxNxK   problem size (or a single N for a square GEMM)
  --configs a,b   names from ladder.LADDER / SWEEP / EXTRA / B200 (or "all"), optionally with a split-K suffix
                  (``cta_n128@sk2``); configs invalid for the shape print SKIP
  --torch         also launch cuBLAS (torch.matmul) on the same inputs
  --check         compare each config once, on NaN-poisoned output, with the fp32 product of the same bf16 inputs
                  (cuBLAS in fp32, TF32 off) before the timed launches
  --time          time each config with CUDA events (best and mean of --reps launches, after warm-up) and print
                  one JSON line per config; without it the script only launches, for Nsight Compute to time
  --flush         with --time: rewrite a 256 MiB buffer between launches so every launch starts with a cold L2

Output lines: ``CHECK <label> rel=... max|ref|=... ok|MISMATCH``, ``KERNEL <label> <kernel>``, ``SKIP <label>: ...``
(the reference's formats, scripts/ncu_workload.py:63-69) and, with --time, ``TIME {json}``.
"""
from __future__ import annotations

import argparse
import json
import statistics


def parse_shape(text: str) -> tuple[int, int, int]:
  dims = [int(x) for x in text.lower().split("x")]
  if len(dims) == 1: dims *= 3
  if len(dims) != 3: raise SystemExit(f"bad --shape {text!r}")
  return dims[0], dims[1], dims[2]


def _time_pair(fn, ref_fn, reps: int, warmup: int, flush=None) -> tuple[list[float], list[float]]:
  """Alternate ``fn`` and ``ref_fn`` launch by launch (each timed alone with CUDA events), so that both see the same
  clock and power state; returns both lists of microseconds."""
  import torch
  for _ in range(warmup):
    fn()
    ref_fn()
  ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(reps)]
  torch.cuda.synchronize()
  for e in ev:
    if flush is not None: flush.zero_()
    e[0].record()
    fn()
    e[1].record()
    if flush is not None: flush.zero_()
    e[2].record()
    ref_fn()
    e[3].record()
  torch.cuda.synchronize()
  return [e[0].elapsed_time(e[1]) * 1e3 for e in ev], [e[2].elapsed_time(e[3]) * 1e3 for e in ev]


def _time(fn, reps: int, warmup: int, flush=None) -> tuple[float, float]:
  import torch
  for _ in range(warmup): fn()
  starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
  ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
  torch.cuda.synchronize()
  for i in range(reps):
    if flush is not None: flush.zero_()
    starts[i].record()
    fn()
    ends[i].record()
  torch.cuda.synchronize()
  us = [s.elapsed_time(e) * 1e3 for s, e in zip(starts, ends)]
  return min(us), sum(us) / len(us)


def main(argv=None) -> int:
  import torch

  from .ladder import B200, EXTRA, LADDER, SWEEP, build, lookup
  ap = argparse.ArgumentParser()
  ap.add_argument("--shape", default="4096")
  ap.add_argument("--configs", default="")
  ap.add_argument("--reps", type=int, default=5)
  ap.add_argument("--warmup", type=int, default=3)
  ap.add_argument("--torch", action="store_true")
  ap.add_argument("--check", action="store_true")
  ap.add_argument("--time", action="store_true")
  ap.add_argument("--flush", action="store_true")
  args = ap.parse_args(argv)
  M, N, K = parse_shape(args.shape)
  table = {**LADDER, **SWEEP, **EXTRA, **B200}
  names = list(table) if args.configs == "all" else [n for n in args.configs.split(",") if n]
  dev = torch.device("cuda", torch.cuda.current_device())
  g = torch.Generator(device=dev).manual_seed(0)
  a = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
  b = torch.randn((K, N), generator=g, device=dev).to(torch.bfloat16)
  c = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
  flush = torch.empty(64 << 20, dtype=torch.int32, device=dev) if args.flush else None   # 256 MiB
  flops = 2.0 * M * N * K
  ref = None
  if args.check:   # fp32 product of the bf16 inputs (no TF32): the oracle's arithmetic, on the GPU
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = a.float() @ b.float()
    torch.backends.cuda.matmul.allow_tf32 = tf32
  cub_us = None
  if args.torch:
    out = torch.empty_like(c)
    for _ in range(args.reps): torch.matmul(a, b, out=out)
    torch.cuda.synchronize()
    print("KERNEL cublas torch", flush=True)
    if args.time:
      best, mean = _time(lambda: torch.matmul(a, b, out=out), args.reps, args.warmup, flush)
      cub_us = best
      print("TIME " + json.dumps({"label": "cublas", "shape": [M, N, K], "us_best": round(best, 2),
                                  "us_mean": round(mean, 2), "tflops": round(flops / best / 1e6, 1)}), flush=True)
  failed = 0
  for name in names:
    try:
      cfg = lookup(name)
      run = build(N, cfg, M, K)
      launch = run(a, b, c)
      c.fill_(float("nan"))          # a skipped write can't pass the check
      launch()
      launch.check()
      if args.check:
        rel = float((c.float() - ref).abs().max() / (ref.abs().max() + 1e-9))
        bad = not rel <= 4e-3 or bool(torch.isnan(c).any())
        print(f"CHECK {name} rel={rel:.5f} max|ref|={float(ref.abs().max()):.1f} {'MISMATCH' if bad else 'ok'}",
              flush=True)
        failed += bad
      for _ in range(args.reps): launch()
      launch.check()
      print(f"KERNEL {name} {run.kernel_name} {launch.info()['kernel']}", flush=True)
      if args.time:
        rec = {"label": name, "shape": [M, N, K], "kernel": launch.info()["kernel"]}
        if args.torch:   # interleaved with cuBLAS: the ratio of medians is robust to clock drift
          ours, cub = _time_pair(launch, lambda: torch.matmul(a, b, out=out), args.reps, args.warmup, flush)
          med, cmed = statistics.median(ours), statistics.median(cub)
          rec.update(us_best=round(min(ours), 2), us_median=round(med, 2), tflops=round(flops / med / 1e6, 1),
                     cublas_us_median=round(cmed, 2), cublas_tflops=round(flops / cmed / 1e6, 1),
                     pct_cublas=round(100.0 * cmed / med, 1))
        else:
          best, mean = _time(launch, args.reps, args.warmup, flush)
          rec.update(us_best=round(best, 2), us_mean=round(mean, 2), tflops=round(flops / best / 1e6, 1))
        print("TIME " + json.dumps(rec), flush=True)
    except ValueError as exc:
      print(f"SKIP {name}: {exc}", flush=True)
  return 1 if failed else 0


if __name__ == "__main__":
  raise SystemExit(main())
