"""Benchmark of the B200 bf16 GEMM (the hot path of narain1/tinygrad-hopper-wgmma) — prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME] [--cfg NAME]
                    [--no-extra-legs] [--no-cpu-baseline] [--no-e2e]

Workloads (per rank; one process per GPU, launched by torch.distributed.run for N > 1):
  gemm4096   (default) M=N=K=4096, the reference's ladder headline. With N GPUs each rank computes its own
             4096-column shard of a 4096 x 4096N x 4096 GEMM (A replicated, B and C split by columns, no collective in
             the GEMM): per-GPU work is fixed, scaling "weak".
  gemm8192   M=N=K=8192 per rank, same sharding.
  shard32k   M=N=K=32768 split by columns over the N GPUs (32768 x 32768/N x 32768 per rank): scaling "strong".
A step is one GEMM launch on resident inputs. Between timed steps a 256 MiB buffer is rewritten to flush the 126 MB
L2, and each step is timed alone with CUDA events on the launching stream; the whole timed region is bracketed by a
barrier and a synchronize, and the reported time is the max over ranks. Throughput = 2*M*N*K of all ranks / time,
with time = the mean step time (every throughput in the line, cuBLAS's included, uses the mean).

Besides the main workload the line carries two more legs of the BASELINE configs, each with its own cuBLAS
comparison, parity gate, roofline and clocks: ``gemm8192`` (one GPU only) and ``shard32k`` (at every N: the
32768^3 GEMM split by columns over the N GPUs, strong scaling, with per-rank clocks). Every leg first runs once on
NaN-poisoned C and is compared with the fp32 product of the same bf16 inputs (cuBLAS fp32, TF32 off); if any leg
misses max|C - ref| / max|ref| <= 4e-3 or leaves a NaN, the line is still printed and the process exits with
status 3.

``--impl reference`` times the reference's CPU path instead: its host reference ``a.float() @ b.float()``
(scripts/smoke.py:41), fp32 accumulate over bf16 inputs plus the bf16 output rounding, on this host's cores
(the reference's stock tinygrad ``A @ B`` cannot run here). Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "tinygrad-hopper-wgmma_b200"), str(ROOT)]

METRIC = "bf16 GEMM TFLOPS at N=4096/8192, % of B200 dense peak and of cuBLAS"
WORKLOADS = {"gemm4096": (4096, 4096, 4096, "weak"), "gemm8192": (8192, 8192, 8192, "weak"),
             "shard32k": (32768, 32768, 32768, "strong")}
FLUSH_BYTES = 256 << 20
CPU_SAMPLE_SECONDS = 10.0
REFERENCE_BUDGET_S = 90.0
TOL = 4e-3              # max|C - ref| / max|ref| against the fp32 product (north_star tolerance)
EXTRA_LEG_STEPS = 20    # timed steps of the gemm8192 / shard32k legs (fewer when --steps is smaller)
GATE_FAILED_EXIT = 3


def parse_args(argv=None):
  ap = argparse.ArgumentParser()
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=200)
  ap.add_argument("--warmup", type=int, default=10)
  ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
  ap.add_argument("--workload", choices=tuple(WORKLOADS), default="gemm4096")
  ap.add_argument("--cfg", default="best")
  ap.add_argument("--no-extra-legs", action="store_true", help="time the main workload only")
  ap.add_argument("--no-cpu-baseline", action="store_true")
  ap.add_argument("--no-e2e", action="store_true")
  return ap.parse_args(argv)


def shapes(workload: str, world: int):
  """(M, n_per_rank, K, N_total, scaling)."""
  M, N, K, scaling = WORKLOADS[workload]
  if scaling == "weak": return M, N, K, N * world, scaling
  if N % world: raise SystemExit(f"{workload}: N={N} does not split over {world} GPUs")
  return M, N // world, K, N, scaling


def measured_peaks() -> dict:
  p = ROOT / "MEASURED_PEAKS.json"
  if p.exists(): return {**json.loads(p.read_text()), "source": "measured"}
  return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic(kernel_tag: str, workload: str, flops_per_launch: float):
  """DRAM bytes (read + write) per launch of this kernel on this workload, from the committed ncu summaries
  (profiles/*.txt lines 'traffic <kernel tag> <workload> <bytes> <flops of the captured launch>'), scaled to this
  launch's FLOPs when the capture ran a per-rank shard of a different width. None if no capture covers it."""
  for f in sorted((ROOT / "profiles").glob("*.txt")):
    for line in f.read_text().splitlines():
      parts = line.split()
      if len(parts) == 5 and parts[0] == "traffic" and parts[1] == kernel_tag and parts[2] == workload:
        return round(float(parts[3]) * flops_per_launch / float(parts[4]))
  return None


def parity_gate(C, ref):
  """Compare the bf16 output C with the fp32 reference product ``ref`` (same device): max|C - ref| / max|ref| and
  the NaN count (C was NaN-poisoned before the launch). ``ok`` is False when either misses the bar."""
  import torch
  nan = int(torch.isnan(C).sum())
  rel = float((C.float() - ref).abs().max() / (ref.abs().max() + 1e-9))
  if rel != rel: rel = float("inf")
  return {"rel_err_vs_fp32": rel, "nan_after_poison": nan, "tol": TOL, "ok": bool(nan == 0 and rel <= TOL)}


def gates_failed(line: dict) -> list[str]:
  """Names of the legs of a result line whose parity gate failed."""
  bad = [] if line.get("parity", {}).get("ok", False) else ["main"]
  for leg in ("gemm8192", "shard32k"):
    sub = line.get(leg)
    if isinstance(sub, dict) and "parity" in sub and not sub["parity"].get("ok", False): bad.append(leg)
  return bad


# ------------------------------------------------------------------------------------------------------------------
# clocks during the timed region (NVML reads only; no setting is changed)
# ------------------------------------------------------------------------------------------------------------------
class ClockSampler:
  REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
             "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
             "display_clock_setting": 0x100}

  def __init__(self, device_index: int, period_s: float = 0.002):
    self.samples, self.reasons, self.period, self.ok = [], 0, period_s, False
    self._stop = threading.Event()
    try:
      import pynvml
      pynvml.nvmlInit()
      self.nv = pynvml
      self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
      self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
      self.ok = True
    except Exception as exc:   # NVML missing: report that instead of clocks
      self.err = repr(exc)

  def _sample(self):
    try:
      self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
      self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
    except Exception:
      pass

  def _run(self):
    while not self._stop.is_set():
      self._sample()
      time.sleep(self.period)

  def __enter__(self):
    if self.ok:
      self._sample()
      self.t = threading.Thread(target=self._run, daemon=True)
      self.t.start()
    return self

  def __exit__(self, *exc):
    if self.ok:
      self._stop.set()
      self.t.join()
      self._sample()

  def summary(self) -> dict:
    if not self.ok: return {"error": self.err}
    active = [k for k, v in self.REASONS.items() if self.reasons & v and k != "gpu_idle"]
    return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples), "reasons": active}


# ------------------------------------------------------------------------------------------------------------------
# reference arm: the CPU path
# ------------------------------------------------------------------------------------------------------------------
def cpu_gemm_tflops(M: int, N: int, K: int, seconds: float, reps_min: int = 1, reps_max: int | None = None):
  """Time the oracle's full operator (fp32 accumulate + bf16 rounding) on this host. Returns (tflops, reps, secs)."""
  from oracle import gemm_ref
  a_bits, b_bits = gemm_ref.randn_bf16_bits((M, K), 0), gemm_ref.randn_bf16_bits((K, N), 1)
  a32, b32 = gemm_ref.bf16_bits_to_f32(a_bits), gemm_ref.bf16_bits_to_f32(b_bits)
  gemm_ref.f32_to_bf16_bits(a32 @ b32)   # warm the BLAS thread pool
  reps, t0 = 0, time.perf_counter()
  while reps < reps_min or (time.perf_counter() - t0 < seconds and (reps_max is None or reps < reps_max)):
    gemm_ref.f32_to_bf16_bits(a32 @ b32)
    reps += 1
  dt = time.perf_counter() - t0
  return 2.0 * M * N * K * reps / dt / 1e12, reps, dt


def blas_threads() -> int:
  try:
    from threadpoolctl import threadpool_info
    return max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"), default=1)
  except Exception:
    return len(os.sched_getaffinity(0))


def run_reference(args):
  if int(os.environ.get("RANK", "0")) != 0: return   # rank 0 alone runs the CPU arm
  M, n, K, N_total, scaling = shapes(args.workload, 1)
  from oracle import gemm_ref
  # One step = the rank-0 GEMM restricted to a sample of cap_M rows, sized so that warm-up + steps take about
  # REFERENCE_BUDGET_S on this host (the metric is per FLOP, so a row sample measures the same throughput).
  probe_rows = 256
  pa, pb = gemm_ref.randn_bf16_bits((probe_rows, K), 2), gemm_ref.randn_bf16_bits((K, n), 3)
  pa32, pb32 = gemm_ref.bf16_bits_to_f32(pa), gemm_ref.bf16_bits_to_f32(pb)
  gemm_ref.f32_to_bf16_bits(pa32 @ pb32)
  t0 = time.perf_counter()
  gemm_ref.f32_to_bf16_bits(pa32 @ pb32)
  per_row = (time.perf_counter() - t0) / probe_rows
  budget_step = REFERENCE_BUDGET_S / max(1, args.steps + args.warmup)
  cap_M = int(min(M, max(64, budget_step / max(per_row, 1e-9))) // 64 * 64) or 64
  a_bits, b_bits = gemm_ref.randn_bf16_bits((cap_M, K), 0), gemm_ref.randn_bf16_bits((K, n), 1)
  a32, b32 = gemm_ref.bf16_bits_to_f32(a_bits), gemm_ref.bf16_bits_to_f32(b_bits)
  for _ in range(args.warmup): gemm_ref.f32_to_bf16_bits(a32 @ b32)
  t0 = time.perf_counter()
  for _ in range(args.steps): gemm_ref.f32_to_bf16_bits(a32 @ b32)
  dt = time.perf_counter() - t0
  tflops = 2.0 * cap_M * n * K * args.steps / dt / 1e12
  cores = blas_threads()
  sample = f"{args.steps} x numpy fp32 GEMM {cap_M}x{n}x{K} + bf16 rounding (rows capped at {cap_M} of {M})"
  emit({
    "impl": "reference", "metric": METRIC, "value": round(tflops, 4), "unit": "TFLOPS", "n_gpus": args.gpus,
    "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
    "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate",
    "data": "synthetic: seeded N(0,1) rounded to bf16",
    "config": {"workload": args.workload, "M": cap_M, "N": n, "K": K,
               "path": "reference CPU path stand-in: numpy fp32 matmul of bf16-exact inputs (scripts/smoke.py:41)"},
    "cpu_baseline": {"value": round(tflops, 4), "unit": "TFLOPS", "cores": cores, "kind": "port", "sample": sample},
    "e2e": {"value": round(tflops, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    "gpu_launches": 0})


# ------------------------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------------------------
def pick_cfg(name: str, m: int, n: int, k: int):
  """``best`` = the fastest config of the ncu shape sweep for this size of per-rank GEMM
  (``hopper_wgmma.ladder.best_config``: 256x256 CTA-pair tiles for the 4096^3 workload, 256x512 pair tiles from 8192^3
  up). Any other name is looked up in the ladder tables (``hopper_wgmma.ladder.lookup``, modifiers such as ``@skA``
  included)."""
  from hopper_wgmma.ladder import best_config, lookup
  if name == "best": return "best", best_config(m, n, k)
  try:
    return name, lookup(name)
  except (KeyError, ValueError) as exc:
    raise SystemExit(f"unknown --cfg {name}: {exc}")


def kernel_tag(info: dict, cfg) -> str:
  return (f"sm100_gemm_ws_{'pair' if info['paired'] else 'cta'}_{'tmast' if cfg.tma_store else 'reg'}"
          f"{'_x2' if cfg.n_mma == 2 else ''}")


class Bench:
  """One rank's benchmark state: device, process group helpers and the L2-flush buffer."""

  def __init__(self, args):
    import torch
    import torch.distributed as dist
    self.torch, self.dist, self.args = torch, dist, args
    self.rank, self.world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    self.local = int(os.environ.get("LOCAL_RANK", "0"))
    if self.world != args.gpus: raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
    torch.cuda.set_device(self.local)
    self.dev = torch.device("cuda", self.local)
    if self.world > 1:
      from datetime import timedelta
      dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)
    self.flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=self.dev)
    self.peaks = measured_peaks()

  def barrier(self):
    if self.world > 1: self.dist.barrier()

  def max_over_ranks(self, v: float) -> float:
    if self.world == 1: return v
    from hopper_wgmma import shard
    return shard.max_over_ranks(v, device=self.dev)

  def gather(self, values: list[float]) -> list[list[float]]:
    """Every rank's list of floats (same length on all ranks), in rank order."""
    torch = self.torch
    t = torch.tensor(values, dtype=torch.float64, device=self.dev)
    if self.world == 1: return [values]
    out = [torch.empty_like(t) for _ in range(self.world)]
    self.dist.all_gather(out, t)
    return [o.tolist() for o in out]

  def timed(self, fn, steps):
    """Per-step device times (ms) with an L2 flush before every step; returns (max over ranks of the total, list)."""
    torch = self.torch
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    self.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
      self.flush.zero_()
      starts[i].record()
      fn()
      ends[i].record()
    torch.cuda.synchronize()
    self.barrier()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return self.max_over_ranks(sum(per)), per

  def interleaved(self, ours, cublas, steps):
    """Ours and cuBLAS alternating launch by launch (same clocks, same flush protocol): mean ms of each, max over
    ranks, plus the medians for reference."""
    torch = self.torch
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    self.barrier()
    torch.cuda.synchronize()
    for e in ev:
      self.flush.zero_()
      e[0].record()
      ours()
      e[1].record()
      self.flush.zero_()
      e[2].record()
      cublas()
      e[3].record()
    torch.cuda.synchronize()
    self.barrier()
    o = [e[0].elapsed_time(e[1]) for e in ev]
    c = [e[2].elapsed_time(e[3]) for e in ev]
    return {"ours_mean_ms": self.max_over_ranks(statistics.mean(o)),
            "cublas_mean_ms": self.max_over_ranks(statistics.mean(c)),
            "ours_median_ms": self.max_over_ranks(statistics.median(o)),
            "cublas_median_ms": self.max_over_ranks(statistics.median(c))}

  def leg(self, workload: str, cfg_name: str, steps: int, warmup: int, per_rank_clocks: bool = False):
    """Time one GEMM workload: parity gate on poisoned C, ``steps`` flushed launches (the leg's value), cuBLAS
    interleaved, roofline and clocks. Returns (result dict, launch, operands) — the operands stay alive for the
    caller's end-to-end leg."""
    torch = self.torch
    from hopper_wgmma import shard
    M, n, K, N_total, scaling = shapes(workload, self.world)
    cfg_name, cfg = pick_cfg(cfg_name, M, n, K)
    flops_rank = 2.0 * M * n * K
    # inputs resident in HBM: A replicated (same seed everywhere), this rank's K-major B shard, this rank's C shard
    g = torch.Generator(device=self.dev).manual_seed(1234)
    A = torch.randn((M, K), generator=g, device=self.dev, dtype=torch.float32).to(torch.bfloat16)
    gb = torch.Generator(device=self.dev).manual_seed(5678 + self.rank)
    BT = torch.randn((n, K), generator=gb, device=self.dev, dtype=torch.float32).to(torch.bfloat16)
    C = torch.full((M, n), float("nan"), dtype=torch.bfloat16, device=self.dev)
    launch = shard.local_gemm(A, BT, C, cfg)
    info = launch.info()

    # parity gate on the leg's own inputs, before timing: NaN-poisoned C against the fp32 product (TF32 off)
    launch()
    launch.check()
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
      ref = A.float() @ BT.float().t()
    finally:
      torch.backends.cuda.matmul.allow_tf32 = tf32
    parity = parity_gate(C, ref)
    del ref
    parity["ok"] = self.max_over_ranks(0.0 if parity["ok"] else 1.0) == 0.0   # every rank passed
    cub_bf16 = A @ BT.t()
    parity["bitwise_equal_fraction_vs_cublas"] = round(float((C == cub_bf16).float().mean()), 4)
    del cub_bf16
    torch.cuda.empty_cache()

    for _ in range(warmup): launch()
    torch.cuda.synchronize()
    with ClockSampler(self.local) as clocks:
      total_ms, per = self.timed(launch, steps)
    launch.check()
    ms = total_ms / steps
    value = flops_rank * self.world / (ms * 1e-3) / 1e12
    achieved = flops_rank / (statistics.mean(per) * 1e-3) / 1e12

    Cc = torch.empty_like(C)
    cub = lambda: torch.matmul(A, BT.t(), out=Cc)
    for _ in range(3): cub()
    pair_steps = max(3, min(steps, 200))
    with ClockSampler(self.local) as clocks_pair:
      cmp = self.interleaved(launch, cub, pair_steps)
    del Cc
    peak = self.peaks["bf16_tflops"]
    # strong scaling changes the per-rank shape with the world size: its captures are keyed "shard32k/<world>"
    traffic = profiled_traffic(kernel_tag(info, cfg), workload if scaling == "weak" else f"{workload}/{self.world}",
                               flops_rank)
    res = {
      "value": round(value, 3), "unit": "TFLOPS", "ms_per_step": round(ms, 5), "steps": steps, "warmup": warmup,
      "statistic": "mean", "scaling": scaling,
      "config": {"workload": workload, "M": M, "N": N_total, "K": K, "n_per_gpu": n, "cfg": cfg_name,
                 "cfg_name": cfg.name, "kernel": info["kernel"], "grid": info["grid"], "smem": info["smem_bytes"],
                 "parallelism": f"N-column shards x{self.world} (A replicated, no collective in the GEMM)",
                 "l2": "flushed between steps (256 MiB write); each step timed alone with CUDA events"},
      "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                   "frac": round(achieved / peak, 4), "traffic": traffic,
                   "peak_source": f"{self.peaks['source']} bf16_tflops (burst, cuBLAS 8192^3)",
                   "algorithmic_flops_per_launch": flops_rank,
                   "algorithmic_bytes_per_launch": 2 * (M * K + n * K + M * n)},
      "cublas": {"value": round(flops_rank * self.world / (cmp["cublas_mean_ms"] * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                 "ours_over_cublas": round(cmp["cublas_mean_ms"] / cmp["ours_mean_ms"], 4), "statistic": "mean",
                 "interleaved_steps": pair_steps, **{k: round(v, 5) for k, v in cmp.items()},
                 "ours_over_cublas_median": round(cmp["cublas_median_ms"] / cmp["ours_median_ms"], 4),
                 "clocks": clocks_pair.summary(),
                 "kernel": "torch.matmul (cuBLAS), same inputs, same flush protocol, alternating with ours"},
      "parity": parity, "clocks": clocks.summary(), "gpu_launches": steps,
    }
    if per_rank_clocks:
      s = clocks.summary()
      mine = [float(s.get("sm_mhz") or 0.0), float(sum(ClockSampler.REASONS[r] for r in s.get("reasons", []))),
              float(s.get("samples", 0))]
      res["clocks_per_rank"] = [
        {"rank": r, "sm_mhz": v[0], "samples": int(v[2]),
         "reasons": [k for k, bit in ClockSampler.REASONS.items() if int(v[1]) & bit]}
        for r, v in enumerate(self.gather(mine))]
    return res, launch, (A, BT, C, cfg, M, n, K)

  def e2e(self, cfg, M, n, K, A, BT, C):
    """End to end through the public API, as a caller streaming batches would run it: every step copies its A and
    B from pinned host memory, runs the reference-facing operator build_gemm_ws(...)(A, B, C)() (plan and launch; B
    is read as given for CTA-pair tiles, copied K-major first otherwise) and copies C back to pinned host memory.
    Steps rotate over three streams and buffer sets (two when a set would exceed 1 GiB), so one step's host-to-device
    copies overlap earlier steps' GEMMs and device-to-host copies without queueing behind them on a shared stream."""
    torch = self.torch
    from hopper_wgmma.gemm import build_gemm_ws
    sets = []
    nsets = 3 if 2 * (M * K + K * n + M * n) <= (1 << 30) else 2
    for _ in range(nsets):
      hA = torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True)
      hB = torch.empty((K, n), dtype=torch.bfloat16, pin_memory=True)
      hC = torch.empty((M, n), dtype=torch.bfloat16, pin_memory=True)
      hA.copy_(A.cpu())
      hB.copy_(BT.t().cpu())
      dA, dB, dC = torch.empty_like(A), torch.empty((K, n), dtype=torch.bfloat16, device=self.dev), torch.empty_like(C)
      sets.append((hA, hB, hC, dA, dB, dC, torch.cuda.Stream(device=self.dev)))
    run = build_gemm_ws(n, cfg, M, K)

    def step(i):
      hA, hB, hC, dA, dB, dC, st = sets[i % nsets]
      with torch.cuda.stream(st):
        dA.copy_(hA, non_blocking=True)
        dB.copy_(hB, non_blocking=True)
        run(dA, dB, dC)()
        hC.copy_(dC, non_blocking=True)
    steps = max(3, min(self.args.steps, 30))
    for i in range(2 * nsets): step(i)
    torch.cuda.synchronize()
    # The copies without the GEMM: each direction alone on one stream, then both directions at once on two streams
    # (a step's device-to-host copy overlaps the next steps' host-to-device copies), whose time per step is the
    # bound the end-to-end step cannot beat.
    hA, hB, hC, dA, dB, dC, st = sets[0]
    st2 = sets[1][6]
    h2d, d2h = ((dA, hA), (dB, hB)), ((hC, dC),)
    rates = {}

    def timed(plan):   # plan: [(stream, copies)]; three rounds after one untimed round, seconds per round
      cur = torch.cuda.current_stream(self.dev)
      e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      for rounds, ev in ((1, None), (3, e0)):
        if ev is not None:
          torch.cuda.synchronize()
          ev.record(cur)
        for s, copies in plan:
          s.wait_stream(cur)
          with torch.cuda.stream(s):
            for _ in range(rounds):
              for dst, src in copies: dst.copy_(src, non_blocking=True)
        for s, _ in plan: cur.wait_stream(s)
      e1.record(cur)
      torch.cuda.synchronize()
      return e0.elapsed_time(e1) * 1e-3 / 3
    rates["h2d"] = 2 * (M * K + K * n) / timed([(st, h2d)]) / 1e9
    rates["d2h"] = 2 * M * n / timed([(st, d2h)]) / 1e9
    copy_bound_ms = timed([(st, h2d), (st2, d2h)]) * 1e3
    self.barrier()
    cur = torch.cuda.current_stream(self.dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(cur)
    for *_, st in sets: st.wait_event(ev0)
    for i in range(steps): step(i)
    for *_, st in sets:
      done = torch.cuda.Event()
      done.record(st)
      cur.wait_event(done)
    ev1.record(cur)
    torch.cuda.synchronize()
    self.barrier()
    e2e_ms = self.max_over_ranks(ev0.elapsed_time(ev1))
    flops_rank = 2.0 * M * n * K
    return {"value": round(flops_rank * self.world / (e2e_ms / steps * 1e-3) / 1e12, 3), "unit": "TFLOPS",
            "h2d_bytes_per_step": 2 * (M * K + K * n), "d2h_bytes_per_step": 2 * M * n,
            "path": "pinned host A,B -> build_gemm_ws(...)(A, B, C)() ("
                    f"{'B read N-major as given' if cfg.reads_b_directly else 'K-major copy of B'}, plan, launch) -> "
                    f"pinned host C; {nsets} streams and buffer sets, steps overlapped",
            "steps": steps, "ms_per_step": round(e2e_ms / steps, 4),
            "h2d_gbs": round(rates["h2d"], 1), "d2h_gbs": round(rates["d2h"], 1),
            "copy_bound_ms": round(copy_bound_ms, 4), "frac_of_copy_bound": round(copy_bound_ms / (e2e_ms / steps), 3)}

  def allgather(self, C, M, n):
    """Optional NCCL all-gather of the C shards over NVLink (A replicated, B and C column-sharded): timed
    separately, never inside the GEMM. Every rank runs the same collectives in the same order."""
    torch = self.torch
    from hopper_wgmma import shard
    for _ in range(3): shard.gather_columns(C, self.world, as_row_major=False)
    torch.cuda.synchronize()
    self.barrier()
    steps = 10
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps): shard.gather_columns(C, self.world, as_row_major=False)
    ev1.record()
    torch.cuda.synchronize()
    ms = self.max_over_ranks(ev0.elapsed_time(ev1) / steps)
    total = 2 * M * n * self.world
    return {"ms": round(ms, 4), "bytes_gathered": total, "algbw_gbs": round(total / (ms * 1e-3) / 1e9, 1),
            "busbw_gbs": round(total * (self.world - 1) / self.world / (ms * 1e-3) / 1e9, 1),
            "what": "torch.distributed.all_gather_into_tensor (NCCL) of the bf16 C shards -> [world, M, N/world]"}


def run_ours(args) -> int:
  b = Bench(args)
  torch = b.torch
  main, launch, (A, BT, C, cfg, M, n, K) = b.leg(args.workload, args.cfg, args.steps, args.warmup)
  e2e = None if args.no_e2e else b.e2e(cfg, M, n, K, A, BT, C)
  allgather = b.allgather(C, M, n) if b.world > 1 else None
  del A, BT, C, launch
  torch.cuda.empty_cache()

  extra = {}
  if not args.no_extra_legs:
    leg_steps, leg_warmup = max(3, min(args.steps, EXTRA_LEG_STEPS)), max(3, min(args.warmup, 5))
    legs = [("shard32k", True)] if b.world > 1 else [("gemm8192", False), ("shard32k", True)]
    for wl, per_rank in legs:
      if wl == args.workload: continue
      res, *_ = b.leg(wl, "best", leg_steps, leg_warmup, per_rank_clocks=per_rank)
      torch.cuda.empty_cache()
      extra[wl] = res

  cpu = None
  if b.rank == 0 and b.world == 1 and not args.no_cpu_baseline:
    tf, reps, secs = cpu_gemm_tflops(M, n, K, CPU_SAMPLE_SECONDS, reps_min=2)
    cpu = {"value": round(tf, 4), "unit": "TFLOPS", "cores": blas_threads(), "kind": "port",
           "sample": f"{reps} x numpy fp32 GEMM {M}x{n}x{K} + bf16 rounding in {secs:.1f} s (the arm's own shape)"}

  if b.world > 1:
    b.dist.barrier()
    b.dist.destroy_process_group()
  line = {
    "metric": METRIC, "value": main["value"], "unit": "TFLOPS", "n_gpus": b.world, "steps": args.steps,
    "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True, "scaling": main["scaling"],
    "vs_baseline": None, "dtype": "bf16", "data": "synthetic: seeded N(0,1) rounded to bf16, resident in HBM",
    "statistic": "mean step time (CUDA events, L2 flushed before every step), max over ranks",
    "config": main["config"], "roofline": main["roofline"], "cublas": main["cublas"], "parity": main["parity"],
    "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": main["clocks"],
    "allgather_c": allgather, **extra,
  }
  bad = gates_failed(line)
  if bad: line["parity_gate_failed"] = bad
  if b.rank == 0: emit(line)
  return GATE_FAILED_EXIT if bad else 0


_JSON_OUT = None


def emit(line: dict) -> None:
  """Print the result line on the real stdout (everything else that writes to stdout goes to stderr)."""
  print(json.dumps(line), file=_JSON_OUT or sys.stdout, flush=True)


def main():
  global _JSON_OUT
  # Keep stdout for the single JSON line: NCCL and other libraries print banners to fd 1, so fd 1 is pointed at
  # stderr and the result goes through a private duplicate of the original stdout.
  _JSON_OUT = os.fdopen(os.dup(1), "w")
  os.dup2(2, 1)
  args = parse_args()
  if args.impl == "reference":
    run_reference(args)
    return 0
  return run_ours(args)


if __name__ == "__main__":
  sys.exit(main())
