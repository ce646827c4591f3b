"""Host-side measurement tools, on the CPU: config lookup with modifiers (hopper_wgmma.ladder.lookup), the Nsight
Compute report pipeline (hopper_wgmma.ncu_table, hopper_wgmma.report; the reference's scripts/ncu_table.py and
scripts/report.py) and bench.py's choice of config per problem size."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_lookup_modifiers():
  from hopper_wgmma.ladder import B200, LADDER, lookup
  assert lookup("cluster_hilbert") is LADDER["cluster_hilbert"]
  assert lookup("pair_wide") is B200["pair_wide"]
  c = lookup("cta_n128@sk2")
  assert c.split_k == 2 and c.BN == 128 and c.tma_store
  assert lookup("cta_n64@skA").split_k == -1
  c = lookup("cta_n64@reg@s4")
  assert not c.tma_store and c.stages == 4 and c.BN == 64
  c = lookup("cluster_hilbert@bT")
  assert c.b_nmajor is False and c.cluster == 2 and LADDER["cluster_hilbert"].b_nmajor is None
  assert lookup("cta_n128@bN").b_nmajor is True
  c = lookup("cta_n128@sk2@skw")
  assert c.split_k == 2 and c.split_k_cluster is False and lookup("cta_n128@sk2@skc").split_k_cluster is True
  assert lookup("cta_n128@sk2").split_k_cluster is None
  with pytest.raises(KeyError):
    lookup("cta_n64@bogus")
  with pytest.raises(KeyError):
    lookup("no_such_config")
  with pytest.raises(ValueError):
    lookup("tma_ring@sk2")   # a gated (non-persistent) config has no split-K


CSV = """==PROF== Connected
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","void sm100::sm100_gemm_ws<128, 1, 1, 1, 0>(CUtensorMap_st, GemmParams)","1","7","(256, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","usecond","95.50"
"1","1","python","h","void sm100::sm100_gemm_ws<128, 1, 1, 1, 0>(CUtensorMap_st, GemmParams)","1","7","(256, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","usecond","93.25"
"2","1","python","h","nvjet_tst_256x256_64x4_2x2_2cta_v_bz_TNT","1","7","(384, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","nsecond","96580"
"""


def test_ncu_table_best_and_launch_list():
  from hopper_wgmma import ncu_table
  best = ncu_table.best(CSV)
  assert best["sm100::sm100_gemm_ws<128, 1, 1, 1, 0>"] == pytest.approx(93.25)
  assert best["nvjet_tst_256x256_64x4_2x2_2cta_v_bz_TNT"] == pytest.approx(96.58)
  rows = ncu_table.launch_list(CSV)
  assert rows[0][0].startswith("sm100::") and rows[0][1] == 2
  assert sum(r[3] for r in rows) == pytest.approx(1.0)
  assert ncu_table.tflops(93.25, 4096, 4096, 4096) == pytest.approx(2 * 4096 ** 3 / 93.25e-6 / 1e12)


def test_ncu_summary_table():
  from hopper_wgmma import report
  recs = [{"label": "cluster_hilbert", "shape": [4096, 4096, 4096], "us_best": 93.0, "tflops": 1478.0,
           "cublas_us_best": 96.0, "cublas_tflops": 1431.0, "pct_cublas": 103.2},
          {"label": "hilbert", "shape": [4096, 4096, 4096], "us_best": 99.0, "tflops": 1388.0,
           "cublas_us_best": 96.0, "cublas_tflops": 1431.0, "pct_cublas": 97.0},
          {"label": "cta_n128", "shape": [512, 512, 512], "us_best": 6.5, "tflops": 41.0,
           "cublas_us_best": 4.3, "cublas_tflops": 62.0, "pct_cublas": 66.0}]
  text = "\n".join("NCU " + json.dumps(r) for r in recs) + "\nERROR 8192x8192x8192: ncu exited 9: x\n"
  md = report.ncu_summary([text], peak_tflops=1624.7)
  lines = md.splitlines()
  assert lines[2].startswith("| 512×512×512 | cta_n128 |")                      # smallest shape first
  assert lines[3].startswith("| 4096×4096×4096 | cluster_hilbert | 93.0 | 1478 | 1431 | 103.2% | 91.0% |")
  assert "**4096×4096×4096** — cluster_hilbert 103.2%, hilbert 97.0%" in md


def test_best_config_by_size():
  from hopper_wgmma.ladder import B200, LADDER, best_config
  assert best_config(8192, 8192, 8192) is B200["pair_wide_hilbert"]
  assert best_config(32768, 4096, 32768) is B200["pair_wide_hilbert"]     # one rank of the 8-GPU 32768^3 shard
  assert best_config(6144, 6144, 6144) is B200["pair_wide_hilbert"]
  assert best_config(16384, 4096, 4096) is B200["pair_wide_hilbert"]
  assert best_config(4096, 4096, 4096) is LADDER["cluster_hilbert"]
  assert best_config(8192, 8192, 2048) is LADDER["cluster_hilbert"]       # short K: 256x256 pairs (104 % of cuBLAS)
  assert best_config(2048, 2048, 16384) is LADDER["cluster_hilbert"]
  assert best_config(2048, 2048, 2048) is LADDER["cluster_hilbert"]
  small = best_config(1024, 1024, 8192)
  assert small.BN == 128 and small.cluster == 1 and small.split_k == -1


def test_bench_picks_the_best_config_for_the_rank_size():
  sys.path.insert(0, str(ROOT))
  import bench
  name, cfg = bench.pick_cfg("best", 4096, 4096, 4096)
  assert name == "best" and cfg.n_mma == 1 and cfg.cluster == 2 and cfg.hilbert
  _, cfg = bench.pick_cfg("best", 8192, 8192, 8192)
  assert cfg.n_mma == 2 and cfg.cluster == 2
  _, cfg = bench.pick_cfg("best", 32768, 4096, 32768)
  assert cfg.n_mma == 2
  name, cfg = bench.pick_cfg("cta_n128@sk2", 1024, 1024, 1024)
  assert name == "cta_n128@sk2" and cfg.split_k == 2
  with pytest.raises(SystemExit):
    bench.pick_cfg("no_such_config", 4096, 4096, 4096)


def test_bench_reads_traffic_lines_of_the_committed_profiles():
  sys.path.insert(0, str(ROOT))
  import bench
  flops = 2.0 * 4096 ** 3
  t = bench.profiled_traffic("sm100_gemm_ws_pair_tmast", "gemm4096", flops)
  assert t is not None and 67_108_864 <= t <= 2 * 101_000_000      # at least the compulsory A + B
  assert bench.profiled_traffic("sm100_gemm_ws_pair_tmast_x2", "gemm8192", 2.0 * 8192 ** 3) is not None
  assert bench.profiled_traffic("no_such_kernel", "gemm4096", flops) is None


def test_bench_parity_gate_fails_on_a_planted_error_or_nan():
  """The bench's correctness gate compares the bf16 output with the fp32 product; an output with one wrong element
  (planted here on the CPU) or one surviving NaN must fail it."""
  import torch
  sys.path.insert(0, str(ROOT))
  import bench
  g = torch.Generator().manual_seed(0)
  ref = torch.randn((64, 96), generator=g) * 10
  C = ref.to(torch.bfloat16)
  assert bench.parity_gate(C, ref)["ok"]
  bad = C.clone()
  bad[3, 7] += 1.0
  res = bench.parity_gate(bad, ref)
  assert not res["ok"] and res["rel_err_vs_fp32"] > bench.TOL
  bad = C.clone()
  bad[5, 5] = float("nan")
  res = bench.parity_gate(bad, ref)
  assert not res["ok"] and res["nan_after_poison"] == 1


def test_bench_exits_nonzero_when_a_leg_misses_the_gate(monkeypatch):
  """run_ours still prints its line but returns the failure status when any leg's gate failed."""
  sys.path.insert(0, str(ROOT))
  import bench
  from hopper_wgmma import WSCfg

  class FakeTorch:
    class cuda:
      @staticmethod
      def empty_cache(): pass

  class FakeBench:
    def __init__(self, args):
      self.torch, self.world, self.rank = FakeTorch, 1, 0

    def leg(self, workload, cfg_name, steps, warmup, per_rank_clocks=False):
      ok = workload != "gemm8192"                  # the planted failure: one extra leg misses the gate
      res = {"value": 1.0, "ms_per_step": 1.0, "scaling": "weak", "config": {}, "roofline": {}, "cublas": {},
             "parity": {"ok": ok}, "clocks": {}}
      return res, None, (None, None, None, WSCfg(), 64, 64, 64)

  printed = []
  monkeypatch.setattr(bench, "Bench", FakeBench)
  monkeypatch.setattr(bench, "emit", printed.append)
  args = bench.parse_args(["--no-e2e", "--no-cpu-baseline"])
  assert bench.run_ours(args) == bench.GATE_FAILED_EXIT
  assert printed and printed[0]["parity_gate_failed"] == ["gemm8192"]
  args = bench.parse_args(["--no-e2e", "--no-cpu-baseline", "--no-extra-legs"])
  printed.clear()
  assert bench.run_ours(args) == 0 and "parity_gate_failed" not in printed[0]
