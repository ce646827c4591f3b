"""GPU parity tests of the sm_100a GEMM against the CPU oracle (oracle/gemm_ref.py).

Mirrors the reference's correctness harness (scripts/smoke.py): every case runs on a poisoned C (NaN here instead of
12345.0, smoke.py:45) three times (smoke.py:26, :43) and must stay within max|out-ref|/max|ref| <= 4e-3 of the fp32
host reference (smoke.py:41, :48; tolerance tightened from 2e-2). The 13 reference cases (smoke.py:19-25) come first,
then B200-specific cases: CTA pairs, ragged Hilbert deals, BN tails of the register epilogue, single k-block problems,
column-shard outputs, device-side timeouts, and full-size problems checked on sampled rows plus against cuBLAS.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 4e-3
REPS = 3
BUDGET_NS = 500_000_000   # per-wait device limit for the tests: a protocol error fails fast instead of stalling


def _torch():
  import torch
  return torch


def to_dev(bits: np.ndarray, dev):
  torch = _torch()
  return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def to_bits(t) -> np.ndarray:
  torch = _torch()
  return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def poison(t):
  t.fill_(float("nan"))


def fp32_product(A, B):
  """A @ B in fp32 on the GPU (cuBLAS, TF32 off): the oracle's arithmetic at sizes the CPU cannot afford."""
  torch = _torch()
  tf32 = torch.backends.cuda.matmul.allow_tf32
  torch.backends.cuda.matmul.allow_tf32 = False
  try:
    return A.float() @ B.float()
  finally:
    torch.backends.cuda.matmul.allow_tf32 = tf32


def inputs(M, N, K, seed=0):
  from oracle import gemm_ref
  return gemm_ref.randn_bf16_bits((M, K), seed), gemm_ref.randn_bf16_bits((K, N), seed + 1)


def run_case(build_fn, M, N, K, dev, reps=REPS):
  """Build, launch ``reps`` times on NaN-poisoned C, return the worst relative error (inf if NaN survived)."""
  from oracle import gemm_ref
  torch = _torch()
  a_bits, b_bits = inputs(M, N, K)
  A, B = to_dev(a_bits, dev), to_dev(b_bits, dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
  ref = gemm_ref.gemm_f32(a_bits, b_bits)
  launch = build_fn()(A, B, C)
  worst = 0.0
  for _ in range(reps):
    poison(C)
    launch()
    launch.check()
    out = to_bits(C)
    worst = max(worst, gemm_ref.rel_err(out, ref))
  return worst, launch


# ------------------------------------------------------------------------------------------------------------------
# the reference's smoke cases (scripts/smoke.py:19-25)
# ------------------------------------------------------------------------------------------------------------------
def _smoke_cases():
  from hopper_wgmma import WSCfg
  from hopper_wgmma.ladder import LADDER
  cases = [(name, cfg, (512, 512, 512)) for name, cfg in LADDER.items()]
  cases += [
    ("rectangular", WSCfg(), (512, 1024, 256)),
    ("rectangular_tma_store", WSCfg(tma_store=True), (1024, 512, 384)),
    ("bn192", WSCfg(BN=192, tma_store=True), (256, 768, 256)),
    ("group_m_1d", WSCfg(group_m=3), (768, 512, 256)),
    ("one_consumer", WSCfg(consumers=1), (512, 512, 512)),
  ]
  return cases


@pytest.mark.parametrize("idx", range(13))
def test_reference_smoke_cases(idx, cuda_dev):
  from hopper_wgmma.ladder import build
  name, cfg, (M, N, K) = _smoke_cases()[idx]
  worst, launch = run_case(lambda: build(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({launch.info()['kernel']})"


# ------------------------------------------------------------------------------------------------------------------
# B200-specific cases
# ------------------------------------------------------------------------------------------------------------------
def _b200_cases():
  from hopper_wgmma import GatedCfg, WSCfg
  return [
    ("pair_bn128", WSCfg(BN=128, tma_store=True, cluster=2), (512, 512, 512)),
    ("pair_regstore", WSCfg(cluster=2), (1024, 512, 256)),
    ("pair_hilbert_ragged", WSCfg(BN=128, tma_store=True, cluster=2, hilbert=True, num_sm=10), (1024, 640, 256)),
    ("hilbert_ragged", WSCfg(tma_store=True, hilbert=True, num_sm=7), (768, 1024, 320)),
    ("grouped_small_grid", WSCfg(BN=64, tma_store=True, num_sm=5), (640, 448, 192)),
    ("one_kblock", WSCfg(BN=128, tma_store=True), (256, 256, 64)),
    ("bn16_tail", WSCfg(BN=16), (256, 64, 128)),
    ("bn48_tail", WSCfg(BN=48, num_sm=4), (384, 240, 192)),
    ("bn112_tail", WSCfg(BN=112, consumers=1), (192, 336, 128)),
    ("bn240", WSCfg(BN=240, acc_bufs=2), (256, 480, 256)),
    ("one_acc_buffer", WSCfg(tma_store=True, acc_bufs=1), (512, 512, 512)),
    ("two_stages", WSCfg(BN=64, stages=2), (512, 256, 640)),
    ("consumer1_cluster2", WSCfg(consumers=1, cluster=2, tma_store=True), (512, 512, 256)),
    ("consumer1_tmast_bn64", WSCfg(consumers=1, BN=64, tma_store=True), (320, 192, 128)),
    ("tall_k", WSCfg(BN=128, tma_store=True, cluster=2), (256, 256, 4096)),
    ("many_tiles_pair", WSCfg(tma_store=True, cluster=2, hilbert=True), (2048, 2048, 512)),
    ("pair_wide", WSCfg(tma_store=True, cluster=2, n_mma=2), (512, 1024, 256)),
    ("wide_cta_regstore", WSCfg(BN=128, n_mma=2), (256, 512, 128)),
    ("wide_pair_hilbert_ragged", WSCfg(BN=128, n_mma=2, cluster=2, tma_store=True, hilbert=True, num_sm=6),
     (768, 1280, 192)),
    ("wide_c1_bn80", WSCfg(BN=80, n_mma=2, consumers=1), (128, 320, 64)),
    ("no_tail_split", WSCfg(tma_store=True, cluster=2, split_tail=False), (512, 512, 512)),
    ("tail_split_cta", WSCfg(BN=128, tma_store=True, num_sm=6), (512, 640, 192)),
    ("tail_split_pair", WSCfg(tma_store=True, cluster=2, hilbert=True, num_sm=18), (1024, 1792, 128)),
    ("tail_split_wide_pair", WSCfg(n_mma=2, cluster=2, tma_store=True, num_sm=10), (1024, 1536, 128)),
    ("tail_split_bm64_reg", WSCfg(consumers=1, BN=128, num_sm=7), (320, 384, 128)),
    ("wide_split_abc", WSCfg(n_mma=2, cluster=2, tma_store=True, split_tail=False), (512, 1024, 1024)),
    ("wide_split_all_phase_a", WSCfg(n_mma=2, cluster=2, tma_store=True, split_tail=False), (512, 1024, 128)),
    ("wide_split_no_phase_b", WSCfg(n_mma=2, cluster=2, tma_store=True, split_tail=False), (512, 1024, 192)),
    ("wide_split_many_tiles", WSCfg(n_mma=2, cluster=2, tma_store=True, hilbert=True, num_sm=6), (1024, 2048, 320)),
    ("wide_split_regstore", WSCfg(n_mma=2, cluster=2, split_tail=False), (256, 1024, 448)),
    ("wide_split_cta", WSCfg(n_mma=2, tma_store=True, split_tail=False, num_sm=3), (384, 1536, 256)),
    ("gated_c1", GatedCfg(consumers=1, BN=128), (512, 512, 512)),
    ("ring_bn256", GatedCfg(consumers=0, BN=256, stages=2), (256, 256, 256)),
    ("ring_bn64", GatedCfg(consumers=0, BN=64, stages=3), (192, 192, 192)),
    # K serpentine (on by default): odd-numbered tiles of a cluster walk K backwards
    ("k_forward_only", WSCfg(tma_store=True, cluster=2, hilbert=True, k_serpentine=False), (2048, 2048, 512)),
    ("k_serpentine_wide_waves", WSCfg(n_mma=2, cluster=2, tma_store=True, num_sm=10), (1024, 2048, 640)),
  ]


@pytest.mark.parametrize("idx", range(36))
def test_b200_cases(idx, cuda_dev):
  from hopper_wgmma.ladder import build
  name, cfg, (M, N, K) = _b200_cases()[idx]
  worst, launch = run_case(lambda: build(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({launch.info()['kernel']})"


# ------------------------------------------------------------------------------------------------------------------
# B operand layouts: B[K,N] read N-major as given (the default where the tile allows it) and the reference's K-major
# copy BT[N,K] (gemm.py:382), on the same configs
# ------------------------------------------------------------------------------------------------------------------
def _layout_cases():
  from hopper_wgmma import WSCfg
  return [
    ("cluster_hilbert", WSCfg(tma_store=True, hilbert=True, cluster=2), (512, 512, 512)),
    ("cta_bn256_regstore", WSCfg(), (512, 512, 320)),                          # 4 boxes of 64 columns per stage
    ("cta_bn192_no_tail", WSCfg(BN=192, tma_store=True, split_tail=False), (256, 768, 256)),
    ("m64_bn128", WSCfg(consumers=1, BN=128, tma_store=True, hilbert=True), (320, 384, 192)),
    ("pair_wide", WSCfg(tma_store=True, cluster=2, n_mma=2), (512, 1024, 256)),
    ("wide_split_abc", WSCfg(n_mma=2, cluster=2, tma_store=True, split_tail=False), (512, 1024, 1024)),
    ("tail_split_pair", WSCfg(tma_store=True, cluster=2, hilbert=True, num_sm=18), (1024, 1792, 128)),
    ("tail_split_cta", WSCfg(BN=128, tma_store=True, num_sm=6), (512, 640, 192)),
    ("tail_split_wide_pair", WSCfg(n_mma=2, cluster=2, tma_store=True, num_sm=10), (1024, 1536, 128)),
    ("ragged_pair", WSCfg(tma_store=True, hilbert=True, cluster=2, ragged=True), (1000, 1000, 520)),
    ("ragged_cta_reg", WSCfg(BN=128, ragged=True, num_sm=9), (333, 712, 136)),
    ("split_k4", WSCfg(BN=128, tma_store=True, split_k=4), (256, 256, 4096)),
    ("split_k2_wide_pair", WSCfg(n_mma=2, cluster=2, tma_store=True, split_k=2), (256, 1024, 2048)),
    ("serpentine_waves", WSCfg(n_mma=2, cluster=2, tma_store=True, num_sm=10), (1024, 2048, 640)),
    # unpaired CTAs in clusters of 2 (BM = 64): each CTA loads the whole N block; the last wave is split
    ("cluster2_unpaired_tail", WSCfg(consumers=1, cluster=2, BN=128, tma_store=True, num_sm=6), (640, 640, 192)),
  ]


@pytest.mark.parametrize("layout", ["N", "K"])
@pytest.mark.parametrize("idx", range(15))
def test_b_operand_layouts(idx, layout, cuda_dev):
  import dataclasses
  from hopper_wgmma import build_gemm_ws
  name, cfg, (M, N, K) = _layout_cases()[idx]
  cfg = dataclasses.replace(cfg, b_nmajor=layout == "N")
  assert cfg.reads_b_directly == (layout == "N"), name
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  kernel = launch.info()["kernel"]
  assert kernel.endswith(f"b={layout}"), kernel
  assert worst <= TOL, f"{name} b={layout} {M}x{N}x{K}: relative_error={worst:.5f} ({kernel})"


def test_n_major_b_column_views(cuda_dev):
  """plan_gemm_b on a column block of B and of C (both row pitches > N): a rank's shard needs no copy of B."""
  torch = _torch()
  from hopper_wgmma import WSCfg
  from hopper_wgmma.gemm import plan_gemm_b
  from oracle import gemm_ref
  M, N, K, W = 512, 2048, 384, 4
  a_bits, b_bits = inputs(M, N, K, seed=5)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda_dev)
  ref = gemm_ref.gemm_f32(a_bits, b_bits)
  n = N // W
  for r, cfg in ((1, WSCfg(tma_store=True, cluster=2, hilbert=True)), (3, WSCfg(BN=128, consumers=1))):
    launch = plan_gemm_b(A, B[:, r * n:(r + 1) * n], C[:, r * n:(r + 1) * n], cfg, wait_budget_ns=BUDGET_NS)
    launch()
    launch.check()
    assert launch.info()["kernel"].endswith("b=N")
  out = to_bits(C)
  for r in (1, 3):
    assert gemm_ref.rel_err(out[:, r * n:(r + 1) * n], ref[:, r * n:(r + 1) * n]) <= TOL
  rest = np.concatenate([out[:, :n], out[:, 2 * n:3 * n]], axis=1)
  assert (gemm_ref.bf16_bits_to_f32(rest) == 7.0).all()


def test_matches_cublas_bitwise_or_close(cuda_dev):
  """Against torch.matmul (cuBLAS) on the same bf16 inputs: the reference printed rel=0.00000 for every CHECK
  (scripts/ncu_workload.py:60-64). Both accumulate in fp32 and round to bf16, so most elements are bitwise equal;
  the summation order differs, so elements near zero or on a rounding boundary may not be. Parity itself is
  measured against the fp32 product."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  g = torch.Generator(device=cuda_dev).manual_seed(0)
  M = N = K = 1024
  A = torch.randn((M, K), generator=g, device=cuda_dev).to(torch.bfloat16)
  B = torch.randn((K, N), generator=g, device=cuda_dev).to(torch.bfloat16)
  C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
  launch = build_gemm_ws(N, WSCfg(tma_store=True, cluster=2, hilbert=True), M, K)(A, B, C)
  launch()
  launch.check()
  assert not torch.isnan(C).any()
  assert float((C == A @ B).float().mean()) >= 0.9
  ref = fp32_product(A, B)
  rel = float((C.float() - ref).abs().max() / (ref.abs().max() + 1e-9))
  assert rel <= TOL, rel


def test_column_shard_view_output(cuda_dev):
  """A GEMM written into a column block of a wider C (row pitch > N) leaves the other columns untouched."""
  torch = _torch()
  from hopper_wgmma import WSCfg
  from hopper_wgmma.gemm import plan_gemm_bt
  from oracle import gemm_ref
  M, N, K, W = 256, 1024, 256, 4
  a_bits, b_bits = inputs(M, N, K, seed=3)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  BT = B.t().contiguous()
  C = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=cuda_dev)
  n = N // W
  r = 2
  launch = plan_gemm_bt(A, BT[r * n:(r + 1) * n], C[:, r * n:(r + 1) * n], WSCfg(BN=128, tma_store=True, cluster=2),
                        wait_budget_ns=BUDGET_NS)
  launch()
  launch.check()
  ref = gemm_ref.gemm_f32(a_bits, b_bits)
  out = to_bits(C)
  assert gemm_ref.rel_err(out[:, r * n:(r + 1) * n], ref[:, r * n:(r + 1) * n]) <= TOL
  rest = np.concatenate([out[:, :r * n], out[:, (r + 1) * n:]], axis=1)
  assert (gemm_ref.bf16_bits_to_f32(rest) == 7.0).all()


@pytest.mark.parametrize("which", ["ws", "pair", "ring"])
def test_device_timeout_reports_error_and_context_survives(which, cuda_dev):
  """A stage the producer never loads makes the kernel's bounded waits run out: the launch reports an error through
  the error word, the kernel returns on its own, and the same context then runs a correct GEMM."""
  torch = _torch()
  from hopper_wgmma import GatedCfg, WSCfg
  from hopper_wgmma.ladder import build
  cfg = {"ws": WSCfg(BN=128, tma_store=True), "pair": WSCfg(BN=128, tma_store=True, cluster=2),
         "ring": GatedCfg(consumers=0, BN=128, stages=2)}[which]
  M = N = K = 256
  A = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda_dev)
  B = torch.zeros((K, N), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  bad = build(N, cfg, M, K, wait_budget_ns=50_000_000, debug_skip_job=1)(A, B, C)
  bad()
  with pytest.raises(RuntimeError, match="timed out"):
    bad.check()
  worst, _ = run_case(lambda: build(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev, reps=1)
  assert worst <= TOL


def test_launch_is_repeatable_and_async(cuda_dev):
  """Many launches back to back on one stream, one check at the end (no per-launch synchronization)."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from oracle import gemm_ref
  M = N = K = 512
  a_bits, b_bits = inputs(M, N, K, seed=5)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  launch = build_gemm_ws(N, WSCfg(tma_store=True, hilbert=True), M, K)(A, B, C)
  poison(C)
  for _ in range(20): launch()
  launch.check()
  assert gemm_ref.rel_err(to_bits(C), gemm_ref.gemm_f32(a_bits, b_bits)) <= TOL


def test_contract_errors_before_launch(cuda_dev):
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  run = build_gemm_ws(512, WSCfg())
  A = torch.zeros((512, 512), dtype=torch.bfloat16, device=cuda_dev)
  with pytest.raises(ValueError, match="shapes"):
    run(A, torch.zeros((512, 256), dtype=torch.bfloat16, device=cuda_dev), A)
  with pytest.raises(ValueError, match="bfloat16"):
    run(A, torch.zeros((512, 512), dtype=torch.float16, device=cuda_dev), A)
  with pytest.raises(ValueError, match="CUDA"):
    run(A.cpu(), A, A)


@pytest.mark.parametrize("size,cfg_name", [(4096, "cluster_hilbert"), (8192, "cluster_hilbert"), (4096, "tma_store")])
def test_full_size_sampled(size, cfg_name, cuda_dev):
  """Headline sizes: 64 sampled rows against the fp32 CPU oracle, every element against the fp32 product on the GPU
  (cuBLAS, TF32 off), NaN scan."""
  torch = _torch()
  from hopper_wgmma.ladder import LADDER, build
  from oracle import gemm_ref
  M = N = K = size
  a_bits, b_bits = inputs(M, N, K, seed=11)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  poison(C)
  launch = build(N, LADDER[cfg_name], M, K)(A, B, C)
  launch()
  launch.check()
  assert not torch.isnan(C).any()
  rows = np.random.default_rng(0).choice(M, 64, replace=False)
  ref_rows = gemm_ref.sampled_rows_ref(a_bits, b_bits, rows)
  out = to_bits(C)
  assert gemm_ref.rel_err(out[rows], ref_rows) <= TOL
  ref = fp32_product(A, B)
  rel = float((C.float() - ref).abs().max() / (ref.abs().max() + 1e-9))
  assert rel <= TOL, rel


# ------------------------------------------------------------------------------------------------------------------
# shapes that are not tile multiples (opt-in WSCfg(ragged=True); the reference rejects them, gemm.py:303)
# ------------------------------------------------------------------------------------------------------------------
def _ragged_cases():
  from hopper_wgmma import WSCfg
  return [
    ("pair_tmast_hilbert", WSCfg(tma_store=True, cluster=2, hilbert=True, ragged=True), (300, 520, 200)),
    ("pair_regstore", WSCfg(cluster=2, ragged=True), (777, 1000, 1000)),
    ("cta_tmast", WSCfg(BN=128, tma_store=True, ragged=True), (129, 136, 72)),
    ("wide_pair", WSCfg(n_mma=2, cluster=2, tma_store=True, ragged=True), (1000, 1200, 328)),
    ("bm64_reg_bn48", WSCfg(consumers=1, BN=48, ragged=True), (70, 104, 136)),
    ("one_row", WSCfg(tma_store=True, ragged=True), (1, 264, 64)),
    ("k8", WSCfg(cluster=2, tma_store=True, ragged=True), (256, 256, 8)),
    ("exact_multiple", WSCfg(tma_store=True, cluster=2, ragged=True), (512, 512, 512)),
  ]


@pytest.mark.parametrize("idx", range(8))
def test_ragged_shapes(idx, cuda_dev):
  from hopper_wgmma import build_gemm_ws
  name, cfg, (M, N, K) = _ragged_cases()[idx]
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({launch.info()['kernel']})"


# ------------------------------------------------------------------------------------------------------------------
# split-K (WSCfg(split_k=S)): S entries per output tile over disjoint K ranges, reduced in-kernel by the last arrival
# ------------------------------------------------------------------------------------------------------------------
def _split_k_cases():
  from hopper_wgmma import WSCfg
  return [
    ("cta_tmast_sk2", WSCfg(BN=128, tma_store=True, hilbert=True, split_k=2, split_k_cluster=False), (512, 512, 1024)),
    ("cta_reg_sk3_uneven_k", WSCfg(BN=128, split_k=3), (256, 256, 448)),               # 7 k-blocks: 2 + 2 + 3
    ("bm64_sk4", WSCfg(consumers=1, BN=128, tma_store=True, split_k=4), (256, 512, 512)),
    ("pair_tmast_sk2", WSCfg(tma_store=True, cluster=2, hilbert=True, split_k=2), (512, 512, 512)),
    ("pair_reg_sk4", WSCfg(cluster=2, split_k=4), (512, 512, 1024)),
    ("wide_pair_sk2", WSCfg(n_mma=2, cluster=2, tma_store=True, split_k=2), (512, 1024, 1024)),
    ("wide_pair_sk3_short", WSCfg(n_mma=2, cluster=2, tma_store=True, split_k=3), (512, 1024, 384)),
    ("waves_sk2", WSCfg(BN=128, tma_store=True, hilbert=True, num_sm=6, split_k=2), (512, 640, 256)),
    ("one_kblock_each_sk8", WSCfg(BN=64, tma_store=True, split_k=8), (128, 256, 512)),
    ("ragged_pair_sk2", WSCfg(tma_store=True, cluster=2, ragged=True, split_k=2), (300, 520, 1000)),
    ("pair_sk5_few_clusters", WSCfg(cluster=2, split_k=5, num_sm=8), (512, 256, 640)),
    ("small_ring_sk2", WSCfg(BN=128, stages=3, split_k=2, split_k_cluster=False), (256, 512, 1024)),   # registers
    ("bm64_reg_sk6", WSCfg(consumers=1, BN=64, split_k=6), (192, 256, 768)),
  ]


@pytest.mark.parametrize("idx", range(13))
def test_split_k(idx, cuda_dev):
  """Three launches of one plan on NaN-poisoned C: also checks that every launch leaves the arrival words zero.
  Single-wave cases reduce through the idle operand ring (cp.async), the others and small rings through registers."""
  from hopper_wgmma import build_gemm_ws
  name, cfg, (M, N, K) = _split_k_cases()[idx]
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  info = launch.info()
  assert info["split_k"] == cfg.split_k and f"splitk={cfg.split_k} " in info["kernel"]   # through the workspace
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({info['kernel']})"


def test_split_k_is_bitwise_reproducible(cuda_dev):
  """The last arrival adds the splits in split order whatever the arrival order, so repeated launches agree bit for
  bit (while the splits race differently each time)."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  M, N, K = 768, 768, 2048
  a_bits, b_bits = inputs(M, N, K, seed=21)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  launch = build_gemm_ws(N, WSCfg(BN=128, tma_store=True, split_k=4), M, K, wait_budget_ns=BUDGET_NS)(A, B, C)
  outs = []
  for _ in range(5):
    poison(C)
    launch()
    launch.check()
    outs.append(to_bits(C))
  assert all((o == outs[0]).all() for o in outs[1:])


def test_split_k_timeout_reports_error_and_plans_recover(cuda_dev):
  """A split that never gets its operands: the other splits of its tile publish and leave (none of them is last),
  the stuck one times out, the launch reports the error and the host clears the arrival words."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  cfg = WSCfg(BN=128, tma_store=True, split_k=2, split_k_cluster=False)
  M = N = K = 256
  A = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda_dev)
  B = torch.zeros((K, N), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  bad = build_gemm_ws(N, cfg, M, K, wait_budget_ns=50_000_000, debug_skip_job=1)(A, B, C)
  bad()
  with pytest.raises(RuntimeError, match="timed out"):
    bad.check()
  worst, _ = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev, reps=2)
  assert worst <= TOL


def test_split_k_auto_choice(cuda_dev):
  """split_k=-1 splits only shapes with few tiles and long K: as many splits as keep one wave of clusters, each
  with at least 32 k-blocks, or 24 where the splits meet inside a cluster."""
  from hopper_wgmma import WSCfg, build_gemm_ws
  from hopper_wgmma._capi import device_info
  sms = device_info(cuda_dev.index or 0)["sm_count"]
  cfg = WSCfg(BN=64, tma_store=True, split_k=-1)
  M, N, K = 256, 1024, 16384                      # 2 x 16 tiles of 128 x 64, 256 k-blocks
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev, reps=2)
  assert worst <= TOL
  assert launch.info()["split_k"] == min(sms // 32, 8, 16)
  _, launch = run_case(lambda: build_gemm_ws(1024, cfg, 1024, 1024, wait_budget_ns=BUDGET_NS), 1024, 1024, 1024,
                       cuda_dev, reps=1)
  assert launch.info()["split_k"] == 1            # 16 k-blocks: too short to split
  cfg = WSCfg(BN=128, tma_store=True, split_k=-1)
  M, N, K = 1024, 1024, 3072                      # 64 tiles, 48 k-blocks: two splits of 24 inside clusters
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev, reps=2)
  assert worst <= TOL
  assert launch.info()["split_k"] == 2 and "splitk=2/cluster" in launch.info()["kernel"]
  _, launch = run_case(lambda: build_gemm_ws(N, cfg, M, 2048, wait_budget_ns=BUDGET_NS), M, N, 2048, cuda_dev, reps=1)
  assert launch.info()["split_k"] == 1            # 32 k-blocks: splits of 16 gain nothing


# ------------------------------------------------------------------------------------------------------------------
# split-K inside a cluster (split_k_cluster): the splits of a tile are the CTAs of one cluster and add up through
# distributed shared memory
# ------------------------------------------------------------------------------------------------------------------
def _split_k_cluster_cases():
  from hopper_wgmma import WSCfg
  return [
    ("cta_tmast_sk2", WSCfg(BN=128, tma_store=True, hilbert=True, split_k=2, split_k_cluster=True), (512, 512, 1024)),
    ("cta_reg_sk2_uneven_k", WSCfg(BN=128, split_k=2, split_k_cluster=True), (256, 384, 448)),   # 7 k-blocks: 3 + 4
    ("cta_bn256_sk2_b_as_given", WSCfg(BN=256, tma_store=True, split_k=2, split_k_cluster=True), (256, 512, 1024)),
    ("cta_bn256_sk4", WSCfg(BN=256, tma_store=True, split_k=4, split_k_cluster=True), (256, 512, 2048)),
    ("cta_reg_sk4_32_columns_each", WSCfg(BN=128, split_k=4, split_k_cluster=True), (256, 256, 1024)),
    ("bm64_sk2", WSCfg(consumers=1, BN=128, tma_store=True, split_k=2, split_k_cluster=True), (192, 256, 512)),
    ("bn64_reg_sk2", WSCfg(BN=64, split_k=2, split_k_cluster=True), (256, 192, 640)),
    ("ragged_sk2", WSCfg(BN=128, tma_store=True, ragged=True, split_k=2, split_k_cluster=True), (300, 520, 1000)),
    ("one_kblock_each_sk4", WSCfg(BN=256, tma_store=True, split_k=4, split_k_cluster=True), (128, 256, 256)),
    ("auto_picks_cluster", WSCfg(BN=128, tma_store=True, split_k=2), (384, 512, 2048)),
    ("bm64_reg_sk2", WSCfg(consumers=1, BN=128, split_k=2, split_k_cluster=True), (256, 256, 512)),
    ("bn192_reg_sk2_three_chunks_each", WSCfg(BN=192, split_k=2, split_k_cluster=True), (256, 384, 512)),
    ("ragged_reg_sk4", WSCfg(BN=256, ragged=True, split_k=4, split_k_cluster=True), (200, 600, 904)),
  ]


@pytest.mark.parametrize("idx", range(13))
def test_split_k_in_cluster(idx, cuda_dev):
  """Three launches of one plan on NaN-poisoned C, against the CPU oracle: every tile's splits run on one cluster and
  exchange their sums through distributed shared memory (the plan's kernel name says so)."""
  from hopper_wgmma import build_gemm_ws
  name, cfg, (M, N, K) = _split_k_cluster_cases()[idx]
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  info = launch.info()
  assert info["split_k"] == cfg.split_k and f"splitk={cfg.split_k}/cluster" in info["kernel"], info["kernel"]
  assert info["grid"] == cfg.split_k * info["tiles"]
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({info['kernel']})"


@pytest.mark.parametrize("cfg_name", ["sk2_tma_store", "sk4_registers"])
def test_split_k_cluster_matches_the_workspace_bitwise(cfg_name, cuda_dev):
  """Both protocols add the splits in split order 0, 1, ..., S - 1 onto the same per-split sums, so their outputs
  agree bit for bit."""
  import dataclasses
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  base, (M, N, K) = {
    "sk2_tma_store": (WSCfg(BN=128, tma_store=True, hilbert=True, split_k=2), (512, 768, 1536)),
    "sk4_registers": (WSCfg(BN=128, split_k=4), (384, 512, 2048)),
  }[cfg_name]
  a_bits, b_bits = inputs(M, N, K, seed=23)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  outs = {}
  for in_cluster in (True, False):
    C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
    poison(C)
    cfg = dataclasses.replace(base, split_k_cluster=in_cluster)
    launch = build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)(A, B, C)
    launch()
    launch.check()
    assert ("/cluster" in launch.info()["kernel"]) == in_cluster
    outs[in_cluster] = to_bits(C)
  assert (outs[True] == outs[False]).all()


def test_split_k_cluster_timeout_reports_error_and_plans_recover(cuda_dev):
  """K = 320 splits 2 + 3 k-blocks: only split 1 has a job 2, which its producer skips, so split 0 sends its share,
  waits for split 1's in vain and reports the timeout; the context stays usable and the next plan is right."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  cfg = WSCfg(BN=128, tma_store=True, split_k=2, split_k_cluster=True)
  M, N, K = 256, 256, 320
  A = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda_dev)
  B = torch.zeros((K, N), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  bad = build_gemm_ws(N, cfg, M, K, wait_budget_ns=50_000_000, debug_skip_job=2)(A, B, C)
  bad()
  with pytest.raises(RuntimeError, match="timed out"):
    bad.check()
  worst, _ = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev, reps=2)
  assert worst <= TOL


@pytest.mark.parametrize("case", ["pair", "three_splits", "narrow_share", "too_many_tiles"])
def test_split_k_cluster_refusals(case, cuda_dev):
  """split_k_cluster=True where a cluster cannot hold the splits fails before any launch, naming the reason; the
  automatic choice falls back to the workspace on the same plan."""
  import dataclasses
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  cfg, (M, N, K), why = {
    "pair": (WSCfg(tma_store=True, cluster=2, split_k=2), (512, 512, 512), "single-CTA tiles"),
    "three_splits": (WSCfg(BN=128, split_k=3), (256, 256, 768), "split_k 2 or 4"),
    "narrow_share": (WSCfg(BN=128, tma_store=True, split_k=4), (256, 256, 1024), "multiple of 64"),
    "too_many_tiles": (WSCfg(BN=128, tma_store=True, split_k=2), (2048, 2048, 512), "own cluster"),
  }[case]
  A = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda_dev)
  B = torch.zeros((K, N), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  with pytest.raises((RuntimeError, ValueError), match=why):
    build_gemm_ws(N, dataclasses.replace(cfg, split_k_cluster=True), M, K)(A, B, C)
  launch = build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)(A, B, C)
  assert "/cluster" not in launch.info()["kernel"]
  launch()
  launch.check()


def test_plan_tables_hold_bounded_device_memory(cuda_dev):
  """Plans for 1000 distinct M values (a caller with ragged batch sizes): each plan's tile table is shared while a
  plan uses it and freed (beyond a small idle cache) once none does, so device memory stays bounded; a shape whose
  table was evicted on the way plans and computes correctly again."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from hopper_wgmma.gemm import plan_gemm_bt
  cfg = WSCfg(tma_store=True, hilbert=True)           # 128 x 256 tiles, Hilbert table
  small = lambda: build_gemm_ws(512, cfg, 512, 320, wait_budget_ns=BUDGET_NS)
  worst, _ = run_case(small, 512, 512, 320, cuda_dev, reps=1)   # its table goes idle when the plan is dropped
  assert worst <= TOL
  N, K, M_max = 4096, 64, 128 * 2000
  A = torch.zeros((M_max, K), dtype=torch.bfloat16, device=cuda_dev)
  BT = torch.zeros((N, K), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.zeros((M_max, N), dtype=torch.bfloat16, device=cuda_dev)

  def plans(lo, hi):
    for i in range(lo, hi):
      M = 128 * (1000 + i)                            # 1000-2000 row tiles x 16 column tiles: 64-128 KB tables
      launch = plan_gemm_bt(A[:M], BT, C[:M], cfg)
      del launch
  plans(0, 100)
  torch.cuda.synchronize(cuda_dev)
  free_warm = torch.cuda.mem_get_info(cuda_dev)[0]
  plans(100, 1000)
  torch.cuda.synchronize(cuda_dev)
  free_after = torch.cuda.mem_get_info(cuda_dev)[0]
  # unbounded, 900 more tables of 64-128 KB would take ~90 MB
  assert free_warm - free_after < (24 << 20), (free_warm, free_after)
  worst, _ = run_case(small, 512, 512, 320, cuda_dev, reps=1)
  assert worst <= TOL


# ------------------------------------------------------------------------------------------------------------------
# wave barrier (WSCfg(wave_sync=True)): the producers of all CTAs meet at every tile boundary
# ------------------------------------------------------------------------------------------------------------------
def _wave_sync_cases():
  from hopper_wgmma import WSCfg
  return [
    ("pair_hilbert_8_waves", WSCfg(tma_store=True, cluster=2, hilbert=True, num_sm=8, wave_sync=True), (1024, 2048, 256)),
    ("pair_ragged_deal", WSCfg(tma_store=True, cluster=2, hilbert=True, num_sm=14, wave_sync=True), (1280, 1536, 192)),
    ("cta_tail_split", WSCfg(BN=128, tma_store=True, num_sm=6, wave_sync=True), (512, 640, 192)),
    ("wide_pair_waves", WSCfg(n_mma=2, cluster=2, tma_store=True, num_sm=10, wave_sync=True), (1024, 2048, 640)),
    ("regstore_bm64", WSCfg(consumers=1, BN=128, num_sm=7, wave_sync=True), (320, 384, 128)),
  ]


@pytest.mark.parametrize("idx", range(5))
def test_wave_sync(idx, cuda_dev):
  """Three launches of one plan: the barrier's counter keeps counting across launches (each launch starts from
  where the previous one left it)."""
  from hopper_wgmma import build_gemm_ws
  name, cfg, (M, N, K) = _wave_sync_cases()[idx]
  worst, launch = run_case(lambda: build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS), M, N, K, cuda_dev)
  assert "wavesync" in launch.info()["kernel"], launch.info()["kernel"]
  assert worst <= TOL, f"{name} {M}x{N}x{K}: relative_error={worst:.5f} ({launch.info()['kernel']})"


def test_wave_sync_many_launches_and_auto_choice(cuda_dev):
  """Fifty launches back to back with one check at the end. The automatic choice turns the barrier on where a wave's
  operand panels outgrow L2 and each cluster runs several tiles (256x512 pair tiles at 8192^3), and leaves it off
  for short K (4096^3 with 256x256 pair tiles, 6144^3 with 256x512)."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from hopper_wgmma.gemm import plan_gemm_bt
  from hopper_wgmma.ladder import LADDER, best_config
  from oracle import gemm_ref
  M, N, K = 1024, 2048, 128
  a_bits, b_bits = inputs(M, N, K, seed=8)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  launch = build_gemm_ws(N, WSCfg(tma_store=True, cluster=2, hilbert=True, num_sm=8, wave_sync=True), M, K,
                         wait_budget_ns=BUDGET_NS)(A, B, C)              # 32 tiles on 4 clusters: 8 each
  assert "wavesync" in launch.info()["kernel"]
  poison(C)
  for _ in range(50): launch()
  launch.check()
  assert gemm_ref.rel_err(to_bits(C), gemm_ref.gemm_f32(a_bits, b_bits)) <= TOL
  for size, cfg, on in ((8192, best_config(8192, 8192, 8192), True), (6144, best_config(6144, 6144, 6144), False),
                        (4096, LADDER["cluster_hilbert"], False)):
    X = torch.empty((size, size), dtype=torch.bfloat16, device=cuda_dev)
    plan = plan_gemm_bt(X, X, X, cfg)                                    # planned only, never launched
    assert ("wavesync" in plan.info()["kernel"]) == on, (size, plan.info()["kernel"])
    del plan, X


def test_wave_sync_timeout_reports_error_and_recovers(cuda_dev):
  """A stage the producer never loads in a plan with the wave barrier: the launch's bounded waits run out, the launch
  reports the error (and the check resets the plan's wave counter), and the GPU then runs wave-barrier plans
  correctly, twice in a row."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from oracle import gemm_ref
  cfg = WSCfg(BN=128, tma_store=True, num_sm=4, wave_sync=True)
  M, N, K = 512, 512, 128                                               # 16 tiles on 4 CTAs
  a_bits, b_bits = inputs(M, N, K, seed=9)
  A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  bad = build_gemm_ws(N, cfg, M, K, wait_budget_ns=50_000_000, debug_skip_job=1)(A, B, C)
  bad()
  with pytest.raises(RuntimeError, match="timed out"):
    bad.check()
  good = build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)(A, B, C)
  for _ in range(2):
    poison(C)
    good()
    good.check()
    assert gemm_ref.rel_err(to_bits(C), gemm_ref.gemm_f32(a_bits, b_bits)) <= TOL


def test_registered_shared_memory_budget_limits_the_ring(cuda_dev):
  """A caller lowers the dynamic shared memory registered for a kernel name (the reference's
  runtime.set_dynamic_smem_bytes) before run(): the plan's ring has the stages that fit, and the GEMM is still right."""
  from hopper_wgmma import WSCfg, build_gemm_ws, runtime
  cfg = WSCfg(tma_store=True, cluster=2, hilbert=True)
  M = N = K = 1024
  holder = {}

  def build():
    run = build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)
    runtime.set_dynamic_smem_bytes(run.kernel_name, 150_000)
    holder["run"] = run
    return run
  worst, launch = run_case(build, M, N, K, cuda_dev, reps=1)
  assert launch.info()["stages"] == cfg.within_smem(150_000).stages == 3
  assert worst <= TOL


def test_wave_sync_launches_side_by_side_on_two_streams(cuda_dev):
  """Two wave-barrier launches of full-GPU persistent grids on two streams at once: their CTAs cannot all be
  resident together, and the soft barrier must let both finish correctly without reporting an error."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from oracle import gemm_ref
  M, N, K = 2048, 4096, 512
  cfg = WSCfg(tma_store=True, cluster=2, hilbert=True, wave_sync=True)   # 128 tiles on 74 clusters
  runs = []
  for seed in (30, 31):
    a_bits, b_bits = inputs(M, N, K, seed=seed)
    A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
    C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
    poison(C)
    runs.append((a_bits, b_bits, C, build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)(A, B, C)))
  assert "wavesync" in runs[0][3].info()["kernel"]
  streams = [torch.cuda.Stream(device=cuda_dev) for _ in runs]
  torch.cuda.synchronize(cuda_dev)
  for _ in range(5):
    for st, (_, _, _, launch) in zip(streams, runs):
      with torch.cuda.stream(st):
        launch()
  for st, (a_bits, b_bits, C, launch) in zip(streams, runs):
    with torch.cuda.stream(st):
      launch.check()
    assert gemm_ref.rel_err(to_bits(C), gemm_ref.gemm_f32(a_bits, b_bits)) <= TOL


def test_split_k_cluster_launches_side_by_side_on_two_streams(cuda_dev):
  """Two split-K-inside-a-cluster launches of 128 CTAs each on two streams at once (more CTAs than SMs together):
  only a cluster's own CTAs wait for each other, and the GPU schedules a cluster whole, so both finish correctly
  without a timeout."""
  torch = _torch()
  from hopper_wgmma import WSCfg, build_gemm_ws
  from oracle import gemm_ref
  M, N, K = 1024, 1024, 2048
  cfg = WSCfg(BN=128, tma_store=True, split_k=2, split_k_cluster=True)   # 64 tiles x 2 splits
  runs = []
  for seed in (40, 41):
    a_bits, b_bits = inputs(M, N, K, seed=seed)
    A, B = to_dev(a_bits, cuda_dev), to_dev(b_bits, cuda_dev)
    C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
    poison(C)
    runs.append((a_bits, b_bits, C, build_gemm_ws(N, cfg, M, K, wait_budget_ns=BUDGET_NS)(A, B, C)))
  assert "splitk=2/cluster" in runs[0][3].info()["kernel"] and runs[0][3].info()["grid"] == 128
  streams = [torch.cuda.Stream(device=cuda_dev) for _ in runs]
  torch.cuda.synchronize(cuda_dev)
  for _ in range(5):
    for st, (_, _, _, launch) in zip(streams, runs):
      with torch.cuda.stream(st):
        launch()
  for st, (a_bits, b_bits, C, launch) in zip(streams, runs):
    with torch.cuda.stream(st):
      launch.check()
    assert gemm_ref.rel_err(to_bits(C), gemm_ref.gemm_f32(a_bits, b_bits)) <= TOL
