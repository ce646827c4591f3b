"""GPU parity at the benchmark configurations' full sizes, for the configs that produce the headline numbers.

Every case launches once on NaN-poisoned C and checks three things: 64 sampled rows against the fp32 CPU oracle
(oracle/gemm_ref.py: fp32 accumulation of the same bf16 inputs, scripts/smoke.py:41), every element against the
fp32 product on the GPU (cuBLAS fp32, TF32 off: the oracle's arithmetic at sizes the CPU cannot afford), both
within max|out - ref| / max|ref| <= 4e-3 (smoke.py:48, tightened from 2e-2), and no NaN left anywhere (smoke.py:45
poisons with 12345.0; NaN here). The configurations are the benchmark's:
  * 1024^3: compared whole with the CPU oracle, for the size-based choice and every ladder rung;
  * 8192^3: ``ladder.best_config`` (256x512 CTA-pair tiles, split accumulator, K serpentine) and the
    reference's best rung (cluster_hilbert), with B read as given (build_gemm_ws) and K-major (the bench's path);
  * the 12 sweep shapes: ``best_config(M, N, K)`` and cluster_hilbert through build_gemm_ws;
  * one rank's shard of the 32768^3 column-sharded GEMM (configs[4], 8 ranks: 32768 x 4096 x 32768) through
    plan_gemm_bt (K-major shard of BT, the bench's path) and plan_gemm_b (a column view of the full B[K, N]).
Inputs are seeded N(0,1) rounded to bf16, drawn on the GPU; the CPU oracle reads the same bits back."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 4e-3
ROWS = 64
SWEEP_SHAPES = [(512, 512, 512), (1024, 1024, 1024), (1536, 1536, 1536), (2048, 2048, 2048), (3072, 3072, 3072),
                (6144, 6144, 6144), (12288, 12288, 12288), (16384, 16384, 16384), (16384, 4096, 4096),
                (4096, 16384, 4096), (8192, 8192, 2048), (2048, 2048, 16384)]

_cache: dict = {}


def _bits(t) -> np.ndarray:
  import torch
  return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _inputs(M, N, K, dev, seed=7):
  """A[M,K] and B[K,N] bf16 on the device (kept for the next case of the same shape)."""
  import torch
  key = (M, N, K, seed)
  if key not in _cache:
    _cache.clear()
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(seed)
    A = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    B = torch.randn((K, N), generator=g, device=dev).to(torch.bfloat16)
    _cache[key] = (A, B)
  return _cache[key]


def _fp32_product(A, B):
  import torch
  tf32 = torch.backends.cuda.matmul.allow_tf32
  torch.backends.cuda.matmul.allow_tf32 = False
  try:
    return A.float() @ B.float()
  finally:
    torch.backends.cuda.matmul.allow_tf32 = tf32


def _check(C, A, B, label):
  """Sampled rows against the CPU oracle, every element against the fp32 product, NaN scan."""
  import torch
  from oracle import gemm_ref
  M = A.shape[0]
  assert not torch.isnan(C).any(), f"{label}: NaN survived"
  rows = np.sort(np.random.default_rng(M).choice(M, min(ROWS, M), replace=False))
  idx = torch.from_numpy(rows).to(A.device)
  ref_rows = gemm_ref.sampled_rows_ref(_bits(A.index_select(0, idx)), _bits(B), np.arange(len(rows)))
  out_rows = _bits(C.index_select(0, idx))
  rel_rows = gemm_ref.rel_err(out_rows, ref_rows)
  assert rel_rows <= TOL, f"{label}: sampled rows vs the CPU oracle rel={rel_rows:.2e}"
  ref = _fp32_product(A, B)
  rel = float((C.float() - ref).abs().max() / (ref.abs().max() + 1e-9))
  del ref
  assert rel <= TOL, f"{label}: full output vs the fp32 product rel={rel:.2e}"


def _run(launch, C):
  C.fill_(float("nan"))
  launch()
  launch.check()


# ------------------------------------------------------------------------------------------------------------------
# 1024^3 against the CPU oracle, whole
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("cfg_name", ["best", "tma_ring", "gated_ws", "role_split", "role_split_regs", "tma_store",
                                      "hilbert", "cluster", "cluster_hilbert"])
def test_1024_cube_against_the_cpu_oracle(cfg_name, cuda_dev):
  import torch
  from hopper_wgmma.ladder import LADDER, best_config, build
  from oracle import gemm_ref
  M = N = K = 1024
  cfg = best_config(M, N, K) if cfg_name == "best" else LADDER[cfg_name]
  a_bits, b_bits = gemm_ref.randn_bf16_bits((M, K), 0), gemm_ref.randn_bf16_bits((K, N), 1)
  to_dev = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(cuda_dev)
  A, B = to_dev(a_bits), to_dev(b_bits)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  launch = build(N, cfg, M, K)(A, B, C)
  _run(launch, C)
  out = _bits(C)
  assert gemm_ref.count_nan(out) == 0
  rel = gemm_ref.rel_err(out, gemm_ref.gemm_f32(a_bits, b_bits))
  assert rel <= TOL, f"{cfg_name}: rel={rel:.2e} ({launch.info()['kernel']})"


# ------------------------------------------------------------------------------------------------------------------
# 8192^3, both B layouts
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("layout", ["B_as_given", "BT_k_major"])
@pytest.mark.parametrize("cfg_name", ["best", "cluster_hilbert"])
def test_8192_cube(cfg_name, layout, cuda_dev):
  import torch
  from hopper_wgmma import build_gemm_ws
  from hopper_wgmma.gemm import plan_gemm_bt
  from hopper_wgmma.ladder import LADDER, best_config
  M = N = K = 8192
  cfg = best_config(M, N, K) if cfg_name == "best" else LADDER[cfg_name]
  A, B = _inputs(M, N, K, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  if layout == "B_as_given":
    launch = build_gemm_ws(N, cfg, M, K)(A, B, C)
  else:
    BT = B.t().contiguous()
    launch = plan_gemm_bt(A, BT, C, cfg)
  _run(launch, C)
  kernel = launch.info()["kernel"]
  assert kernel.endswith("b=N" if layout == "B_as_given" else "b=K"), kernel
  _check(C, A, B, f"8192^3 {cfg_name} {layout} ({kernel})")


# ------------------------------------------------------------------------------------------------------------------
# the 12 sweep shapes
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("cfg_name", ["best", "cluster_hilbert"])
@pytest.mark.parametrize("shape", SWEEP_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_sweep_shape(shape, cfg_name, cuda_dev):
  import torch
  from hopper_wgmma import build_gemm_ws
  from hopper_wgmma.ladder import LADDER, best_config
  M, N, K = shape
  cfg = best_config(M, N, K) if cfg_name == "best" else LADDER[cfg_name]
  A, B = _inputs(M, N, K, cuda_dev)
  C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
  launch = build_gemm_ws(N, cfg, M, K)(A, B, C)
  _run(launch, C)
  _check(C, A, B, f"{M}x{N}x{K} {cfg_name} ({launch.info()['kernel']})")


# ------------------------------------------------------------------------------------------------------------------
# one rank's shard of the 32768^3 column-sharded GEMM (rank 3 of 8)
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("entry", ["plan_gemm_bt", "plan_gemm_b"])
def test_32768_cube_rank_shard(entry, cuda_dev):
  import torch
  from hopper_wgmma import shard
  from hopper_wgmma.gemm import plan_gemm_b
  from hopper_wgmma.ladder import best_config
  M = N = K = 32768
  world, rank = 8, 3
  c0, c1 = shard.column_range(N, world, rank)
  cfg = best_config(M, c1 - c0, K)
  A, B = _inputs(M, N, K, cuda_dev)
  Bs = B[:, c0:c1]
  C = torch.empty((M, c1 - c0), dtype=torch.bfloat16, device=cuda_dev)
  if entry == "plan_gemm_bt":
    BT = shard.shard_bt(B.t().contiguous(), world, rank)   # the rank's rows of the K-major copy
    launch = shard.local_gemm(A, BT, C, cfg)
  else:
    launch = plan_gemm_b(A, Bs, C, cfg)                     # B's column block read in place (row pitch N)
  _run(launch, C)
  _check(C, A, Bs, f"32768^3 rank {rank}/{world} via {entry} ({launch.info()['kernel']})")
