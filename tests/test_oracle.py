"""The CPU oracle, pinned before it is trusted: exact known answers for the GEMM oracle and the reference's own
outputs (tests/golden/reference_host.json) for the tile-order oracle."""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

from oracle import gemm_ref, schedule_ref


def bf16_round_exact(v: Fraction) -> Fraction:
  """Round a rational to bf16 (8 significant bits, ties to even) with exact arithmetic: independent of numpy."""
  if v == 0: return Fraction(0)
  sign = -1 if v < 0 else 1
  a = abs(v)
  e = 0
  while a >= 2: a /= 2; e += 1
  while a < 1: a *= 2; e -= 1
  q = a * 128                      # 1.xxxxxxx -> 8 significant bits
  r = round(q)                     # Python rounds Fractions half to even
  return sign * Fraction(r, 128) * Fraction(2) ** e


def test_bf16_rounding_known_answers():
  x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0, -0.0, 3.0e38, 1e-40, np.inf, -np.inf],
               dtype=np.float32)
  bits = gemm_ref.f32_to_bf16_bits(x)
  # 1 + 2^-8 is the tie between 1 and 1 + 2^-7: even mantissa (1.0) wins; 1 + 3*2^-8 rounds up to 1 + 2^-6
  assert list(bits[:6]) == [0x3F80, 0x3F80, 0x3F82, 0xC020, 0x0000, 0x8000]
  assert bits[8] == 0x7F80 and bits[9] == 0xFF80
  assert gemm_ref.f32_to_bf16_bits(np.array([np.nan], np.float32))[0] == 0x7FC0
  back = gemm_ref.bf16_bits_to_f32(bits[:4])
  assert back.tolist() == [1.0, 1.0, 1.0 + 2 ** -6, -2.5]


def test_bf16_rounding_matches_exact_rounding_on_random_values():
  rng = np.random.default_rng(7)
  x = (rng.standard_normal(2000) * 10.0 ** rng.integers(-3, 4, 2000)).astype(np.float32)
  bits = gemm_ref.f32_to_bf16_bits(x)
  got = gemm_ref.bf16_bits_to_f32(bits)
  for xi, gi in zip(x.tolist(), got.tolist()):
    assert Fraction(gi) == bf16_round_exact(Fraction(xi))


@pytest.mark.parametrize("M,N,K", [(8, 8, 8), (16, 24, 64), (5, 7, 130)])
def test_gemm_oracle_exact_on_integer_inputs(M, N, K):
  """Integer-valued bf16 inputs in [-4, 4]: every fp32 partial sum is an exact integer, so the fp32 oracle must equal
  the Python-integer product exactly, and the bf16 operator must equal its exact RNE rounding."""
  rng = np.random.default_rng(M * 1000 + N * 10 + K)
  a = rng.integers(-4, 5, (M, K))
  b = rng.integers(-4, 5, (K, N))
  a_bits = gemm_ref.f32_to_bf16_bits(a.astype(np.float32))
  b_bits = gemm_ref.f32_to_bf16_bits(b.astype(np.float32))
  exact = [[sum(int(a[i, k]) * int(b[k, j]) for k in range(K)) for j in range(N)] for i in range(M)]
  f32 = gemm_ref.gemm_f32(a_bits, b_bits)
  assert (f32 == np.array(exact, dtype=np.float64)).all()
  out = gemm_ref.bf16_bits_to_f32(gemm_ref.gemm_bf16(a_bits, b_bits))
  for i in range(M):
    for j in range(N):
      assert Fraction(float(out[i, j])) == bf16_round_exact(Fraction(exact[i][j]))


def test_rel_err_metric_and_nan():
  ref = np.array([[100.0, -50.0], [25.0, 0.0]], np.float32)
  out = gemm_ref.f32_to_bf16_bits(np.array([[100.0, -49.0], [25.0, 0.5]], np.float32))
  assert gemm_ref.rel_err(out, ref) == pytest.approx(1.0 / 100.0, rel=1e-6)
  poisoned = out.copy()
  poisoned[0, 0] = 0x7FC0
  assert gemm_ref.rel_err(poisoned, ref) == float("inf")
  assert gemm_ref.count_nan(poisoned) == 1


def test_seeded_inputs_are_deterministic_and_normal():
  a = gemm_ref.randn_bf16_bits((256, 256), seed=0)
  b = gemm_ref.randn_bf16_bits((256, 256), seed=0)
  assert (a == b).all()
  f = gemm_ref.bf16_bits_to_f32(a)
  assert abs(float(f.mean())) < 0.02 and abs(float(f.std()) - 1.0) < 0.02


def test_scale_of_reference_sized_products():
  """The reference printed max|ref| ~ 5.4-6.4 sqrt(K) for N(0,1) inputs (results/*: 100.5 at 512^3, 159 at 1024^3);
  the oracle's seeded products land in the same band (a sanity check of the distribution, not of values)."""
  M = N = K = 512
  ref = gemm_ref.gemm_f32(gemm_ref.randn_bf16_bits((M, K), 0), gemm_ref.randn_bf16_bits((K, N), 1))
  assert 4.5 * K ** 0.5 < float(np.abs(ref).max()) < 7.0 * K ** 0.5


def test_sampled_rows_match_full_product():
  a = gemm_ref.randn_bf16_bits((64, 128), 3)
  b = gemm_ref.randn_bf16_bits((128, 32), 4)
  rows = np.array([0, 5, 63])
  assert np.array_equal(gemm_ref.sampled_rows_ref(a, b, rows), gemm_ref.gemm_f32(a, b)[rows])


# ----------------------------------------------------------------------------------------------------------------
# tile-order oracle pinned against the reference's own functions
# ----------------------------------------------------------------------------------------------------------------
def test_hilbert_schedule_oracle_matches_reference(golden):
  for case in golden["hilbert_schedule"]:
    if "error" in case:
      with pytest.raises(ValueError) as exc:
        schedule_ref.hilbert_schedule(case["M"], case["N"], case["cores"])
      assert str(exc.value) == case["error"]
    else:
      assert schedule_ref.hilbert_schedule(case["M"], case["N"], case["cores"]) == case["ok"]


def test_grouped_order_oracle_matches_reference(golden):
  for case in golden["grouped_tile_order"]:
    CMT, NT, GM, GN = case["CMT"], case["NT"], case["GM"], case["GN"]
    assert schedule_ref.is_grouped_2d(CMT, NT, GM, GN) == case["grouped_2d"]
    got = [list(schedule_ref.grouped_coords(CMT, NT, GM, GN, t)) for t in range(CMT * NT)]
    assert got == case["coords"]


def test_dealt_tables_cover_every_tile_once():
  for CMT, NT, cores in [(16, 16, 74), (7, 3, 5), (32, 16, 148), (1, 1, 3)]:
    curve = schedule_ref.hilbert_curve(CMT, NT)
    assert sorted(curve) == sorted((m << 16) | n for m in range(CMT) for n in range(NT))
    per = schedule_ref.assignment(curve, cores)
    assert sum(len(p) for p in per) == CMT * NT
    assert max(len(p) for p in per) - min(len(p) for p in per) <= 1
