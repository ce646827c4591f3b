"""CPU oracle for the bf16 GEMM. TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline may use it, as the checker or the timed CPU stand-in; the product path never calls it.

What it restates (reference citations are paths inside narain1/tinygrad-hopper-wgmma):
  * the host reference of the correctness harness, ``ref = a.float().numpy() @ b.float().numpy()``
    (scripts/smoke.py:41): fp32 accumulation over bf16-exact inputs, here numpy's float32 matmul;
  * the comparison metric ``max|to_f32(out) - ref| / (max|ref| + 1e-9)`` (scripts/smoke.py:48) with ``to_f32`` =
    bf16 bits shifted into the high half of a float32 (scripts/smoke.py:30-31);
  * the poisoned-output check (scripts/smoke.py:45), with NaN as the poison: no NaN may survive a launch;
  * the tolerance, tightened from 2e-2 (scripts/smoke.py:27) to 4e-3.
Inputs: seeded i.i.d. N(0,1) float32 rounded to bf16 (round to nearest even), generated here so that the GPU and the
oracle see identical bits. The reference draws them with tinygrad's RNG (scripts/smoke.py:38-39), whose stream is not
reproducible without tinygrad; only the distribution matches.

Parity pinning: the reference stores no GEMM value vectors, and its stock tinygrad CPU ``A @ B`` cannot run here (the
tinygrad submodule is empty and not installable offline), so the numerics oracle is pinned against exact known
answers instead (integer-valued inputs whose fp32 sums are exact, checked with Python integers in
tests/test_oracle.py). At the tinygrad boundary itself parity is unpinned.
"""
from __future__ import annotations

import numpy as np

TOL = 4e-3


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
  """float32 -> bf16 bit patterns (uint16), round to nearest, ties to even; NaN stays a quiet NaN."""
  x = np.ascontiguousarray(x, dtype=np.float32)
  u = x.view(np.uint32).astype(np.uint64)
  lsb = (u >> 16) & 1
  r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
  nan = np.isnan(x)
  if nan.any(): r[nan] = 0x7FC0
  return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
  """bf16 bit patterns -> float32 (exact): the bits become the high half (scripts/smoke.py:30-31)."""
  return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def randn_bf16_bits(shape: tuple[int, ...], seed: int) -> np.ndarray:
  """Seeded i.i.d. N(0,1) float32 rounded to bf16; returns uint16 bits."""
  rng = np.random.default_rng(seed)
  return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))


def gemm_f32(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
  """fp32-accumulated A @ B over bf16 inputs (A: M x K bits, B: K x N bits), float32 result before output rounding."""
  return bf16_bits_to_f32(a_bits) @ bf16_bits_to_f32(b_bits)


def gemm_bf16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
  """The full operator: fp32 accumulate, one rounding to bf16 at the end. Returns uint16 bits."""
  return f32_to_bf16_bits(gemm_f32(a_bits, b_bits))


def rel_err(out_bits: np.ndarray, ref: np.ndarray) -> float:
  """max|to_f32(out) - ref| / (max|ref| + 1e-9) (scripts/smoke.py:48). NaN anywhere in out gives inf."""
  out = bf16_bits_to_f32(out_bits).astype(np.float64)
  ref = np.asarray(ref, dtype=np.float64)
  if np.isnan(out).any(): return float("inf")
  return float(np.max(np.abs(out - ref)) / (np.max(np.abs(ref)) + 1e-9))


def count_nan(out_bits: np.ndarray) -> int:
  return int(np.isnan(bf16_bits_to_f32(out_bits)).sum())


def sampled_rows_ref(a_bits: np.ndarray, b_bits: np.ndarray, rows: np.ndarray) -> np.ndarray:
  """fp32 reference for a subset of output rows (for problems too large to multiply whole on the CPU)."""
  return bf16_bits_to_f32(a_bits[rows]) @ bf16_bits_to_f32(b_bits)
