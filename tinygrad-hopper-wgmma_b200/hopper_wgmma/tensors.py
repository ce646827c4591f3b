"""Tensor adapters: what the GEMM needs from an operand (device pointer, shape, dtype, device, layout).

The reference's ``launch()`` works over tinygrad Tensors and reads the raw CUDA pointer from a tinygrad internal
(hopper_wgmma/tensor_map.py:20-24). This build works over ``torch.Tensor`` (CUDA, bf16, row-major) and, when tinygrad
is importable, over realized tinygrad CUDA Tensors read the same way.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Operand:
  ptr: int
  shape: tuple[int, ...]
  bf16: bool
  device: int           # CUDA ordinal
  row_pitch: int        # elements between rows (row-major, unit inner stride)
  obj: object           # the original tensor, kept alive by the caller of the plan


def _torch_operand(t) -> Operand:
  import torch
  if t.device.type != "cuda": raise ValueError("tensors must live on a CUDA device")
  if t.dim() != 2: raise ValueError("tensors must be 2-D")
  if t.stride(1) != 1 or t.stride(0) < t.shape[1]: raise ValueError("tensors must be row-major with unit inner stride")
  return Operand(t.data_ptr(), tuple(t.shape), t.dtype == torch.bfloat16, t.device.index or 0, t.stride(0), t)


def _tinygrad_operand(t) -> Operand:
  from tinygrad import dtypes
  t.realize()
  try:
    ptr = int(t.uop.base.buffer._buf)
  except (AttributeError, TypeError, ValueError) as exc:
    raise ValueError("tensor must be a realized CUDA tensor") from exc
  dev = str(t.device)
  if not dev.upper().startswith("CUDA"): raise ValueError("tensors must live on a CUDA device")
  ordinal = int(dev.split(":")[1]) if ":" in dev else 0
  shape = tuple(int(s) for s in t.shape)
  return Operand(ptr, shape, t.dtype == dtypes.bfloat16, ordinal, shape[1], t)


def operand(t) -> Operand:
  mod = type(t).__module__
  if mod.startswith("torch"): return _torch_operand(t)
  if mod.startswith("tinygrad"): return _tinygrad_operand(t)
  raise ValueError(f"unsupported tensor type {type(t).__name__}: pass a torch.Tensor (or a tinygrad Tensor)")


def transpose_contiguous(B):
  """K-major copy of B (the reference's ``B.T.contiguous().realize()``, gemm.py:387), on B's own framework/stream."""
  mod = type(B).__module__
  if mod.startswith("torch"): return B.t().contiguous()
  return B.T.contiguous().realize()


def current_stream(t) -> int:
  """The stream a launch on ``t``'s device should use: torch's current stream (0 = legacy default otherwise)."""
  if type(t).__module__.startswith("torch"):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream
  return 0
