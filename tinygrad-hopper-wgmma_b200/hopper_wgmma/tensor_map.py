"""CUDA tensor-map construction for the reference's 3-D bf16 TMA layout (hopper_wgmma/tensor_map.py).

The GEMM itself encodes 2-D maps in C++ and passes them to the kernel as ``__grid_constant__`` parameters, so it needs
neither a device upload nor a device synchronization per ``run`` (the reference does both, tensor_map.py:22, :33).
This function keeps the reference's helper for callers that want the raw descriptor: the same 3-D view
(64, height, width/64) with strides (2*width, 128) bytes, box (64, box_h, box_w/64) and 128-byte swizzle, returned
as a 128-byte ``torch.uint8`` tensor on the source tensor's device."""
from __future__ import annotations

import ctypes

from . import _capi
from .tensors import operand


def make_tensor_map(tensor, box_h: int, box_w: int, height: int, width: int):
  if box_h <= 0 or box_w <= 0 or height <= 0 or width <= 0:
    raise ValueError("tensor-map dimensions must be positive")
  if box_w % 64 or width % 64:
    raise ValueError("tensor-map tile and width must be multiples of 64 bf16 elements")
  import torch
  op = operand(tensor)
  desc = (ctypes.c_uint8 * 128)()
  _capi.check(_capi.LIB.bg_encode_tensor_map_3d(desc, op.ptr, height, width, box_h, box_w), "cuTensorMapEncodeTiled")
  return torch.frombuffer(bytearray(bytes(desc)), dtype=torch.uint8).to(f"cuda:{op.device}")
