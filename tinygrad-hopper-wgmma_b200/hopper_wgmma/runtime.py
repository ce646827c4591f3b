"""Launch-time settings of the GEMM kernels.

The reference needs process-global tinygrad monkey-patches for three things tinygrad's CUDA backend lacks
(hopper_wgmma/runtime.py:20-98): opt-in dynamic shared memory above 48 KiB, cluster dimensions, and the dynamic
shared-memory size in the launch arguments. Here the C ABI sets them explicitly per plan (cudaFuncSetAttribute and a
cluster-dimension launch attribute on cudaLaunchKernelEx), so nothing global is patched. ``install_runtime_hooks``
stays as a no-op so that code written for the reference (README:44-47) keeps working.
"""
from __future__ import annotations

from . import _capi

_MAX_DYNAMIC_SHARED = 227 * 1024
_dynamic_bytes_by_kernel: dict[str, int] = {}


def install_runtime_hooks() -> None:
  """Kept for API compatibility. Launch attributes are set per plan; there is nothing to install."""


def set_dynamic_smem_bytes(kernel_name: str, nbytes: int) -> None:
  """Record a dynamic shared-memory request (validated as runtime.py:20-25 does). Plans compute their own size;
  this registry only serves callers that query it."""
  if not kernel_name.startswith("sm100_"):
    raise ValueError("dynamic shared memory can only be configured for sm100_ kernels")
  if not isinstance(nbytes, int) or not 0 <= nbytes <= _MAX_DYNAMIC_SHARED:
    raise ValueError(f"dynamic shared-memory size must be an integer from 0 to {_MAX_DYNAMIC_SHARED}")
  _dynamic_bytes_by_kernel[kernel_name] = nbytes


def device_info(device: int = 0) -> dict:
  """SM count, opt-in shared memory per block and compute capability of a CUDA device."""
  return _capi.device_info(device)
