"""Launch-time settings of the GEMM kernels.

The reference needs process-global tinygrad monkey-patches for three things tinygrad's CUDA backend lacks
(hopper_wgmma/runtime.py:20-98): opt-in dynamic shared memory above 48 KiB, cluster dimensions, and the dynamic
shared-memory size in the launch arguments, which its builders register per kernel name (gemm.py:315-316,
gated.py:64-65) and its launch hook reads back. Here the C ABI sets the launch attributes explicitly per plan
(cudaFuncSetAttribute and a cluster-dimension attribute on cudaLaunchKernelEx), so nothing global is patched and
``install_runtime_hooks`` is a no-op kept for code written against the reference (README:44-47).

The per-kernel registry keeps its role as the record of each kernel's dynamic shared memory: ``build_gemm_ws`` and
``build_gated_gemm`` register their configuration's size under the kernel name, as the reference's builders do, and
``build_gemm_ws``'s ``run`` reads it back as the budget of the plan it makes: a caller that registers a smaller size
for a kernel name (before calling ``run``) gets a plan whose shared-memory ring has as many stages as fit in it.
"""
from __future__ import annotations

from . import _capi

_MAX_DYNAMIC_SHARED = 227 * 1024
_dynamic_bytes_by_kernel: dict[str, int] = {}


def install_runtime_hooks() -> None:
  """Kept for API compatibility. Launch attributes are set per plan; there is nothing to install."""


def set_dynamic_smem_bytes(kernel_name: str, nbytes: int) -> None:
  """Register the dynamic shared memory of a kernel (validated as runtime.py:20-25 does)."""
  if not kernel_name.startswith("sm100_"):
    raise ValueError("dynamic shared memory can only be configured for sm100_ kernels")
  if not isinstance(nbytes, int) or not 0 <= nbytes <= _MAX_DYNAMIC_SHARED:
    raise ValueError(f"dynamic shared-memory size must be an integer from 0 to {_MAX_DYNAMIC_SHARED}")
  _dynamic_bytes_by_kernel[kernel_name] = nbytes


def dynamic_smem_bytes(kernel_name: str) -> int | None:
  """The size registered for a kernel name, or None."""
  return _dynamic_bytes_by_kernel.get(kernel_name)


def device_info(device: int = 0) -> dict:
  """SM count, opt-in shared memory per block and compute capability of a CUDA device."""
  return _capi.device_info(device)
