"""B200 (sm_100a) bf16 GEMM with the operator API of the Hopper wgmma experiment (narain1/tinygrad-hopper-wgmma).

Public names are the reference's (hopper_wgmma/__init__.py:2-5)."""
from .gated import GatedCfg, build_gated_gemm
from .gemm import Ring, WSCfg, build_gemm_ws, hilbert_schedule, region

__all__ = ["GatedCfg", "Ring", "WSCfg", "build_gated_gemm", "build_gemm_ws", "hilbert_schedule", "region"]
