"""omlx_exl3_b200: the EXL3 quantized-linear hot path for NVIDIA B200 (sm_100a).

A drop-in for daig/omlx-exl3's `omlx.exl3` package on PyTorch/CUDA: the same EXL3Linear /
EXL3SiblingGroup module API and kernel entry points, backed by hand-written sm_100a CUDA behind the
C ABI in include/exl3_b200.h (libexl3b200.so).
"""
from .kernels import MAX_GEMV_ROWS, TrellisGemvPlan, decode_wt, had_svh, norm_rot, rot, swiglu_rot
from .linear import EXL3Linear, EXL3SiblingGroup

__all__ = ["MAX_GEMV_ROWS", "TrellisGemvPlan", "decode_wt", "had_svh", "norm_rot", "rot", "swiglu_rot",
           "EXL3Linear", "EXL3SiblingGroup"]
