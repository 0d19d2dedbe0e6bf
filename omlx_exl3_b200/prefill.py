"""Prefill (rows > MAX_GEMV_ROWS) path of EXL3Linear (daig/omlx-exl3 src/omlx/exl3/linear.py:97-121).

xh = rot(x, suh) in fp16 (the reference casts the activations to fp16 before rotating), then the fused
tcgen05 kernel (kernels.gemm: trellis decoded into shared memory, tensor-core product, output rotation
and svh in the epilogue). Shapes the fused kernel does not take (k % 64 != 0) decode W^T to fp16 in
column chunks (kernels.decode_wt, bit-exact), multiply, and rotate with kernels.had_svh.
"""
from __future__ import annotations

import torch

from .kernels import decode_wt, gemm, had_svh, rot

PREFILL_COL_CHUNK = 16384
# Up to this many rows (one 256-row tile: every weight decoded once) the fused kernel is used. Up to
# FUSED_WIDE_ROWS it is used too when the output has at least FUSED_WIDE_BLOCKS 128-column blocks: it
# then runs 512-row tiles (every weight still decoded once) on about one CTA per SM. Beyond that, or
# for narrower outputs (too few CTAs without a k split), decoding W once to fp16 plus a library GEMM
# is faster on B200 at the 27B-class shapes (measured: M=512, 5120->17408: fused 793 TFLOP/s against
# 617; 17408->5120: 414 against 667; M=4096: 892 / 790 against 1086 / 1268).
FUSED_MAX_ROWS = 256
FUSED_WIDE_ROWS = 512
FUSED_WIDE_BLOCKS = 128


def use_fused(rows: int, n: int) -> bool:
    return rows <= FUSED_MAX_ROWS or (rows <= FUSED_WIDE_ROWS and n // 128 >= FUSED_WIDE_BLOCKS)


def linear_prefill(x2: torch.Tensor, tr: torch.Tensor, k: int, n: int, K: int, cb: int, suh: torch.Tensor,
                   svh: torch.Tensor, out_dtype: torch.dtype = torch.float32, fused: bool | None = None) -> torch.Tensor:
    """(rows, n) = had128(had128(x2 * suh) @ W) * svh for x2 (rows, k)."""
    rows = x2.shape[0]
    xh = rot(x2, suh.reshape(1, -1))[0]
    if fused is None:
        fused = use_fused(rows, n)
    if fused and k % 64 == 0 and n % 128 == 0:
        return gemm(xh, tr, k, n, K, cb, svh, out_dtype)
    y = torch.empty((rows, n), dtype=torch.float16, device=x2.device)
    for c0 in range(0, n, PREFILL_COL_CHUNK):
        c = min(PREFILL_COL_CHUNK, n - c0)
        wt = decode_wt(tr, k, n, K, cb, nt0=c0 // 16, ntc=c // 16)
        torch.matmul(xh, wt.t(), out=y[:, c0:c0 + c])
    return had_svh(y, svh, out_dtype)
