"""Prefill (rows > MAX_GEMV_ROWS) path of EXL3Linear (daig/omlx-exl3 src/omlx/exl3/linear.py:97-121).

xh = rot(x, suh) in fp16 (the reference casts the activations to fp16 before rotating), then one of two
tcgen05 paths of this package, both with the output rotation and svh in the GEMM's epilogue:

- fused (kernels.gemm): the trellis is decoded into shared memory inside the GEMM. Each weight is
  decoded once per row tile, so it wins while the rows fit one or two tiles;
- decode-once (kernels.decode_wt + kernels.gemm_wt): W^T is decoded to fp16 once per column chunk, then
  multiplied by the pair-of-SMs GEMM that loads both operands with TMA. Above a few hundred rows the
  product is tensor-core bound and the decode cost is amortised over all rows.
"""
from __future__ import annotations

import torch

from .kernels import decode_wt, gemm, gemm_wt, rot

PREFILL_COL_CHUNK = 16384          # decoded columns per chunk: bounds the fp16 W^T scratch to 32 KB per k
# Up to FUSED_MAX_ROWS rows the fused kernel decodes each weight once (256- or 512-row tiles; narrow
# outputs split k over more CTAs) and beats decoding W^T to HBM first; above it the decode cost is
# amortised and decode-once + the SM-pair GEMM is faster. Measured at the 27B-class shapes, 6 bpw,
# TFLOP/s fused / decode-once: M=512 5120->17408 776 / 601, 17408->5120 660 / 542; M=4096 893 / 1241,
# 739 / 1241.
FUSED_MAX_ROWS = 512


def use_fused(rows: int, n: int) -> bool:
    return rows <= FUSED_MAX_ROWS


def linear_prefill(x2: torch.Tensor, tr: torch.Tensor, k: int, n: int, K: int, cb: int, suh: torch.Tensor,
                   svh: torch.Tensor, out_dtype: torch.dtype = torch.float32, fused: bool | None = None) -> torch.Tensor:
    """(rows, n) = had128(had128(x2 * suh) @ W) * svh for x2 (rows, k)."""
    rows = x2.shape[0]
    xh = rot(x2, suh.reshape(1, -1))[0]
    if fused is None:
        fused = use_fused(rows, n)
    if fused:
        return gemm(xh, tr, k, n, K, cb, svh, out_dtype)
    svh = svh.reshape(-1)
    y = torch.empty((rows, n), dtype=out_dtype, device=x2.device)
    for c0 in range(0, n, PREFILL_COL_CHUNK):
        c = min(PREFILL_COL_CHUNK, n - c0)
        wt = decode_wt(tr, k, n, K, cb, nt0=c0 // 16, ntc=c // 16)
        gemm_wt(xh, wt, svh[c0:c0 + c], out=y[:, c0:c0 + c])
    return y
