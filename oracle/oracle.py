"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the EXL3 hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only as
the checker (or the timed CPU baseline). The product package never does.

Pieces and the reference code each one restates (daig/omlx-exl3):
  decode_wt / decode_w      exl3_oracle.c (C): trellis format + codebooks, kernels.py:4-8, 26-55, 304-351
  gemv                      had128(xh @ W) / sqrt(128) * svh in fp32, kernels.py:114-209 (test formula
                            of src/tools/exl3_kernel_test.py:34-50)
  rot / norm_rot / swiglu_rot   kernels.py:354-483, fp32 with the reference's FWHT stage order
  prefill (linear forward for rows > 8)   linear.py:97-121
  kl_div                    src/tools/exl3_kld.py:210-212, 244 (logits clamped at -200)
  unpack_signs              linear.py:36-40

The decode is bit-exact and pinned against the reference's own decode source (oracle/build_ref.py ->
oracle/_ref/libexl3_ref.so, and the golden fixtures in tests/golden/). The fp32 GEMV / rotations are
pinned only to the tolerance of the reference's own kernel tests, since MLX is not available here.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB_PATH = BUILD / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libexl3_ref.so"
SRC = HERE / "exl3_oracle.c"

HAD_SCALE = np.float32(0.08838834764831845)

_lib = None
_ref = None


def build(force: bool = False) -> Path:
    """Compile exl3_oracle.c (gcc, OpenMP) into oracle/_build/liboracle.so."""
    BUILD.mkdir(exist_ok=True)
    if LIB_PATH.exists() and not force and LIB_PATH.stat().st_mtime > SRC.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    subprocess.run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"], check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SRC.stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i = ctypes.c_int
        L.exl3o_decode_wt.argtypes = [P, i, i, i, i, i, i, P]
        L.exl3o_decode_w_f32.argtypes = [P, i, i, i, i, P]
        L.exl3o_gemv_f32.argtypes = [P, i, i, i, i, P, i, P, P]
        L.exl3o_dec1.argtypes = [ctypes.c_uint32, i]
        L.exl3o_dec1.restype = ctypes.c_uint16
        L.exl3o_fwht128.argtypes = [P]
        L.exl3o_set_threads.argtypes = [i]
        L.exl3o_num_threads.restype = i
        _lib = L
    return _lib


def ref_lib():
    """The reference's own decode compiled for the CPU (oracle/_ref), or None when it was not built."""
    global _ref
    if _ref is None and REF_LIB_PATH.exists():
        L = ctypes.CDLL(str(REF_LIB_PATH))
        P = ctypes.c_void_p
        i = ctypes.c_int
        L.exl3_ref_decode_wt.argtypes = [i, i, P, i, i, i, i, P]
        L.exl3_ref_gemv.argtypes = [i, i, P, i, i, P, i, P, P]
        L.exl3_ref_threads.restype = i
        L.exl3_ref_set_threads.argtypes = [i]
        _ref = L
    return _ref


def _ptr(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------------------ synthetic inputs

def random_trellis(k: int, n: int, K: int, seed: int, bit31: bool = True) -> np.ndarray:
    """int16 [k/16, n/16, 16K] trellis, uniform over the full range (bit31=False: the reference
    test's 31-bit words, src/tools/exl3_kernel_test.py:29-31)."""
    rng = np.random.default_rng(seed)
    words = rng.integers(0, 2 ** 32 if bit31 else 2 ** 31, size=(k // 16) * (n // 16) * 8 * K, dtype=np.uint64)
    return words.astype(np.uint32).view(np.int16).reshape(k // 16, n // 16, 16 * K)


def trellis_u32(trellis: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(trellis).view(np.uint32).reshape(-1)


# ------------------------------------------------------------------------------ decode

def decode_wt(trellis: np.ndarray, k: int, n: int, K: int, cb: int, nt0: int = 0, ntc: int | None = None) -> np.ndarray:
    """(16*ntc, k) float16: W^T columns [16*nt0, 16*(nt0+ntc)) (kernels.py:340-351)."""
    ntc = n // 16 - nt0 if ntc is None else ntc
    t = trellis_u32(trellis)
    out = np.empty((ntc * 16, k), dtype=np.uint16)
    rc = lib().exl3o_decode_wt(_ptr(t), k, n, K, cb, nt0, ntc, _ptr(out))
    if rc:
        raise ValueError(f"oracle decode_wt rejected its arguments ({rc})")
    return out.view(np.float16)


def decode_w(trellis: np.ndarray, k: int, n: int, K: int, cb: int) -> np.ndarray:
    """W (k, n) float32, k-major: y = x @ W."""
    t = trellis_u32(trellis)
    out = np.empty((k, n), dtype=np.float32)
    rc = lib().exl3o_decode_w_f32(_ptr(t), k, n, K, cb, _ptr(out))
    if rc:
        raise ValueError(f"oracle decode_w rejected its arguments ({rc})")
    return out


def ref_decode_wt(trellis: np.ndarray, k: int, n: int, K: int, cb: int, nt0: int = 0, ntc: int | None = None):
    """Same as decode_wt through the reference's own decode source (None if oracle/_ref is absent)."""
    L = ref_lib()
    if L is None:
        return None
    ntc = n // 16 - nt0 if ntc is None else ntc
    t = trellis_u32(trellis)
    out = np.empty((ntc * 16, k), dtype=np.uint16)
    if L.exl3_ref_decode_wt(K, cb, _ptr(t), k, n, nt0, ntc, _ptr(out)):
        raise ValueError("reference decode rejected its arguments")
    return out.view(np.float16)


# ------------------------------------------------------------------------------ rotations

def fwht128(v: np.ndarray) -> np.ndarray:
    """Sylvester-order FWHT over the last axis in 128-blocks, fp32, stages h = 1..64 in the
    reference's order (kernels.py:194-204, 374-386). Unscaled."""
    v = np.array(v, dtype=np.float32, copy=True)
    shp = v.shape
    b = v.reshape(-1, 128)
    h = 1
    while h < 128:
        x = b.reshape(-1, 128 // (2 * h), 2, h)
        a0 = x[:, :, 0, :].copy()
        a1 = x[:, :, 1, :].copy()
        x[:, :, 0, :] = a0 + a1
        x[:, :, 1, :] = a0 - a1
        h *= 2
    return b.reshape(shp)


def had128(v: np.ndarray) -> np.ndarray:
    """fp32 had128(v) / sqrt(128) (linear.py:31-33 / exl3_kernel_test.py:24-27)."""
    return fwht128(v) * HAD_SCALE


def rot(x: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """xh[m] = fp16(FWHT128(x * suh[m]) * 1/sqrt(128)), (NM, rows, k) (kernels.py:396-406, 451-458)."""
    x = np.asarray(x, dtype=np.float32)
    suh = np.asarray(suh).reshape(-1, x.shape[-1]).astype(np.float32)
    out = [(fwht128(x * suh[m]) * HAD_SCALE).astype(np.float16) for m in range(suh.shape[0])]
    return np.stack(out)


def _round_to(v: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 to fp16 / bf16 (nearest even) and back to fp32."""
    v = np.asarray(v, dtype=np.float32)
    if dtype == "float16":
        return v.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        u = v.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        nan = np.isnan(v)
        out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
        out[nan] = np.nan
        return out
    return v


def norm_rot(x: np.ndarray, w: np.ndarray, eps: float, suh: np.ndarray, dtype: str):
    """RMSNorm with MLX's rounding, then the rotations (kernels.py:408-425, 461-473).
    x, w: fp32 arrays holding `dtype` values. Returns (xn fp32 holding dtype values, xh fp16)."""
    x = np.asarray(x, dtype=np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(ss / x.shape[-1] + eps)).astype(np.float32)
    xn = _round_to(np.asarray(w, dtype=np.float32) * _round_to(x * inv, dtype), dtype)
    return xn, rot(xn, suh)


def swiglu_rot(gu: np.ndarray, suh: np.ndarray) -> np.ndarray:
    """had128(silu(gate) * up * suh) / sqrt(128) as fp16, (1, rows, n) (kernels.py:428-433, 476-483)."""
    gu = np.asarray(gu, dtype=np.float32)
    n = gu.shape[-1] // 2
    g, u = gu[:, :n], gu[:, n:]
    v = g / (np.float32(1.0) + np.exp(-g)) * u * np.asarray(suh, dtype=np.float32).reshape(-1)
    return (fwht128(v) * HAD_SCALE).astype(np.float16)[None]


# ------------------------------------------------------------------------------ GEMV / linear

def gemv(trellises, k: int, ns, K: int, cb: int, xh: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """fp32 had128(xh[m] @ W_m) * svh_m for each member, concatenated: (rows, sum(ns)).
    The reference test's formula (exl3_kernel_test.py:44-46); xh (NM, rows, k) fp16."""
    outs = []
    svh = np.asarray(svh, dtype=np.float16).reshape(-1)
    o = 0
    for m, (t, n) in enumerate(zip(trellises, ns)):
        W = decode_w(t, k, n, K, cb)
        y = np.asarray(xh[m], dtype=np.float32) @ W
        outs.append(had128(y) * svh[o:o + n].astype(np.float32))
        o += n
    return np.concatenate(outs, axis=1)


def gemv_c(trellis, k: int, n: int, K: int, cb: int, xh: np.ndarray, svh: np.ndarray) -> np.ndarray:
    """Single-member fp32 GEMV in C (fused decode, no k x n buffer): for the larger shapes."""
    t = trellis_u32(trellis)
    x = np.ascontiguousarray(np.asarray(xh, dtype=np.float16).reshape(-1, k)).view(np.uint16)
    s = np.ascontiguousarray(np.asarray(svh, dtype=np.float16).reshape(-1)).view(np.uint16)
    y = np.empty((x.shape[0], n), dtype=np.float32)
    if lib().exl3o_gemv_f32(_ptr(t), k, n, K, cb, _ptr(x), x.shape[0], _ptr(s), _ptr(y)):
        raise ValueError("oracle gemv rejected its arguments")
    return y


def linear_forward(trellis, k: int, n: int, K: int, cb: int, x: np.ndarray, suh: np.ndarray, svh: np.ndarray,
                   bias: np.ndarray | None = None) -> np.ndarray:
    """fp32 y = had128(had128(x * suh) @ W) * svh (+ bias), the EXL3Linear forward (linear.py:107-121)
    without the reference's intermediate fp16 roundings."""
    x = np.asarray(x, dtype=np.float32)
    xh = had128(x * np.asarray(suh, dtype=np.float32).reshape(-1))
    y = had128(xh @ decode_w(trellis, k, n, K, cb)) * np.asarray(svh, dtype=np.float32).reshape(-1)
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y


def unpack_signs(bits: np.ndarray) -> np.ndarray:
    """Packed int16 sign bitfield -> +-1 fp16 (linear.py:36-40): bit i of word j = element 16j+i, set = -1."""
    b = np.asarray(bits).view(np.uint16).astype(np.uint32).reshape(-1)
    e = (b[:, None] >> np.arange(16, dtype=np.uint32)) & 1
    return (1.0 - 2.0 * e.reshape(-1)).astype(np.float16)


def kl_div(ref_logits: np.ndarray, logits: np.ndarray) -> np.ndarray:
    """Per-row KL(ref || model) with logits clamped at -200 (exl3_kld.py:210-212, 244)."""
    def lsm(z):
        z = np.maximum(np.asarray(z, dtype=np.float64), -200.0)
        m = z.max(axis=-1, keepdims=True)
        return z - (m + np.log(np.exp(z - m).sum(axis=-1, keepdims=True)))
    lr, lq = lsm(ref_logits), lsm(logits)
    return np.sum(np.exp(lr) * (lr - lq), axis=-1)


def max_rel(a, b) -> float:
    """max |a - b| / max |b| (exl3_kernel_test.py:20-22)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
