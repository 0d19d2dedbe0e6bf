"""ctypes binding of libexl3b200.so (include/exl3_b200.h).

The library is the only compute path: there is no CPU or library fallback. If it cannot be loaded
(not built and no nvcc to build it) every op raises. Status codes from the C ABI become exceptions:
shape / bits / codebook / dtype problems raise ValueError (the reference asserts or raises on the same
preconditions, kernels.py:269-270, :465; linear.py:60-61), CUDA failures raise RuntimeError.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import build as _build

EXL3_F16, EXL3_BF16, EXL3_F32 = 0, 1, 2

_STATUS_EXC = {
    -1: ValueError,    # EXL3_E_SHAPE
    -2: ValueError,    # EXL3_E_BITS
    -3: ValueError,    # EXL3_E_CODEBOOK
    -4: TypeError,     # EXL3_E_DTYPE
    -5: ValueError,    # EXL3_E_ALIGN
    -6: ValueError,    # EXL3_E_NULL
    -7: RuntimeError,  # EXL3_E_CUDA
    -8: ValueError,    # EXL3_E_WORKSPACE
    -9: RuntimeError,  # EXL3_E_DEVICE
}


class GemvDesc(ctypes.Structure):
    _fields_ = [("k", ctypes.c_int32), ("n_members", ctypes.c_int32), ("n", ctypes.c_int32 * 3),
                ("bits", ctypes.c_int32), ("codebook", ctypes.c_int32), ("rows", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("grid", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("member_bits", ctypes.c_int32 * 3)]


GEMV_ROW_EXACT = 1


class PeerGroupDesc(ctypes.Structure):
    """exl3_peer_group: one tensor-parallel group as seen by one rank."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("base", ctypes.c_void_p * 8),
                ("flag_off", ctypes.c_uint64), ("data_off", ctypes.c_uint64), ("inbox_bytes", ctypes.c_uint64)]


PEER_HANDLE_BYTES = 64


class QkvPostArgs(ctypes.Structure):
    """exl3_qkv_post_args: the q/k/v GEMV epilogue's extra operands."""
    _fields_ = [("q_norm_w", ctypes.c_void_p), ("k_norm_w", ctypes.c_void_p), ("cos_table", ctypes.c_void_p),
                ("sin_table", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("k_cache", ctypes.c_void_p),
                ("v_cache", ctypes.c_void_p), ("q_out", ctypes.c_void_p), ("hq", ctypes.c_int32),
                ("hkv", ctypes.c_int32), ("max_len", ctypes.c_int32), ("eps", ctypes.c_float)]


_lib = None
_lock = threading.Lock()

# Every symbol include/exl3_b200.h declares: name -> (restype, argtypes)
_P, _I, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "exl3_strerror": (ctypes.c_char_p, [_I]),
    "exl3_version": (_I, []),
    "exl3_decode_wt": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "exl3_gemv_workspace": (_I, [ctypes.POINTER(GemvDesc), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "exl3_gemv_reset": (_I, [_P, _SZ, _P]),
    "exl3_gemv": (_I, [ctypes.POINTER(GemvDesc), _P, _P, _P, _P, _P, _P, _P]),
    "exl3_gemv_noalloc": (_I, [ctypes.POINTER(GemvDesc), _P, _P, _P, _P, _P]),
    "exl3_gemv_qkv_post": (_I, [ctypes.POINTER(GemvDesc), _P, _P, _P, _P, _P, ctypes.POINTER(QkvPostArgs), _P]),
    "exl3_rot": (_I, [_P, _I, _I, _I, _P, _I, _P, _P]),
    "exl3_norm_rot": (_I, [_P, _P, _I, _I, _I, _F, _P, _I, _P, _P, _P]),
    "exl3_swiglu_rot": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "exl3_had_svh": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "exl3_gemm": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _P, _I, _P, _SZ, _P, _P]),
    "exl3_gemm_workspace": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "exl3_gemm_wt_workspace": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "exl3_gemm_wt": (_I, [_P, _I, _I, _I, _P, _P, _P, _I, _I, _P, _SZ, _P, _P]),
    "exl3_qkv_post": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P, _P, _P, _I, _P, _P]),
    "exl3_add_norm_rot": (_I, [_P, _P, _P, _I, _I, _I, _F, _P, _I, _P, _P, _P, _P]),
    "exl3_peer_create": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    "exl3_peer_destroy": (_I, [_P]),
    "exl3_peer_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "exl3_peer_close": (_I, [_P]),
    "exl3_ar_add_norm_rot": (_I, [ctypes.POINTER(PeerGroupDesc), _I, _P, _P, _I, _I, _I, _F, _P, _I, _P, _P, _P,
                                  _P]),
    "exl3_peer_status": (_I, [ctypes.POINTER(PeerGroupDesc), ctypes.POINTER(ctypes.c_uint32)]),
    "exl3_attn_workspace": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(ctypes.c_size_t)]),
    "exl3_attn_decode_rot": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "exl3_peer_put": (_I, [ctypes.POINTER(PeerGroupDesc), _I, _P, _I, _I, _P]),
    "exl3_argmax": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "exl3_gemv_peer": (_I, [ctypes.POINTER(GemvDesc), _P, _P, _P, _P, _P, ctypes.POINTER(PeerGroupDesc), _I, _P]),
    "exl3_gemv_prologue_workspace": (_I, [ctypes.POINTER(GemvDesc), ctypes.POINTER(_SZ)]),
    "exl3_gemv_rot": (_I, [ctypes.POINTER(GemvDesc), _P, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "exl3_gemv_swiglu": (_I, [ctypes.POINTER(GemvDesc), _P, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "exl3_gemv_swiglu_peer": (_I, [ctypes.POINTER(GemvDesc), _P, _I, _P, _P, _P, _P, _P, _P, _SZ,
                                   ctypes.POINTER(PeerGroupDesc), _I, _P]),
}


def lib():
    """Load (building first if the sources are newer) and return the native library."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = _build.LIB
                if not _build.up_to_date():
                    path = _build.build()
                L = ctypes.CDLL(str(path))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().exl3_strerror(status).decode()
        raise _STATUS_EXC.get(status, RuntimeError)(f"{what}: {msg} (status {status})")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return EXL3_F16
    if dt == torch.bfloat16:
        return EXL3_BF16
    if dt == torch.float32:
        return EXL3_F32
    raise TypeError(f"unsupported dtype {dt}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device | int | None = None) -> int:
    """The current CUDA stream of `device` as a raw cudaStream_t. Every launch asks for it, so the
    raw accessor is used where torch has it (torch.cuda.current_stream builds a Stream object)."""
    if _raw_stream is not None:
        idx = device.index if isinstance(device, torch.device) else device
        return _raw_stream(torch.cuda.current_device() if idx is None else idx)
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
