"""Host side of the EXL3 kernels: the reference's kernels.py interface over the sm_100a C ABI.

Mirrors daig/omlx-exl3 src/omlx/exl3/kernels.py (same names, argument meaning and preconditions),
with torch CUDA tensors in place of MLX arrays:

  TrellisGemvPlan   kernels.py:263-299   decode GEMV (rows <= MAX_GEMV_ROWS), 1-3 sibling members
  decode_wt         kernels.py:340-351   trellis -> W^T (n_chunk, k) fp16, bit-exact
  rot               kernels.py:451-458   xh = had128(x * suh) / sqrt(128), member-major (NM, rows, k)
  norm_rot          kernels.py:461-473   RMSNorm (MLX rounding) + rotations
  swiglu_rot        kernels.py:476-483   had128(silu(g) * u * suh) / sqrt(128)

Every op launches native code from libexl3b200.so on the current CUDA stream; nothing here falls back
to another implementation.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import GemvDesc, check, dtype_code, lib, ptr, stream_ptr

MAX_GEMV_ROWS = 8


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("EXL3 kernels take CUDA tensors")


class TrellisGemvPlan:
    """A reusable launch of the decode GEMV for fixed shapes: 1-3 members (linears read together, one
    codebook), `rows` input rows, output dtype. A call takes the members' rotated inputs, stacked
    member-major as xh (n_members, rows, k), and their trellis words, and returns every member's
    H(xh_m @ W_m) * svh side by side as (rows, sum(member_ns)). K is one bitrate for all members or one
    per member (members of different bitrates still take one launch, each on its own share of the
    CTAs; the reference's groups share one K).

    The plan owns the launch descriptor, an fp16 copy of svh and the scratch (split-k partials and
    per-block arrival counters that every call leaves at zero). One plan must not run on two streams
    at once (the reference plan has the same restriction, kernels.py:284-286)."""

    def __init__(self, k: int, member_ns: list[int], K: int | list[int], cb: int, svh: torch.Tensor, rows: int,
                 out_dtype: torch.dtype = torch.float16, grid: int = 0):
        Ks = [int(x) for x in K] if isinstance(K, (list, tuple)) else [int(K)] * len(member_ns)
        assert len(Ks) == len(member_ns) and all(1 <= x <= 8 for x in Ks)
        assert k % 16 == 0 and all(n % 128 == 0 for n in member_ns) and cb in (0, 1, 2)
        assert 1 <= len(member_ns) <= 3 and 1 <= rows <= MAX_GEMV_ROWS
        assert out_dtype in (torch.float16, torch.bfloat16)
        self.k, self.n, self.K, self.cb, self.rows = k, sum(member_ns), Ks[0], cb, rows
        self.Ks = Ks
        self.out_dtype = out_dtype
        self.nsub = len(member_ns)
        self.member_ns = list(member_ns)
        self.KT, self.NT = k // 16, self.n // 16
        self.blocks = self.n // 128
        d = GemvDesc()
        d.k, d.n_members = k, self.nsub
        for i in range(3):
            d.n[i] = member_ns[i] if i < self.nsub else 0
        d.bits, d.codebook, d.rows = Ks[0], cb, rows
        mixed = any(x != Ks[0] for x in Ks)
        for i in range(3):
            d.member_bits[i] = Ks[i] if mixed and i < self.nsub else 0
        d.out_dtype = dtype_code(out_dtype)
        d.grid = grid
        d.flags = 0
        self.desc = d
        self.device = svh.device
        _need_cuda(svh)
        pb, cbytes = ctypes.c_size_t(), ctypes.c_size_t()
        with torch.cuda.device(self.device):
            check(lib().exl3_gemv_workspace(ctypes.byref(d), ctypes.byref(pb), ctypes.byref(cbytes)),
                  "exl3_gemv_workspace")
            self.svh = svh.to(torch.float16).reshape(-1).contiguous()
            assert self.svh.numel() == self.n
            self.partials = torch.empty(max(pb.value // 4, 4), dtype=torch.float32, device=self.device)
            self.counters = torch.zeros(max(cbytes.value // 4, 1), dtype=torch.int32, device=self.device)
        self._tptr = (ctypes.c_void_p * 3)()
        # argument objects of every launch, built once
        self._desc_ref = ctypes.byref(self.desc)
        self._tptr_arg = ctypes.cast(self._tptr, ctypes.c_void_p)

    def __call__(self, xh: torch.Tensor, trellises: list[torch.Tensor], out: torch.Tensor | None = None) -> torch.Tensor:
        """trellises: one flat uint32/int32 view per member. Returns (rows, n) in out_dtype."""
        assert len(trellises) == self.nsub
        xh = xh.contiguous()
        if xh.dtype != torch.float16:
            raise TypeError("xh must be fp16")
        if xh.numel() != self.nsub * self.rows * self.k:
            raise ValueError(f"xh has {xh.numel()} elements, expected {self.nsub}x{self.rows}x{self.k}")
        _need_cuda(xh, *trellises)
        for t, n, Km in zip(trellises, self.member_ns, self.Ks):
            if t.numel() * t.element_size() != self.k * n * Km // 8:
                raise ValueError(f"trellis holds {t.numel() * t.element_size()} bytes, expected "
                                 f"{self.k * n * Km // 8} for {self.k}x{n} at {Km} bpw")
        y = out if out is not None else torch.empty((self.rows, self.n), dtype=self.out_dtype, device=xh.device)
        for i in range(3):
            self._tptr[i] = trellises[i if i < self.nsub else 0].data_ptr()
        check(lib().exl3_gemv(self._desc_ref, xh.data_ptr(), self._tptr_arg,
                              self.svh.data_ptr(), y.data_ptr(), self.partials.data_ptr(), self.counters.data_ptr(),
                              stream_ptr(xh.device)), "exl3_gemv")
        return y


    def _xs(self) -> torch.Tensor:
        """Scratch of the input prologue (exl3_gemv_prologue_workspace bytes), made on first use."""
        xs = self.__dict__.get("_xs_buf")
        if xs is None:
            nb = ctypes.c_size_t()
            check(lib().exl3_gemv_prologue_workspace(self._desc_ref, ctypes.byref(nb)), "exl3_gemv_prologue_workspace")
            xs = self._xs_buf = torch.empty(max(nb.value // 2, 8), dtype=torch.float16, device=self.device)
        return xs

    def _check_trellises(self, trellises):
        assert len(trellises) == self.nsub
        _need_cuda(*trellises)
        for t, n, Km in zip(trellises, self.member_ns, self.Ks):
            if t.numel() * t.element_size() != self.k * n * Km // 8:
                raise ValueError(f"trellis holds {t.numel() * t.element_size()} bytes, expected "
                                 f"{self.k * n * Km // 8} for {self.k}x{n} at {Km} bpw")
        for i in range(3):
            self._tptr[i] = trellises[i if i < self.nsub else 0].data_ptr()

    def rot_call(self, x: torch.Tensor, suh: torch.Tensor, trellises: list[torch.Tensor],
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """rot(x, suh) and the GEMV in one launch (exl3_gemv_rot): x (rows, k) fp16/bf16/fp32, suh fp16
        (n_members, k) -> (rows, n) in out_dtype; bit-identical to plan(rot(x, suh), trellises)."""
        x = x.reshape(self.rows, self.k)
        if not x.is_contiguous():
            x = x.contiguous()
        if suh.dtype != torch.float16 or not suh.is_contiguous():
            suh = suh.to(torch.float16).contiguous()
        if suh.numel() != self.nsub * self.k:
            raise ValueError(f"suh has {suh.numel()} elements, expected {self.nsub}x{self.k}")
        _need_cuda(x, suh)
        self._check_trellises(trellises)
        xs = self._xs()
        y = out if out is not None else torch.empty((self.rows, self.n), dtype=self.out_dtype, device=x.device)
        check(lib().exl3_gemv_rot(self._desc_ref, x.data_ptr(), dtype_code(x.dtype), suh.data_ptr(), self._tptr_arg,
                                  self.svh.data_ptr(), y.data_ptr(), self.partials.data_ptr(),
                                  self.counters.data_ptr(), xs.data_ptr(), xs.numel() * 2, stream_ptr(x.device)),
              "exl3_gemv_rot")
        return y

    def bind_rot(self, suh: torch.Tensor, trellises: list[torch.Tensor]):
        """rot_call with suh and the trellises fixed, for a module's eager path: returns f(x, out=None) -> y
        that validates x and makes exactly one C call (every other argument was checked and converted
        here, once). The callable keeps suh and the trellises alive; rebind after replacing them."""
        suh = suh.to(torch.float16).contiguous()
        if suh.numel() != self.nsub * self.k:
            raise ValueError(f"suh has {suh.numel()} elements, expected {self.nsub}x{self.k}")
        _need_cuda(suh)
        self._check_trellises(trellises)
        tptr = (ctypes.c_void_p * 3)(*[trellises[i if i < self.nsub else 0].data_ptr() for i in range(3)])
        xs = self._xs()
        fn = lib().exl3_gemv_rot
        desc, tp = self._desc_ref, ctypes.cast(tptr, ctypes.c_void_p)
        suh_p, svh_p = suh.data_ptr(), self.svh.data_ptr()
        part_p, cnt_p, xs_p, xs_b = self.partials.data_ptr(), self.counters.data_ptr(), xs.data_ptr(), xs.numel() * 2
        rows, k, n, odt, dev = self.rows, self.k, self.n, self.out_dtype, self.device
        codes = {torch.float16: _lib.EXL3_F16, torch.bfloat16: _lib.EXL3_BF16, torch.float32: _lib.EXL3_F32}
        keep = (suh, list(trellises), tptr, xs)

        def call(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
            if x.shape != (rows, k) or not x.is_contiguous():
                x = x.reshape(rows, k).contiguous()
            code = codes.get(x.dtype)
            if code is None:
                raise TypeError(f"unsupported dtype {x.dtype}")
            if not x.is_cuda:
                raise ValueError("EXL3 kernels take CUDA tensors")
            y = out if out is not None else torch.empty((rows, n), dtype=odt, device=dev)
            st = fn(desc, x.data_ptr(), code, suh_p, tp, svh_p, y.data_ptr(), part_p, cnt_p, xs_p, xs_b,
                    stream_ptr(dev))
            if st:
                check(st, "exl3_gemv_rot")
            return y

        call.keep = keep
        return call

    def swiglu_call(self, gu: torch.Tensor, suh: torch.Tensor, trellises: list[torch.Tensor], peers=None,
                    slot: int = 0, out: torch.Tensor | None = None) -> torch.Tensor | None:
        """swiglu_rot(gu, suh) and the GEMV in one launch for a one-member plan (k = the MLP width):
        gu (rows, 2k) = [gate | up] fp16/bf16. Returns (rows, n) in out_dtype (exl3_gemv_swiglu), or,
        with peers (comm.PeerGroup), pushes the rows into inbox (slot, rank) of every rank and returns
        None (exl3_gemv_swiglu_peer)."""
        assert self.nsub == 1
        if gu.shape != (self.rows, 2 * self.k):
            raise ValueError(f"gu must be ({self.rows}, {2 * self.k})")
        if not gu.is_contiguous():
            gu = gu.contiguous()
        suh = suh.reshape(-1)
        if suh.dtype != torch.float16 or not suh.is_contiguous():
            suh = suh.to(torch.float16).contiguous()
        _need_cuda(gu, suh)
        self._check_trellises(trellises)
        xs = self._xs()
        if peers is not None:
            check(lib().exl3_gemv_swiglu_peer(self._desc_ref, gu.data_ptr(), dtype_code(gu.dtype), suh.data_ptr(),
                                              self._tptr_arg, self.svh.data_ptr(), self.partials.data_ptr(),
                                              self.counters.data_ptr(), xs.data_ptr(), xs.numel() * 2,
                                              ctypes.byref(peers.desc), slot, stream_ptr(gu.device)),
                  "exl3_gemv_swiglu_peer")
            return None
        y = out if out is not None else torch.empty((self.rows, self.n), dtype=self.out_dtype, device=gu.device)
        check(lib().exl3_gemv_swiglu(self._desc_ref, gu.data_ptr(), dtype_code(gu.dtype), suh.data_ptr(),
                                     self._tptr_arg, self.svh.data_ptr(), y.data_ptr(), self.partials.data_ptr(),
                                     self.counters.data_ptr(), xs.data_ptr(), xs.numel() * 2, stream_ptr(gu.device)),
              "exl3_gemv_swiglu")
        return y

    def qkv_post(self, xh: torch.Tensor, trellises: list[torch.Tensor], q_norm_w: torch.Tensor,
                 k_norm_w: torch.Tensor, eps: float, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor,
                 k_cache: torch.Tensor, v_cache: torch.Tensor, q_out: torch.Tensor | None = None) -> torch.Tensor:
        """For a q/k/v group plan: the GEMV with qkv_post as its epilogue (exl3_gemv_qkv_post). Writes this
        step's k/v into the caches at pos and returns q (rows, hq, 128) fp16."""
        assert self.nsub == 3 and len(trellises) == 3
        hq, hkv = self.member_ns[0] // 128, self.member_ns[1] // 128
        xh = xh.contiguous()
        if xh.dtype != torch.float16 or xh.numel() != 3 * self.rows * self.k:
            raise ValueError("xh must be fp16 (3, rows, k)")
        _need_cuda(xh, *trellises)
        assert k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape[0] == hkv
        assert cos.dtype == sin.dtype == torch.float32 and pos.dtype == torch.int64
        if q_out is None:
            q_out = torch.empty((self.rows, hq, 128), dtype=torch.float16, device=xh.device)
        a = _lib.QkvPostArgs()
        a.q_norm_w, a.k_norm_w = q_norm_w.data_ptr(), k_norm_w.data_ptr()
        a.cos_table, a.sin_table, a.pos = cos.data_ptr(), sin.data_ptr(), pos.data_ptr()
        a.k_cache, a.v_cache, a.q_out = k_cache.data_ptr(), v_cache.data_ptr(), q_out.data_ptr()
        a.hq, a.hkv, a.max_len, a.eps = hq, hkv, k_cache.shape[1], float(eps)
        for i in range(3):
            self._tptr[i] = trellises[i].data_ptr()
        check(lib().exl3_gemv_qkv_post(self._desc_ref, xh.data_ptr(), self._tptr_arg,
                                       self.svh.data_ptr(), self.partials.data_ptr(), self.counters.data_ptr(),
                                       ctypes.byref(a), stream_ptr(xh.device)), "exl3_gemv_qkv_post")
        return q_out

    def peer(self, xh: torch.Tensor, trellises: list[torch.Tensor], peers, slot: int) -> None:
        """The GEMV with its output rows pushed into inbox (slot, rank) of every rank of `peers`
        (comm.PeerGroup) for the next ar_add_norm_rot on that slot (exl3_gemv_peer); no y."""
        assert len(trellises) == self.nsub
        xh = xh.contiguous()
        if xh.dtype != torch.float16 or xh.numel() != self.nsub * self.rows * self.k:
            raise ValueError(f"xh must be fp16 ({self.nsub}, {self.rows}, {self.k})")
        _need_cuda(xh, *trellises)
        for i in range(3):
            self._tptr[i] = trellises[i if i < self.nsub else 0].data_ptr()
        check(lib().exl3_gemv_peer(self._desc_ref, xh.data_ptr(), self._tptr_arg,
                                   self.svh.data_ptr(), self.partials.data_ptr(), self.counters.data_ptr(),
                                   ctypes.byref(peers.desc), slot, stream_ptr(xh.device)), "exl3_gemv_peer")


def decode_wt(trellis_u32: torch.Tensor, k: int, n: int, K: int, cb: int, nt0: int = 0, ntc: int | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """W_inner^T columns [16*nt0, 16*(nt0+ntc)) as an (16*ntc, k) fp16 matrix (rows = output features)."""
    ntc = n // 16 - nt0 if ntc is None else ntc
    _need_cuda(trellis_u32)
    if trellis_u32.numel() * trellis_u32.element_size() < k * n * K // 8:
        raise ValueError(f"trellis holds {trellis_u32.numel() * trellis_u32.element_size()} bytes, "
                         f"expected {k * n * K // 8} for {k}x{n} at {K} bpw")
    w = out if out is not None else torch.empty((ntc * 16, k), dtype=torch.float16, device=trellis_u32.device)
    check(lib().exl3_decode_wt(trellis_u32.data_ptr(), k, n, K, cb, nt0, ntc, w.data_ptr(),
                               stream_ptr(trellis_u32.device)), "exl3_decode_wt")
    return w


def rot(x: torch.Tensor, suh: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x (rows, K) any float dtype, suh (NM, K) fp16 -> xh (NM, rows, K) fp16."""
    rows, k = x.shape
    suh = suh.reshape(-1, k)
    nm = suh.shape[0]
    _need_cuda(x, suh)
    x = x.contiguous()
    suh = suh.to(torch.float16).contiguous()
    xh = out if out is not None else torch.empty((nm, rows, k), dtype=torch.float16, device=x.device)
    check(lib().exl3_rot(x.data_ptr(), dtype_code(x.dtype), rows, k, suh.data_ptr(), nm, xh.data_ptr(),
                         stream_ptr(x.device)), "exl3_rot")
    return xh


def norm_rot(x: torch.Tensor, w: torch.Tensor, eps: float, suh: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm(x) * w in x.dtype (as mx.fast.rms_norm rounds it) and its rotations xh (NM, rows, K) fp16."""
    rows, k = x.shape
    suh = suh.reshape(-1, k)
    nm = suh.shape[0]
    assert k % 1024 == 0 and x.dtype in (torch.bfloat16, torch.float16)
    _need_cuda(x, w, suh)
    x = x.contiguous()
    w = w.to(x.dtype).contiguous()
    suh = suh.to(torch.float16).contiguous()
    xn = torch.empty_like(x)
    xh = torch.empty((nm, rows, k), dtype=torch.float16, device=x.device)
    check(lib().exl3_norm_rot(x.data_ptr(), w.data_ptr(), dtype_code(x.dtype), rows, k, float(eps), suh.data_ptr(),
                              nm, xn.data_ptr(), xh.data_ptr(), stream_ptr(x.device)), "exl3_norm_rot")
    return xn, xh


def swiglu_rot(gu: torch.Tensor, suh: torch.Tensor) -> torch.Tensor:
    """gu (rows, 2N) = [gate | up], suh (N,) fp16 -> had128(silu(gate) * up * suh) / sqrt(128), (1, rows, N) fp16."""
    rows, n2 = gu.shape
    n = n2 // 2
    _need_cuda(gu, suh)
    gu = gu.contiguous()
    suh = suh.to(torch.float16).reshape(-1).contiguous()
    xh = torch.empty((1, rows, n), dtype=torch.float16, device=gu.device)
    check(lib().exl3_swiglu_rot(gu.data_ptr(), dtype_code(gu.dtype), rows, n, suh.data_ptr(), xh.data_ptr(),
                                stream_ptr(gu.device)), "exl3_swiglu_rot")
    return xh


def had_svh(y: torch.Tensor, svh: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """out_dtype(had128(y) / sqrt(128) * svh) for y (rows, n): the prefill output rotation (linear.py:105)."""
    rows, n = y.shape
    _need_cuda(y, svh)
    y = y.contiguous()
    svh = svh.to(torch.float16).reshape(-1).contiguous()
    out = torch.empty((rows, n), dtype=out_dtype, device=y.device)
    check(lib().exl3_had_svh(y.data_ptr(), dtype_code(y.dtype), rows, n, svh.data_ptr(), out.data_ptr(),
                             dtype_code(out_dtype), stream_ptr(y.device)), "exl3_had_svh")
    return out


def _rows_view(t: torch.Tensor, width: int) -> int:
    """Row stride (elements) of a (rows, width) view whose elements are contiguous within a row."""
    assert t.dim() == 2 and t.shape[1] == width and t.stride(1) == 1, "need (rows, width) with unit column stride"
    return t.stride(0)


def qkv_post(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
             eps: float, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor, k_cache: torch.Tensor,
             v_cache: torch.Tensor, q_out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-head q/k RMSNorm + rotate-half RoPE, k/v into the fp16 caches at pos; returns q fp16 (rows, hq, 128).

    q (rows, hq*128), k and v (rows, hkv*128) in one dtype (views into a fused projection output are
    fine); cos/sin f32 (max_len, 64); pos int64 (rows); caches fp16 (hkv, max_len, 128).
    """
    rows = q.shape[0]
    hq, hkv = q.shape[1] // 128, k.shape[1] // 128
    max_len = k_cache.shape[1]
    _need_cuda(q, k, v, k_cache, v_cache)
    assert q.dtype == k.dtype == v.dtype and k_cache.dtype == v_cache.dtype == torch.float16
    assert k_cache.is_contiguous() and v_cache.is_contiguous() and tuple(k_cache.shape) == (hkv, max_len, 128)
    assert cos.dtype == sin.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous()
    assert cos.shape[1] == 64 and pos.dtype == torch.int64 and pos.is_contiguous()
    sq, sk, sv = _rows_view(q, hq * 128), _rows_view(k, hkv * 128), _rows_view(v, hkv * 128)
    if q_out is None:
        q_out = torch.empty((rows, hq, 128), dtype=torch.float16, device=q.device)
    check(lib().exl3_qkv_post(q.data_ptr(), k.data_ptr(), v.data_ptr(), sq, sk, sv, dtype_code(q.dtype), rows, hq, hkv,
                              q_norm_w.data_ptr(), k_norm_w.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(),
                              pos.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), max_len, q_out.data_ptr(),
                              stream_ptr(q.device)), "exl3_qkv_post")
    return q_out


_ATTN_WS: dict = {}


def attn_fits(rows: int, hq: int, hkv: int) -> bool:
    """Whether attn_rot handles this shape: up to 64 q vectors (rows x heads per kv head), in groups of
    16 per CTA."""
    return hq % hkv == 0 and rows * (hq // hkv) <= 64


def attn_rot(q16: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, T: int, suh: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention of q16 (rows, hq, 128) fp16 over cache[:, :T] (causal among the new rows, which
    sit at T - rows ..) fused with o_proj's input rotation: returns xh (1, rows, hq*128) fp16
    (exl3_attn_decode_rot). The split scratch is one cached buffer per device, shared by calls that run
    one after another on a stream."""
    rows, hq = q16.shape[0], q16.shape[1]
    hkv, max_len = k_cache.shape[0], k_cache.shape[1]
    _need_cuda(q16, k_cache, v_cache, suh)
    assert q16.dtype == k_cache.dtype == v_cache.dtype == torch.float16 and q16.shape[2] == 128
    assert q16.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()
    assert tuple(v_cache.shape) == tuple(k_cache.shape) and k_cache.shape[2] == 128
    suh = suh.to(torch.float16).reshape(-1).contiguous()
    assert suh.numel() == hq * 128
    nb = ctypes.c_size_t()
    with torch.cuda.device(q16.device):
        check(lib().exl3_attn_workspace(rows, hq, hkv, max_len, T, ctypes.byref(nb)), "exl3_attn_workspace")
        key = q16.device.index
        ws = _ATTN_WS.get(key)
        if ws is None or ws.numel() * 4 < nb.value:
            ws = torch.zeros(max(nb.value // 4 + 64, 1 << 16), dtype=torch.int32, device=q16.device)
            _ATTN_WS[key] = ws
    xh = out if out is not None else torch.empty((1, rows, hq * 128), dtype=torch.float16, device=q16.device)
    check(lib().exl3_attn_decode_rot(q16.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), rows, hq, hkv, max_len,
                                     int(T), suh.data_ptr(), xh.data_ptr(), ws.data_ptr(), nb.value,
                                     stream_ptr(q16.device)), "exl3_attn_decode_rot")
    return xh


def argmax(x: torch.Tensor, n: int | None = None, index_base: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Per row of x (rows, ld) fp16/bf16/fp32: (max of the first n values as fp32, its column +
    index_base as int64); the first column wins ties (exl3_argmax)."""
    rows, ld = x.shape
    n = ld if n is None else n
    _need_cuda(x)
    assert x.stride(1) == 1 and 1 <= n <= ld
    val = torch.empty(rows, dtype=torch.float32, device=x.device)
    idx = torch.empty(rows, dtype=torch.int64, device=x.device)
    check(lib().exl3_argmax(x.data_ptr(), dtype_code(x.dtype), rows, x.stride(0), n, index_base, val.data_ptr(),
                            idx.data_ptr(), stream_ptr(x.device)), "exl3_argmax")
    return val, idx


def add_norm_rot(x: torch.Tensor, d: torch.Tensor, w: torch.Tensor, eps: float, suh: torch.Tensor,
                 want_xn: bool = True) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
    """h = x + d, RMSNorm(h) * w (MLX rounding) and its rotations: returns (h, xn, xh (NM, rows, K) fp16);
    xn is None (not computed into memory) when want_xn is False."""
    rows, k = x.shape
    suh = suh.reshape(-1, k)
    nm = suh.shape[0]
    assert k % 128 == 0 and x.dtype in (torch.bfloat16, torch.float16) and d.dtype == x.dtype
    _need_cuda(x, d, w, suh)
    x, d = x.contiguous(), d.contiguous()
    w = w.to(x.dtype).contiguous()
    suh = suh.to(torch.float16).contiguous()
    h = torch.empty_like(x)
    xn = torch.empty_like(x) if want_xn else None
    xh = torch.empty((nm, rows, k), dtype=torch.float16, device=x.device)
    check(lib().exl3_add_norm_rot(x.data_ptr(), d.data_ptr(), w.data_ptr(), dtype_code(x.dtype), rows, k, float(eps),
                                  suh.data_ptr(), nm, h.data_ptr(), xn.data_ptr() if xn is not None else None,
                                  xh.data_ptr(), stream_ptr(x.device)), "exl3_add_norm_rot")
    return h, xn, xh


class _StatusWord:
    """A device's prefill-GEMM status word (the kernel ORs an error bit into it when a bounded wait
    gives up) and a pinned host mirror of it. After every GEMM launch outside stream capture the word
    is copied into the mirror asynchronously; each launch first looks at the mirror, so an error raises
    at a later call without the host ever waiting for the GPU. `read()` is the synchronous check."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.word = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.mirror = torch.zeros(4, dtype=torch.int32).pin_memory()

    def raise_if_set(self, value: int):
        if value:
            raise RuntimeError(f"exl3_gemm on {self.device}: a pipeline wait timed out (status 0x{value:x}); "
                               "the outputs of the failed call are invalid")

    def before_launch(self):
        self.raise_if_set(int(self.mirror[0]))

    def after_launch(self):
        if not torch.cuda.is_current_stream_capturing():
            self.mirror.copy_(self.word, non_blocking=True)

    def read(self) -> int:
        return int(self.word[0].item())


_status_words: dict = {}


def _status(device: torch.device) -> _StatusWord:
    key = torch.device(device)
    if key not in _status_words:
        _status_words[key] = _StatusWord(key)
    return _status_words[key]


def gemm(xh: torch.Tensor, trellis_u32: torch.Tensor, k: int, n: int, K: int, cb: int, svh: torch.Tensor,
         out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None, split: bool = True) -> torch.Tensor:
    """Prefill product with the trellis decoded in the kernel: out_dtype(had128(xh @ W) / sqrt(128) * svh)
    for xh fp16 (M, k). Needs k % 64 == 0 and n % 128 == 0 (EXL3Linear._prefill, linear.py:97-105).
    With `split`, narrow outputs may split k over several CTAs per tile, summed in a fixed part order (a
    per-device workspace: calls on one device must not run concurrently on several streams). Raises
    RuntimeError once an earlier launch on this device reported a timed-out wait."""
    M = xh.shape[0]
    _need_cuda(xh, trellis_u32, svh)
    if xh.dtype != torch.float16:
        raise TypeError("xh must be fp16")
    if trellis_u32.numel() * trellis_u32.element_size() != k * n * K // 8:
        raise ValueError(f"trellis holds {trellis_u32.numel() * trellis_u32.element_size()} bytes, "
                         f"expected {k * n * K // 8} for {k}x{n} at {K} bpw")
    st = _status(xh.device)
    st.before_launch()
    xh = xh.contiguous()
    svh = svh.to(torch.float16).reshape(-1).contiguous()
    y = out if out is not None else torch.empty((M, n), dtype=out_dtype, device=xh.device)
    ws, ws_bytes = _workspace(xh.device, "exl3_gemm_workspace", M, k, n) if split else (0, 0)
    check(lib().exl3_gemm(xh.data_ptr(), M, k, n, trellis_u32.data_ptr(), K, cb, svh.data_ptr(), y.data_ptr(),
                          dtype_code(y.dtype), ws, ws_bytes, st.word.data_ptr(), stream_ptr(xh.device)), "exl3_gemm")
    st.after_launch()
    return y


_split_workspaces: dict = {}


def _workspace(device: torch.device, query: str, M: int, k: int, n: int) -> tuple[int, int]:
    """(pointer, bytes) of this device's k-split workspace of one prefill kernel (`query` names its size
    query) for an M x k x n call, grown on demand. Each kernel has its own buffer: the kernels place
    their arrival counters and partials differently, and the counters must stay zero at rest (new
    buffers are zeroed; every completed call leaves them zero). (0, 0) when the call runs unsplit."""
    need = ctypes.c_size_t()
    check(getattr(lib(), query)(M, k, n, ctypes.byref(need)), query)
    if need.value == 0:
        return 0, 0
    key = (torch.device(device), query)
    buf = _split_workspaces.get(key)
    if buf is None or buf.numel() < need.value:
        buf = torch.zeros(need.value, dtype=torch.uint8, device=key[0])
        _split_workspaces[key] = buf
    return buf.data_ptr(), buf.numel()


def gemm_wt(xh: torch.Tensor, wt: torch.Tensor, svh: torch.Tensor, out_dtype: torch.dtype = torch.float32,
            out: torch.Tensor | None = None, split: bool = True) -> torch.Tensor:
    """Prefill product on decoded weights: out_dtype(had128(xh @ wt^T) / sqrt(128) * svh) for xh fp16 (M, k)
    and wt fp16 (n, k) as decode_wt returns it (linear.py:101-105). `out` may be a column slice of a wider
    row-major matrix (unit column stride); the rows are written in place. Needs k % 64 == 0, n % 128 == 0.
    With `split` the call may cut k into parts summed in a fixed order (a per-device workspace; calls on
    one device must not run concurrently on several streams). Raises RuntimeError once an earlier launch
    on this device reported a timed-out wait."""
    M, k = xh.shape
    n = wt.shape[0]
    _need_cuda(xh, wt, svh)
    if xh.dtype != torch.float16 or wt.dtype != torch.float16:
        raise TypeError("xh and wt must be fp16")
    if wt.shape[1] != k:
        raise ValueError(f"wt is {tuple(wt.shape)}, expected ({n}, {k})")
    st = _status(xh.device)
    st.before_launch()
    xh, wt = xh.contiguous(), wt.contiguous()
    svh = svh.to(torch.float16).reshape(-1).contiguous()
    y = out if out is not None else torch.empty((M, n), dtype=out_dtype, device=xh.device)
    if y.shape != (M, n) or y.stride(1) != 1:
        raise ValueError("out must be (M, n) with unit column stride")
    ws, ws_bytes = _workspace(xh.device, "exl3_gemm_wt_workspace", M, k, n) if split else (0, 0)
    check(lib().exl3_gemm_wt(xh.data_ptr(), M, k, n, wt.data_ptr(), svh.data_ptr(), y.data_ptr(), y.stride(0),
                             dtype_code(y.dtype), ws, ws_bytes, st.word.data_ptr(), stream_ptr(xh.device)),
          "exl3_gemm_wt")
    st.after_launch()
    return y


def gemm_status(device: torch.device | None = None) -> int:
    """The prefill kernel's error word on `device` (0 = no bounded wait ever gave up); synchronises."""
    return _status(device or torch.device("cuda", torch.cuda.current_device())).read()


def check_gemm_status(device: torch.device | None = None) -> None:
    """Raise RuntimeError if a prefill GEMM on `device` ever reported a timed-out wait (synchronises)."""
    st = _status(device or torch.device("cuda", torch.cuda.current_device()))
    st.raise_if_set(st.read())
