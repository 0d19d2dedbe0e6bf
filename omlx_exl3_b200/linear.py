"""EXL3 linear layers for PyTorch on B200: the drop-in for the reference's linear.py.

Mirrors daig/omlx-exl3 src/omlx/exl3/linear.py. EXL3Linear holds exactly the checkpoint tensors of
one ExLlamaV3 linear (trellis, suh/su, svh/sv, mul1/mcg marker, optional bias) as module buffers
named after the checkpoint parts, so strict state-dict loading fills it like any layer. Forward
computes  y = had128( had128(x * suh) @ W_inner ) * svh  (+ bias):

  rows <= MAX_GEMV_ROWS (decode, speculative verify): the input rotation (one kernel, or none when
      the producer primed it, see fusion.py), then one trellis GEMV kernel that also reduces, applies
      the output rotation and svh, and writes the caller's dtype (kernels.TrellisGemvPlan)
  more rows (prefill): input rotation, trellis decode, fp16 GEMM, output rotation and svh
      (prefill.py)

EXL3SiblingGroup runs same-input siblings (q/k/v, gate/up, in_proj_qkv/z) as one GEMV launch over
their own trellis buffers when they share K and codebook; each member returns its slice, served from
a single-slot cache keyed on the input tensor's identity.
"""
from __future__ import annotations

import torch
from torch import nn

from . import prefill
from .kernels import MAX_GEMV_ROWS, TrellisGemvPlan, rot

PREFILL_COL_CHUNK = 16384          # output columns decoded per chunk on the unfused prefill path


def unpack_signs(bits: torch.Tensor) -> torch.Tensor:
    """Packed int16 sign bitfield (legacy su/sv) -> +-1 fp16 vector, bit i of word j = element 16j+i
    (linear.py:36-40)."""
    b = bits.reshape(-1).view(torch.int16).to(torch.int32) & 0xFFFF
    expanded = (b[:, None] >> torch.arange(16, dtype=torch.int32, device=bits.device)) & 1
    return (1.0 - 2.0 * expanded.reshape(-1).to(torch.float32)).to(torch.float16)


class EXL3Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, tensors: dict[str, tuple[tuple[int, ...], torch.dtype]],
                 device: torch.device | str | None = None):
        """tensors: checkpoint tensor name (trellis, suh, svh, su, sv, mul1, mcg, bias) -> (shape, dtype)."""
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        for name, (shape, dtype) in tensors.items():
            self.register_buffer(name, torch.zeros(shape, dtype=dtype, device=device))
        self._group = None
        self._idx = 0
        self._ready = False
        self._primed = None

    def __contains__(self, name: str) -> bool:
        """`"mul1" in linear`: whether the checkpoint declared that part (MLX module semantics)."""
        return name in self._buffers and self._buffers[name] is not None

    # -- runtime state, derived once from the loaded tensors -------------------------------------
    def _prepare(self):
        if self._ready:
            return
        w16 = self.trellis.shape[-1]
        if w16 % 16:
            raise NotImplementedError(f"half-integer EXL3 bitrate ({w16 / 16} bpw) is not supported yet")
        self._K = w16 // 16
        self._cb = 2 if "mul1" in self else 1 if "mcg" in self else 0
        suh = self.suh if "suh" in self else unpack_signs(self.su)
        svh = self.svh if "svh" in self else unpack_signs(self.sv)
        self._suh = suh.to(torch.float16).reshape(-1).contiguous()
        self._svh = svh.to(torch.float16).reshape(-1).contiguous()
        self._suh2d = self._suh.reshape(1, -1)
        self._tr = self.trellis.contiguous().view(torch.int32).reshape(-1)
        self._plans = {}
        self._ready = True

    def reset_runtime(self):
        """Drop derived state (after the buffers were replaced or moved)."""
        self._ready = False
        self._primed = None

    @property
    def rot_suh(self) -> torch.Tensor:
        """(1, in_features): this linear's input scales, as rotation kernels take them."""
        self._prepare()
        return self._suh2d

    def prime(self, x: torch.Tensor, xh: torch.Tensor):
        """The next call with exactly this tensor uses xh as its rotated input (fusion.py)."""
        self._primed = (x, xh)

    def plan(self, rows: int, out_dtype: torch.dtype) -> TrellisGemvPlan:
        self._prepare()
        plan = self._plans.get((rows, out_dtype))
        if plan is None:
            plan = self._plans[(rows, out_dtype)] = TrellisGemvPlan(
                self.in_features, [self.out_features], self._K, self._cb, self._svh, rows, out_dtype)
        return plan

    def gemv_rotated(self, xh: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """(rows, out_features) from an already rotated input xh, (1, rows, k) or (rows, k)."""
        rows = xh.shape[-2]
        return self.plan(rows, out_dtype)(xh, [self._tr])

    def _bias(self, y):
        return y + self.bias.to(y.dtype) if "bias" in self else y

    def _prefill(self, x2: torch.Tensor) -> torch.Tensor:
        return prefill.linear_prefill(x2, self._tr, self.in_features, self.out_features, self._K, self._cb,
                                      self._suh, self._svh)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._group is not None:
            return self._group.member_output(x, self._idx)
        self._prepare()
        in_shape, dtype = x.shape, x.dtype
        rows = x.numel() // self.in_features
        if rows <= MAX_GEMV_ROWS:
            primed, self._primed = self._primed, None
            xh = primed[1] if primed is not None and primed[0] is x else \
                rot(x.reshape(rows, self.in_features), self.rot_suh)
            y = self.gemv_rotated(xh, dtype if dtype in (torch.float16, torch.bfloat16) else torch.float16)
            y = y.to(dtype)
        else:
            y = self._prefill(x.reshape(rows, self.in_features)).to(dtype)
        return self._bias(y).reshape(in_shape[:-1] + (self.out_features,))


class EXL3SiblingGroup:
    """Same-input EXL3 siblings computed in one launch (rows <= MAX_GEMV_ROWS)."""

    def __init__(self, members: list[EXL3Linear]):
        for m in members:
            m._prepare()
        first = members[0]
        self.members = members
        self.k = first.in_features
        self.ns = [m.out_features for m in members]
        self.K, self.cb = first._K, first._cb
        self.suh = torch.stack([m._suh for m in members]).contiguous()          # (n_members, k)
        self.svh = torch.cat([m._svh for m in members]).contiguous()
        self.trs = [m._tr for m in members]
        self.plans: dict[tuple, TrellisGemvPlan] = {}
        self._cache_x = None
        self._cache_out = None
        self._served: set[int] = set()
        self._primed = None
        for i, m in enumerate(members):
            m._group, m._idx = self, i

    @staticmethod
    def fusable(members: list[EXL3Linear]) -> bool:
        for m in members:
            m._prepare()
        f = members[0]
        return (2 <= len(members) <= 3
                and all(m.in_features == f.in_features and m._K == f._K and m._cb == f._cb for m in members)
                and all(m.out_features % 128 == 0 and "bias" not in m for m in members))

    @property
    def rot_suh(self) -> torch.Tensor:
        return self.suh

    def prime(self, x: torch.Tensor, xh: torch.Tensor):
        """The next call with exactly this tensor uses xh (n_members, rows, k) as its rotated input."""
        self._primed = (x, xh)

    def plan(self, rows: int, out_dtype: torch.dtype) -> TrellisGemvPlan:
        plan = self.plans.get((rows, out_dtype))
        if plan is None:
            plan = self.plans[(rows, out_dtype)] = TrellisGemvPlan(self.k, self.ns, self.K, self.cb, self.svh,
                                                                   rows, out_dtype)
        return plan

    def gemv(self, x: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """All members' outputs, concatenated: (rows, sum(ns)) in out_dtype (rows <= MAX_GEMV_ROWS)."""
        rows = x.numel() // self.k
        primed, self._primed = self._primed, None
        xh = primed[1] if primed is not None and primed[0] is x else rot(x.reshape(rows, self.k), self.suh)
        return self.plan(rows, out_dtype)(xh, self.trs)

    def member_output(self, x: torch.Tensor, idx: int) -> torch.Tensor:
        """Member idx's output. The group computes once per input and serves each member once from
        the cache (torch tensors are mutable, so a cached result is not reused for a later call)."""
        if self._cache_x is x and idx not in self._served:
            self._served.add(idx)
            return self._cache_out[idx]
        out = self(x)
        self._served = {idx}
        return out[idx]

    def __call__(self, x: torch.Tensor) -> tuple[torch.Tensor, ...]:
        if self._cache_x is x and not self._served:
            return self._cache_out
        in_shape, dtype = x.shape, x.dtype
        rows = x.numel() // self.k
        if rows > MAX_GEMV_ROWS:   # prefill: each member on its own path
            outs = []
            for m in self.members:
                m._group = None
                try:
                    outs.append(m(x))
                finally:
                    m._group = self
            out = tuple(outs)
        else:
            odt = dtype if dtype in (torch.float16, torch.bfloat16) else torch.float16
            y = self.gemv(x, odt).to(dtype)
            out = tuple(o.reshape(in_shape[:-1] + (n,)) for o, n in zip(torch.split(y, self.ns, dim=-1), self.ns))
        self._cache_x, self._cache_out = x, out
        self._served = set()
        return out
