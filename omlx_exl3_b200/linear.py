"""PyTorch modules for EXL3-quantised linears, backed by the sm_100a kernels of this package.

An EXL3 checkpoint stores each quantised linear as a handful of tensors under one prefix: the
trellis bitstream (int16, [k/16, n/16, 16*bits]), the input and output sign vectors (fp16 `suh` /
`svh`, or the older bit-packed int16 `su` / `sv`), an optional codebook marker (`mul1` or `mcg`; its
presence is what matters) and an optional bias. `EXL3Linear` registers exactly the tensors the
checkpoint declares, under those names, so loading a state dict fills it without any renaming.

The product it computes, for an input x of any leading shape, is

    y = H(H(x * suh) @ W) * svh  (+ bias)          H: 128-point Walsh-Hadamard blocks scaled by 1/sqrt(128)

where W is the k x n matrix the trellis decodes to. Up to MAX_GEMV_ROWS rows (batch decode, speculative
verify) it is one GEMV launch that rotates its own input, decodes the trellis on the fly and applies
the output rotation (or, when a fused producer has already written the rotated input, see `prime`, the
GEMV alone). Larger inputs take the prefill path (prefill.py).

`EXL3SiblingGroup` ties 2-3 linears that read the same input (q/k/v, gate/up, in_proj_qkv/z) into a
single GEMV launch over their separate trellis buffers.

Reference: daig/omlx-exl3 src/omlx/exl3/linear.py (EXL3Linear :43-121, EXL3SiblingGroup :124-193);
constructor, buffer names, forward signature and the fusion hooks (rot_suh, prime, gemv_rotated,
fusable, gemv) are kept as there.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from . import prefill
from .kernels import MAX_GEMV_ROWS, TrellisGemvPlan

PREFILL_COL_CHUNK = 16384          # output columns decoded per chunk on the unfused prefill path


def unpack_signs(bits: torch.Tensor) -> torch.Tensor:
    """Legacy packed sign vector -> +-1 fp16. Word j of the int16 bitfield carries elements 16j..16j+15,
    least significant bit first; a set bit means -1 (reference linear.py:36-40)."""
    words = bits.reshape(-1).view(torch.int16).to(torch.int32) & 0xFFFF
    shifts = torch.arange(16, dtype=torch.int32, device=bits.device)
    neg = ((words.unsqueeze(1) >> shifts) & 1).reshape(-1)
    return torch.where(neg.bool(), -1.0, 1.0).to(torch.float16)


def trellis_bitrate(trellis: torch.Tensor) -> int:
    """Bits per weight of a trellis tensor: each 16x16 tile holds 256*K bits = 16*K int16 words."""
    words = int(trellis.shape[-1])
    if words % 16:
        raise NotImplementedError(f"EXL3 tensor at {words / 16} bpw: half-integer bitrates are not supported")
    return words // 16


@dataclass
class _Runtime:
    """What the kernels need from a loaded EXL3Linear, derived once from its checkpoint tensors."""
    bits: int
    codebook: int                  # 0 = 3inst (no marker), 1 = mcg, 2 = mul1
    suh: torch.Tensor              # (k,) fp16
    svh: torch.Tensor              # (n,) fp16
    words: torch.Tensor            # trellis as a flat int32 view (the kernels read uint32 words)
    plans: dict


class EXL3Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, tensors: dict[str, tuple[tuple[int, ...], torch.dtype]],
                 device: torch.device | str | None = None):
        """tensors maps each checkpoint part present for this linear (trellis, suh / su, svh / sv, mul1 /
        mcg, bias) to its (shape, dtype); a zero buffer of that shape is registered under the part's name."""
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        for part, (shape, dtype) in tensors.items():
            self.register_buffer(part, torch.zeros(shape, dtype=dtype, device=device))
        self._rt: _Runtime | None = None
        self._group = None           # EXL3SiblingGroup this linear belongs to, if any
        self._idx = 0                # its position in that group
        self._primed = None          # (input tensor, its rotation) handed over by a fused producer

    def __contains__(self, part: str) -> bool:
        """Whether the checkpoint declared `part` for this linear (e.g. `"mul1" in lin`)."""
        return self._buffers.get(part) is not None

    # -- derived state ---------------------------------------------------------------------------
    def runtime(self) -> _Runtime:
        """Bitrate, codebook, fp16 sign vectors and the trellis word view, computed on first use."""
        if self._rt is None:
            marker = next((m for m in ("mul1", "mcg") if m in self), None)
            signs_in = self.suh if "suh" in self else unpack_signs(self.su)
            signs_out = self.svh if "svh" in self else unpack_signs(self.sv)
            self._rt = _Runtime(bits=trellis_bitrate(self.trellis), codebook={"mul1": 2, "mcg": 1, None: 0}[marker],
                                suh=signs_in.reshape(-1).to(torch.float16).contiguous(),
                                svh=signs_out.reshape(-1).to(torch.float16).contiguous(),
                                words=self.trellis.contiguous().view(torch.int32).reshape(-1), plans={})
        return self._rt

    def reset_runtime(self):
        """Forget the derived state (call after the buffers were replaced, reloaded or moved)."""
        self._rt = None
        self._primed = None

    @property
    def bits(self) -> int:
        return self.runtime().bits

    @property
    def codebook(self) -> int:
        return self.runtime().codebook

    @property
    def trellis_words(self) -> torch.Tensor:
        return self.runtime().words

    @property
    def output_signs(self) -> torch.Tensor:
        return self.runtime().svh

    # -- fusion hooks ----------------------------------------------------------------------------
    @property
    def rot_suh(self) -> torch.Tensor:
        """Input sign vector shaped (1, in_features): the `suh` operand of the rotation kernels."""
        return self.runtime().suh.view(1, -1)

    def prime(self, x: torch.Tensor, xh: torch.Tensor):
        """Hand over xh = H(x * suh) computed by a fused producer; used only if the next forward gets
        this very tensor object x."""
        self._primed = (x, xh)

    def _take_primed(self, x: torch.Tensor) -> torch.Tensor | None:
        handed, self._primed = self._primed, None
        return handed[1] if handed is not None and handed[0] is x else None

    def plan(self, rows: int, out_dtype: torch.dtype) -> TrellisGemvPlan:
        rt = self.runtime()
        key = (rows, out_dtype)
        if key not in rt.plans:
            rt.plans[key] = TrellisGemvPlan(self.in_features, [self.out_features], rt.bits, rt.codebook, rt.svh,
                                            rows, out_dtype)
        return rt.plans[key]

    def gemv_rotated(self, xh: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """GEMV of an input already rotated by H(. * suh): xh (1, rows, k) or (rows, k) fp16 ->
        (rows, out_features) in out_dtype."""
        return self.plan(xh.shape[-2], out_dtype)(xh, [self.trellis_words])

    # -- forward ---------------------------------------------------------------------------------
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._group is not None:
            return self._group.member_output(x, self._idx)
        rt = self._rt if self._rt is not None else self.runtime()
        x2 = x if x.dim() == 2 else x.reshape(-1, self.in_features)
        rows = x2.shape[0]
        if rows > MAX_GEMV_ROWS:
            y = prefill.linear_prefill(x2, rt.words, self.in_features, self.out_features, rt.bits, rt.codebook,
                                       rt.suh, rt.svh)
        else:
            xh = self._take_primed(x) if self._primed is not None else None
            gemv_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
            if xh is not None:
                y = self.gemv_rotated(xh, gemv_dtype)
            else:            # one launch: the GEMV rotates its own input (exl3_gemv_rot)
                # the launch with every argument but x bound once per (rows, dtype): the eager module
                # call is otherwise dominated by host work (argument checks and conversions)
                key = ("rot", rows, gemv_dtype)
                f = rt.plans.get(key)
                if f is None:
                    f = rt.plans[key] = self.plan(rows, gemv_dtype).bind_rot(rt.suh, [rt.words])
                y = f(x2)
        if y.dtype != x.dtype:
            y = y.to(x.dtype)
        bias = self._buffers.get("bias")
        if bias is not None:
            y = y + bias.to(y.dtype)
        return y if x.dim() == 2 else y.reshape(*x.shape[:-1], self.out_features)


class EXL3SiblingGroup:
    """2-3 EXL3 linears fed by one input, computed by one GEMV launch for rows <= MAX_GEMV_ROWS.

    Eligible members share in_features, bitrate and codebook, have output widths that are multiples
    of 128 and no bias (`fusable`). Joining a group redirects each member's forward here: the first
    member called with an input runs the group's launch, and the other members take their column
    slice of that result for the same input.
    """

    def __init__(self, members: list[EXL3Linear]):
        rts = [m.runtime() for m in members]
        self.members = list(members)
        self.k = members[0].in_features
        self.ns = [m.out_features for m in members]
        self.K, self.cb = rts[0].bits, rts[0].codebook
        self.suh = torch.stack([rt.suh for rt in rts])               # (n_members, k): one rotation per member
        self.svh = torch.cat([rt.svh for rt in rts])                 # output signs in member order
        self.trs = [rt.words for rt in rts]
        self.plans: dict[tuple, TrellisGemvPlan] = {}
        self._primed = None
        self._last: tuple | None = None        # (input, per-member outputs, members not yet served)
        for idx, m in enumerate(members):
            m._group, m._idx = self, idx

    @staticmethod
    def fusable(members: list[EXL3Linear]) -> bool:
        if not 2 <= len(members) <= 3:
            return False
        key = {(m.in_features, m.bits, m.codebook) for m in members}
        return len(key) == 1 and not any(m.out_features % 128 or "bias" in m for m in members)

    @property
    def rot_suh(self) -> torch.Tensor:
        return self.suh

    def prime(self, x: torch.Tensor, xh: torch.Tensor):
        """Hand over the members' rotated inputs xh (n_members, rows, k) for the input tensor x."""
        self._primed = (x, xh)

    def plan(self, rows: int, out_dtype: torch.dtype) -> TrellisGemvPlan:
        key = (rows, out_dtype)
        if key not in self.plans:
            self.plans[key] = TrellisGemvPlan(self.k, self.ns, self.K, self.cb, self.svh, rows, out_dtype)
        return self.plans[key]

    def gemv(self, x: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """One launch for all members: (rows, sum(ns)) in out_dtype, members side by side."""
        handed, self._primed = self._primed, None
        x2 = x.reshape(-1, self.k)
        plan = self.plan(x2.shape[0], out_dtype)
        if handed is not None and handed[0] is x:
            return plan(handed[1], self.trs)
        return plan.rot_call(x2, self.suh, self.trs)         # one launch: the GEMV rotates its input

    def member_output(self, x: torch.Tensor, idx: int) -> torch.Tensor:
        """Output of member idx for input x. A group result is handed to each member once: tensors are
        mutable, so the same object passed again later (a reused static buffer) is recomputed."""
        if self._last is not None and self._last[0] is x and idx in self._last[2]:
            self._last[2].discard(idx)
            return self._last[1][idx]
        outs = self(x)
        self._last = (x, outs, set(range(len(self.members))) - {idx})
        return outs[idx]

    def __call__(self, x: torch.Tensor) -> tuple[torch.Tensor, ...]:
        lead = x.shape[:-1]
        rows = x.numel() // self.k
        if rows > MAX_GEMV_ROWS:
            # prefill: every member on its own path (detached from the group for the call)
            outs = []
            for m in self.members:
                m._group = None
                try:
                    outs.append(m(x))
                finally:
                    m._group = self
            return tuple(outs)
        gemv_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
        y = self.gemv(x, gemv_dtype).to(x.dtype)
        return tuple(part.reshape(*lead, n) for part, n in zip(y.split(self.ns, dim=-1), self.ns))
