"""Fused input rotations for eager decode: the producer of an EXL3 input writes its rotation too.

Each EXL3 consumer (a linear, or a sibling group of them) reads xh = H(x * suh), the 128-point
Walsh-Hadamard rotation of its input. Called module by module, every consumer launches that rotation
itself after the kernel that produced x. At decode widths (rows <= MAX_GEMV_ROWS) two kinds of producer
can emit the rotations as a by-product instead:

  norm sites   an RMSNorm read only by EXL3 consumers (attention input norm -> q/k/v or
               in_proj_qkv/z, MLP input norm -> gate/up, final norm -> lm_head): kernels.norm_rot writes
               the normalised tensor and the rotated input of every consumer in one launch
  MLP sites    gate/up sibling group -> SwiGLU -> down_proj: down_proj's GEMV computes SwiGLU and its
               own input rotation from the gate/up GEMV output in the same launch
               (TrellisGemvPlan.swiglu_call)

`fuse_decode(model)` finds the sites and attaches a `FusionSite` to each producer module. The site
replaces the module's forward through an instance attribute only, so the module keeps its class,
parameters and state-dict keys; the site's forward runs the fused kernel at decode widths while
`ENABLED` is true and the original forward otherwise. The rotations are handed over through the
consumers' `prime(x, xh)` hook, which a consumer honours only when its next input is the very tensor
object the norm returned; a consumer reached through anything else (a view, a cast) rotates for
itself, so a missed hand-over costs a launch, never a wrong result. `unfuse(model)` restores the
original forwards.

Reference: daig/omlx-exl3 src/omlx/exl3/fusion.py (the same two fusions on MLX modules; `fuse_decode`,
`ENABLED` and the consumer hooks are the names the oMLX integration calls).
"""
from __future__ import annotations

import torch
from torch import nn

from .kernels import MAX_GEMV_ROWS, norm_rot
from .linear import EXL3Linear

ENABLED = True          # False sends every fused module down its original forward (for A/B timing)

# (module holding the linears, linear names) whose outputs a decoder layer's input norm feeds
_ATTENTION_INPUTS = (("self_attn", ("q_proj", "k_proj", "v_proj")), ("linear_attn", ("in_proj_qkv", "in_proj_z")))


def _decode_rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1]


class FusionSite:
    """One producer module whose forward is taken over for decode widths."""

    kind = "site"

    def __init__(self, module: nn.Module):
        self.module = module
        self.original = module.forward                 # bound method of the module's class

    def install(self):
        self.module.forward = self.forward             # instance attribute: shadows the class method

    def uninstall(self):
        self.module.__dict__.pop("forward", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not ENABLED or _decode_rows(x) > MAX_GEMV_ROWS:
            return self.original(x)
        return self.fused(x)

    def fused(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class NormSite(FusionSite):
    """RMSNorm -> its EXL3 consumers: one norm_rot launch writes xn and every consumer's xh."""

    kind = "norm"

    def __init__(self, norm: nn.Module, units: list, kind: str = "norm"):
        super().__init__(norm)
        self.kind = kind                  # "norm", or "head" for the final norm before the output head
        self.units = units
        self.widths = [u.rot_suh.shape[0] for u in units]                  # rotations per unit
        self.suh = torch.cat([u.rot_suh for u in units]).contiguous()      # (sum(widths), k)
        self.eps = _eps_of(norm)

    def fused(self, x: torch.Tensor) -> torch.Tensor:
        k = x.shape[-1]
        xn, xh = norm_rot(x.reshape(-1, k), self.module.weight, self.eps, self.suh)
        xn = xn.view(x.shape)
        start = 0
        for unit, width in zip(self.units, self.widths):
            unit.prime(xn, xh[start:start + width])
            start += width
        return xn


class MlpSite(FusionSite):
    """gate/up group -> SwiGLU -> down_proj: down_proj's GEMV takes the gate/up output and computes
    SwiGLU and its input rotation itself (one launch less than swiglu_rot + GEMV, bit-identical)."""

    kind = "mlp"

    def __init__(self, mlp: nn.Module, gate_up, down: EXL3Linear):
        super().__init__(mlp)
        self.gate_up, self.down = gate_up, down

    def fused(self, x: torch.Tensor) -> torch.Tensor:
        gu = self.gate_up.gemv(x, torch.float16)                           # (rows, 2 * n): gate | up
        d = self.down
        y = d.plan(gu.shape[0], x.dtype).swiglu_call(gu, d.rot_suh, [d.trellis_words])
        return y.view(*x.shape[:-1], y.shape[-1])


def _eps_of(norm: nn.Module) -> float:
    for attr in ("eps", "variance_epsilon"):
        v = getattr(norm, attr, None)
        if v is not None:
            return float(v)
    return float(torch.finfo(norm.weight.dtype).eps)


def _is_rms_norm(m) -> bool:
    return isinstance(m, nn.RMSNorm) or bool(getattr(m, "_exl3_rms_norm", False))


def _units_of(owner: nn.Module | None, names) -> list | None:
    """The distinct consumers (sibling group, else the linear) behind the named linears of owner, in
    first-use order; None unless every name is an EXL3Linear."""
    if owner is None:
        return None
    units: list = []
    for name in names:
        lin = getattr(owner, name, None)
        if not isinstance(lin, EXL3Linear):
            return None
        unit = lin._group or lin
        if not any(unit is u for u in units):
            units.append(unit)
    return units


def _norm_site(norm, units, kind: str = "norm") -> NormSite | None:
    w = getattr(norm, "weight", None)
    if not units or not _is_rms_norm(norm) or w is None:
        return None
    if w.dtype not in (torch.float16, torch.bfloat16) or w.shape[0] % 1024:   # norm_rot's shape rule
        return None
    return NormSite(norm, units, kind)


def _mlp_site(mlp) -> MlpSite | None:
    gate, up, down = (getattr(mlp, n, None) for n in ("gate_proj", "up_proj", "down_proj"))
    if not all(isinstance(m, EXL3Linear) for m in (gate, up, down)) or "bias" in down:
        return None
    group = gate._group
    if group is None or group.members != [gate, up] or gate.out_features != up.out_features:
        return None
    return MlpSite(mlp, group, down)


def find_sites(model: nn.Module) -> list[FusionSite]:
    """Every fusable producer of the model: per decoder layer its two norms and its MLP, then the
    final norm in front of the output head."""
    sites: list[FusionSite | None] = []
    for _, layer in model.named_modules():
        if not all(hasattr(layer, a) for a in ("input_layernorm", "post_attention_layernorm", "mlp")):
            continue
        attn_units = None
        for owner_name, names in _ATTENTION_INPUTS:
            owner = getattr(layer, owner_name, None)
            if owner is not None:
                attn_units = _units_of(owner, names)
                break
        sites.append(_norm_site(layer.input_layernorm, attn_units))
        sites.append(_norm_site(layer.post_attention_layernorm, _units_of(layer.mlp, ("gate_proj", "up_proj"))))
        sites.append(_mlp_site(layer.mlp))
    lm = getattr(model, "language_model", model)
    inner = getattr(lm, "model", None)
    if inner is not None and hasattr(inner, "norm"):
        sites.append(_norm_site(inner.norm, _units_of(lm, ("lm_head",)), kind="head"))
    return [s for s in sites if s is not None]


def fuse_decode(model: nn.Module) -> dict[str, int]:
    """Install the decode-width fusions on every eligible site; returns how many of each kind."""
    unfuse(model)
    sites = find_sites(model)
    for s in sites:
        s.install()
    model.__dict__["_exl3_fusion_sites"] = sites
    counts = {"norm": 0, "mlp": 0, "head": 0}
    for s in sites:
        counts[s.kind] += 1
    return counts


def unfuse(model: nn.Module) -> None:
    """Remove the fusions installed by fuse_decode (the modules' own forwards run again)."""
    for s in model.__dict__.pop("_exl3_fusion_sites", []):
        s.uninstall()
