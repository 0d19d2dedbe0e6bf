"""Qwen3-style dense decoder with EXL3 linears, tensor-parallel over the GPUs of one box.

The reference runs its EXL3 linears inside mlx-vlm's Qwen3.5 model (not part of the reference repo);
this module is the host model the EXL3 hot path is measured in (BASELINE configs 4 and 5): RMSNorm ->
q/k/v (+ per-head q/k RMSNorm, RoPE) -> GQA attention over a KV cache -> o_proj -> residual ->
RMSNorm -> SwiGLU MLP -> residual, then the final norm and an EXL3 output head. Module paths follow
the Hugging Face checkpoint naming (model.layers.N.self_attn.q_proj, ..., lm_head), so a checkpoint's
EXL3 tensors load by name (loader.py) and fusion.fuse_decode finds its targets.

Tensor parallelism (tp_size > 1, one process per GPU): q/k/v, gate/up and the head are column-parallel
(whole 128-column Hadamard blocks per rank), o_proj and down_proj row-parallel (whole 128-row blocks of
k per rank, the input rotation is local per block); the row-parallel outputs are summed with one
all-reduce each. The head's logits are gathered (or arg-maxed) across ranks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from .kernels import (MAX_GEMV_ROWS, TrellisGemvPlan, add_norm_rot, argmax, attn_fits, attn_rot, norm_rot, qkv_post,
                      rot, swiglu_rot)
from .linear import EXL3Linear

# Up to this MLP width (per rank) the decode step's down_proj GEMV computes SwiGLU and its input rotation
# itself (TrellisGemvPlan.swiglu_call), one launch less. Every CTA rotates the k blocks its units read, so
# the work is repeated once per 128-column block of the output: measured on B200 (graphs of 50 calls,
# 6 bpw, 5120 outputs, 1 row) 9.9 -> 9.2 us at k = 2176 and 13.9 -> 13.1 at 4352, but 32.2 -> 33.7 at
# 17408, where the separate SwiGLU kernel stays.
FUSED_SWIGLU_MAX_K = 4352


@dataclass
class ModelConfig:
    hidden_size: int = 5120
    num_attention_heads: int = 40
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 17408
    num_hidden_layers: int = 64
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 8192
    dtype: torch.dtype = torch.bfloat16
    tie_word_embeddings: bool = False
    extra: dict = field(default_factory=dict)

    @staticmethod
    def from_hf(cfg: dict) -> "ModelConfig":
        c = cfg.get("text_config", cfg)
        hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
        dt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}.get(
            str(c.get("torch_dtype", "bfloat16")), torch.bfloat16)
        return ModelConfig(hidden_size=c["hidden_size"], num_attention_heads=c["num_attention_heads"],
                           num_key_value_heads=c.get("num_key_value_heads", c["num_attention_heads"]), head_dim=hd,
                           intermediate_size=c["intermediate_size"], num_hidden_layers=c["num_hidden_layers"],
                           vocab_size=c["vocab_size"], rms_norm_eps=c.get("rms_norm_eps", 1e-6),
                           rope_theta=c.get("rope_theta", 1e6),
                           max_position_embeddings=c.get("max_position_embeddings", 8192), dtype=dt,
                           tie_word_embeddings=c.get("tie_word_embeddings", False))


# ------------------------------------------------------------------------------------------ TP

@dataclass
class TP:
    rank: int = 0
    size: int = 1
    group: object = None
    peers: object = None      # comm.PeerGroup once setup_peers() ran: fused NVLink all-reduce

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def blocks(self, n_blocks: int) -> tuple[int, int]:
        """This rank's share [b0, b1) of n_blocks 128-wide blocks (uneven shares differ by one)."""
        return n_blocks * self.rank // self.size, n_blocks * (self.rank + 1) // self.size


def column_shard(n: int, tp: TP) -> tuple[int, int]:
    """Output columns [c0, c1) of a column-parallel linear with n outputs on this rank."""
    b0, b1 = tp.blocks(n // 128)
    return b0 * 128, b1 * 128


def row_shard(k: int, tp: TP) -> tuple[int, int]:
    """Input rows [r0, r1) of a row-parallel linear with k inputs on this rank."""
    b0, b1 = tp.blocks(k // 128)
    return b0 * 128, b1 * 128


# ------------------------------------------------------------------------------------------ layers

class RMSNorm(nn.Module):
    """RMSNorm with MLX's rounding (mx.fast.rms_norm): xn = T(w * T(x * rsqrt(mean(x^2) + eps)))."""

    _exl3_rms_norm = True

    def __init__(self, dim: int, eps: float, dtype: torch.dtype, device=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype, device=device), requires_grad=False)
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (self.weight.float() * (xf * inv).to(x.dtype).float()).to(x.dtype)


def rope_tables(cfg: ModelConfig, device) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, dtype=torch.float64) / cfg.head_dim))
    t = torch.arange(cfg.max_position_embeddings, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cos(f).float().to(device), torch.sin(f).float().to(device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x (rows, heads, hd), cos/sin (rows, hd/2): rotate-half convention."""
    xf = x.float()
    h = xf.shape[-1] // 2
    x1, x2 = xf[..., :h], xf[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class KVCache:
    """Per-layer fp16 K/V cache (n_kv_local, max_len, head_dim) with a length counter."""

    def __init__(self, n_layers: int, n_kv: int, max_len: int, head_dim: int, device, dtype=torch.float16):
        self.k = [torch.zeros((n_kv, max_len, head_dim), dtype=dtype, device=device) for _ in range(n_layers)]
        self.v = [torch.zeros((n_kv, max_len, head_dim), dtype=dtype, device=device) for _ in range(n_layers)]
        self.max_len = max_len
        self.length = 0

    def fill_random(self, length: int, seed: int = 0):
        g = torch.Generator(device=self.k[0].device)
        g.manual_seed(seed)
        for t in self.k + self.v:
            t[:, :length].normal_(generator=g)
        self.length = length


def _exl3(k: int, n: int, K: int, device, cb: int = 0, bias: bool = False) -> EXL3Linear:
    parts = {"trellis": ((k // 16, n // 16, 16 * K), torch.int16), "suh": ((k,), torch.float16),
             "svh": ((n,), torch.float16)}
    if cb == 1:
        parts["mcg"] = ((1,), torch.int32)
    elif cb == 2:
        parts["mul1"] = ((1,), torch.int32)
    if bias:
        parts["bias"] = ((n,), torch.float16)
    return EXL3Linear(k, n, parts, device=device)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: TP, bits: dict, device):
        super().__init__()
        self.cfg, self.tp = cfg, tp
        hd = cfg.head_dim
        self.hq = cfg.num_attention_heads // tp.size
        self.hkv = cfg.num_key_value_heads // tp.size
        h = cfg.hidden_size
        self.q_proj = _exl3(h, self.hq * hd, bits["q_proj"], device)
        self.k_proj = _exl3(h, self.hkv * hd, bits["k_proj"], device)
        self.v_proj = _exl3(h, self.hkv * hd, bits["v_proj"], device)
        self.o_proj = _exl3(self.hq * hd, h, bits["o_proj"], device)
        self.q_norm = RMSNorm(hd, cfg.rms_norm_eps, cfg.dtype, device)
        self.k_norm = RMSNorm(hd, cfg.rms_norm_eps, cfg.dtype, device)

    def forward(self, x: torch.Tensor, layer: int, cache: KVCache, pos: torch.Tensor, cos, sin) -> torch.Tensor:
        rows = x.shape[0]
        hd = self.cfg.head_dim
        q = self.q_norm(self.q_proj(x).reshape(rows, self.hq, hd))
        k = self.k_norm(self.k_proj(x).reshape(rows, self.hkv, hd))
        v = self.v_proj(x).reshape(rows, self.hkv, hd)
        c, s = cos.index_select(0, pos), sin.index_select(0, pos)
        q, k = apply_rope(q, c, s), apply_rope(k, c, s)
        kc, vc = cache.k[layer], cache.v[layer]
        kc.index_copy_(1, pos, k.transpose(0, 1).to(kc.dtype))
        vc.index_copy_(1, pos, v.transpose(0, 1).to(vc.dtype))
        T = cache.length + rows
        qh = q.transpose(0, 1)[None].to(kc.dtype)                  # (1, hq, rows, hd)
        kk, vv = kc[None, :, :T], vc[None, :, :T]
        mask = None
        if rows > 1:   # causal among the new rows
            i = torch.arange(rows, device=x.device)[:, None]
            j = torch.arange(T, device=x.device)[None, :]
            mask = (j <= (T - rows + i))[None, None]
        o = F.scaled_dot_product_attention(qh, kk, vv, attn_mask=mask, enable_gqa=True)
        o = o[0].transpose(0, 1).reshape(rows, self.hq * hd).to(x.dtype)
        return self.tp.all_reduce(self.o_proj(o))


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: TP, bits: dict, device):
        super().__init__()
        ni = cfg.intermediate_size // tp.size
        h = cfg.hidden_size
        self.gate_proj = _exl3(h, ni, bits["gate_proj"], device)
        self.up_proj = _exl3(h, ni, bits["up_proj"], device)
        self.down_proj = _exl3(ni, h, bits["down_proj"], device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: TP, bits: dict, device):
        super().__init__()
        self.tp = tp
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, cfg.dtype, device)
        self.self_attn = Attention(cfg, tp, bits, device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, cfg.dtype, device)
        self.mlp = MLP(cfg, tp, bits, device)

    def forward(self, x, layer, cache, pos, cos, sin):
        h = x + self.self_attn(self.input_layernorm(x), layer, cache, pos, cos, sin)
        return h + self.tp.all_reduce(self.mlp(self.post_attention_layernorm(h)))


def _consumer_of(lin: EXL3Linear):
    return lin._group if lin._group is not None else lin


class _Targets:
    """The distinct EXL3 consumers (sibling groups or single linears) of one normalised input, with
    their stacked input scales: one rotation kernel writes all their rotated inputs."""

    def __init__(self, linears: list[EXL3Linear], units: list | None = None):
        self.units = list(units) if units is not None else []
        if units is None:
            for lin in linears:
                c = _consumer_of(lin)
                if all(c is not u for u in self.units):
                    self.units.append(c)
        self.nms = [u.rot_suh.shape[0] for u in self.units]
        self.suh = torch.cat([u.rot_suh for u in self.units]).contiguous()

    def outputs(self, xh: torch.Tensor, rows: int, out_dtype: torch.dtype) -> list[torch.Tensor]:
        """Every unit's GEMV output from the stacked rotations xh (sum(nms), rows, k)."""
        outs, o = [], 0
        for u, nm in zip(self.units, self.nms):
            if isinstance(u, EXL3Linear):
                outs.append(u.gemv_rotated(xh[o:o + nm], out_dtype))
            else:
                outs.append(u.plan(rows, out_dtype)(xh[o:o + nm], u.trs))
            o += nm
        return outs


class _MixedGroup:
    """Linears of one input that are not one sibling group (their bitrates differ) but share in_features
    and the codebook (q/k/v, gate/up): one GEMV launch with a bitrate per member (TrellisGemvPlan with a
    list of K); for q/k/v the decode step still finishes with qkv_post's math in that launch."""

    def __init__(self, members: list[EXL3Linear]):
        self.members = members
        self.k = members[0].in_features
        self.ns = [m.out_features for m in members]
        self.Ks = [m.bits for m in members]
        self.cb = members[0].codebook
        self.rot_suh = torch.cat([m.rot_suh for m in members]).contiguous()     # (3, k)
        self.svh = torch.cat([m.output_signs for m in members]).contiguous()
        self.trs = [m.trellis_words for m in members]
        self.plans: dict[tuple, TrellisGemvPlan] = {}

    @staticmethod
    def fits(members: list[EXL3Linear]) -> bool:
        f = members[0]
        return all(m.in_features == f.in_features and m.codebook == f.codebook and "bias" not in m and
                   m.out_features % 128 == 0 for m in members)

    def plan(self, rows: int, out_dtype: torch.dtype) -> TrellisGemvPlan:
        plan = self.plans.get((rows, out_dtype))
        if plan is None:
            plan = self.plans[(rows, out_dtype)] = TrellisGemvPlan(self.k, self.ns, self.Ks, self.cb, self.svh,
                                                                   rows, out_dtype)
        return plan


class _LayerDecode:
    """Per-layer state of the fused decode step (rows <= MAX_GEMV_ROWS)."""

    def __init__(self, layer: DecoderLayer):
        a, m = layer.self_attn, layer.mlp
        self.qkv = _Targets([a.q_proj, a.k_proj, a.v_proj])
        self.gate_up = _Targets([m.gate_proj, m.up_proj])
        # column slices of each projection inside the unit outputs: (unit index, column offset, width)
        self.qkv_at = [self._locate(self.qkv, lin) for lin in (a.q_proj, a.k_proj, a.v_proj)]
        self.gu_at = [self._locate(self.gate_up, lin) for lin in (m.gate_proj, m.up_proj)]
        # one q/k/v sibling group in that order: its GEMV can finish with qkv_post as the epilogue; q/k/v
        # of different bitrates become one mixed-bitrate launch with the same finish
        u = self.qkv.units[0]
        self.qkv_group = (u if len(self.qkv.units) == 1 and not isinstance(u, EXL3Linear)
                          and list(u.members) == [a.q_proj, a.k_proj, a.v_proj] else None)
        qkv, gu = [a.q_proj, a.k_proj, a.v_proj], [m.gate_proj, m.up_proj]
        if self.qkv_group is None and _MixedGroup.fits(qkv):
            self.qkv_group = _MixedGroup(qkv)
            self.qkv = _Targets(qkv, units=[self.qkv_group])       # the norm writes xh in q, k, v order
            self.qkv_at = self._spans(qkv)
        if len(self.gate_up.units) > 1 and _MixedGroup.fits(gu):
            self.gate_up = _Targets(gu, units=[_MixedGroup(gu)])
            self.gu_at = self._spans(gu)

    @staticmethod
    def _spans(lins: list[EXL3Linear]) -> list[tuple[int, int, int]]:
        """(unit 0, column offset, width) of each linear inside one mixed group's output."""
        out, off = [], 0
        for lin in lins:
            out.append((0, off, lin.out_features))
            off += lin.out_features
        return out

    @staticmethod
    def _locate(t: _Targets, lin: EXL3Linear) -> tuple[int, int, int]:
        c = _consumer_of(lin)
        ui = next(i for i, u in enumerate(t.units) if u is c)
        off = sum(c.ns[:lin._idx]) if c is not lin else 0
        return ui, off, lin.out_features


def _cols(outs: list[torch.Tensor], at: tuple[int, int, int]) -> torch.Tensor:
    ui, off, n = at
    return outs[ui][:, off:off + n]


class Inner(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: TP, layer_bits: list[dict], device):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size, device=device, dtype=cfg.dtype)
        self.embed_tokens.weight.requires_grad_(False)
        self.layers = nn.ModuleList([DecoderLayer(cfg, tp, b, device) for b in layer_bits])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, cfg.dtype, device)


class Qwen3EXL3(nn.Module):
    """Decoder with EXL3 linears. forward(tokens, pos) -> this rank's logits (rows, vocab_local)."""

    def __init__(self, cfg: ModelConfig, layer_bits: list[dict], head_bits: int | None, tp: TP | None = None,
                 device=None):
        super().__init__()
        self.cfg = cfg
        self.tp = tp or TP()
        self.model = Inner(cfg, self.tp, layer_bits, device)
        self.vocab_range = column_shard(((cfg.vocab_size + 127) // 128) * 128, self.tp)
        v0, v1 = self.vocab_range
        self.vocab_range = (v0, min(v1, cfg.vocab_size))
        self.lm_head = _exl3(cfg.hidden_size, v1 - v0, head_bits, device) if head_bits else None
        cos, sin = rope_tables(cfg, device)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def make_cache(self, max_len: int, device=None) -> KVCache:
        dev = device or self.rope_cos.device
        return KVCache(self.cfg.num_hidden_layers, self.cfg.num_key_value_heads // self.tp.size, max_len,
                       self.cfg.head_dim, dev)

    def hidden(self, tokens: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        x = self.model.embed_tokens(tokens)
        for i, layer in enumerate(self.model.layers):
            x = layer(x, i, cache, pos, self.rope_cos, self.rope_sin)
        return self.model.norm(x)

    def forward(self, tokens: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        if tokens.shape[0] <= MAX_GEMV_ROWS and self.fused_decode and self._decode_ready():
            return self._forward_decode(tokens, cache, pos)
        h = self.hidden(tokens, cache, pos)
        return self.lm_head(h) if self.lm_head is not None else h

    # -- fused decode step ----------------------------------------------------------------------
    # rows <= MAX_GEMV_ROWS: per layer  [add+]norm+rotate -> q/k/v GEMV with qkv_post (q/k norm, RoPE,
    # cache write) as its epilogue -> attention -> rotate -> o GEMV -> all-reduce -> add+norm+rotate -> gate/up GEMV ->
    # SwiGLU+rotate -> down GEMV -> all-reduce; the MLP residual add is folded into the next layer's
    # input norm (and the last one into the final norm). Same arithmetic and roundings as the module
    # path above (the residual sums round to the model dtype in both).
    fused_decode = True

    def _decode_ready(self) -> bool:
        plans = self.__dict__.get("_decode_plans")
        if plans is None:
            cfg = self.cfg
            ok = (cfg.head_dim == 128 and cfg.hidden_size % 1024 == 0
                  and cfg.dtype in (torch.float16, torch.bfloat16)
                  and all(isinstance(getattr(l.self_attn, n), EXL3Linear) for l in self.model.layers
                          for n in ("q_proj", "k_proj", "v_proj", "o_proj"))
                  and all(isinstance(getattr(l.mlp, n), EXL3Linear) and "bias" not in getattr(l.mlp, n)
                          for l in self.model.layers for n in ("gate_proj", "up_proj", "down_proj"))
                  and all("bias" not in getattr(l.self_attn, n) for l in self.model.layers
                          for n in ("q_proj", "k_proj", "v_proj", "o_proj")))
            plans = [_LayerDecode(l) for l in self.model.layers] if ok else []
            self.__dict__["_decode_plans"] = plans
            self.__dict__["_head_targets"] = _Targets([self.lm_head]) if ok and self.lm_head is not None else None
        return bool(plans)

    def reset_decode_plans(self):
        """Drop the fused-decode plans (after regrouping siblings or replacing linears)."""
        self.__dict__.pop("_decode_plans", None)

    def _forward_decode(self, tokens: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        rows = tokens.shape[0]
        dt = cfg.dtype
        hs = cfg.hidden_size
        peers = self.tp.peers if self.tp.size > 1 else None
        x = self.model.embed_tokens(tokens)
        T = cache.length + rows
        pending = None          # the row-parallel output still to be summed over ranks and added to x
        slot = 0                # peer-buffer slot of the next row-parallel output (alternates)

        def row_parallel(lin: EXL3Linear, xh_in: torch.Tensor):
            nonlocal slot
            if peers is None:
                return self.tp.all_reduce(lin.gemv_rotated(xh_in, dt))
            lin.plan(rows, dt).peer(xh_in, [lin.trellis_words], peers, slot)   # pushed into every rank's inbox
            slot ^= 1
            return slot ^ 1

        def add_norm(x, pend, w, suh, want_xn=False):
            if peers is None:
                return add_norm_rot(x, pend, w, eps, suh, want_xn=want_xn)
            return peers.ar_add_norm_rot(pend, x, w, eps, suh, want_xn=want_xn)

        for i, (layer, lp) in enumerate(zip(self.model.layers, self.__dict__["_decode_plans"])):
            attn = layer.self_attn
            w_in = layer.input_layernorm.weight
            if pending is None:
                _, xh = norm_rot(x, w_in, eps, lp.qkv.suh)
            else:
                x, _, xh = add_norm(x, pending, w_in, lp.qkv.suh)
            kc, vc = cache.k[i], cache.v[i]
            if lp.qkv_group is not None:                    # q/k/v GEMV with qkv_post as its epilogue
                g = lp.qkv_group
                q16 = g.plan(rows, dt).qkv_post(xh, g.trs, attn.q_norm.weight, attn.k_norm.weight, eps,
                                                self.rope_cos, self.rope_sin, pos, kc, vc)
            else:
                outs = lp.qkv.outputs(xh, rows, dt)
                q16 = qkv_post(_cols(outs, lp.qkv_at[0]), _cols(outs, lp.qkv_at[1]), _cols(outs, lp.qkv_at[2]),
                               attn.q_norm.weight, attn.k_norm.weight, eps, self.rope_cos, self.rope_sin, pos, kc, vc)
            if attn_fits(rows, q16.shape[1], kc.shape[0]):     # attention fused with o_proj's input rotation
                xo = attn_rot(q16, kc, vc, T, attn.o_proj.rot_suh)
            else:
                xo = rot(self._attend(q16, kc, vc, T, rows), attn.o_proj.rot_suh)
            a = row_parallel(attn.o_proj, xo)
            x, _, xh = add_norm(x, a, layer.post_attention_layernorm.weight, lp.gate_up.suh)
            gu_outs = lp.gate_up.outputs(xh, rows, torch.float16)
            gu = gu_outs[0] if len(gu_outs) == 1 else torch.cat(
                [_cols(gu_outs, lp.gu_at[0]), _cols(gu_outs, lp.gu_at[1])], dim=1)
            down = layer.mlp.down_proj
            if down.in_features <= FUSED_SWIGLU_MAX_K:
                # down_proj's GEMV computes SwiGLU and its own input rotation from gu in the same launch
                dplan = down.plan(rows, dt)
                if peers is None:
                    pending = self.tp.all_reduce(dplan.swiglu_call(gu, down.rot_suh, [down.trellis_words]))
                else:
                    dplan.swiglu_call(gu, down.rot_suh, [down.trellis_words], peers=peers, slot=slot)
                    pending = slot
                    slot ^= 1
            else:
                pending = row_parallel(down, swiglu_rot(gu, down.rot_suh.reshape(-1)))
        w_out = self.model.norm.weight
        head = self.__dict__["_head_targets"]
        if head is None:
            return add_norm(x, pending, w_out, torch.ones((1, hs), dtype=torch.float16, device=x.device),
                            want_xn=True)[1]
        _, _, xh = add_norm(x, pending, w_out, head.suh)
        return head.outputs(xh, rows, dt)[0]

    def close_peers(self):
        """Release the peer buffers (every rank, after the last decode step of the group)."""
        if self.tp.peers is not None:
            self.tp.peers.close()
            self.tp.peers = None

    def setup_peers(self, max_rows: int = MAX_GEMV_ROWS):
        """Collective over the tensor-parallel group: map the ranks' NVLink peer buffers so the decode
        step sums row-parallel outputs with the fused all-reduce kernel instead of NCCL."""
        if self.tp.size > 1 and self.tp.peers is None:
            from .comm import PeerGroup
            dev = self.rope_cos.device
            self.tp.peers = PeerGroup(self.tp.size, self.tp.rank, dev, max_rows, self.cfg.hidden_size,
                                      group=self.tp.group)

    @staticmethod
    def _attend(q16: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, T: int, rows: int) -> torch.Tensor:
        """GQA attention of the new rows (causal among themselves) over cache[:T]: (rows, hq*128) fp16."""
        hq = q16.shape[1]
        qh = q16.transpose(0, 1)[None]                                   # (1, hq, rows, 128)
        mask = None
        if rows > 1:
            i = torch.arange(rows, device=q16.device)[:, None]
            j = torch.arange(T, device=q16.device)[None, :]
            mask = (j <= (T - rows + i))[None, None]
        o = F.scaled_dot_product_attention(qh, kc[None, :, :T], vc[None, :, :T], attn_mask=mask, enable_gqa=True)
        return o[0].transpose(0, 1).reshape(rows, hq * 128)

    def gather_logits(self, local: torch.Tensor) -> torch.Tensor:
        """All ranks' logit shards -> (rows, vocab) on every rank."""
        if self.tp.size == 1:
            return local[:, : self.cfg.vocab_size]
        n_local = torch.tensor([local.shape[1]], device=local.device)
        sizes = [torch.zeros_like(n_local) for _ in range(self.tp.size)]
        dist.all_gather(sizes, n_local, group=self.tp.group)
        mx = int(max(s.item() for s in sizes))
        pad = torch.zeros((local.shape[0], mx), dtype=local.dtype, device=local.device)
        pad[:, : local.shape[1]] = local
        parts = [torch.empty_like(pad) for _ in range(self.tp.size)]
        dist.all_gather(parts, pad, group=self.tp.group)
        out = torch.cat([p[:, : int(s.item())] for p, s in zip(parts, sizes)], dim=1)
        return out[:, : self.cfg.vocab_size]

    def greedy(self, local: torch.Tensor) -> torch.Tensor:
        """Global argmax token per row from the local logit shard (one small all-gather). Without an
        output head the argmax is over the (replicated) final hidden state."""
        if self.lm_head is None:
            v0, n_valid = 0, local.shape[1]
        else:
            v0 = self.vocab_range[0]
            n_valid = self.vocab_range[1] - v0
        val, idx = argmax(local, n_valid, v0)                           # one pass over the fp16/bf16 logits
        if self.tp.size == 1:
            return idx
        pack = torch.stack([val, idx.float()], dim=-1)                  # (rows, 2); indices < 2^24 are exact
        flat = torch.empty((self.tp.size * pack.shape[0], 2), dtype=pack.dtype, device=pack.device)
        dist.all_gather_into_tensor(flat, pack, group=self.tp.group)    # ranks concatenated, no per-rank copies
        allp = flat.view(self.tp.size, pack.shape[0], 2)                 # (tp, rows, 2)
        best = allp[..., 0].argmax(dim=0)                                # (rows,)
        return allp[best, torch.arange(pack.shape[0], device=pack.device), 1].long()
