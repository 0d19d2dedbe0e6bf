"""Place EXL3 checkpoints (or seeded synthetic EXL3 tensors) in HBM, sharded across the GPUs of a box.

Functions with a counterpart in daig/omlx-exl3 src/omlx/exl3/loader.py (same names and results):
  is_exl3_config      loader.py:45-47    does config.json declare EXL3 quantisation
  _read_header        loader.py:50-55    tensor table of one safetensors shard
  inventory           loader.py:58-72    EXL3 linear prefix -> {part: (shape, dtype)}, from headers only
  group_siblings      loader.py:137-156  same-input linears tied into single-launch groups per rate
  unify_float_dtypes  loader.py:159-180  non-EXL3 float parameters at the embedding dtype
  load                loader.py:183-223  model with EXL3 linears from a checkpoint directory
The model is this package's Qwen3-style decoder (model.py) instead of mlx-vlm's, and load() takes the
tensor-parallel rank and size: column-parallel linears (q/k/v, gate/up, lm_head) get whole 128-column
blocks of the trellis ([:, nt0:nt1, :]) and of svh; row-parallel ones (o_proj, down_proj) get whole
128-row blocks ([kt0:kt1, :, :]) and the matching suh slice. Only this rank's slice is read from disk.
"""
from __future__ import annotations

import json
import logging
import os
import struct
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .fusion import fuse_decode
from .linear import EXL3Linear, EXL3SiblingGroup
from .model import TP, ModelConfig, Qwen3EXL3, column_shard, row_shard

logger = logging.getLogger(__name__)

_DTYPES = {"I16": torch.int16, "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32,
           "I32": torch.int32, "U16": torch.int16, "U32": torch.int32, "I8": torch.int8, "U8": torch.uint8}
_NP = {"I16": np.int16, "F16": np.float16, "BF16": np.uint16, "F32": np.float32, "I32": np.int32,
       "U16": np.int16, "U32": np.int32, "I8": np.int8, "U8": np.uint8}
_EXL3_PARTS = ("trellis", "suh", "svh", "su", "sv", "mul1", "mcg", "bias")
_SIBLINGS = (("q_proj", "k_proj", "v_proj"), ("gate_proj", "up_proj"), ("in_proj_qkv", "in_proj_z"))
COLUMN_PARALLEL = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "lm_head")
ROW_PARALLEL = ("o_proj", "down_proj")


def is_exl3_config(config: dict[str, Any]) -> bool:
    """Whether a Hugging Face config.json declares EXL3 quantisation (quant_method "exl3", any case)."""
    method = (config.get("quantization_config") or {}).get("quant_method")
    return isinstance(method, str) and method.casefold() == "exl3"


def _read_header(path: Path) -> dict[str, Any]:
    """Tensor table of one safetensors file: a little-endian u64 byte count, then that many bytes of
    JSON mapping each tensor name to its dtype, shape and offsets (the `__metadata__` entry dropped)."""
    with open(path, "rb") as fh:
        (size,) = struct.unpack("<Q", fh.read(8))
        table = json.loads(fh.read(size).decode("utf-8"))
    return {name: entry for name, entry in table.items() if name != "__metadata__"}


def _files(model_path: Path) -> list[str]:
    """The checkpoint's safetensors shards: those the index names, else the single model.safetensors."""
    index = model_path / "model.safetensors.index.json"
    if not index.exists():
        return ["model.safetensors"]
    return sorted(set(json.loads(index.read_text())["weight_map"].values()))


def inventory(model_path: Path) -> dict[str, dict[str, tuple[tuple[int, ...], Any]]]:
    """For every EXL3 linear of the checkpoint (a tensor name prefix with a `.trellis` part), the parts
    present (`_EXL3_PARTS`) with their (shape, torch dtype), read from the shard headers only."""
    parts_by_prefix: dict[str, dict[str, tuple[tuple[int, ...], Any]]] = {}
    for f in _files(model_path):
        for name, entry in _read_header(model_path / f).items():
            prefix, _, part = name.rpartition(".")
            if part in _EXL3_PARTS:
                parts_by_prefix.setdefault(prefix, {})[part] = (tuple(entry["shape"]), _DTYPES[entry["dtype"]])
    return {prefix: parts for prefix, parts in parts_by_prefix.items() if "trellis" in parts}


def _sibling_sets(model: torch.nn.Module):
    """Every complete set of same-input EXL3 linears (one of _SIBLINGS found under one module)."""
    for _, owner in model.named_modules():
        for names in _SIBLINGS:
            found = [getattr(owner, nm, None) for nm in names]
            if all(isinstance(lin, EXL3Linear) for lin in found):
                yield found


def group_siblings(model: torch.nn.Module) -> int:
    """Tie same-input EXL3 linears into EXL3SiblingGroups (one GEMV launch each). A group launch runs
    one bitrate and codebook, so a set is first split by (bits, codebook): a checkpoint that gives q
    its own rate still gets k and v as a pair. Returns the number of groups made."""
    made = 0
    for found in _sibling_sets(model):
        rates = sorted({(lin.bits, lin.codebook) for lin in found})
        for rate in rates:
            subset = [lin for lin in found if (lin.bits, lin.codebook) == rate]
            if EXL3SiblingGroup.fusable(subset):
                EXL3SiblingGroup(subset)
                made += 1
    return made


def unify_float_dtypes(model: torch.nn.Module) -> int:
    """Bring every floating-point parameter outside the EXL3 linears to the token embedding's dtype, so
    no elementwise op mixes fp16 and bf16 operands (which would promote to fp32). EXL3Linear keeps its
    checkpoint dtypes: it computes in fp16 internally and returns its caller's dtype. Returns the
    number of parameters cast."""
    embed = next((m for name, m in model.named_modules() if name.endswith("embed_tokens")), None)
    if embed is None or getattr(embed, "weight", None) is None:
        return 0
    want = embed.weight.dtype
    casts = [p for m in model.modules() if not isinstance(m, EXL3Linear)
             for p in m.parameters(recurse=False) if p.dtype.is_floating_point and p.dtype != want]
    for p in casts:
        p.data = p.data.to(want)
    return len(casts)


# ------------------------------------------------------------------------------ shard helpers

def _kind(prefix: str) -> str:
    leaf = prefix.rsplit(".", 1)[-1]
    if leaf in ROW_PARALLEL:
        return "row"
    if leaf in COLUMN_PARALLEL:
        return "col"
    return "rep"


def shard_exl3_part(part: str, arr, kind: str, k: int, n: int, tp: TP):
    """This rank's slice of one EXL3 tensor (numpy or torch, checkpoint layout)."""
    if tp.size == 1 or kind == "rep":
        return arr
    if kind == "col":
        c0, c1 = column_shard(n, tp)
        if part == "trellis":
            return arr[:, c0 // 16:c1 // 16, :]
        if part in ("svh", "bias"):
            return arr[c0:c1]
        if part == "sv":
            return arr[c0 // 16:c1 // 16]
        return arr
    r0, r1 = row_shard(k, tp)
    if part == "trellis":
        return arr[r0 // 16:r1 // 16, :, :]
    if part == "suh":
        return arr[r0:r1]
    if part == "su":
        return arr[r0 // 16:r1 // 16]
    if part == "bias":
        return arr if tp.rank == 0 else arr * 0
    return arr


def _layer_bits_from_inventory(cfg: ModelConfig, inv) -> tuple[list[dict], int | None]:
    layer_bits = []
    for i in range(cfg.num_hidden_layers):
        b = {}
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            b[name] = inv[f"model.layers.{i}.self_attn.{name}"]["trellis"][0][-1] // 16
        for name in ("gate_proj", "up_proj", "down_proj"):
            b[name] = inv[f"model.layers.{i}.mlp.{name}"]["trellis"][0][-1] // 16
        layer_bits.append(b)
    head = inv.get("lm_head")
    return layer_bits, (head["trellis"][0][-1] // 16 if head else None)


def _finish(model: Qwen3EXL3, fuse: bool) -> Qwen3EXL3:
    for m in model.modules():
        if isinstance(m, EXL3Linear):
            m.reset_runtime()
    cast = unify_float_dtypes(model)
    groups = group_siblings(model)
    fuse = fuse and os.environ.get("OMLX_EXL3_FUSE", "1") != "0"
    fused = fuse_decode(model) if fuse else {}
    model.fused_decode = fuse        # the fused decode step of Qwen3EXL3 (rows <= MAX_GEMV_ROWS)
    model.reset_decode_plans()
    logger.info("EXL3: %d sibling groups, %d float tensors cast, fused rotations %s", groups, cast, fused)
    return model


def _sharded_shape(part: str, shape: tuple, kind: str, k: int, n: int, tp: TP) -> tuple:
    if tp.size == 1 or kind == "rep":
        return tuple(shape)
    if kind == "col":
        c0, c1 = column_shard(n, tp)
        if part == "trellis":
            return (shape[0], (c1 - c0) // 16, shape[2])
        if part in ("svh", "bias"):
            return (c1 - c0,)
        if part == "sv":
            return ((c1 - c0) // 16,)
        return tuple(shape)
    r0, r1 = row_shard(k, tp)
    if part == "trellis":
        return ((r1 - r0) // 16, shape[1], shape[2])
    if part == "suh":
        return (r1 - r0,)
    if part == "su":
        return ((r1 - r0) // 16,)
    return tuple(shape)


def _slice_index(part: str, kind: str, k: int, n: int, tp: TP):
    """Index tuple selecting this rank's slice of a checkpoint tensor (read lazily from disk)."""
    if tp.size == 1 or kind == "rep":
        return None
    if kind == "col":
        c0, c1 = column_shard(n, tp)
        return {"trellis": (slice(None), slice(c0 // 16, c1 // 16)), "svh": (slice(c0, c1),),
                "bias": (slice(c0, c1),), "sv": (slice(c0 // 16, c1 // 16),)}.get(part)
    r0, r1 = row_shard(k, tp)
    return {"trellis": (slice(r0 // 16, r1 // 16),), "suh": (slice(r0, r1),),
            "su": (slice(r0 // 16, r1 // 16),)}.get(part)


def load(model_name: str | Path, *, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
         device: torch.device | str | None = None, fuse: bool = True) -> Qwen3EXL3:
    """Model with EXL3 linears from a checkpoint directory (config.json + safetensors), this rank's shard."""
    from safetensors import safe_open

    model_path = Path(model_name)
    cfg_json = json.loads((model_path / "config.json").read_text())
    if not is_exl3_config(cfg_json):
        logger.warning("EXL3: %s has no exl3 quantization_config; loading its trellis tensors anyway", model_path)
    inv = inventory(model_path)
    if not inv:
        raise ValueError(f"no EXL3 trellis tensors found in {model_path}")
    cfg = ModelConfig.from_hf(cfg_json)
    tp = TP(tp_rank, tp_size, tp_group)
    layer_bits, head_bits = _layer_bits_from_inventory(cfg, inv)
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    model = Qwen3EXL3(cfg, layer_bits, head_bits, tp, device)

    # each EXL3 linear declares exactly its checkpoint's parts (legacy su/sv, codebook marker, bias)
    full_kn = {}
    for prefix, parts in inv.items():
        old = model.get_submodule(prefix)
        if not isinstance(old, EXL3Linear):
            raise TypeError(f"EXL3 tensor at {prefix} targets a {type(old).__name__}, expected Linear")
        tshape = parts["trellis"][0]
        k_full, n_full = tshape[0] * 16, tshape[1] * 16
        kind = _kind(prefix)
        full_kn[prefix] = (k_full, n_full, kind)
        tensors = {part: (_sharded_shape(part, shape, kind, k_full, n_full, tp), dt)
                   for part, (shape, dt) in parts.items()}
        new = EXL3Linear(old.in_features, old.out_features, tensors, device=device)
        parent_name, _, leaf = prefix.rpartition(".")
        setattr(model.get_submodule(parent_name) if parent_name else model, leaf, new)

    state = model.state_dict()
    loaded = set()
    for f in _files(model_path):
        with safe_open(str(model_path / f), framework="pt") as fh:
            for key in fh.keys():
                prefix, _, part = key.rpartition(".")
                if prefix in inv:
                    k_full, n_full, kind = full_kn[prefix]
                    idx = _slice_index(part, kind, k_full, n_full, tp)
                    t = fh.get_slice(key)[idx] if idx is not None else fh.get_tensor(key)
                    if part == "bias" and kind == "row" and tp.rank != 0:
                        t = torch.zeros_like(t)
                    dst = model.get_submodule(prefix)._buffers[part]
                    dst.copy_(t.view(dst.dtype) if t.dtype != dst.dtype and t.element_size() == dst.element_size()
                              else t)
                    loaded.add(key)
                elif key in state:
                    state[key].copy_(fh.get_tensor(key).to(state[key].dtype))
                    loaded.add(key)
    missing = [k for k in state if k not in loaded]
    if missing:
        logger.warning("EXL3: %d tensors not in the checkpoint (left at init): %s", len(missing), missing[:5])
    return _finish(model, fuse)


# ------------------------------------------------------------------------------ synthetic weights

# Sibling tensors that self-calibrated EXL3 checkpoints quantize at one rate (k/v, gate/up), so that
# they can share one GEMV launch; q, o and down get their own rates.
_RATE_GROUPS = (("q_proj",), ("k_proj", "v_proj"), ("o_proj",), ("gate_proj", "up_proj"), ("down_proj",))


def draw_bits(n_layers: int, seed: int, choices=(5, 6, 7, 8), target: float = 6.0, cfg: ModelConfig | None = None
              ) -> list[dict]:
    """Seeded per-tensor bitrates in 5..8 bpw whose weight-count-weighted mean is `target` (BASELINE
    config 5). One rate per rate group (_RATE_GROUPS); drawn, then nudged group by group until the
    weighted mean is within 0.01 of the target."""
    cfg = cfg or ModelConfig()
    h, hd, ni = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    sizes = {"q_proj": h * cfg.num_attention_heads * hd, "k_proj": h * cfg.num_key_value_heads * hd,
             "v_proj": h * cfg.num_key_value_heads * hd, "o_proj": cfg.num_attention_heads * hd * h,
             "gate_proj": h * ni, "up_proj": h * ni, "down_proj": ni * h}
    gsize = {grp: sum(sizes[nm] for nm in grp) for grp in _RATE_GROUPS}
    rng = np.random.default_rng(seed)
    p = np.array([0.35, 0.35, 0.2, 0.1])[: len(choices)]
    p = p / p.sum()
    groups = [{grp: int(rng.choice(choices, p=p)) for grp in _RATE_GROUPS} for _ in range(n_layers)]
    total = sum(gsize.values()) * n_layers

    def mean():
        return sum(gsize[grp] * b[grp] for b in groups for grp in gsize) / total

    order = [(li, grp) for li in range(n_layers) for grp in _RATE_GROUPS]
    rng.shuffle(order)
    it = 0
    while abs(mean() - target) > 0.01 and it < 100 * len(order):
        li, grp = order[it % len(order)]
        b = groups[li][grp]
        # a step of the smallest groups first keeps the final mean close to the target
        if mean() > target and b > min(choices):
            groups[li][grp] = b - 1
        elif mean() < target and b < max(choices):
            groups[li][grp] = b + 1
        it += 1
    return [{nm: b[grp] for grp in _RATE_GROUPS for nm in grp} for b in groups]


def synthetic_model(cfg: ModelConfig, layer_bits: list[dict], head_bits: int | None, *, tp_rank: int = 0,
                    tp_size: int = 1, tp_group=None, device=None, seed: int = 0, fuse: bool = True,
                    codebook: int = 0, svh_scale: float = 1.0) -> Qwen3EXL3:
    """Random-init model with seeded uniform trellis, +-1 suh, +-svh_scale/(1.244 sqrt(k)) svh (0 gives
    +-1) and N(1, 0.1) norm weights, generated
    directly on the device. Every rank draws the same full tensors and keeps its shard, so any TP size
    describes the same model."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    tp = TP(tp_rank, tp_size, tp_group)
    model = Qwen3EXL3(cfg, layer_bits, head_bits, tp, device)
    gen = torch.Generator(device=device)
    for idx, (name, mod) in enumerate(sorted(model.named_modules(), key=lambda x: x[0])):
        if isinstance(mod, EXL3Linear):
            kind = _kind(name)
            k_full = mod.in_features * (tp_size if kind == "row" else 1)
            n_full = mod.out_features * (tp_size if kind == "col" else 1)
            if name == "lm_head":
                n_full = ((cfg.vocab_size + 127) // 128) * 128
            K = mod.trellis.shape[-1] // 16
            gen.manual_seed(seed * 1000003 + idx)
            words = torch.randint(-2 ** 31, 2 ** 31 - 1, (k_full // 16, n_full // 16, 8 * K), dtype=torch.int32,
                                  device=device, generator=gen)
            tr = words.view(torch.int16)
            suh = torch.randint(0, 2, (k_full,), device=device, generator=gen).to(torch.float16) * 2 - 1
            # +-svh_scale / sqrt(k): with decoded weights of std ~1.24 each linear keeps the activation
            # scale, so a deep random model stays inside the fp16 range of the rotated inputs
            sv = svh_scale / (1.244 * float(k_full) ** 0.5) if svh_scale else 1.0
            svh = (torch.randint(0, 2, (n_full,), device=device, generator=gen).to(torch.float32) * 2 - 1) * sv
            svh = svh.to(torch.float16)
            mod.trellis.copy_(shard_exl3_part("trellis", tr, kind, k_full, n_full, tp))
            mod.suh.copy_(shard_exl3_part("suh", suh, kind, k_full, n_full, tp))
            mod.svh.copy_(shard_exl3_part("svh", svh, kind, k_full, n_full, tp))
            del words, tr
            if codebook:
                mod.register_buffer("mcg" if codebook == 1 else "mul1", torch.zeros(1, dtype=torch.int32, device=device))
    gen.manual_seed(seed * 7919 + 1)
    model.model.embed_tokens.weight.normal_(0, 1.0, generator=gen)
    for name, mod in model.named_modules():
        if getattr(mod, "_exl3_rms_norm", False):
            mod.weight.normal_(1.0, 0.1, generator=gen)
    return _finish(model, fuse)
