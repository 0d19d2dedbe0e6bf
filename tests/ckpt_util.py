"""Test helper: write an EXL3 checkpoint directory (config.json + sharded safetensors + index) from an
unsharded model of omlx_exl3_b200.model, in the layout ExLlamaV3 checkpoints use: per quantised linear
`<prefix>.trellis` (int16 [k/16, n/16, 16K]) with `<prefix>.suh` / `.svh` (fp16) or the older packed
`<prefix>.su` / `.sv` (int16 bitfields), an optional codebook marker (`.mcg` / `.mul1`) and an optional
`.bias`; every other parameter under its module path."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch


def pack_signs(pm1: torch.Tensor) -> torch.Tensor:
    """+-1 vector -> int16 words, bit i of word j set when element 16j+i is negative."""
    neg = (pm1.float().cpu().numpy() < 0).astype(np.uint32).reshape(-1, 16)
    words = (neg << np.arange(16, dtype=np.uint32)).sum(axis=1).astype(np.uint16)
    return torch.from_numpy(words.view(np.int16).copy())


def write_checkpoint(model, path: Path, n_shards: int = 2, legacy: tuple = (), markers: dict | None = None,
                     biases: dict | None = None) -> dict[str, torch.Tensor]:
    """Write `model` (tp_size 1) to `path`. legacy: linear prefixes stored with packed su/sv; markers:
    prefix -> "mcg" | "mul1"; biases: prefix -> fp16 tensor. Returns every written tensor by name."""
    from omlx_exl3_b200.linear import EXL3Linear
    markers, biases = markers or {}, biases or {}
    path.mkdir(parents=True, exist_ok=True)
    tensors: dict[str, torch.Tensor] = {}
    exl3 = {name: m for name, m in model.named_modules() if isinstance(m, EXL3Linear)}
    for prefix, lin in exl3.items():
        tensors[f"{prefix}.trellis"] = lin.trellis.cpu()
        if prefix in legacy:
            tensors[f"{prefix}.su"] = pack_signs(lin.suh)
            tensors[f"{prefix}.sv"] = pack_signs(lin.svh)
        else:
            tensors[f"{prefix}.suh"] = lin.suh.cpu()
            tensors[f"{prefix}.svh"] = lin.svh.cpu()
        if prefix in markers:
            tensors[f"{prefix}.{markers[prefix]}"] = torch.zeros(1, dtype=torch.int32)
        if prefix in biases:
            tensors[f"{prefix}.bias"] = biases[prefix].to(torch.float16).cpu()
    for name, p in model.named_parameters():
        owner = name.rpartition(".")[0]
        if owner not in exl3:
            tensors[name] = p.detach().cpu()
    names = sorted(tensors)
    shards = [names[i::n_shards] for i in range(n_shards)]
    weight_map = {}
    from safetensors.torch import save_file
    for i, group in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{n_shards:05d}.safetensors"
        save_file({nm: tensors[nm].contiguous() for nm in group}, str(path / fname))
        weight_map.update({nm: fname for nm in group})
    (path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    cfg = model.cfg
    (path / "config.json").write_text(json.dumps({
        "model_type": "qwen3", "hidden_size": cfg.hidden_size, "num_attention_heads": cfg.num_attention_heads,
        "num_key_value_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim,
        "intermediate_size": cfg.intermediate_size, "num_hidden_layers": cfg.num_hidden_layers,
        "vocab_size": cfg.vocab_size, "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta,
        "max_position_embeddings": cfg.max_position_embeddings, "torch_dtype": "bfloat16",
        "quantization_config": {"quant_method": "exl3"}}))
    return tensors
