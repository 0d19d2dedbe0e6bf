"""TEST INFRASTRUCTURE ONLY -- fp32 numpy forward of the Qwen3-style EXL3 decoder (omlx_exl3_b200.model).

Only tests/ use this module, as the checker of the model path's logits (logit KL). Every EXL3 linear is
evaluated with oracle.linear_forward (the reference's EXL3Linear forward, linear.py:107-121, in fp32
without the intermediate fp16 roundings); norms are exact fp32 RMSNorm, attention is exact softmax
attention over the given fp16 KV cache plus the new rows (causal among them), RoPE rotate-half.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def _np(t):
    return t.detach().float().cpu().numpy()


def _lin(mod, x):
    """fp32 forward of one EXL3Linear from its buffers."""
    tr = mod.trellis.detach().cpu().numpy()
    k, n = mod.in_features, mod.out_features
    K = tr.shape[-1] // 16
    cb = 2 if "mul1" in mod else 1 if "mcg" in mod else 0
    suh = _np(mod.suh) if "suh" in mod else O.unpack_signs(mod.su.cpu().numpy()).astype(np.float32)
    svh = _np(mod.svh) if "svh" in mod else O.unpack_signs(mod.sv.cpu().numpy()).astype(np.float32)
    bias = _np(mod.bias) if "bias" in mod else None
    return O.linear_forward(tr, k, n, K, cb, x, suh, svh, bias)


def _rms(x, w, eps):
    x = np.asarray(x, np.float64)
    return (x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * np.asarray(w, np.float64)).astype(np.float32)


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def forward(model, tokens: np.ndarray, cache_k: list, cache_v: list, length: int) -> np.ndarray:
    """Logits (rows, vocab_local) for `tokens` at positions length.., given per-layer fp16 caches
    (n_kv, >= length, hd) as numpy float arrays. The caches are not modified."""
    cfg = model.cfg
    hd = cfg.head_dim
    rows = len(tokens)
    pos = np.arange(length, length + rows)
    cos, sin = _np(model.rope_cos)[pos], _np(model.rope_sin)[pos]
    x = _np(model.model.embed_tokens.weight)[tokens]
    for li, layer in enumerate(model.model.layers):
        at = layer.self_attn
        xn = _rms(x, _np(layer.input_layernorm.weight), cfg.rms_norm_eps)
        q = _lin(at.q_proj, xn).reshape(rows, at.hq, hd)
        k = _lin(at.k_proj, xn).reshape(rows, at.hkv, hd)
        v = _lin(at.v_proj, xn).reshape(rows, at.hkv, hd)
        q = _rms(q, _np(at.q_norm.weight), cfg.rms_norm_eps)
        k = _rms(k, _np(at.k_norm.weight), cfg.rms_norm_eps)
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        K_all = np.concatenate([cache_k[li][:, :length], k.transpose(1, 0, 2).astype(np.float16).astype(np.float32)], 1)
        V_all = np.concatenate([cache_v[li][:, :length], v.transpose(1, 0, 2).astype(np.float16).astype(np.float32)], 1)
        g = at.hq // at.hkv
        T = length + rows
        out = np.zeros((rows, at.hq, hd), np.float32)
        for hh in range(at.hq):
            kv = hh // g
            s = (q[:, hh, :].astype(np.float64) @ K_all[kv].T.astype(np.float64)) / np.sqrt(hd)
            mask = np.arange(T)[None, :] <= (length + np.arange(rows))[:, None]
            s = np.where(mask, s, -np.inf)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[:, hh, :] = (p @ V_all[kv].astype(np.float64)).astype(np.float32)
        x = x + _lin(at.o_proj, out.reshape(rows, at.hq * hd))
        xn = _rms(x, _np(layer.post_attention_layernorm.weight), cfg.rms_norm_eps)
        mlp = layer.mlp
        gt, up = _lin(mlp.gate_proj, xn), _lin(mlp.up_proj, xn)
        x = x + _lin(mlp.down_proj, gt / (1.0 + np.exp(-gt)) * up)
    xn = _rms(x, _np(model.model.norm.weight), cfg.rms_norm_eps)
    return _lin(model.lm_head, xn) if model.lm_head is not None else xn
