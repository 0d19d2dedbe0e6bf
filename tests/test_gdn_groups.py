"""Gated-DeltaNet (linear attention) layers: their input projections in_proj_qkv and in_proj_z read the
same normed input, so the loader ties them into one sibling group and fuse_decode hands the input norm's
rotation to that group (reference: src/omlx/exl3/loader.py:39 `_SIBLINGS`, fusion.py:114-117). The
delta-rule mixer itself is the model library's code; a stand-in mixer (qkv * sigmoid(z)) exercises the
projections here. CPU: grouping and fusion sites. GPU: the fused decode path against the unfused one and
against the fp32 oracle of each projection."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O

H = 1024


class _LinearAttn(nn.Module):
    def __init__(self, qkv, z, out):
        super().__init__()
        self.in_proj_qkv, self.in_proj_z, self.out_proj = qkv, z, out

    def forward(self, x):
        a = self.in_proj_qkv(x)
        g = torch.sigmoid(self.in_proj_z(x).float())
        return self.out_proj((a[..., : g.shape[-1]].float() * g).to(x.dtype))


class _Mlp(nn.Module):
    def __init__(self, gate, up, down):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down

    def forward(self, x):
        g, u = self.gate_proj(x).float(), self.up_proj(x).float()
        return self.down_proj((g / (1 + torch.exp(-g)) * u).to(x.dtype))


class _Layer(nn.Module):
    def __init__(self, attn, mlp, device):
        super().__init__()
        from omlx_exl3_b200.model import RMSNorm
        self.input_layernorm = RMSNorm(H, 1e-6, torch.bfloat16, device)
        self.post_attention_layernorm = RMSNorm(H, 1e-6, torch.bfloat16, device)
        self.linear_attn, self.mlp = attn, mlp

    def forward(self, x):
        h = x + self.linear_attn(self.input_layernorm(x))
        return h + self.mlp(self.post_attention_layernorm(h))


class _Model(nn.Module):
    def __init__(self, layer):
        super().__init__()
        self.layers = nn.ModuleList([layer])

    def forward(self, x):
        return self.layers[0](x)


SHAPES = {"in_proj_qkv": (H, 768, 4), "in_proj_z": (H, 256, 4), "out_proj": (256, H, 5),
          "gate_proj": (H, 512, 5), "up_proj": (H, 512, 5), "down_proj": (512, H, 5)}


def _build(device, seed=0, fill=True):
    from omlx_exl3_b200.model import _exl3
    rng = np.random.default_rng(seed)
    lins, tensors = {}, {}
    for i, (name, (k, n, K)) in enumerate(SHAPES.items()):
        lin = _exl3(k, n, K, device)
        if fill:
            t = O.random_trellis(k, n, K, seed + 10 + i)
            suh = np.where(rng.random(k) < 0.5, -1, 1).astype(np.float16)
            svh = (rng.standard_normal(n) * 0.05).astype(np.float16)
            lin.load_state_dict({"trellis": torch.from_numpy(t), "suh": torch.from_numpy(suh),
                                 "svh": torch.from_numpy(svh)})
            tensors[name] = (t, suh, svh)
        lins[name] = lin
    attn = _LinearAttn(lins["in_proj_qkv"], lins["in_proj_z"], lins["out_proj"])
    mlp = _Mlp(lins["gate_proj"], lins["up_proj"], lins["down_proj"])
    return _Model(_Layer(attn, mlp, device)), lins, tensors


def test_gdn_projections_group_and_fusion_sites():
    from omlx_exl3_b200 import fusion
    from omlx_exl3_b200.loader import group_siblings
    model, lins, _ = _build("cpu", fill=False)
    assert group_siblings(model) == 2                   # in_proj_qkv/z and gate/up
    g = lins["in_proj_qkv"]._group
    assert g is not None and g is lins["in_proj_z"]._group and g.ns == [768, 256]
    sites = fusion.find_sites(model)
    layer = model.layers[0]
    norm_sites = [s for s in sites if isinstance(s, fusion.NormSite)]
    assert any(s.module is layer.input_layernorm and s.units == [g] for s in norm_sites)
    assert any(s.module is layer.post_attention_layernorm for s in norm_sites)
    assert any(isinstance(s, fusion.MlpSite) for s in sites)


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 4])
def test_gdn_fused_decode_matches_unfused_and_oracle(cuda, rows):
    from omlx_exl3_b200 import fusion
    from omlx_exl3_b200.loader import group_siblings
    model, lins, tensors = _build(cuda, seed=3)
    group_siblings(model)
    x = torch.randn((rows, H), generator=torch.Generator().manual_seed(rows)).to(cuda, torch.bfloat16)
    with torch.no_grad():
        ref = model(x).float()
        counts = fusion.fuse_decode(model)
        assert counts["norm"] == 2 and counts["mlp"] == 1
        fused = model(x).float()
        # the grouped projections of the normed input against the fp32 oracle of each linear
        xn = model.layers[0].input_layernorm(x)
        outs = lins["in_proj_qkv"]._group(xn)
    fusion.unfuse(model)
    torch.cuda.synchronize()
    assert O.max_rel(fused.cpu().numpy(), ref.cpu().numpy()) < 1e-2
    for name, y in zip(("in_proj_qkv", "in_proj_z"), outs):
        t, suh, svh = tensors[name]
        k, n, K = SHAPES[name]
        want = O.linear_forward(t, k, n, K, 0, xn.float().cpu().numpy(), suh, svh)
        assert O.max_rel(y.float().cpu().numpy(), want) < 1e-2, name
