"""GPU: decode attention fused with o_proj's input rotation (exl3_attn_decode_rot).

Expected values: attention computed in fp32 by torch on the same fp16 q and cache (scores / sqrt(128),
causal rule for the new rows, softmax, P V), rounded to fp16 as the framework's attention output is,
then the oracle's rotation (numpy, Sylvester FWHT / sqrt(128) after * suh). The kernel's probabilities
enter the P V product in fp16, so the bound is relative to the output's largest magnitude."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _reference(q, kc, vc, T, suh):
    rows, hq = q.shape[0], q.shape[1]
    hkv = kc.shape[0]
    grp = hq // hkv
    qf = q.float()                                                     # (rows, hq, 128)
    k = kc[:, :T].float().repeat_interleave(grp, dim=0)                # (hq, T, 128)
    v = vc[:, :T].float().repeat_interleave(grp, dim=0)
    s = torch.einsum("rhd,htd->hrt", qf, k) / math.sqrt(128.0)
    pos = torch.arange(T, device=q.device)[None, :]
    lim = (T - rows + torch.arange(rows, device=q.device))[:, None]
    s = s.masked_fill((pos > lim)[None], float("-inf"))
    o = torch.einsum("hrt,htd->rhd", torch.softmax(s, dim=-1), v)      # (rows, hq, 128)
    o16 = o.reshape(rows, hq * 128).half()
    return O.rot(o16.float().cpu().numpy(), suh.reshape(1, -1).cpu().numpy())


@pytest.mark.parametrize("rows,hq,hkv,T,max_len", [
    (1, 40, 8, 4097, 4200),      # 27B-class layer, one GPU
    (1, 20, 4, 4097, 4200),      # tensor-parallel 2
    (1, 5, 1, 4097, 4200),       # tensor-parallel 8
    (1, 40, 8, 1, 16),           # a single cached position
    (1, 40, 8, 100, 128),        # ragged: positions end inside a 16-position step
    (3, 40, 8, 257, 300),        # three new rows (15 q vectors per kv head), causal among them
    (2, 16, 2, 50, 64),          # exactly one 16-row tile of q vectors
    (1, 8, 8, 33, 40),           # no grouping
    (4, 40, 8, 4100, 4200),      # 4-token MTP verify at the 27B-class layer: 20 q vectors, two q groups
    (8, 40, 8, 300, 320),        # 8-token verify: 40 q vectors, three q groups (the last one partial)
    (4, 5, 1, 4100, 4200),       # 4-token verify at tensor-parallel 8
    (6, 40, 8, 70, 80),          # 6 rows, 30 q vectors, positions end inside a step
])
def test_attn_decode_rot_matches_fp32(cuda, rows, hq, hkv, T, max_len):
    from omlx_exl3_b200 import kernels
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 1000 + hq * 10 + T)
    q = torch.randn((rows, hq, 128), device=cuda, generator=g).half()
    kc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    vc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    kc[:, T:] = float("nan")                                            # never read
    vc[:, T:] = float("nan")
    suh = (torch.randint(0, 2, (hq * 128,), device=cuda, generator=g) * 2 - 1).half()
    xh = kernels.attn_rot(q, kc, vc, T, suh)
    torch.cuda.synchronize()
    assert tuple(xh.shape) == (1, rows, hq * 128)
    got = xh.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref = _reference(q, kc, vc, T, suh)
    err = float(np.abs(got - ref).max()) / float(np.abs(ref).max())
    assert err < 4e-3, err


def test_attn_decode_rot_matches_sdpa_and_is_deterministic(cuda):
    """Against the framework path it replaces (SDPA then rot) and bitwise stable across calls."""
    import torch.nn.functional as F
    from omlx_exl3_b200 import kernels
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    rows, hq, hkv, T, max_len = 1, 40, 8, 2049, 2100
    q = torch.randn((rows, hq, 128), device=cuda, generator=g).half()
    kc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    vc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    suh = (torch.randint(0, 2, (hq * 128,), device=cuda, generator=g) * 2 - 1).half()
    a = kernels.attn_rot(q, kc, vc, T, suh)
    b = kernels.attn_rot(q, kc, vc, T, suh)
    o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], kc[None, :, :T], vc[None, :, :T], enable_gqa=True)
    ref = kernels.rot(o[0].transpose(0, 1).reshape(rows, hq * 128), suh)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    err = float((a.float() - ref.float()).abs().max()) / float(ref.float().abs().max())
    assert err < 4e-3, err


def test_attn_rejects_wide_groups(cuda):
    """Up to 64 q vectors per kv head (4 groups of 16): every MTP-verify width at GQA 5 fits; wider
    groups are rejected with an error, not computed wrongly."""
    from omlx_exl3_b200 import kernels
    assert kernels.attn_fits(8, 40, 8) and kernels.attn_fits(4, 40, 8) and not kernels.attn_fits(8, 72, 8)
    q = torch.zeros((8, 72, 128), device=cuda).half()
    kc = torch.zeros((8, 64, 128), device=cuda).half()
    with pytest.raises(Exception):
        kernels.attn_rot(q, kc, kc.clone(), 32, torch.ones(72 * 128, device=cuda).half())


def test_attn_verify_rows_are_row_exact(cuda):
    """Row r of a multi-row (verify) call equals a single-row call at the same position over the same
    cache, bit for bit: every q vector is reduced over the same positions in the same order whatever
    the number of rows, so MTP verification reproduces plain decoding."""
    from omlx_exl3_b200 import kernels
    g = torch.Generator(device=cuda)
    g.manual_seed(21)
    rows, hq, hkv, T, max_len = 4, 40, 8, 4100, 4200
    q = torch.randn((rows, hq, 128), device=cuda, generator=g).half()
    kc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    vc = torch.randn((hkv, max_len, 128), device=cuda, generator=g).half()
    suh = (torch.randint(0, 2, (hq * 128,), device=cuda, generator=g) * 2 - 1).half()
    multi = kernels.attn_rot(q, kc, vc, T, suh)
    for r in range(rows):
        one = kernels.attn_rot(q[r:r + 1].contiguous(), kc, vc, T - rows + 1 + r, suh)
        torch.cuda.synchronize()
        assert torch.equal(one[0, 0], multi[0, r]), r
