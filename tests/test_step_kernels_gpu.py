"""GPU: the decode-step glue kernels (qkv_post, add_norm_rot) against plain fp32 PyTorch / the oracle.

qkv_post: per-head q/k RMSNorm with MLX rounding, rotate-half RoPE, cache writes at each row's position.
add_norm_rot: residual add (rounded to the model dtype) + norm_rot (oracle.norm_rot restates the
reference's kernels.py:408-425, :461-473). Tolerances: the residual sum is bit-exact; norm outputs may
differ from the fp32 reference by one unit of the storage dtype in a small fraction of elements (the
sum of squares is reduced in another order), rotations within rel 1e-3 as the reference's own test."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rms_mlx(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * (xf * inv).to(x.dtype).float()).to(x.dtype)


def _rope(x: torch.Tensor, c: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    x1, x2 = xf[..., :64], xf[..., 64:]
    c, s = c[:, None, :], s[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def _close_frac(a: torch.Tensor, b: torch.Tensor, rtol: float, atol: float) -> float:
    a, b = a.float(), b.float()
    return float((~torch.isclose(a, b, rtol=rtol, atol=atol)).float().mean())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hq,hkv", [(1, 40, 8), (3, 8, 2), (8, 20, 4)])
@pytest.mark.parametrize("fused_layout", [True, False])
def test_qkv_post(cuda, dtype, rows, hq, hkv, fused_layout):
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.model import ModelConfig, rope_tables
    g = torch.Generator().manual_seed(rows * 100 + hq)
    nq, nk = hq * 128, hkv * 128
    if fused_layout:     # q/k/v are column views of one (rows, nq + 2 nk) projection output
        y = (torch.randn((rows, nq + 2 * nk), generator=g) * 2).to(dtype).to(cuda)
        q, k, v = y[:, :nq], y[:, nq:nq + nk], y[:, nq + nk:]
    else:
        q = (torch.randn((rows, nq), generator=g) * 2).to(dtype).to(cuda)
        k = (torch.randn((rows, nk), generator=g) * 2).to(dtype).to(cuda)
        v = (torch.randn((rows, nk), generator=g) * 2).to(dtype).to(cuda)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype).to(cuda)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype).to(cuda)
    cfg = ModelConfig(max_position_embeddings=600)
    cos, sin = rope_tables(cfg, cuda)
    max_len = 600
    pos = torch.tensor([5, 599, 300, 17, 0, 250, 251, 252][:rows], dtype=torch.int64, device=cuda)
    kc = torch.zeros((hkv, max_len, 128), dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    q16 = kernels.qkv_post(q, k, v, qw, kw, 1e-6, cos, sin, pos, kc, vc)

    c, s = cos.index_select(0, pos), sin.index_select(0, pos)
    rq = _rope(_rms_mlx(q.reshape(rows, hq, 128), qw, 1e-6), c, s).to(torch.float16)
    rk = _rope(_rms_mlx(k.reshape(rows, hkv, 128), kw, 1e-6), c, s).to(torch.float16)
    rv = v.reshape(rows, hkv, 128).to(torch.float16)
    assert q16.shape == (rows, hq, 128) and q16.dtype == torch.float16
    ulp = 1.6e-2 if dtype == torch.bfloat16 else 2e-3
    assert _close_frac(q16, rq, ulp, 1e-2) < 5e-3
    assert torch.allclose(q16.float(), rq.float(), rtol=ulp, atol=3e-2)
    got_k = kc[:, pos].transpose(0, 1)
    got_v = vc[:, pos].transpose(0, 1)
    assert _close_frac(got_k, rk, ulp, 1e-2) < 5e-3
    assert torch.equal(got_v, rv)
    # nothing else in the cache was written
    mask = torch.ones(max_len, dtype=torch.bool, device=cuda)
    mask[pos] = False
    assert not kc[:, mask].any() and not vc[:, mask].any()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("k,nm", [(5120, 1), (5120, 2), (5120, 3), (2560, 1)])
def test_add_norm_rot(cuda, dtype, rows, k, nm):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(rows * 7 + nm + k)
    x = torch.from_numpy((rng.standard_normal((rows, k)) * 3).astype(np.float32)).to(dtype)
    d = torch.from_numpy((rng.standard_normal((rows, k)) * 2).astype(np.float32)).to(dtype)
    w = torch.from_numpy((1 + 0.1 * rng.standard_normal(k)).astype(np.float32)).to(dtype)
    suh = torch.from_numpy((rng.standard_normal((nm, k)) * 0.5).astype(np.float16))
    h, xn, xh = kernels.add_norm_rot(x.to(cuda), d.to(cuda), w.to(cuda), 1e-6, suh.to(cuda))

    h_ref = (x.float() + d.float()).to(dtype)
    assert torch.equal(h.cpu(), h_ref)
    xn_ref = _rms_mlx(h_ref, w, 1e-6)
    assert _close_frac(xn.cpu(), xn_ref, 1e-2 if dtype == torch.bfloat16 else 1e-3, 1e-3) < 1e-3
    ref = O.rot(xn.float().cpu().numpy(), suh.numpy())
    assert O.max_rel(xh.float().cpu().numpy(), ref) < 1e-3
    # and the same values norm_rot gives on the summed residual
    xn2, xh2 = kernels.norm_rot(h, w.to(cuda), 1e-6, suh.to(cuda)) if k % 1024 == 0 else (xn, xh)
    assert _close_frac(xn, xn2, 1e-2, 1e-3) < 1e-3


def test_add_norm_rot_rejects_alias(cuda):
    from omlx_exl3_b200 import _lib
    x = torch.zeros((1, 1024), dtype=torch.bfloat16, device=cuda)
    d = torch.zeros_like(x)
    w = torch.ones(1024, dtype=torch.bfloat16, device=cuda)
    suh = torch.ones((1, 1024), dtype=torch.float16, device=cuda)
    xn = torch.empty_like(x)
    xh = torch.empty((1, 1, 1024), dtype=torch.float16, device=cuda)
    rc = _lib.lib().exl3_add_norm_rot(x.data_ptr(), d.data_ptr(), w.data_ptr(), 1, 1, 1024, 1e-6, suh.data_ptr(), 1,
                                      x.data_ptr(), xn.data_ptr(), xh.data_ptr(), None)
    assert rc == -1     # EXL3_E_SHAPE


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hq,hkv,K", [(1, 40, 8, 6), (3, 8, 2, 5), (8, 20, 4, 4), (1, 40, 8, [6, 5, 8]),
                                           (2, 5, 1, [7, 6, 5])])
def test_gemv_qkv_post_epilogue_matches_two_kernels(cuda, dtype, rows, hq, hkv, K):
    """exl3_gemv_qkv_post == exl3_gemv (y in dtype) followed by exl3_qkv_post, bit for bit; also with
    q/k/v at different bitrates (one mixed-bitrate launch)."""
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.model import ModelConfig, rope_tables
    k = 1024
    ns = [hq * 128, hkv * 128, hkv * 128]
    Ks = K if isinstance(K, list) else [K] * 3
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 7 + hq + sum(Ks))
    trs = [torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * Km // 32,), dtype=torch.int32, device=cuda, generator=g)
           for n, Km in zip(ns, Ks)]
    svh = ((torch.randint(0, 2, (sum(ns),), device=cuda, generator=g) * 2 - 1) * 0.03).half()
    xh = torch.randn((3, rows, k), device=cuda, generator=g).half()
    qw = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).to(dtype)
    cos, sin = rope_tables(ModelConfig(max_position_embeddings=700), cuda)
    pos = torch.tensor([3, 650, 17, 0, 100, 101, 102, 400][:rows], dtype=torch.int64, device=cuda)
    plan = kernels.TrellisGemvPlan(k, ns, K, 0, svh, rows, dtype)
    kc1 = torch.zeros((hkv, 700, 128), dtype=torch.float16, device=cuda)
    vc1, kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(kc1), torch.zeros_like(kc1)
    y = plan(xh, trs)
    q1 = kernels.qkv_post(y[:, :ns[0]], y[:, ns[0]:ns[0] + ns[1]], y[:, ns[0] + ns[1]:], qw, kw, 1e-6, cos, sin, pos,
                          kc1, vc1)
    q2 = plan.qkv_post(xh, trs, qw, kw, 1e-6, cos, sin, pos, kc2, vc2)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    assert int(plan.counters.abs().sum().item()) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,ld,n", [(1, 151936, 151936), (3, 19008, 18992), (8, 1000, 999), (2, 37, 5)])
def test_argmax_matches_torch(cuda, dtype, rows, ld, n):
    """exl3_argmax against torch on the first n columns: same maximum and, with ties planted, the first
    column; index_base is added to the index."""
    from omlx_exl3_b200 import kernels
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 31 + n)
    x = (4 * torch.randn((rows, ld), device=cuda, generator=g)).to(dtype)
    x[:, n:] = 1000.0                                               # never read
    if n > 10:
        x[0, 3] = x[0, n - 2] = 900.0                               # a tie: the first wins
    val, idx = kernels.argmax(x, n, index_base=7)
    ref_v, ref_i = x[:, :n].float().max(dim=-1)
    torch.cuda.synchronize()
    assert torch.equal(val, ref_v)
    first = torch.stack([(x[r, :n].float() == ref_v[r]).nonzero()[0, 0] for r in range(rows)])
    assert torch.equal(idx, first + 7)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_argmax_nan_order_matches_torch(cuda, dtype):
    """NaN logits: exl3_argmax picks what torch.argmax picks (NaN above every number, the first NaN
    of a row wins), including a row that is all NaN and one whose NaN lies in another CTA's eighth."""
    from omlx_exl3_b200 import kernels
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    rows, n = 4, 151936
    x = torch.randn((rows, n), device=cuda, generator=g).to(dtype)
    x[0, 5000] = float("nan")
    x[1, 140000] = float("nan")
    x[1, 90000] = float("nan")                 # the first of two NaNs, in an earlier CTA's share
    x[2, :] = float("nan")
    x[3, 77] = float("inf")                    # no NaN: plain maximum
    _, idx = kernels.argmax(x)
    torch.cuda.synchronize()
    assert torch.equal(idx, x.argmax(dim=-1))
    assert idx.tolist() == [5000, 90000, 0, 77]
