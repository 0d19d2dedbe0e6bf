"""GPU: the fused prefill GEMM (exl3_gemm: trellis decoded in shared memory, tcgen05 MMAs into tensor
memory, FWHT + svh epilogue) against the fp32 oracle. BASELINE's GEMV/GEMM bar is max-rel <= 1e-2; the
reference's own kernel test uses 2e-3 for fp16 outputs (src/tools/exl3_kernel_test.py:50), which the
fp32-output comparisons here also meet."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(t, dev):
    return torch.from_numpy(O.trellis_u32(t).view(np.int32).copy()).to(dev)


def _case(dev, M, k, n, K, cb, out=torch.float32, seed=0):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(seed)
    t = O.random_trellis(k, n, K, seed + 1)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    y = kernels.gemm(torch.from_numpy(xh).to(dev), _t(t, dev), k, n, K, cb, torch.from_numpy(svh).to(dev), out)
    torch.cuda.synchronize()
    ref = O.gemv([t], k, [n], K, cb, xh[None], svh)
    assert kernels.gemm_status(dev) == 0
    return y.float().cpu().numpy(), ref


@pytest.mark.parametrize("M", [1, 7, 100, 256, 257, 600, 1100])
def test_gemm_rows(cuda, M):
    y, ref = _case(cuda, M, 512, 256, 6, 0, seed=M)
    assert O.max_rel(y, ref) < 2e-3, M


@pytest.mark.parametrize("M", [600, 1100])
def test_gemm_tall_tiles(cuda, M):
    """Wide enough (148 column blocks) that M > 256 runs 512-row tiles: four accumulators, two TMA
    boxes per stage, a two-pass epilogue, and a partial last row tile."""
    y, ref = _case(cuda, M, 256, 148 * 128, 5, 0, seed=M + 3)
    assert O.max_rel(y, ref) < 2e-3, M


@pytest.mark.parametrize("K", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("cb", [0, 1, 2])
def test_gemm_bits_codebooks(cuda, K, cb):
    y, ref = _case(cuda, 64, 256, 384, K, cb, seed=10 * K + cb)
    assert O.max_rel(y, ref) < 2e-3, (K, cb)


@pytest.mark.parametrize("out", [torch.float16, torch.bfloat16])
def test_gemm_out_dtypes(cuda, out):
    y, ref = _case(cuda, 300, 1024, 512, 5, 0, out=out, seed=4)
    assert O.max_rel(y, ref) < (2e-3 if out == torch.float16 else 1e-2)


def test_gemm_config3_shape_slice(cuda):
    """BASELINE config 3 (6 bpw): 5120 -> 17408 at M = 512, checked on 512 of the columns in C."""
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(5)
    M, k, n, K = 512, 5120, 17408, 6
    t = O.random_trellis(k, n, K, 7)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    y = kernels.gemm(torch.from_numpy(xh).to(cuda), _t(t, cuda), k, n, K, 0, torch.from_numpy(svh).to(cuda))
    torch.cuda.synchronize()
    nc = 512
    ref = O.gemv_c(t[:, : nc // 16].copy(), k, nc, K, 0, xh[:64], svh[:nc])
    assert O.max_rel(y[:64, :nc].cpu().numpy(), ref) < 2e-3
    # every row: linearity check against the row-sum (sum of rows of y == gemm of the summed xh rows)
    assert kernels.gemm_status(cuda) == 0


def test_gemm_rejects_bad_shapes(cuda):
    from omlx_exl3_b200 import kernels
    t = torch.zeros(96 * 128 * 4 // 32, dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError):
        kernels.gemm(torch.zeros((4, 96), dtype=torch.float16, device=cuda), t, 96, 128, 4, 0,
                     torch.ones(128, dtype=torch.float16, device=cuda))


def test_gemm_k_split_deterministic(cuda):
    """4 tiles over 64 k-steps: the call splits k over 4 CTAs per tile and the last arriving part sums the
    parts in part order. Matches the oracle, the unsplit call within fp32 rounding, and itself bit for
    bit; the arrival counters are left at zero (the second call gives the same bits)."""
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(60)
    M, k, n, K = 300, 4096, 512, 5
    t = O.random_trellis(k, n, K, 61)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    x, tr, s = torch.from_numpy(xh).to(cuda), _t(t, cuda), torch.from_numpy(svh).to(cuda)
    a = kernels.gemm(x, tr, k, n, K, 0, s)
    b = kernels.gemm(x, tr, k, n, K, 0, s)
    c = kernels.gemm(x, tr, k, n, K, 0, s, split=False)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert torch.equal(a, b)
    assert not torch.equal(a, c)
    assert O.max_rel(a.cpu().numpy(), c.cpu().numpy()) < 1e-5
    assert O.max_rel(a.cpu().numpy(), O.gemv([t], k, [n], K, 0, xh[None], svh)) < 2e-3


def test_gemm_config3_narrow_split(cuda):
    """BASELINE config 3's narrow case (17408 -> 5120, M = 512, 6 bpw): 40 column blocks, so k is split
    over 3 CTAs per tile. Checked on 256 columns in C, and every column against the unsplit kernel."""
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(62)
    M, k, n, K = 512, 17408, 5120, 6
    t = O.random_trellis(k, n, K, 63)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    x, tr, s = torch.from_numpy(xh).to(cuda), _t(t, cuda), torch.from_numpy(svh).to(cuda)
    a = kernels.gemm(x, tr, k, n, K, 0, s)
    c = kernels.gemm(x, tr, k, n, K, 0, s, split=False)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert O.max_rel(a.cpu().numpy(), c.cpu().numpy()) < 1e-4
    nc = 256
    ref = O.gemv_c(t[:, : nc // 16].copy(), k, nc, K, 0, xh[:32], svh[:nc])
    assert O.max_rel(a[:32, :nc].cpu().numpy(), ref) < 2e-3


@pytest.mark.parametrize("M", [100, 300, 600])
def test_gemm_pair_matches_one_cta_kernel(cuda, M, monkeypatch):
    """With EXL3_GEMM_PAIR=1, outputs whose width is a multiple of 256 run on SM pairs
    (exl3_gemm_pair.cu); by default the one-CTA kernel runs. Both decode every weight exactly and
    accumulate in fp32 in k order."""
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(70 + M)
    k, n, K = 1024, 512, 5
    t = O.random_trellis(k, n, K, 71)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    x, tr, s = torch.from_numpy(xh).to(cuda), _t(t, cuda), torch.from_numpy(svh).to(cuda)
    monkeypatch.setenv("EXL3_GEMM_PAIR", "1")
    a = kernels.gemm(x, tr, k, n, K, 0, s, split=False)
    monkeypatch.setenv("EXL3_GEMM_PAIR", "0")
    b = kernels.gemm(x, tr, k, n, K, 0, s, split=False)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert O.max_rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-5
    assert O.max_rel(a.cpu().numpy(), O.gemv([t], k, [n], K, 0, xh[None], svh)) < 2e-3


def test_gemm_pair_k_split(cuda, monkeypatch):
    """The pair kernel's k split (few pair tiles over a long k) against the oracle and itself."""
    from omlx_exl3_b200 import kernels
    monkeypatch.setenv("EXL3_GEMM_PAIR", "1")
    rng = np.random.default_rng(80)
    M, k, n, K = 300, 4096, 512, 4
    t = O.random_trellis(k, n, K, 81)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    x, tr, s = torch.from_numpy(xh).to(cuda), _t(t, cuda), torch.from_numpy(svh).to(cuda)
    a = kernels.gemm(x, tr, k, n, K, 0, s)
    b = kernels.gemm(x, tr, k, n, K, 0, s)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert torch.equal(a, b)
    assert O.max_rel(a.cpu().numpy(), O.gemv([t], k, [n], K, 0, xh[None], svh)) < 2e-3
