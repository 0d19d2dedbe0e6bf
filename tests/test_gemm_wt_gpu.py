"""GPU: the prefill GEMM on decoded weights (exl3_gemm_wt: tcgen05 pair tiles over two SMs, TMA for both
operands, FWHT + svh epilogue, persistent with two tensor-memory accumulators) against the fp32 oracle.
The weights come from exl3_decode_wt, which is bit-exact to the oracle's decode (test_decode_gpu.py).
Tolerance: the reference's kernel test bar of 2e-3 for fp16 outputs (src/tools/exl3_kernel_test.py:50),
which the fp32 outputs here meet too; 1e-2 for bf16."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(t, dev):
    return torch.from_numpy(O.trellis_u32(t).view(np.int32).copy()).to(dev)


def _inputs(dev, M, k, n, K, cb, seed):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(seed)
    t = O.random_trellis(k, n, K, seed + 1)
    wt = kernels.decode_wt(_t(t, dev), k, n, K, cb)
    xh = rng.standard_normal((M, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    return t, wt, xh, svh


def _case(dev, M, k, n, K=6, cb=0, out=torch.float32, seed=0):
    from omlx_exl3_b200 import kernels
    t, wt, xh, svh = _inputs(dev, M, k, n, K, cb, seed)
    y = kernels.gemm_wt(torch.from_numpy(xh).to(dev), wt, torch.from_numpy(svh).to(dev), out)
    torch.cuda.synchronize()
    assert kernels.gemm_status(dev) == 0
    return y.float().cpu().numpy(), O.gemv([t], k, [n], K, cb, xh[None], svh)


@pytest.mark.parametrize("M", [1, 5, 128, 255, 256, 257, 600])
def test_gemm_wt_rows(cuda, M):
    """Row tails inside a pair tile: the second CTA's rows past M read TMA zero fill and are not stored."""
    y, ref = _case(cuda, M, 512, 512, seed=M)
    assert O.max_rel(y, ref) < 2e-3, M


def test_gemm_wt_half_tile_columns(cuda):
    """n % 256 == 128: the last tile's second column block is outside the matrix."""
    y, ref = _case(cuda, 300, 256, 384, seed=11)
    assert O.max_rel(y, ref) < 2e-3


def test_gemm_wt_long_k(cuda):
    """80 k-steps: the 6-stage ring wraps many times within one tile."""
    y, ref = _case(cuda, 256, 5120, 256, K=5, seed=12)
    assert O.max_rel(y, ref) < 2e-3


def test_gemm_wt_many_tiles(cuda):
    """370 tiles over at most 74 SM pairs: every pair runs several tiles, alternating accumulators, so
    epilogues overlap the next tile's MMAs and each accumulator is reused after its read-out."""
    y, ref = _case(cuda, 1100, 256, 148 * 128, K=4, seed=13)
    assert O.max_rel(y, ref) < 2e-3


@pytest.mark.parametrize("out", [torch.float16, torch.bfloat16])
def test_gemm_wt_out_dtypes(cuda, out):
    y, ref = _case(cuda, 300, 1024, 512, K=5, out=out, seed=4)
    assert O.max_rel(y, ref) < (2e-3 if out == torch.float16 else 1e-2)


@pytest.mark.parametrize("cb", [1, 2])
def test_gemm_wt_codebooks(cuda, cb):
    y, ref = _case(cuda, 200, 256, 256, K=3, cb=cb, seed=20 + cb)
    assert O.max_rel(y, ref) < 2e-3


def test_gemm_wt_column_chunk_in_place(cuda):
    """A column chunk written into a wider output (row stride > n) leaves the other columns untouched."""
    from omlx_exl3_b200 import kernels
    M, k, n, c0, width = 300, 512, 256, 384, 1024
    t, wt, xh, svh = _inputs(cuda, M, k, n, 6, 0, 5)
    y = torch.full((M, width), float("nan"), dtype=torch.float16, device=cuda)
    kernels.gemm_wt(torch.from_numpy(xh).to(cuda), wt, torch.from_numpy(svh).to(cuda), out=y[:, c0:c0 + n])
    torch.cuda.synchronize()
    ref = O.gemv([t], k, [n], 6, 0, xh[None], svh)
    assert O.max_rel(y[:, c0:c0 + n].float().cpu().numpy(), ref) < 2e-3
    assert torch.isnan(y[:, :c0]).all() and torch.isnan(y[:, c0 + n:]).all()


def test_gemm_wt_matches_fused_kernel(cuda):
    """Decode-once + exl3_gemm_wt and the fused exl3_gemm compute the same product (both fp32 accumulate)."""
    from omlx_exl3_b200 import kernels
    M, k, n, K = 512, 1024, 1024, 6
    t, wt, xh, svh = _inputs(cuda, M, k, n, K, 0, 6)
    x, s = torch.from_numpy(xh).to(cuda), torch.from_numpy(svh).to(cuda)
    a = kernels.gemm_wt(x, wt, s)
    b = kernels.gemm(x, _t(t, cuda), k, n, K, 0, s)
    torch.cuda.synchronize()
    assert O.max_rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-5


def test_gemm_wt_rejects_bad_input(cuda):
    from omlx_exl3_b200 import kernels
    x = torch.zeros((4, 96), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        kernels.gemm_wt(x, torch.zeros((128, 96), dtype=torch.float16, device=cuda),
                        torch.ones(128, dtype=torch.float16, device=cuda))       # k % 64 != 0
    x = torch.zeros((4, 128), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        kernels.gemm_wt(x, torch.zeros((200, 128), dtype=torch.float16, device=cuda),
                        torch.ones(200, dtype=torch.float16, device=cuda))       # n % 128 != 0
    with pytest.raises(TypeError):
        kernels.gemm_wt(x.float(), torch.zeros((128, 128), dtype=torch.float16, device=cuda),
                        torch.ones(128, dtype=torch.float16, device=cuda))


@pytest.mark.parametrize("fused", [True, False])
def test_linear_prefill_paths_match_oracle(cuda, fused):
    """Both prefill paths of EXL3Linear (fused decode-in-GEMM, decode-once + exl3_gemm_wt) on the same
    input: rotation of x, product, output rotation and svh, against the fp32 oracle of the whole linear."""
    from omlx_exl3_b200.prefill import linear_prefill
    rng = np.random.default_rng(31)
    k, n, K, rows = 1024, 768, 5, 600
    t = O.random_trellis(k, n, K, 32)
    suh = np.where(rng.random(k) < 0.5, -1, 1).astype(np.float16)
    svh = (rng.standard_normal(n) * 0.02).astype(np.float16)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    y = linear_prefill(torch.from_numpy(x).to(cuda), _t(t, cuda), k, n, K, 0, torch.from_numpy(suh).to(cuda),
                       torch.from_numpy(svh).to(cuda), torch.float32, fused=fused)
    ref = O.linear_forward(t, k, n, K, 0, x, suh, svh, None)
    assert O.max_rel(y.cpu().numpy(), ref) < 2e-3


def test_linear_prefill_default_is_decode_once_for_tall_inputs():
    """Fused up to 512 rows, decode-once above (the measured crossover at the 27B-class shapes)."""
    from omlx_exl3_b200.prefill import use_fused
    assert use_fused(256, 5120) and use_fused(512, 17408) and use_fused(512, 5120)
    assert not use_fused(513, 5120) and not use_fused(4096, 17408)


def test_gemm_wt_k_split_deterministic(cuda):
    """Few output tiles (4) over a long k (256 k-steps): the call splits k into parts whose partials the
    last arriving unit sums in part order. Same result as the unsplit call within fp32 rounding,
    bit-identical from call to call, and the arrival counters are left at zero (a second call still
    gives the same bits)."""
    from omlx_exl3_b200 import kernels
    M, k, n, K = 300, 16384, 512, 4
    t, wt, xh, svh = _inputs(cuda, M, k, n, K, 0, 40)
    x, s = torch.from_numpy(xh).to(cuda), torch.from_numpy(svh).to(cuda)
    a = kernels.gemm_wt(x, wt, s)
    b = kernels.gemm_wt(x, wt, s)
    c = kernels.gemm_wt(x, wt, s, split=False)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert torch.equal(a, b)
    ref = O.gemv([t], k, [n], K, 0, xh[None], svh)
    assert O.max_rel(a.cpu().numpy(), ref) < 2e-3
    assert O.max_rel(a.cpu().numpy(), c.cpu().numpy()) < 1e-4     # fp32 sums of 16384 terms, two orders
    assert not torch.equal(a, c)          # the split really ran (a different summation order)


def _torch_ref(xh, wt, svh):
    """fp32 reference of had128(xh @ wt^T) / sqrt(128) * svh on the GPU (no TF32)."""
    import math
    h = torch.ones((1, 1), dtype=torch.float32, device=xh.device)
    while h.shape[0] < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y = xh.float() @ wt.float().t()
        y = (y.reshape(y.shape[0], -1, 128) @ h).reshape(y.shape) / math.sqrt(128)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return y * svh.float()


def test_gemm_wt_tail_split(cuda):
    """80 tiles on 74 SM pairs: the first 74 tiles run whole, the last 6 run as k parts spread over the
    pairs (a whole round and a split tail in one launch). Against an fp32 torch reference built from the
    same decoded weights."""
    from omlx_exl3_b200 import kernels
    M, k, n, K = 256, 8192, 80 * 256, 2
    g = torch.Generator(device=cuda)
    g.manual_seed(50)
    tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * K // 32,), dtype=torch.int32, device=cuda, generator=g)
    wt = kernels.decode_wt(tr, k, n, K, 0)
    xh = torch.randn((M, k), device=cuda, generator=g).half()
    svh = torch.randint(0, 2, (n,), device=cuda, generator=g).half() * 2 - 1
    a = kernels.gemm_wt(xh, wt, svh)
    b = kernels.gemm_wt(xh, wt, svh)
    c = kernels.gemm_wt(xh, wt, svh, split=False)
    ref = _torch_ref(xh, wt, svh)
    torch.cuda.synchronize()
    assert kernels.gemm_status(cuda) == 0
    assert torch.equal(a, b)
    assert O.max_rel(a.cpu().numpy(), ref.cpu().numpy()) < 2e-3
    assert O.max_rel(c.cpu().numpy(), ref.cpu().numpy()) < 2e-3
    if torch.cuda.get_device_properties(cuda).multi_processor_count == 148:
        assert not torch.equal(a[:, -256:], c[:, -256:])      # the tail tiles really ran split
        assert torch.equal(a[:, :256], c[:, :256])            # a whole tile: same bits as unsplit
