"""GPU: the decode GEMV (TrellisGemvPlan -> exl3_gemv) against the fp32 oracle.

The reference's own kernel test (src/tools/exl3_kernel_test.py:34-50) checks
max|y - ref| / max|ref| < 2e-3 (fp16 out) / 1e-2 (bf16 out) against had128(xh @ W) * svh built from
the same trellises; the same cases and tolerances are used here, plus every codebook, the bench
shapes, determinism, row-exactness and the scratch protocol."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _t(t: np.ndarray, dev):
    return torch.from_numpy(O.trellis_u32(t).view(np.int32).copy()).to(dev)


def _run(dev, k, ns, K, cb, rows, out_dtype, seed=0, bit31=False, svh_scale=0.01):
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(seed)
    trs = [O.random_trellis(k, n, K, seed * 10 + i, bit31=bit31) for i, n in enumerate(ns)]
    svh = (rng.standard_normal(sum(ns)) * svh_scale).astype(np.float16)
    xh = rng.standard_normal((len(ns), rows, k)).astype(np.float16)
    plan = TrellisGemvPlan(k, ns, K, cb, torch.from_numpy(svh).to(dev), rows, out_dtype)
    y = plan(torch.from_numpy(xh).to(dev), [_t(t, dev) for t in trs])
    torch.cuda.synchronize()
    ref = O.gemv(trs, k, ns, K, cb, xh, svh)
    return y, ref, plan


# the reference test's cases: k = 1024, mul1, 31-bit words
REF_CASES = [(6, [256]), (6, [256, 384]), (6, [128, 256, 128]), (5, [256, 128]), (7, [384]), (8, [128, 128]),
             (4, [256]), (3, [128])]


@pytest.mark.parametrize("bits,ns", REF_CASES)
def test_gemv_reference_cases(cuda, bits, ns):
    for rows in (1, 3, 8):
        for dt in (torch.float16, torch.bfloat16):
            y, ref, plan = _run(cuda, 1024, ns, bits, 2, rows, dt, seed=bits + rows, bit31=False)
            assert y.dtype == dt and tuple(y.shape) == (rows, sum(ns))
            e = O.max_rel(y.float().cpu().numpy(), ref)
            assert e < TOL[dt], (bits, ns, rows, dt, e)
            assert int(plan.counters.abs().sum().item()) == 0


@pytest.mark.parametrize("cb", [0, 1, 2])
@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 6, 7, 8])
def test_gemv_all_bits_codebooks(cuda, bits, cb):
    y, ref, _ = _run(cuda, 2048, [384], bits, cb, 2, torch.float16, seed=100 + bits * 3 + cb)
    assert O.max_rel(y.float().cpu().numpy(), ref) < TOL[torch.float16]


def test_gemv_config1_shape(cuda):
    """4096 -> 4096 at 4 bpw, batch 1, 3inst, +-1 svh."""
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(7)
    k = n = 4096
    t = O.random_trellis(k, n, 4, 1)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    xh = rng.standard_normal((1, 1, k)).astype(np.float16)
    plan = TrellisGemvPlan(k, [n], 4, 0, torch.from_numpy(svh).to(cuda), 1, torch.float16)
    y = plan(torch.from_numpy(xh).to(cuda), [_t(t, cuda)]).float().cpu().numpy()
    ref = O.gemv_c(t, k, n, 4, 0, xh[0], svh)
    assert O.max_rel(y, ref) < TOL[torch.float16]


@pytest.mark.parametrize("k,n", [(5120, 17408), (17408, 5120), (5120, 6144), (5120, 5120)])
def test_gemv_bench_shapes(cuda, k, n):
    """BASELINE config 2 shapes at 6 bpw, rows 1 and 8 (oracle in C on a 1024-column slice)."""
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(k + n)
    K = 6
    t = O.random_trellis(k, n, K, 3)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    tt = _t(t, cuda)
    for rows in (1, 8):
        xh = rng.standard_normal((1, rows, k)).astype(np.float16)
        plan = TrellisGemvPlan(k, [n], K, 0, torch.from_numpy(svh).to(cuda), rows, torch.float16)
        y = plan(torch.from_numpy(xh).to(cuda), [tt]).float().cpu().numpy()
        nc = 1024
        tsub = t[:, : nc // 16, :].copy()
        ref = O.gemv_c(tsub, k, nc, K, 0, xh[0], svh[:nc])
        assert O.max_rel(y[:, :nc], ref) < TOL[torch.float16], (k, n, rows)
        assert int(plan.counters.abs().sum().item()) == 0


def test_gemv_deterministic_and_row_exact(cuda):
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(5)
    k, n, K = 5120, 1024, 4
    t = _t(O.random_trellis(k, n, K, 9), cuda)
    svh = torch.from_numpy(np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)).to(cuda)
    xh8 = torch.from_numpy(rng.standard_normal((1, 8, k)).astype(np.float16)).to(cuda)
    p8 = TrellisGemvPlan(k, [n], K, 0, svh, 8, torch.float16)
    a = p8(xh8, [t]).clone()
    b = p8(xh8, [t]).clone()
    assert torch.equal(a, b)
    for r in (2, 3, 5):
        pr = TrellisGemvPlan(k, [n], K, 0, svh, r, torch.float16)
        yr = pr(xh8[:, :r].contiguous(), [t])
        assert torch.equal(yr, a[:r]), r
    # one row takes the same fp32-accumulating path: bitwise row 0 of the 8-row call
    p1 = TrellisGemvPlan(k, [n], K, 0, svh, 1, torch.float16)
    assert torch.equal(p1(xh8[:, :1].contiguous(), [t]), a[:1])


# Worst case for the accumulation: the longest reduction of the 27B-class shapes (down_proj, k = 17408)
# at batch 1, every bitrate of the sweep. The reference multiplies each fp16 weight by x with fp32 FMAs
# into fp32 accumulators (src/omlx/exl3/kernels.py:215-218); here each product is exact and summed in
# fp32 on the tensor cores, so the error against the fp32 oracle stays at the fp16 output rounding.
WORST_TOL = 2e-3


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_gemv_worst_case_accumulation(cuda, bits):
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(900 + bits)
    k, n, nc = 17408, 5120, 512
    t = O.random_trellis(k, n, bits, 40 + bits)
    svh = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float16)
    xh = rng.standard_normal((1, 1, k)).astype(np.float16)
    plan = TrellisGemvPlan(k, [n], bits, 0, torch.from_numpy(svh).to(cuda), 1, torch.float16)
    y = plan(torch.from_numpy(xh).to(cuda), [_t(t, cuda)]).float().cpu().numpy()
    ref = O.gemv_c(t[:, : nc // 16, :].copy(), k, nc, bits, 0, xh[0], svh[:nc])
    e = O.max_rel(y[:, :nc], ref)
    print(f"k=17408 n=5120 K={bits} rows=1 max-rel {e:.3e}")
    assert e < WORST_TOL, (bits, e)


def test_gemv_small_grids_and_many_segments(cuda):
    """Forced small grids make every CTA span several blocks and every block several CTAs."""
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(6)
    k, ns, K = 1024, [640, 256], 5
    trs = [O.random_trellis(k, n, K, 30 + i) for i, n in enumerate(ns)]
    svh = rng.standard_normal(sum(ns)).astype(np.float16)
    xh = rng.standard_normal((2, 4, k)).astype(np.float16)
    ref = O.gemv(trs, k, ns, K, 0, xh, svh)
    for grid in (1, 3, 7, 13, 64, 300):
        plan = TrellisGemvPlan(k, ns, K, 0, torch.from_numpy(svh).to(cuda), 4, torch.float16, grid=grid)
        y = plan(torch.from_numpy(xh).to(cuda), [_t(t, cuda) for t in trs]).float().cpu().numpy()
        assert O.max_rel(y, ref) < TOL[torch.float16], grid
        assert int(plan.counters.abs().sum().item()) == 0


def _ref_mixed(trs, k, ns, Ks, cb, xh, svh):
    outs, o = [], 0
    for m, (t, n, Km) in enumerate(zip(trs, ns, Ks)):
        outs.append(O.gemv([t], k, [n], Km, cb, xh[m:m + 1], svh[o:o + n]))
        o += n
    return np.concatenate(outs, axis=1)


@pytest.mark.parametrize("Ks,ns", [([5, 3, 8], [256, 128, 384]), ([6, 7], [640, 128]), ([8, 5, 5], [1280, 256, 256]),
                                   ([2, 6, 4], [128, 128, 128])])
@pytest.mark.parametrize("rows", [1, 2, 8])
def test_gemv_mixed_bitrates(cuda, Ks, ns, rows):
    """Members of different bitrates in one launch (each on its own CTA segment) against the oracle of
    each member, with forced grids too, and the scratch left at rest."""
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    rng = np.random.default_rng(sum(Ks) * 10 + rows)
    k, cb = 1024, 0
    trs = [O.random_trellis(k, n, Km, 70 + i) for i, (n, Km) in enumerate(zip(ns, Ks))]
    svh = (rng.standard_normal(sum(ns)) * 0.01).astype(np.float16)
    xh = rng.standard_normal((len(ns), rows, k)).astype(np.float16)
    ref = _ref_mixed(trs, k, ns, Ks, cb, xh, svh)
    for grid in (0, 5, 40):
        for dt in (torch.float16, torch.bfloat16):
            plan = TrellisGemvPlan(k, ns, Ks, cb, torch.from_numpy(svh).to(cuda), rows, dt, grid=grid)
            y = plan(torch.from_numpy(xh).to(cuda), [_t(t, cuda) for t in trs])
            torch.cuda.synchronize()
            assert tuple(y.shape) == (rows, sum(ns))
            assert O.max_rel(y.float().cpu().numpy(), ref) < TOL[dt], (grid, dt)
            assert int(plan.counters.abs().sum().item()) == 0
    # every member's result equals its own single-member launch within tolerance, deterministic
    plan = TrellisGemvPlan(k, ns, Ks, cb, torch.from_numpy(svh).to(cuda), rows, torch.float16)
    args = (torch.from_numpy(xh).to(cuda), [_t(t, cuda) for t in trs])
    assert torch.equal(plan(*args), plan(*args))


def test_gemv_rejects_bad_input(cuda):
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    svh = torch.ones(256, dtype=torch.float16, device=cuda)
    with pytest.raises(AssertionError):
        TrellisGemvPlan(1000, [256], 4, 0, svh, 1)
    with pytest.raises(AssertionError):
        TrellisGemvPlan(1024, [256], 4, 0, svh, 9)
    plan = TrellisGemvPlan(1024, [256], 4, 0, svh, 1)
    with pytest.raises(ValueError):
        plan(torch.zeros((1, 2, 1024), dtype=torch.float16, device=cuda),
             [torch.zeros(1024 * 256 * 4 // 32, dtype=torch.int32, device=cuda)])


# ---------------------------------------------------------------------------------------------- fused input
# The GEMV that computes its own rotated input (exl3_gemv_rot / exl3_gemv_swiglu): every CTA rotates
# the k blocks its units read with the arithmetic of exl3_rot / exl3_swiglu_rot, so the result must
# equal the two-launch path bit for bit. Forced small grids make CTAs span one, two (disjoint k
# ranges) and several blocks, which exercises every prologue range.

@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("ns,K", [([1024], 6), ([512, 256, 256], 4), ([384, 128], 5)])
def test_gemv_rot_equals_rot_then_gemv(cuda, xdtype, rows, ns, K):
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 7 + K)
    k = 2048
    trs = [_t(O.random_trellis(k, n, K, 50 + i), cuda) for i, n in enumerate(ns)]
    svh = (torch.randn(sum(ns), device=cuda, generator=g) * 0.02).half()
    suh = (torch.randint(0, 2, (len(ns), k), device=cuda, generator=g) * 2 - 1).half()
    x = torch.randn((rows, k), device=cuda, generator=g).to(xdtype)
    for grid in (0, 3, 7, 50):
        plan = TrellisGemvPlan(k, ns, K, 0, svh, rows, torch.float16, grid=grid)
        ref = plan(kernels.rot(x, suh), trs).clone()
        got = plan.rot_call(x, suh, trs)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), grid
        assert int(plan.counters.abs().sum().item()) == 0


@pytest.mark.parametrize("gdtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows", [1, 4, 8])
def test_gemv_swiglu_equals_swiglu_rot_then_gemv(cuda, gdtype, rows):
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    g = torch.Generator(device=cuda)
    g.manual_seed(rows)
    k, n, K = 4352, 1024, 6                   # down_proj-like: k = the MLP width
    tr = _t(O.random_trellis(k, n, K, 60), cuda)
    svh = (torch.randn(n, device=cuda, generator=g) * 0.02).half()
    suh = (torch.randint(0, 2, (k,), device=cuda, generator=g) * 2 - 1).half()
    gu = (2 * torch.randn((rows, 2 * k), device=cuda, generator=g)).to(gdtype)
    for grid in (0, 5, 33):
        plan = TrellisGemvPlan(k, [n], K, 0, svh, rows, torch.bfloat16, grid=grid)
        ref = plan(kernels.swiglu_rot(gu, suh), [tr]).clone()
        got = plan.swiglu_call(gu, suh, [tr])
        torch.cuda.synchronize()
        assert torch.equal(got, ref), grid


def test_gemv_prologue_rejects_bad_input(cuda):
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    svh = torch.ones(256, dtype=torch.float16, device=cuda)
    tr = torch.zeros(1040 * 256 * 4 // 32, dtype=torch.int32, device=cuda)
    plan = TrellisGemvPlan(1040, [256], 4, 0, svh, 1)            # k % 128 != 0: no in-kernel rotation
    with pytest.raises(ValueError):
        plan.rot_call(torch.zeros((1, 1040), dtype=torch.float16, device=cuda),
                      torch.ones((1, 1040), dtype=torch.float16, device=cuda), [tr])
