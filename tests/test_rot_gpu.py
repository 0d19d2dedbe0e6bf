"""GPU: rot / norm_rot / swiglu_rot / had_svh against the oracle.

The reference's test (src/tools/exl3_kernel_test.py:53-77) uses rows 1/3/8, k 5120 (1-3 members)
and 6144, bf16 x = 3 N(0,1), w = 1 + 0.1 N(0,1), suh = 0.5 N(0,1); rotations within rel 1e-3, the
norm output differing from rms_norm in < 0.1% of elements, swiglu_rot at n = 17408 within 1e-3."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _bf16(a):
    return torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("k,nm", [(5120, 1), (5120, 2), (5120, 3), (6144, 1)])
def test_rot_and_norm_rot(cuda, rows, k, nm):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(rows * 10 + nm + k)
    x = _bf16(rng.standard_normal((rows, k)) * 3)
    w = _bf16(1 + 0.1 * rng.standard_normal(k))
    suh = torch.from_numpy((rng.standard_normal((nm, k)) * 0.5).astype(np.float16))
    xf, wf = x.float().numpy(), w.float().numpy()

    xh = kernels.rot(x.to(cuda), suh.to(cuda)).cpu().numpy()
    ref = O.rot(xf, suh.numpy())
    assert xh.shape == (nm, rows, k)
    assert O.max_rel(xh, ref) < 1e-3
    # same fp32 inputs and the reference's stage order: bit-identical rotations
    assert np.array_equal(xh.view(np.uint16), ref.view(np.uint16))

    xn, xh2 = kernels.norm_rot(x.to(cuda), w.to(cuda), 1e-6, suh.to(cuda))
    xn_ref, xh2_ref = O.norm_rot(xf, wf, 1e-6, suh.numpy(), "bfloat16")
    differ = np.mean(xn.float().cpu().numpy() != xn_ref)
    assert differ < 1e-3
    assert O.max_rel(xh2.cpu().numpy(), xh2_ref) < 1e-3


@pytest.mark.parametrize("rows", [1, 3, 8])
def test_swiglu_rot(cuda, rows):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(rows)
    n = 17408
    gu = (rng.standard_normal((rows, 2 * n)) * 2).astype(np.float16)
    suh = (rng.standard_normal(n) * 0.5).astype(np.float16)
    xh = kernels.swiglu_rot(torch.from_numpy(gu).to(cuda), torch.from_numpy(suh).to(cuda)).cpu().numpy()
    ref = O.swiglu_rot(gu.astype(np.float32), suh)
    assert xh.shape == (1, rows, n)
    assert O.max_rel(xh, ref) < 1e-3


def test_norm_rot_fp16(cuda):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(11)
    rows, k = 4, 5120
    x = (rng.standard_normal((rows, k))).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(k)).astype(np.float16)
    suh = np.where(rng.random((2, k)) < 0.5, -1, 1).astype(np.float16)
    xn, xh = kernels.norm_rot(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), 1e-6,
                              torch.from_numpy(suh).to(cuda))
    xn_ref, xh_ref = O.norm_rot(x.astype(np.float32), w.astype(np.float32), 1e-6, suh, "float16")
    assert np.mean(xn.float().cpu().numpy() != xn_ref) < 1e-3
    assert O.max_rel(xh.cpu().numpy(), xh_ref) < 1e-3


def test_norm_rot_precondition(cuda):
    from omlx_exl3_b200 import kernels
    x = torch.zeros((1, 640), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(AssertionError):
        kernels.norm_rot(x, torch.ones(640, dtype=torch.bfloat16, device=cuda), 1e-6,
                         torch.ones((1, 640), dtype=torch.float16, device=cuda))


@pytest.mark.parametrize("out", [torch.float16, torch.bfloat16, torch.float32])
def test_had_svh(cuda, out):
    from omlx_exl3_b200 import kernels
    rng = np.random.default_rng(3)
    y = rng.standard_normal((5, 1024)).astype(np.float32)
    svh = np.where(rng.random(1024) < 0.5, -1, 1).astype(np.float16)
    got = kernels.had_svh(torch.from_numpy(y).to(cuda), torch.from_numpy(svh).to(cuda), out).float().cpu().numpy()
    ref = O.had128(y) * svh.astype(np.float32)
    assert O.max_rel(got, ref) < (1e-6 if out == torch.float32 else 1e-2)
