"""GPU: the allocation-free GEMV entry point (exl3_gemv_noalloc) through the C ABI.

Some callers cannot allocate device memory at all: code running while a CUDA graph is captured,
hosts whose own pool allocator owns every byte of device memory, and thin bindings that only get the
input and output pointers. exl3_gemv_noalloc serves them from a fixed scratch array inside the
library instead of caller-provided scratch. This file is collected last (test_zz_) so that a run that
stops at the first failure has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _desc(k, ns, K, cb, rows):
    from omlx_exl3_b200._lib import GemvDesc
    d = GemvDesc()
    d.k, d.n_members = k, len(ns)
    for i in range(3):
        d.n[i] = ns[i] if i < len(ns) else 0
    d.bits, d.codebook, d.rows, d.out_dtype, d.grid, d.flags = K, cb, rows, 0, 0, 0
    return d


def test_noalloc_matches_gemv_twice(cuda):
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(17)
    k, ns, K, cb, rows = 2048, [512, 256], 5, 0, 3
    trs = [O.random_trellis(k, n, K, 40 + i) for i, n in enumerate(ns)]
    tt = [torch.from_numpy(O.trellis_u32(t).view(np.int32).copy()).to(cuda) for t in trs]
    svh = torch.from_numpy(np.where(rng.random(sum(ns)) < 0.5, -1.0, 1.0).astype(np.float16)).to(cuda)
    d = _desc(k, ns, K, cb, rows)
    tptr = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in tt], tt[0].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream

    # the existing entry point, with caller-allocated scratch
    pb, cbytes = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.exl3_gemv_workspace(ctypes.byref(d), ctypes.byref(pb), ctypes.byref(cbytes)) == 0
    partials = torch.empty(pb.value // 4, dtype=torch.float32, device=cuda)
    counters = torch.zeros(cbytes.value // 4, dtype=torch.int32, device=cuda)

    for call in range(2):
        xh = torch.from_numpy(rng.standard_normal((len(ns), rows, k)).astype(np.float16)).to(cuda)
        y_ref = torch.empty((rows, sum(ns)), dtype=torch.float16, device=cuda)
        y = torch.full((rows, sum(ns)), float("nan"), dtype=torch.float16, device=cuda)
        assert L.exl3_gemv(ctypes.byref(d), xh.data_ptr(), ctypes.cast(tptr, ctypes.c_void_p), svh.data_ptr(),
                           y_ref.data_ptr(), partials.data_ptr(), counters.data_ptr(), stream) == 0
        assert L.exl3_gemv_noalloc(ctypes.byref(d), xh.data_ptr(), ctypes.cast(tptr, ctypes.c_void_p),
                                   svh.data_ptr(), y.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        a, b = y.float().cpu().numpy(), y_ref.float().cpu().numpy()
        assert np.isfinite(a).all(), call
        assert O.max_rel(a, b) < 2e-3, call
        oracle_y = O.gemv(trs, k, ns, K, cb, xh.cpu().numpy(), svh.cpu().numpy())
        assert O.max_rel(a, oracle_y) < 2e-3, call


def test_noalloc_rejects_oversize(cuda):
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    # 4096 column blocks need more arrival counters than the fixed scratch holds
    d = _desc(1024, [4096 * 128], 4, 0, 1)
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda)
    tptr = (ctypes.c_void_p * 3)(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr())
    rc = L.exl3_gemv_noalloc(ctypes.byref(d), dummy.data_ptr(), ctypes.cast(tptr, ctypes.c_void_p),
                             dummy.data_ptr(), dummy.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -8                      # EXL3_E_WORKSPACE
    assert b"workspace" in L.exl3_strerror(rc)
