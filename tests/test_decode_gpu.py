"""GPU: trellis -> W^T decode through the C ABI, bit-exact against the reference's own decode
(golden fixtures and digests made from it) and against the oracle."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
pytestmark = pytest.mark.gpu


def _dev_trellis(t: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(O.trellis_u32(t).view(np.int32).copy()).to(dev)


def test_decode_matches_golden_fixtures(cuda):
    from omlx_exl3_b200 import kernels
    z = np.load(GOLDEN / "decode_golden.npz")
    for K in range(1, 9):
        for cb in range(3):
            for tag in ("u32", "u31"):
                t = z[f"trellis_k{K}_cb{cb}_{tag}"]
                w = kernels.decode_wt(_dev_trellis(t, cuda), 16, 128, K, cb)
                got = w.cpu().numpy().view(np.uint16)
                assert np.array_equal(got, z[f"wt_k{K}_cb{cb}_{tag}"]), (K, cb, tag)


def test_decode_matches_reference_digests(cuda):
    from omlx_exl3_b200 import kernels
    d = json.loads((GOLDEN / "decode_digest.json").read_text())
    nt0, ntc = d["window"]
    for c in d["cases"]:
        t = _dev_trellis(O.random_trellis(c["k"], c["n"], c["K"], c["seed"]), cuda)
        w = kernels.decode_wt(t, c["k"], c["n"], c["K"], c["cb"]).cpu().numpy().view(np.uint16)
        assert hashlib.sha256(w.tobytes()).hexdigest() == c["sha256"], c
        ww = kernels.decode_wt(t, c["k"], c["n"], c["K"], c["cb"], nt0=nt0, ntc=ntc).cpu().numpy().view(np.uint16)
        assert hashlib.sha256(ww.tobytes()).hexdigest() == c["sha256_window"], c


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6, 8])
def test_decode_large_shape_matches_oracle(cuda, K):
    """A 27B-class shape (5120 -> 1024 columns of gate/up), ragged k-chunking (KT = 320 = 5 x 64)."""
    from omlx_exl3_b200 import kernels
    k, n = 5120, 1024
    t = O.random_trellis(k, n, K, 900 + K)
    for cb in range(3):
        got = kernels.decode_wt(_dev_trellis(t, cuda), k, n, K, cb).cpu().numpy().view(np.uint16)
        ref = O.decode_wt(t, k, n, K, cb).view(np.uint16)
        assert np.array_equal(got, ref), (K, cb)


def test_decode_tail_k_and_windows(cuda):
    """k not a multiple of the 64-tile CTA chunk, and column windows at both ends."""
    from omlx_exl3_b200 import kernels
    k, n, K = 16 * 70, 256, 7
    t = O.random_trellis(k, n, K, 4242)
    tt = _dev_trellis(t, cuda)
    for nt0, ntc in ((0, 16), (0, 1), (15, 1), (3, 9)):
        got = kernels.decode_wt(tt, k, n, K, 1, nt0=nt0, ntc=ntc).cpu().numpy().view(np.uint16)
        ref = O.decode_wt(t, k, n, K, 1, nt0=nt0, ntc=ntc).view(np.uint16)
        assert np.array_equal(got, ref), (nt0, ntc)


def test_decode_rejects_bad_window(cuda):
    from omlx_exl3_b200 import kernels
    tt = _dev_trellis(O.random_trellis(16, 128, 4, 1), cuda)
    with pytest.raises(ValueError):
        kernels.decode_wt(tt, 16, 128, 4, 0, nt0=5, ntc=4)
