"""CPU: the oracle against the reference's own decode (golden fixtures, digests, and when the reference
checkout is present, the reference decode compiled for the CPU)."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases():
    z = np.load(GOLDEN / "decode_golden.npz")
    for K in range(1, 9):
        for cb in range(3):
            for tag in ("u32", "u31"):
                yield K, cb, z[f"trellis_k{K}_cb{cb}_{tag}"], z[f"wt_k{K}_cb{cb}_{tag}"]


@pytest.mark.parametrize("K", range(1, 9))
def test_oracle_matches_golden_fixtures(K):
    n_checked = 0
    for KK, cb, t, wt in _cases():
        if KK != K:
            continue
        got = O.decode_wt(t, 16, 128, K, cb).view(np.uint16)
        assert np.array_equal(got, wt), (K, cb)
        n_checked += 1
    assert n_checked == 6


def test_oracle_matches_reference_digests():
    d = json.loads((GOLDEN / "decode_digest.json").read_text())
    nt0, ntc = d["window"]
    assert len(d["cases"]) == 24
    for c in d["cases"]:
        t = O.random_trellis(c["k"], c["n"], c["K"], c["seed"])
        w = O.decode_wt(t, c["k"], c["n"], c["K"], c["cb"]).view(np.uint16)
        assert hashlib.sha256(w.tobytes()).hexdigest() == c["sha256"], c
        ww = O.decode_wt(t, c["k"], c["n"], c["K"], c["cb"], nt0=nt0, ntc=ntc).view(np.uint16)
        assert hashlib.sha256(ww.tobytes()).hexdigest() == c["sha256_window"], c


def test_oracle_matches_compiled_reference_decode():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    for K in range(1, 9):
        for cb in range(3):
            t = O.random_trellis(64, 384, K, 77 + K * 3 + cb)
            a = O.decode_wt(t, 64, 384, K, cb).view(np.uint16)
            b = O.ref_decode_wt(t, 64, 384, K, cb).view(np.uint16)
            assert np.array_equal(a, b), (K, cb)


def test_codebook_statistics():
    """Value ranges of the three codebooks over all 65536 states (3inst/mcg std ~1.24, mul1 ~1.0)."""
    L = O.lib()
    for cb, std, amax in ((0, 1.2437, 3.98), (1, 1.2441, 3.95), (2, 1.0003, 3.46)):
        v = np.array([L.exl3o_dec1(s, cb) for s in range(65536)], dtype=np.uint16).view(np.float16)
        v = v.astype(np.float64)
        assert abs(v.std() - std) < 2e-3 and np.abs(v).max() < amax, cb


def test_position_map_is_a_bijection():
    """Runs x positions cover the 16x16 tile exactly once (kernels.py:52-55)."""
    t = O.random_trellis(16, 16, 4, 3)
    w = O.decode_w(t, 16, 16, 4, 0)
    assert w.shape == (16, 16) and np.isfinite(w).all()
    seen = set()
    for g in range(8):
        for p in range(32):
            j = p & 7
            col = g + 8 * (j >= 4)
            kk = 2 * (p >> 3) + (j & 1) + 8 * ((j & 3) >= 2)
            seen.add((kk, col))
    assert len(seen) == 256


def test_decode_w_is_transpose_of_decode_wt():
    t = O.random_trellis(64, 256, 5, 11)
    wt = O.decode_wt(t, 64, 256, 5, 1).astype(np.float32)
    w = O.decode_w(t, 64, 256, 5, 1)
    assert np.array_equal(w, wt.T)


def test_fwht_properties():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    y = O.had128(O.had128(x))            # H/sqrt(128) is an involution
    assert np.allclose(y, x, atol=1e-5)
    e = np.zeros(128, np.float32)
    e[0] = 1
    assert np.allclose(O.fwht128(e), np.ones(128))
    # Sylvester order: row i, column j of H is (-1)^popcount(i & j)
    H = np.array([[(-1) ** bin(i & j).count("1") for j in range(128)] for i in range(128)], np.float32)
    assert np.allclose(O.fwht128(x[:, :128]), x[:, :128] @ H.T, atol=1e-4)


def test_gemv_numpy_and_c_agree():
    rng = np.random.default_rng(1)
    k, n, K, cb = 256, 384, 4, 0
    t = O.random_trellis(k, n, K, 5)
    xh = rng.standard_normal((1, 3, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1, 1).astype(np.float16)
    a = O.gemv([t], k, [n], K, cb, xh, svh)
    b = O.gemv_c(t, k, n, K, cb, xh[0], svh)
    assert O.max_rel(b, a) < 1e-5


def test_unpack_signs():
    bits = np.array([0b1, 0x8000, 0xFFFF], dtype=np.uint16).view(np.int16)
    s = O.unpack_signs(bits)
    assert s.shape == (48,)
    assert s[0] == -1 and (s[1:16] == 1).all()
    assert s[31] == -1 and (s[16:31] == 1).all()
    assert (s[32:] == -1).all()


def test_kl_div_zero_for_equal_logits():
    z = np.random.default_rng(2).standard_normal((4, 100))
    assert np.allclose(O.kl_div(z, z), 0)
    assert (O.kl_div(z, z + np.random.default_rng(3).standard_normal((4, 100))) > 0).all()
