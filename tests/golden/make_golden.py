"""Generate the EXL3 decode golden fixtures from the reference's own decode source.

Run here, where the reference checkout exists (it is compiled by oracle/build_ref.py into
oracle/_ref/libexl3_ref.so); the GPU box and the CPU test suite only read the committed outputs:

  decode_golden.npz   for every bitrate K = 1..8 and codebook cb = 0..2 (3inst, mcg, mul1): a seeded
                      trellis of one 16 x 128 slice (8 tiles) and the reference's decoded W^T (128, 16)
                      fp16, once with full-range 32-bit words and once with the reference test's
                      31-bit words (src/tools/exl3_kernel_test.py:29-31).
  decode_digest.json  sha256 of the reference decode of larger seeded trellises (k = 256, n = 512 per
                      K and cb, plus a windowed nt0/ntc case): the GPU decode is checked against it.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build_ref, oracle  # noqa: E402

OUT = Path(__file__).resolve().parent

# (k, n, seed) of the digest cases; seeds are offset by K and cb inside digest_cases()
DIGEST_SHAPE = (256, 512)
DIGEST_WINDOW = (5, 11)      # nt0, ntc of the windowed decode case


def small_cases():
    for K in range(1, 9):
        for cb in range(3):
            for bit31 in (True, False):
                yield K, cb, bit31, 1000 + 37 * K + 7 * cb + (0 if bit31 else 1)


def digest_cases():
    k, n = DIGEST_SHAPE
    for K in range(1, 9):
        for cb in range(3):
            yield K, cb, k, n, 5000 + 11 * K + cb


def main():
    if build_ref.build() is None:
        raise SystemExit("the reference checkout is needed to build oracle/_ref")
    arrays = {}
    for K, cb, bit31, seed in small_cases():
        t = oracle.random_trellis(16, 128, K, seed, bit31=bit31)
        w = oracle.ref_decode_wt(t, 16, 128, K, cb)
        mine = oracle.decode_wt(t, 16, 128, K, cb)
        assert np.array_equal(w.view(np.uint16), mine.view(np.uint16)), (K, cb, bit31)
        tag = f"k{K}_cb{cb}_{'u32' if bit31 else 'u31'}"
        arrays[f"trellis_{tag}"] = t
        arrays[f"wt_{tag}"] = w.view(np.uint16)
    np.savez_compressed(OUT / "decode_golden.npz", **arrays)

    digests = {"shape": list(DIGEST_SHAPE), "window": list(DIGEST_WINDOW), "cases": []}
    for K, cb, k, n, seed in digest_cases():
        t = oracle.random_trellis(k, n, K, seed)
        w = oracle.ref_decode_wt(t, k, n, K, cb).view(np.uint16)
        nt0, ntc = DIGEST_WINDOW
        ww = oracle.ref_decode_wt(t, k, n, K, cb, nt0=nt0, ntc=ntc).view(np.uint16)
        assert np.array_equal(w, oracle.decode_wt(t, k, n, K, cb).view(np.uint16))
        digests["cases"].append({
            "K": K, "cb": cb, "k": k, "n": n, "seed": seed,
            "sha256": hashlib.sha256(w.tobytes()).hexdigest(),
            "sha256_window": hashlib.sha256(ww.tobytes()).hexdigest(),
        })
    (OUT / "decode_digest.json").write_text(json.dumps(digests, indent=1) + "\n")
    print("wrote", OUT / "decode_golden.npz", OUT / "decode_digest.json")


if __name__ == "__main__":
    main()
