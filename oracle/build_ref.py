"""TEST INFRASTRUCTURE ONLY -- builds oracle/_ref/libexl3_ref.so from the reference's own decode source.

The reference (daig/omlx-exl3) keeps its trellis decode as Metal source text that Python assembles at
run time: HEADER (src/omlx/exl3/kernels.py:26-49) plus _decode_source(K) (kernels.py:304-334). This
recipe imports that kernels.py from the read-only reference checkout with a stub `mlx.core` (the
module only needs the name at import time), takes the generated text for K = 1..8 unchanged, and
compiles it as C++20 against oracle/ref_shim.h. The result is the reference's decode running on the
CPU, used to pin oracle/exl3_oracle.c and to generate the golden fixtures in tests/golden/. It also
holds the timed CPU baseline of bench.py (`--impl reference`): the reference decode, then an fp32
GEMV and the 128-point output rotation.

Generated sources and the library go to oracle/_ref/ only (git-ignored). Needs a read-only checkout of
the reference: the directory named by EXL3_REFERENCE_ROOT, else a `reference` directory beside this
repository's root. Without one, build() keeps an existing library and otherwise builds nothing; the
GPU box uses the prebuilt library.
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libexl3_ref.so"
REF_ROOT = Path(os.environ["EXL3_REFERENCE_ROOT"]) if os.environ.get("EXL3_REFERENCE_ROOT") \
    else HERE.parent.parent / "reference"
KERNELS_PY = REF_ROOT / "src" / "omlx" / "exl3" / "kernels.py"


def _load_reference_kernels():
    """Import the reference's kernels.py with a stand-in mlx.core (nothing in it runs at import)."""
    mx = types.ModuleType("mlx.core")
    for name in ("float16", "float32", "bfloat16", "uint32", "int32", "int16", "uint16"):
        setattr(mx, name, name)
    mx.Dtype = type("Dtype", (), {})
    mlx = types.ModuleType("mlx")
    mlx.core = mx
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core")}
    sys.modules["mlx"], sys.modules["mlx.core"] = mlx, mx
    try:
        spec = importlib.util.spec_from_file_location("_exl3_reference_kernels", KERNELS_PY)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod


_WRAPPER = r"""
// ---- CPU driver around the reference decode bodies (oracle test infrastructure) ----
#include <immintrin.h>
#include <omp.h>
#include <vector>

typedef void (*body_fn)(uint3, const uint*, const uint*, half*);

static body_fn pick(int K, int cb)
{
    switch (K * 4 + cb) {
@CASES@
    default: return nullptr;
    }
}

// W^T columns [16*nt0, 16*(nt0+ntc)) as (16*ntc, k) fp16 bits, exactly as the reference's decode
// kernel computes them; one emulated Metal thread per (k-slice, n-tile, run).
extern "C" int exl3_ref_decode_wt(int K, int cb, const uint32_t* trellis, int k, int n, int nt0, int ntc,
                                  uint16_t* w)
{
    body_fn f = pick(K, cb);
    if (!f || k % 16 || n % 16 || nt0 < 0 || ntc < 0 || nt0 + ntc > n / 16) return -1;
    const uint params[4] = {(uint)(k / 16), (uint)(n / 16), (uint)nt0, (uint)ntc};
    const long total = (long)(k / 16) * ntc * 8;
#pragma omp parallel for schedule(static)
    for (long gid = 0; gid < total; ++gid)
        f(uint3{(uint)gid, 0, 0}, trellis, params, reinterpret_cast<half*>(w));
    return 0;
}

static void fwht128(float* v)
{
    for (int h = 1; h < 128; h <<= 1)
        for (int b = 0; b < 64; ++b) {
            const int i0 = (b / h) * (2 * h) + (b % h), i1 = i0 + h;
            const float a0 = v[i0], a1 = v[i1];
            v[i0] = a0 + a1;
            v[i1] = a0 - a1;
        }
}

// CPU baseline of one EXL3 linear at decode shapes: per 128-column block, the reference decode of
// those columns, an fp32 GEMV (F16C + FMA), the 128-point output rotation, * 1/sqrt(128) * svh.
// xh: (rows, k) fp16 bits, svh: (n) fp16 bits, y: (rows, n) fp32.
extern "C" int exl3_ref_gemv(int K, int cb, const uint32_t* trellis, int k, int n, const uint16_t* xh,
                             int rows, const uint16_t* svh, float* y)
{
    body_fn f = pick(K, cb);
    if (!f || k % 16 || n % 128 || rows < 1 || rows > 8) return -1;
    const int blocks = n / 128;
    std::vector<float> xf((size_t)rows * k);
    for (size_t i = 0; i < xf.size(); ++i) xf[i] = _cvtsh_ss(xh[i]);
#pragma omp parallel
    {
        std::vector<uint16_t> wt((size_t)128 * k);
        float acc[8][128];
#pragma omp for schedule(dynamic, 1)
        for (int blk = 0; blk < blocks; ++blk) {
            const uint params[4] = {(uint)(k / 16), (uint)(n / 16), (uint)(blk * 8), 8u};
            const long total = (long)(k / 16) * 8 * 8;
            for (long gid = 0; gid < total; ++gid)
                f(uint3{(uint)gid, 0, 0}, trellis, params, reinterpret_cast<half*>(wt.data()));
            for (int c = 0; c < 128; ++c) {
                const uint16_t* wr = wt.data() + (size_t)c * k;
                for (int r = 0; r < rows; ++r) {
                    const float* xr = xf.data() + (size_t)r * k;
                    __m256 s = _mm256_setzero_ps();
                    for (int i = 0; i < k; i += 8) {
                        const __m256 wv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wr + i)));
                        s = _mm256_fmadd_ps(wv, _mm256_loadu_ps(xr + i), s);
                    }
                    alignas(32) float t[8];
                    _mm256_store_ps(t, s);
                    acc[r][c] = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
                }
            }
            for (int r = 0; r < rows; ++r) {
                fwht128(acc[r]);
                for (int c = 0; c < 128; ++c)
                    y[(size_t)r * n + blk * 128 + c] = acc[r][c] * 0.08838834764831845f * _cvtsh_ss(svh[blk * 128 + c]);
            }
        }
    }
    return 0;
}

extern "C" int exl3_ref_threads(void) { return omp_get_max_threads(); }
extern "C" void exl3_ref_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
"""


def generate() -> Path:
    """Write oracle/_ref/ref_decode.cpp from the reference's generated decode source."""
    ref = _load_reference_kernels()
    OUT.mkdir(parents=True, exist_ok=True)
    parts = ['#include "ref_shim.h"', "", "// ---- reference HEADER (kernels.py:26-49), verbatim ----",
             ref.HEADER]
    cases = []
    for K in range(1, 9):
        parts.append(f"// ---- reference _decode_source({K}) (kernels.py:304-334), verbatim ----")
        parts.append(f"namespace dec_k{K} {{")
        parts.append("template <int BITS, int CB>")
        parts.append("static void body(uint3 thread_position_in_grid, const device uint* trellis, "
                     "const device uint* params, device half* w) {")
        parts.append(ref._decode_source(K))
        parts.append("}")
        parts.append("}")
        for cb in range(3):
            cases.append(f"    case {K * 4 + cb}: return &dec_k{K}::body<{K}, {cb}>;")
    parts.append(_WRAPPER.replace("@CASES@", "\n".join(cases)))
    src = OUT / "ref_decode.cpp"
    src.write_text("\n".join(parts))
    return src


def build(force: bool = False) -> Path | None:
    """Compile the reference decode for the CPU. Returns the library path, or None without the reference."""
    if not KERNELS_PY.exists():
        return LIB if LIB.exists() else None
    if LIB.exists() and not force and LIB.stat().st_mtime > max(
            KERNELS_PY.stat().st_mtime, Path(__file__).stat().st_mtime, (HERE / "ref_shim.h").stat().st_mtime):
        return LIB
    src = generate()
    cmd = ["g++", "-std=c++20", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared",
           "-fno-strict-aliasing", f"-I{HERE}", "-o", str(LIB), str(src)]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
