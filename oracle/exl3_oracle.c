/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the EXL3 hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this library, and
 * only as the checker or the timed CPU baseline.  The product (omlx_exl3_b200) never calls it.
 *
 * A plain-C restatement of the EXL3 (ExLlamaV3 trellis) weight format as the reference documents
 * and decodes it (daig/omlx-exl3, src/omlx/exl3/kernels.py):
 *   - format docstring                        kernels.py:4-8
 *   - codebook hash dec1<CB>                  kernels.py:26-48
 *   - run/position -> (k, n) tile map (_kk)   kernels.py:52-55, 216, 332
 *   - decode_wt output layout (n_chunk, k)    kernels.py:304-351
 * It is written from the format description, not from the generated Metal code.  Parity with the
 * reference's own decode is pinned by oracle/build_ref.py, which compiles the reference's decode
 * source for the CPU, and by the golden fixtures under tests/golden/.
 *
 * fp16 arithmetic is done exactly: conversions are written out by hand (round to nearest even),
 * and each fp16 operation is evaluated exactly in double and rounded once, which is what a single
 * IEEE fp16 add / fma does.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 helpers (exact) ---- */

static double h2d(uint16_t h)
{
    const int s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | 0x400), e - 25);
    return s ? -v : v;
}

/* Round a double to the nearest fp16 (ties to even). */
static uint16_t d2h(double x)
{
    uint16_t sign = 0;
    if (signbit(x)) { sign = 0x8000; x = -x; }
    if (isnan(x)) return sign | 0x7e00;
    if (x >= 65520.0) return sign | 0x7c00;            /* rounds to inf */
    if (x < ldexp(1.0, -14)) {                         /* subnormal: units of 2^-24 */
        double q = x * ldexp(1.0, 24);
        double r = nearbyint(q);                       /* default rounding mode: ties to even */
        return sign | (uint16_t)r;                     /* r == 1024 becomes the smallest normal */
    }
    int e;
    double f = frexp(x, &e);                           /* x = f * 2^e, f in [0.5, 1) */
    double q = ldexp(f, 11);                           /* 11 significant bits -> [1024, 2048) */
    double r = nearbyint(q);
    if (r >= 2048.0) { r = 1024.0; e += 1; }
    int be = e - 1 + 15;                               /* biased exponent of 1.m * 2^(e-1) */
    if (be >= 31) return sign | 0x7c00;
    return sign | (uint16_t)(be << 10) | (uint16_t)((int)r - 1024);
}

float exl3o_h2f(uint16_t h) { return (float)h2d(h); }
uint16_t exl3o_f2h(float x) { return d2h((double)x); }

/* ---------------------------------------------------------------- codebooks ---------------- */

/* fp16 constants of the mul1 codebook (kernels.py:27-28, 46): 1/K and the bias, as fp16 bits */
#define MUL1_INV_BITS 0x1eeeu
#define MUL1_BIAS_BITS 0xc931u

/* One 16-bit trellis state -> fp16 weight bits, codebook cb (0 = 3inst, 1 = mcg, 2 = mul1). */
uint16_t exl3o_dec1(uint32_t s, int cb)
{
    s &= 0xffffu;
    if (cb == 0 || cb == 1) {
        const uint32_t h = cb == 0 ? s * 89226354u + 64248484u : s * 0xCBAC1FEDu;
        const uint32_t v = (h & 0x8fff8fffu) ^ 0x3b603b60u;
        /* two fp16 halves, one fp16 add */
        return d2h(h2d((uint16_t)(v & 0xffffu)) + h2d((uint16_t)(v >> 16)));
    } else {
        const uint32_t h = s * 0x83DCD12Du;
        const uint32_t bytesum = (h & 0xffu) + ((h >> 8) & 0xffu) + ((h >> 16) & 0xffu) + (h >> 24);
        const double r = 1024.0 + (double)bytesum;    /* fp16 0x6400 + bytesum, exact */
        /* one fp16 fma: r * inv + bias, rounded once */
        return d2h(r * h2d(MUL1_INV_BITS) + h2d(MUL1_BIAS_BITS));
    }
}

/* ---------------------------------------------------------------- bitstream --------------- */

/* 16-bit state of position t (0..255) of one tile: stream bits [(t+1)K-16, (t+1)K) modulo the
 * tile's 256*K bits.  Stream bit b is bit (31 - b%32) of little-endian word b/32. */
static uint32_t tile_state(const uint32_t* tw, int K, int t)
{
    const int nbits = 256 * K, nwords = 8 * K;
    int e = (t + 1) * K;                               /* exclusive end bit */
    if (e > nbits) e -= nbits;
    const int iw = (e - 1) >> 5;                       /* word holding bit e-1 */
    const int ip = (iw + nwords - 1) % nwords;         /* word before it (tail-biting) */
    const uint64_t cat = ((uint64_t)tw[ip] << 32) | tw[iw];
    const int shift = 32 * (iw + 1) - e;               /* bit e-1 lands at bit 0 */
    return (uint32_t)(cat >> shift) & 0xffffu;
}

/* Position p (0..31) of run g (0..7) -> tile column and tile k-row. */
static void run_pos(int g, int p, int* col, int* kk)
{
    const int j = p & 7;
    *col = g + 8 * (j >= 4);
    *kk = 2 * (p >> 3) + (j & 1) + 8 * ((j & 3) >= 2);
}

/*
 * decode_wt: W^T columns [16*nt0, 16*(nt0+ntc)) of a k x n EXL3 tensor as an (16*ntc, k) fp16
 * matrix, row = output feature (kernels.py:340-351).  trellis is the flat uint32 view of the
 * int16 [k/16, n/16, 16K] checkpoint tensor.  Returns 0 or a negative error.
 */
int exl3o_decode_wt(const uint32_t* trellis, int k, int n, int K, int cb, int nt0, int ntc, uint16_t* w)
{
    if (k % 16 || n % 16 || K < 1 || K > 8 || cb < 0 || cb > 2) return -1;
    const int KT = k / 16, NT = n / 16, TW = 8 * K;
    if (ntc < 0) ntc = NT - nt0;
    if (nt0 < 0 || nt0 + ntc > NT) return -2;
#pragma omp parallel for collapse(2) schedule(static)
    for (int kt = 0; kt < KT; ++kt)
        for (int ntl = 0; ntl < ntc; ++ntl) {
            const uint32_t* tw = trellis + ((size_t)kt * NT + (nt0 + ntl)) * TW;
            for (int g = 0; g < 8; ++g)
                for (int p = 0; p < 32; ++p) {
                    int col, kk;
                    run_pos(g, p, &col, &kk);
                    const uint32_t s = tile_state(tw, K, 32 * g + p);
                    w[((size_t)ntl * 16 + col) * k + (size_t)kt * 16 + kk] = exl3o_dec1(s, cb);
                }
        }
    return 0;
}

/* Same decode as fp32 W (k, n) row-major (k-major), for the fp32 GEMV/GEMM oracles. */
int exl3o_decode_w_f32(const uint32_t* trellis, int k, int n, int K, int cb, float* w)
{
    if (k % 16 || n % 16 || K < 1 || K > 8 || cb < 0 || cb > 2) return -1;
    const int KT = k / 16, NT = n / 16, TW = 8 * K;
#pragma omp parallel for collapse(2) schedule(static)
    for (int kt = 0; kt < KT; ++kt)
        for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* tw = trellis + ((size_t)kt * NT + nt) * TW;
            for (int g = 0; g < 8; ++g)
                for (int p = 0; p < 32; ++p) {
                    int col, kk;
                    run_pos(g, p, &col, &kk);
                    const uint32_t s = tile_state(tw, K, 32 * g + p);
                    w[((size_t)kt * 16 + kk) * n + (size_t)nt * 16 + col] = (float)h2d(exl3o_dec1(s, cb));
                }
        }
    return 0;
}

/* ---------------------------------------------------------------- fp32 GEMV oracle -------- */

/* 128-point fast Walsh-Hadamard transform, Sylvester order, stages h = 1, 2, ..., 64, in fp32
 * (kernels.py:194-204, 374-386): lower index gets a0 + a1, upper gets a0 - a1. */
void exl3o_fwht128(float* v)
{
    for (int h = 1; h < 128; h <<= 1)
        for (int b = 0; b < 64; ++b) {
            const int i0 = (b / h) * (2 * h) + (b % h), i1 = i0 + h;
            const float a0 = v[i0], a1 = v[i1];
            v[i0] = a0 + a1;
            v[i1] = a0 - a1;
        }
}

/*
 * y = had128(xh @ W) * (1/sqrt(128)) * svh for one member, fp32 accumulation (the reference's
 * GEMV, kernels.py:114-209, restated without its split-k reduction order).  xh: (rows, k) fp16
 * bits; svh: (n) fp16 bits; y: (rows, n) fp32 (the caller rounds to the output dtype).
 * Threads: one per (row, 128-column block).
 */
int exl3o_gemv_f32(const uint32_t* trellis, int k, int n, int K, int cb, const uint16_t* xh, int rows,
                   const uint16_t* svh, float* y)
{
    if (k % 16 || n % 128 || K < 1 || K > 8 || cb < 0 || cb > 2 || rows < 1) return -1;
    const int KT = k / 16, NT = n / 16, TW = 8 * K;
    const int blocks = n / 128;
#pragma omp parallel for schedule(dynamic, 1)
    for (int blk = 0; blk < blocks; ++blk) {
        float acc[8][128];
        uint16_t wt[16 * 16];
        for (int r0 = 0; r0 < rows; r0 += 8) {
            const int rr = rows - r0 < 8 ? rows - r0 : 8;
            memset(acc, 0, sizeof(acc));
            for (int kt = 0; kt < KT; ++kt)
                for (int j = 0; j < 8; ++j) {
                    const int nt = blk * 8 + j;
                    const uint32_t* tw = trellis + ((size_t)kt * NT + nt) * TW;
                    for (int g = 0; g < 8; ++g)
                        for (int p = 0; p < 32; ++p) {
                            int col, kk;
                            run_pos(g, p, &col, &kk);
                            wt[kk * 16 + col] = exl3o_dec1(tile_state(tw, K, 32 * g + p), cb);
                        }
                    for (int kk = 0; kk < 16; ++kk)
                        for (int r = 0; r < rr; ++r) {
                            const float xv = (float)h2d(xh[(size_t)(r0 + r) * k + kt * 16 + kk]);
                            for (int col = 0; col < 16; ++col)
                                acc[r][j * 16 + col] += xv * (float)h2d(wt[kk * 16 + col]);
                        }
                }
            for (int r = 0; r < rr; ++r) {
                exl3o_fwht128(acc[r]);
                for (int c = 0; c < 128; ++c)
                    y[(size_t)(r0 + r) * n + blk * 128 + c] =
                        acc[r][c] * 0.08838834764831845f * (float)h2d(svh[blk * 128 + c]);
            }
        }
    }
    return 0;
}

int exl3o_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void exl3o_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
