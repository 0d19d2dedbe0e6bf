/*
 * exl3_b200.h -- C ABI of the B200 (sm_100a) EXL3 quantized-linear hot path.
 *
 * One shared library, libexl3b200.so, built from omlx_exl3_b200/csrc/. Plain pointers and sizes, no
 * framework types: device buffers are owned by the caller, `stream` is a cudaStream_t passed as void*,
 * and every entry point returns 0 (EXL3_OK) or a negative EXL3_E* status (exl3_strerror() names it).
 * Compute entry points allocate no device memory: scratch space is passed in by the caller (or, for
 * exl3_gemv_noalloc, lives in a fixed array inside the library). The one allocating entry point is
 * exl3_peer_create, which makes the tensor-parallel peer buffer.
 *
 * The reference (daig/omlx-exl3) has no C ABI: its kernels are Metal source JIT-compiled through MLX
 * (src/omlx/exl3/kernels.py). Each entry point below names the reference function it replaces. The
 * package omlx_exl3_b200 binds this header through ctypes (omlx_exl3_b200/_lib.py), the way a
 * reference-side Python binding would.
 *
 * Dtype codes: EXL3_F16 = 0, EXL3_BF16 = 1, EXL3_F32 = 2.
 * Trellis buffers are the checkpoint's int16 [k/16][n/16][16K] tensors viewed as uint32 words and
 * must be 16-byte aligned.
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EXL3_API __attribute__((visibility("default")))
#else
#define EXL3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    EXL3_OK = 0,
    EXL3_E_SHAPE = -1,      /* k, n, rows or member count out of range / not a multiple */
    EXL3_E_BITS = -2,       /* bits per weight not in 1..8 */
    EXL3_E_CODEBOOK = -3,   /* codebook not in 0..2 */
    EXL3_E_DTYPE = -4,      /* unsupported dtype code */
    EXL3_E_ALIGN = -5,      /* a pointer is not aligned as required */
    EXL3_E_NULL = -6,       /* a required pointer is NULL */
    EXL3_E_CUDA = -7,       /* a CUDA launch or attribute call failed */
    EXL3_E_WORKSPACE = -8,  /* scratch buffer too small */
    EXL3_E_DEVICE = -9      /* device is not sm_100 */
};

enum { EXL3_F16 = 0, EXL3_BF16 = 1, EXL3_F32 = 2 };

/* Human-readable name of a status code. */
EXL3_API const char* exl3_strerror(int status);

/* ABI version, (major << 16) | minor. */
EXL3_API int exl3_version(void);

/*
 * Trellis -> W^T decode, bit-exact fp16.
 * Replaces: kernels.decode_wt (src/omlx/exl3/kernels.py:340-351).
 * Writes columns [16*nt0, 16*(nt0+ntc)) of the k x n weight as an (16*ntc, k) row-major fp16
 * matrix `w` (row = output feature). ntc < 0 means "to the end".
 */
EXL3_API int exl3_decode_wt(const uint32_t* trellis, int k, int n, int bits, int codebook, int nt0, int ntc,
                   void* w, void* stream);

/*
 * Decode GEMV for 1..8 rows (decode / speculative verify), one launch for a linear or a sibling group.
 * Replaces: kernels.TrellisGemvPlan.__call__ (src/omlx/exl3/kernels.py:263-299, kernel :114-209).
 *   y[r, :] = concat_m( had128(xh[m, r, :] @ W_m) / sqrt(128) ) * svh      (y in out_dtype)
 * xh: fp16 (n_members, rows, k); trellis[m]: member m's k x n[m] trellis; svh: fp16 (sum n);
 * y: (rows, sum n) fp16 or bf16. All members share k, bits and codebook; each n[m] % 128 == 0.
 * partials / counters: scratch from exl3_gemv_workspace(). `counters` must be zeroed once when it is
 * allocated (exl3_gemv_reset); every completed call leaves it zeroed again. Calls that share one
 * scratch buffer must not overlap on the GPU (use one scratch per stream).
 */
typedef struct exl3_gemv_desc {
    int32_t k;           /* in_features, multiple of 16 */
    int32_t n_members;   /* 1..3 */
    int32_t n[3];        /* out_features of each member, multiples of 128 */
    int32_t bits;        /* 1..8 */
    int32_t codebook;    /* 0 = 3inst, 1 = mcg, 2 = mul1 */
    int32_t rows;        /* 1..8 */
    int32_t out_dtype;   /* EXL3_F16 or EXL3_BF16 */
    int32_t grid;        /* CTAs to use; 0 = one per SM of the current device */
    int32_t flags;       /* reserved, 0 (EXL3_GEMV_ROW_EXACT is accepted: every call is row-exact) */
    int32_t member_bits[3]; /* bits of each member; 0 = `bits`. Members may differ (a q/k/v group quantised
                               at different bpw): each then runs on its own share of the CTAs, still one
                               launch (exl3_gemv, exl3_gemv_qkv_post; not exl3_gemv_peer) */
} exl3_gemv_desc;

/* exl3_gemv_desc.flags. Every row count multiplies exact fp16 products into fp32 accumulators on the
 * tensor cores, so row r of any call gives the same bits whatever `rows` is (the reference kernel's
 * row-exact property, src/omlx/exl3/kernels.py:13-15). The flag is kept for callers that set it. */
enum { EXL3_GEMV_ROW_EXACT = 1 };

/*
 * Allocation-free variant of exl3_gemv. It has no counterpart in the reference: it exists for callers
 * that cannot allocate device memory (code running during CUDA graph capture, hosts whose pool
 * allocator owns all device memory, bindings that only receive input/output pointers). The split-k
 * scratch lives in one fixed 4 MiB array inside this library (per device, held until exit), so a
 * call whose scratch would not fit (more than 4096 column blocks of 128, or more than 4 MiB - 16 KiB
 * of partials, e.g. a very wide output on a large grid) returns EXL3_E_WORKSPACE. The first call on
 * each device (and the first after that device's context was reset) looks the array's device address
 * up; make that first call before any stream capture.
 * Every call clears the counters it uses (one memset on `stream`). All calls on one device share the
 * array, so calls that overlap on that GPU (e.g. on two streams) race and corrupt each other's
 * results: issue them one after another on one stream. Each device has its own copy of the array.
 */
EXL3_API int exl3_gemv_noalloc(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                               const void* svh, void* y, void* stream);

EXL3_API int exl3_gemv_workspace(const exl3_gemv_desc* desc, size_t* partial_bytes, size_t* counter_bytes);
EXL3_API int exl3_gemv_reset(uint32_t* counters, size_t counter_bytes, void* stream);
EXL3_API int exl3_gemv(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis, const void* svh,
              void* y, float* partials, uint32_t* counters, void* stream);

/*
 * exl3_gemv whose rotated input is computed inside the same launch: each CTA rotates the 128-column
 * k blocks its units read (the arithmetic of exl3_rot / exl3_swiglu_rot, bit-identical results) into
 * its own region of the scratch `xs`, then runs the GEMV on them. Same scratch rules as exl3_gemv, plus
 * xs of exl3_gemv_prologue_workspace bytes (16-byte aligned, no initial contents needed). k % 128 == 0;
 * members of one bitrate (no member_bits).
 *   exl3_gemv_rot:          xh[m] = rot(x, suh[m]) for x (rows, k) of x_dtype (EXL3_F16 / BF16 / F32)
 *                           and suh fp16 (n_members, k). Replaces: kernels.rot + TrellisGemvPlan.__call__,
 *                           the two launches of EXL3Linear's decode forward (src/omlx/exl3/linear.py:
 *                           111-117, kernels.py:451-458) and EXL3SiblingGroup.gemv (linear.py:163-172).
 *   exl3_gemv_swiglu:       xh = swiglu_rot(gu, suh) for gu = [gate | up] (rows, 2k) of gu_dtype, suh
 *                           fp16 (k); one member. Replaces: kernels.swiglu_rot + down_proj's
 *                           gemv_rotated in the fused MLP (src/omlx/exl3/fusion.py:288-295).
 *   exl3_gemv_swiglu_peer:  the same with the output rows pushed into the peers' inboxes as
 *                           exl3_gemv_peer does (the row-parallel down_proj of a tensor-parallel step).
 */
EXL3_API int exl3_gemv_prologue_workspace(const exl3_gemv_desc* desc, size_t* xs_bytes);
EXL3_API int exl3_gemv_rot(const exl3_gemv_desc* desc, const void* x, int x_dtype, const void* suh,
                           const uint32_t* const* trellis, const void* svh, void* y, float* partials,
                           uint32_t* counters, void* xs, size_t xs_bytes, void* stream);
EXL3_API int exl3_gemv_swiglu(const exl3_gemv_desc* desc, const void* gu, int gu_dtype, const void* suh,
                              const uint32_t* const* trellis, const void* svh, void* y, float* partials,
                              uint32_t* counters, void* xs, size_t xs_bytes, void* stream);

/*
 * Input rotation for 1..3 members: xh[m, r, :] = fp16( had128(x[r, :] * suh[m, :]) / sqrt(128) ).
 * Replaces: kernels.rot (src/omlx/exl3/kernels.py:451-458). x: (rows, k) of x_dtype; suh: fp16
 * (n_members, k); xh: fp16 (n_members, rows, k); k % 128 == 0.
 */
EXL3_API int exl3_rot(const void* x, int x_dtype, int rows, int k, const void* suh, int n_members, void* xh, void* stream);

/*
 * RMSNorm (MLX rounding: xn = T(w * T(x * rsqrt(mean(x^2) + eps)))) fused with the input rotation
 * of every consumer. Replaces: kernels.norm_rot (src/omlx/exl3/kernels.py:461-473).
 * x, w, xn: (rows, k) / (k) / (rows, k) of dtype (EXL3_F16 or EXL3_BF16); suh: fp16 (n_members, k);
 * xh: fp16 (n_members, rows, k); k % 128 == 0.
 */
EXL3_API int exl3_norm_rot(const void* x, const void* w, int dtype, int rows, int k, float eps, const void* suh,
                  int n_members, void* xn, void* xh, void* stream);

/*
 * SwiGLU fused with down_proj's input rotation: xh[r, :] = fp16(had128(silu(g) * u * suh) / sqrt(128))
 * with gu = [g | u] (rows, 2n) of gu_dtype. Replaces: kernels.swiglu_rot (src/omlx/exl3/kernels.py:476-483).
 * suh: fp16 (n); xh: fp16 (1, rows, n); n % 128 == 0.
 */
EXL3_API int exl3_swiglu_rot(const void* gu, int gu_dtype, int rows, int n, const void* suh, void* xh, void* stream);

/*
 * Prefill GEMM with the trellis decoded in-kernel (tcgen05 / tensor memory):
 *   y = out_dtype( had128(xh @ W) / sqrt(128) * svh ),  xh fp16 (M, k), W the k x n trellis, y (M, n).
 * Replaces: EXL3Linear._prefill (src/omlx/exl3/linear.py:97-105: decode_wt chunks, MLX matmul, _had128,
 * * svh). k % 64 == 0, n % 128 == 0, any M >= 1; out_dtype EXL3_F16, EXL3_BF16 or EXL3_F32. `status`
 * is a device uint32 that the kernel ORs an error bit into if a bounded wait gives up (0 = fine).
 * xh, trellis and y must be 16-byte aligned.
 */
EXL3_API int exl3_gemm(const void* xh, int M, int k, int n, const uint32_t* trellis, int bits, int codebook,
                       const void* svh, void* y, int out_dtype, void* workspace, size_t workspace_bytes,
                       uint32_t* status, void* stream);
/* Bytes of the optional exl3_gemm workspace (256-byte aligned) for an M x k x n call; 0 when the call
 * would not split k. With it, calls whose row tiles x column blocks fill at most half of the SMs (narrow
 * outputs) split k over several CTAs per tile; the first bytes are arrival counters that must be zero
 * before the first call (every completed call leaves them zero). A null or smaller workspace runs
 * unsplit. Calls that share a workspace must not overlap. */
EXL3_API int exl3_gemm_workspace(int M, int k, int n, size_t* bytes);

/*
 * Prefill GEMM on weights already decoded by exl3_decode_wt (tcgen05 pairs of SMs, both operands by TMA):
 *   y[:, 0:n] = out_dtype( had128(xh @ wt^T) / sqrt(128) * svh ),  xh fp16 (M, k), wt fp16 (n, k) row-major
 *   (the decode_wt layout: row j = output column j), y rows ldy elements apart (ldy >= n), so a column
 *   chunk of a wider output is written in place.
 * Replaces: the matmul, _had128 and * svh of EXL3Linear._prefill (src/omlx/exl3/linear.py:101-105) for one
 * chunk of decode_wt columns. k % 64 == 0, n % 128 == 0, any M >= 1; out_dtype EXL3_F16, EXL3_BF16 or
 * EXL3_F32; xh, wt and y 16-byte aligned, ldy * element size a multiple of 16. `status` as for exl3_gemm.
 * workspace (256-byte aligned) of exl3_gemm_wt_workspace bytes lets the call split k over several work
 * units for shapes with few output tiles; its first bytes are arrival counters that must be zero before
 * the first call (every completed call leaves them zero). A null or smaller workspace runs unsplit.
 * Calls that share a workspace must not overlap.
 */
EXL3_API int exl3_gemm_wt_workspace(int M, int k, int n, size_t* bytes);
EXL3_API int exl3_gemm_wt(const void* xh, int M, int k, int n, const void* wt, const void* svh, void* y, int ldy,
                          int out_dtype, void* workspace, size_t workspace_bytes, uint32_t* status, void* stream);

/*
 * Output rotation: out[r, :] = out_dtype(had128(y[r, :]) / sqrt(128) * svh), y (rows, n) of y_dtype.
 * Replaces: the prefill tail `_had128(y) * self._svh` (src/omlx/exl3/linear.py:105, :31-33).
 * svh: fp16 (n); n % 128 == 0.
 */
EXL3_API int exl3_had_svh(const void* y, int y_dtype, int rows, int n, const void* svh, void* out, int out_dtype,
                          void* stream);

/*
 * Decode-step attention glue after the fused q/k/v GEMV (head_dim 128, rotate-half RoPE):
 *   q_out[r, h]           = fp16(T(rope(rms_norm(q[r, h]) * q_norm_w)))          for h < hq
 *   k_cache[h, pos[r]]    = fp16(T(rope(rms_norm(k[r, h]) * k_norm_w)))          for h < hkv
 *   v_cache[h, pos[r]]    = fp16(v[r, h])
 * q/k/v rows of dtype T (EXL3_F16 / EXL3_BF16) with element strides q_stride/k_stride/v_stride between
 * rows; norms round as mx.fast.rms_norm does. cos_table/sin_table: f32 (max_len, 64); pos: int64
 * (rows); caches fp16 (hkv, max_len, 128); q_out fp16 (rows, hq, 128).
 * Replaces: the q_norm / k_norm / RoPE / KV-cache update of the attention module the EXL3 q/k/v
 * projections feed (the fused-norm consumer set of src/omlx/exl3/fusion.py:8-10; the attention
 * module itself is the model library's, outside the reference tree). No counterpart kernel in the
 * reference: there these are separate framework ops.
 */
EXL3_API int exl3_qkv_post(const void* q, const void* k, const void* v, int q_stride, int k_stride, int v_stride,
                           int dtype, int rows, int hq, int hkv, const void* q_norm_w, const void* k_norm_w, float eps,
                           const float* cos_table, const float* sin_table, const long long* pos, void* k_cache,
                           void* v_cache, int max_len, void* q_out, void* stream);

/*
 * The q/k/v sibling group's GEMV with exl3_qkv_post as its epilogue: members 0/1/2 are q (hq heads),
 * k and v (hkv heads each, head_dim 128). Each finished 128-column block is one head; it is rounded to
 * desc->out_dtype exactly as exl3_gemv would store it and then written as exl3_qkv_post writes it
 * (q_out fp16 (rows, hq, 128); k/v into the fp16 caches at pos[r]). No y. Same scratch as exl3_gemv.
 * Replaces: kernels.TrellisGemvPlan for the q/k/v group + the attention module's q/k norm, RoPE and
 * cache update (see exl3_qkv_post).
 */
typedef struct exl3_qkv_post_args {
    const void* q_norm_w;        /* (128) in desc->out_dtype */
    const void* k_norm_w;
    const float* cos_table;      /* (max positions, 64) */
    const float* sin_table;
    const long long* pos;        /* (rows) int64 */
    void* k_cache;               /* fp16 (hkv, max_len, 128) */
    void* v_cache;
    void* q_out;                 /* fp16 (rows, hq, 128) */
    int32_t hq, hkv, max_len;
    float eps;
} exl3_qkv_post_args;

EXL3_API int exl3_gemv_qkv_post(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                                const void* svh, float* partials, uint32_t* counters, const exl3_qkv_post_args* post,
                                void* stream);

/*
 * Residual add fused into norm_rot: x_out = T(x + d); xn = T(w * T(x_out * rsqrt(mean(x_out^2) + eps)));
 * xh[m] = fp16(had128(xn * suh[m]) / sqrt(128)). Replaces: `h = x + attn_out` followed by
 * kernels.norm_rot (src/omlx/exl3/kernels.py:408-425, :461-473). x_out must not alias x or d
 * (every block of a row reads the whole row); k % 128 == 0; suh fp16 (n_members, k); xn may be NULL
 * (the norm output is then not stored).
 */
EXL3_API int exl3_add_norm_rot(const void* x, const void* d, const void* w, int dtype, int rows, int k, float eps,
                               const void* suh, int n_members, void* x_out, void* xn, void* xh, void* stream);

/*
 * Greedy selection: for each of `rows` rows of x (row stride ld elements, dtype EXL3_F16 / EXL3_BF16 /
 * EXL3_F32), the largest of the first n values (val, as fp32) and its column + index_base (idx); the
 * first column wins ties and a NaN counts as the largest value, as in torch.argmax. Replaces: the cast + max reduction of the decode step's greedy
 * token (the reference samples in oMLX's generate loop).
 */
EXL3_API int exl3_argmax(const void* x, int dtype, int rows, int ld, int n, int index_base, float* val,
                         long long* idx, void* stream);

/*
 * Decode attention fused with o_proj's input rotation, for rows new tokens (head_dim 128, GQA,
 * rows * hq / hkv <= 64: every speculative-verify width up to 8 rows at 8 heads per kv head) over an
 * fp16 KV cache. Row r's result does not depend on `rows` (bitwise equal to a one-row call at its
 * position):
 *   xh[r, h*128 : h*128+128] = fp16( had128( fp16(softmax(q k^T / sqrt(128)) v) * suh[h*128 ..] ) / sqrt(128) )
 * q: fp16 (rows, hq, 128); k_cache, v_cache: fp16 (hkv, max_len, 128), positions [0, T) valid, new
 * row i at position T - rows + i sees positions <= that; suh: fp16 (hq * 128); xh: fp16 (rows, hq * 128).
 * workspace: exl3_attn_workspace bytes, 16-byte aligned: 16 reserved bytes, then the split partials. Replaces: the model's
 * scaled-dot-product attention + kernels.rot (src/omlx/exl3/kernels.py:451-458) of the decode step.
 */
EXL3_API int exl3_attn_workspace(int rows, int hq, int hkv, int max_len, int T, size_t* bytes);
EXL3_API int exl3_attn_decode_rot(const void* q, const void* k_cache, const void* v_cache, int rows, int hq, int hkv,
                                  int max_len, int T, const void* suh, void* xh, void* workspace,
                                  size_t workspace_bytes, void* stream);

/*
 * Tensor-parallel peer buffers (CUDA IPC over NVLink). Each rank of a tensor-parallel group creates
 * one buffer with exl3_peer_create (the one entry point that allocates device memory: the buffer
 * must be its own cudaMalloc allocation to be shared), sends the 64-byte handle to the other ranks
 * (any host transport), and maps theirs with exl3_peer_open. exl3_peer_close / exl3_peer_destroy
 * undo the two. No counterpart in the reference (one Apple GPU); they carry the fused all-reduce.
 */
#define EXL3_PEER_HANDLE_BYTES 64
EXL3_API int exl3_peer_create(size_t bytes, void** ptr, void* handle);
EXL3_API int exl3_peer_destroy(void* ptr);
EXL3_API int exl3_peer_open(const void* handle, void** ptr);
EXL3_API int exl3_peer_close(void* ptr);

/* One tensor-parallel group as seen by one rank. Buffer layout (byte offsets, same on every rank):
 * a flag block at flag_off (zeroed at creation; word 8 = epoch of the last completed all-reduce,
 * word 9 = CTA arrival count, word 10 = status bits), then two slots, each holding `world` inboxes of
 * inbox_bytes: the inbox of (slot s, source rank p) starts at data_off + (s * world + p) * inbox_bytes.
 * An inbox holds one source rank's (rows, k) partial as "LL" words, 8 bytes per pair of columns:
 * bits 0..31 the two 16-bit values (column 2j in the low half), bits 32..63 the epoch of the call
 * that wrote them. A reader takes a word once its epoch matches, so data and flag arrive together. */
typedef struct exl3_peer_group {
    int32_t world;           /* 1..8 */
    int32_t rank;            /* this process's rank */
    void* base[8];           /* every rank's buffer as mapped in this process (base[rank] = own) */
    uint64_t flag_off;       /* multiple of 64 */
    uint64_t data_off;       /* multiple of 16 */
    uint64_t inbox_bytes;    /* multiple of 16, >= rows * k * 4 */
} exl3_peer_group;

/*
 * Push this rank's (rows, k) partial (16-bit values, 4-byte aligned) into inbox (slot, rank) of every
 * rank of the group, tagged with the epoch of the next exl3_ar_add_norm_rot. For producers other than
 * exl3_gemv_peer. No counterpart in the reference (one Apple GPU).
 */
EXL3_API int exl3_peer_put(const exl3_peer_group* g, int slot, const void* src, int rows, int k, void* stream);

/*
 * exl3_gemv whose output rows go, as LL words, straight into inbox (slot, rank) of every rank of the
 * group (P2P stores over NVLink from the CTAs that finish each 128-column block) instead of into y.
 * The output width n_total is the all-reduce's k. Replaces: kernels.TrellisGemvPlan for a
 * row-parallel projection followed by its all-reduce.
 */
EXL3_API int exl3_gemv_peer(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                            const void* svh, float* partials, uint32_t* counters, const exl3_peer_group* g, int slot,
                            void* stream);

/* exl3_gemv_swiglu with exl3_gemv_peer's output (see exl3_gemv_swiglu above). */
EXL3_API int exl3_gemv_swiglu_peer(const exl3_gemv_desc* desc, const void* gu, int gu_dtype, const void* suh,
                                   const uint32_t* const* trellis, const void* svh, float* partials,
                                   uint32_t* counters, void* xs, size_t xs_bytes, const exl3_peer_group* g,
                                   int slot, void* stream);

/*
 * All-reduce of the row-parallel partials fused with residual add + RMSNorm + input rotation:
 *   d = sum over ranks (in rank order, fp32) of the partials in this rank's inboxes of slot `slot`,
 *   (rows, k) of dtype T, then exactly exl3_add_norm_rot(x, T(d), w, ...). Every rank must have
 *   pushed its partial for this call (exl3_gemv_peer / exl3_peer_put) into slot `slot`; consecutive
 *   calls alternate slot 0 / 1; every rank makes the same sequence of calls. Polls its own inboxes
 *   for at most 2 s, then sets a status bit (exl3_peer_status) and continues. Replaces: the NCCL
 *   all-reduce + exl3_add_norm_rot pair of the tensor-parallel decode step (the reference runs on
 *   one GPU; its norm-rotation is src/omlx/exl3/kernels.py:408-425). k % 128 == 0, k <= 16384,
 *   rows <= 8; x, w, suh, x_out 16-byte aligned; xn may be NULL.
 */
EXL3_API int exl3_ar_add_norm_rot(const exl3_peer_group* g, int slot, const void* x, const void* w, int dtype,
                                  int rows, int k, float eps, const void* suh, int n_members, void* x_out,
                                  void* xn, void* xh, void* stream);
/* Status bits of the group's own flag block (4 = a wait for another rank timed out). */
EXL3_API int exl3_peer_status(const exl3_peer_group* g, uint32_t* status);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
