/*
 * CPU oracle for the quantized-weight QLoRA path.  TEST INFRASTRUCTURE ONLY:
 * the parity tests, the smoke check and the CPU-baseline leg of the bench
 * link this file as the checker; the product path never calls it.
 *
 * What it restates
 * ----------------
 * The reference (takahashim/torobi) binds no quantized op: its CHANGELOG.md:136
 * says quantized ops are not implemented, and the complete mlx-c call table
 * (docs/vendoring.md:299-329, engine/src/mlxc/ops.rs:91-130) has no
 * mlx_quantize / mlx_dequantize / mlx_quantized_matmul.  The arithmetic lives
 * in the pinned third-party dependency MLX 0.32.2 (mlx-c commit
 * c74db5307cc8ce122f48d97ef951b30578674e7f, lib/torobi/mlx_prebuilt.json:4-9),
 * which is absent from the reference tree and from this machine.  This file
 * restates MLX's published affine-quantization algorithm (mx.quantize with
 * mode "affine"):
 *
 *   per group of `group` consecutive elements along the last axis
 *     w_min, w_max          = min / max of the group, in f32
 *     side                  = |w_min| > |w_max|
 *     scale                 = max((w_max - w_min) / (2^bits - 1), 1e-7)
 *     scale                 = side ? scale : -scale
 *     edge                  = side ? w_min : w_max
 *     q0                    = rint(edge / scale)
 *     if q0 != 0: scale = edge / q0, bias = edge     (zero is exactly a code)
 *     else:       bias  = 0
 *     code[i]               = clamp(rint((w[i] - bias) / scale), 0, 2^bits - 1)
 *   codes packed low-bits-first, 32/bits codes per uint32 along the last axis;
 *   scale and bias stored in the weight's dtype (bf16, round-to-nearest-even).
 *
 * Parity unpinned for quantize / dequantize / quantized_matmul: MLX itself
 * cannot be run here and the reference holds no golden vectors for these
 * ops, so bit-exactness against MLX is unverified.  The conventions this file
 * fixes (the kernels are held bit-exact to THIS file):
 *   - all group arithmetic in IEEE f32 with round-to-nearest-even, no FMA
 *     contraction (compiled with -ffp-contract=off);
 *   - max/min follow C++ std::max/std::min (`a < b ? b : a`), so a NaN element
 *     never becomes the group's min or max;
 *   - a NaN element quantizes to code 0;
 *   - dequantized value = RNE_bf16(scale * q + bias), rounded ONCE from the
 *     exact value (the product of an 8-bit code and a bf16 scale is exact, and
 *     the sum is formed in double, which is exact for every group this
 *     quantizer emits: |scale| <= |bias| whenever bias != 0).
 *
 * Linear-layer semantics: y = x . W^T with W in PyTorch layout [d_out, d_in]
 * (reference lib/torobi/dsl/layers.rb:16-25).  The GEMMs here accumulate in
 * f32 (the tolerance the parity tests apply is stated there).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bf16 --- */

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* f32 -> bf16, round to nearest even; NaN -> 0x7FC0. */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if (f != f) return 0x7FC0;
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* double -> bf16 with a single round-to-nearest-even from the double. */
static inline uint16_t f64_to_bf16(double d) {
    if (d != d) return 0x7FC0;
    if (d == 0.0) return signbit(d) ? 0x8000 : 0x0000;
    double a = fabs(d);
    if (isinf(d)) return d > 0 ? 0x7F80 : 0xFF80;
    int e;
    frexp(a, &e);                 /* a = m * 2^e, m in [0.5, 1) */
    int lead = e - 1;             /* a in [2^lead, 2^(lead+1)) */
    if (lead < -126) lead = -126; /* subnormal range: fixed quantum */
    double quantum = ldexp(1.0, lead - 7);
    double r = nearbyint(a / quantum) * quantum; /* exact scaling by 2^k */
    if (r >= ldexp(1.0, 128)) return d > 0 ? 0x7F80 : 0xFF80;
    float f = (float)r;           /* exact: r has <= 8 significant bits */
    uint32_t u;
    memcpy(&u, &f, 4);
    uint16_t h = (uint16_t)(u >> 16);
    return d < 0 ? (uint16_t)(h | 0x8000) : h;
}

void or_f32_to_bf16(const float *in, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(in[i]);
}

void or_bf16_to_f32(const uint16_t *in, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

static inline float mlx_max(float a, float b) { return a < b ? b : a; }
static inline float mlx_min(float a, float b) { return b < a ? b : a; }

/* ------------------------------------------------------------ quantize --- */

/* One group: chooses scale/bias (f32) and writes the packed codes. */
static void quantize_group(const uint16_t *w, int group, int bits,
                           uint32_t *codes, float *scale_out, float *bias_out) {
    const float n_bins = (float)((1 << bits) - 1);
    const float eps = 1e-7f;
    float w_min = INFINITY, w_max = -INFINITY;
    for (int j = 0; j < group; ++j) {
        float v = bf16_to_f32(w[j]);
        w_max = mlx_max(w_max, v);
        w_min = mlx_min(w_min, v);
    }
    int side = fabsf(w_min) > fabsf(w_max);
    float scale = mlx_max((w_max - w_min) / n_bins, eps);
    scale = side ? scale : -scale;
    float edge = side ? w_min : w_max;
    float q0 = rintf(edge / scale);
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = edge / q0;
        bias = edge;
    }
    const int per_word = 32 / bits;
    for (int word = 0; word < group / per_word; ++word) {
        uint32_t packed = 0;
        for (int k = 0; k < per_word; ++k) {
            float v = bf16_to_f32(w[word * per_word + k]);
            float q = rintf((v - bias) / scale);
            q = mlx_min(mlx_max(q, 0.0f), n_bins);
            uint32_t code = (q == q) ? (uint32_t)q : 0u;
            packed |= code << (k * bits);
        }
        codes[word] = packed;
    }
    *scale_out = scale;
    *bias_out = bias;
}

/*
 * w      [rows, cols] bf16 (row-major, cols contiguous)
 * codes  [rows, cols * bits / 32] u32
 * scales [rows, cols / group] bf16, biases likewise
 * Returns 0, or -1 for an unsupported bits/group/shape.
 */
int or_quantize(const uint16_t *w, int64_t rows, int64_t cols, int bits, int group,
                uint32_t *codes, uint16_t *scales, uint16_t *biases) {
    if (!(bits == 4 || bits == 8)) return -1;
    if (!(group == 32 || group == 64 || group == 128)) return -1;
    if (rows < 0 || cols < 0 || cols % group != 0) return -1;
    const int64_t groups_per_row = cols / group;
    const int64_t words_per_group = group * bits / 32;
    const int64_t n_groups = rows * groups_per_row;
#pragma omp parallel for schedule(static)
    for (int64_t gi = 0; gi < n_groups; ++gi) {
        float s, b;
        quantize_group(w + gi * group, group, bits, codes + gi * words_per_group, &s, &b);
        scales[gi] = f32_to_bf16(s);
        biases[gi] = f32_to_bf16(b);
    }
    return 0;
}

/* Also exposes the f32 scale/bias before storage rounding (used by tests). */
int or_quantize_f32_params(const uint16_t *w, int64_t rows, int64_t cols, int bits,
                           int group, uint32_t *codes, float *scales, float *biases) {
    if (!(bits == 4 || bits == 8)) return -1;
    if (!(group == 32 || group == 64 || group == 128)) return -1;
    if (rows < 0 || cols < 0 || cols % group != 0) return -1;
    const int64_t n_groups = rows * (cols / group);
    const int64_t words_per_group = group * bits / 32;
    for (int64_t gi = 0; gi < n_groups; ++gi)
        quantize_group(w + gi * group, group, bits, codes + gi * words_per_group,
                       scales + gi, biases + gi);
    return 0;
}

/* ---------------------------------------------------------- dequantize --- */

static inline uint32_t code_at(const uint32_t *codes_row, int64_t col, int bits) {
    const int per_word = 32 / bits;
    uint32_t word = codes_row[col / per_word];
    return (word >> ((col % per_word) * bits)) & ((1u << bits) - 1u);
}

static inline uint16_t dequant_one(uint32_t q, uint16_t s, uint16_t b) {
    const float sf = bf16_to_f32(s), bf = bf16_to_f32(b), qf = (float)q;
    /* Fast path: when the f32 fma is exact it IS the exact value, and one
       rounding of it to bf16 is the single rounding we want. */
    const float v32 = fmaf(sf, qf, bf);
    const double exact = (double)sf * (double)qf + (double)bf;
    if ((double)v32 == exact) return f32_to_bf16(v32);
    return f64_to_bf16(exact);
}

int or_dequantize(const uint32_t *codes, const uint16_t *scales, const uint16_t *biases,
                  int64_t rows, int64_t cols, int bits, int group, uint16_t *out) {
    if (!(bits == 4 || bits == 8)) return -1;
    if (!(group == 32 || group == 64 || group == 128)) return -1;
    if (rows < 0 || cols < 0 || cols % group != 0) return -1;
    const int64_t words_per_row = cols * bits / 32;
    const int64_t groups_per_row = cols / group;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint32_t *crow = codes + r * words_per_row;
        for (int64_t c = 0; c < cols; ++c) {
            int64_t gi = r * groups_per_row + c / group;
            out[r * cols + c] = dequant_one(code_at(crow, c, bits), scales[gi], biases[gi]);
        }
    }
    return 0;
}

/* Dequantize one row into f32 (exact values of the bf16 results). */
static void dequant_row_f32(const uint32_t *crow, const uint16_t *srow, const uint16_t *brow,
                            int64_t cols, int bits, int group, float *out) {
    for (int64_t c = 0; c < cols; ++c)
        out[c] = bf16_to_f32(dequant_one(code_at(crow, c, bits), srow[c / group], brow[c / group]));
}

/* ------------------------------------------------------ quantized GEMMs --- */

/*
 * y[m, n] = sum_k x[m, k] * Wdq[n, k]        (quantized_matmul, transpose=True)
 * x bf16 [M, K]; W codes [N, K*bits/32]; y f32 [M, N].  f32 accumulation in a
 * fixed order (16 interleaved partial sums, then summed).
 */
int or_qmm_fwd(const uint16_t *x, const uint32_t *codes, const uint16_t *scales,
               const uint16_t *biases, int64_t M, int64_t N, int64_t K, int bits,
               int group, float *y) {
    if (!(bits == 4 || bits == 8) || !(group == 32 || group == 64 || group == 128)) return -1;
    if (M < 0 || N < 0 || K < 0 || K % group != 0) return -1;
    const int64_t words_per_row = K * bits / 32;
    const int64_t groups_per_row = K / group;
#pragma omp parallel
    {
        float *wrow = (float *)__builtin_alloca(sizeof(float) * (size_t)(K > 0 ? K : 1));
        float *xrow = NULL;
        (void)xrow;
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            dequant_row_f32(codes + n * words_per_row, scales + n * groups_per_row,
                            biases + n * groups_per_row, K, bits, group, wrow);
            for (int64_t m = 0; m < M; ++m) {
                const uint16_t *xr = x + m * K;
                float acc[16] = {0};
                int64_t k = 0;
                for (; k + 16 <= K; k += 16)
                    for (int l = 0; l < 16; ++l) acc[l] += bf16_to_f32(xr[k + l]) * wrow[k + l];
                for (; k < K; ++k) acc[k & 15] += bf16_to_f32(xr[k]) * wrow[k];
                float s = 0.0f;
                for (int l = 0; l < 16; ++l) s += acc[l];
                y[m * N + n] = s;
            }
        }
    }
    return 0;
}

/*
 * dx[m, k] = sum_n dy[m, n] * Wdq[n, k]      (the VJP of quantized_matmul wrt x)
 * dy bf16 [M, N]; dx f32 [M, K].  Each thread owns a slab of dx columns and
 * walks n in order, so every dx element accumulates in the same fixed order.
 */
int or_qmm_dx(const uint16_t *dy, const uint32_t *codes, const uint16_t *scales,
              const uint16_t *biases, int64_t M, int64_t N, int64_t K, int bits,
              int group, float *dx) {
    if (!(bits == 4 || bits == 8) || !(group == 32 || group == 64 || group == 128)) return -1;
    if (M < 0 || N < 0 || K < 0 || K % group != 0) return -1;
    const int64_t words_per_row = K * bits / 32;
    const int64_t groups_per_row = K / group;
    const int64_t slab = group; /* columns per work item: whole groups */
    const int64_t n_slabs = K / slab;
    memset(dx, 0, sizeof(float) * (size_t)(M * K));
#pragma omp parallel
    {
        float *wslab = (float *)__builtin_alloca(sizeof(float) * (size_t)slab);
#pragma omp for schedule(static)
        for (int64_t si = 0; si < n_slabs; ++si) {
            const int64_t k0 = si * slab;
            for (int64_t n = 0; n < N; ++n) {
                const uint32_t *crow = codes + n * words_per_row;
                const uint16_t s = scales[n * groups_per_row + si];
                const uint16_t b = biases[n * groups_per_row + si];
                for (int64_t c = 0; c < slab; ++c)
                    wslab[c] = bf16_to_f32(dequant_one(code_at(crow, k0 + c, bits), s, b));
                for (int64_t m = 0; m < M; ++m) {
                    const float g = bf16_to_f32(dy[m * N + n]);
                    float *dr = dx + m * K + k0;
                    for (int64_t c = 0; c < slab; ++c) dr[c] += g * wslab[c];
                }
            }
        }
    }
    return 0;
}

/* Plain bf16 GEMM with f32 accumulate: c[m, n] = sum_k a[m, k] * b[n, k]. */
int or_gemm_nt(const uint16_t *a, const uint16_t *b, int64_t M, int64_t N, int64_t K,
               float *c) {
    if (M < 0 || N < 0 || K < 0) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float acc[16] = {0};
            int64_t k = 0;
            for (; k + 16 <= K; k += 16)
                for (int l = 0; l < 16; ++l)
                    acc[l] += bf16_to_f32(a[m * K + k + l]) * bf16_to_f32(b[n * K + k + l]);
            for (; k < K; ++k) acc[k & 15] += bf16_to_f32(a[m * K + k]) * bf16_to_f32(b[n * K + k]);
            float s = 0.0f;
            for (int l = 0; l < 16; ++l) s += acc[l];
            c[m * N + n] = s;
        }
    }
    return 0;
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
