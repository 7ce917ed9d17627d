/*
 * q4_oracle.c -- CPU restatement of ARIA's Q4_0 path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker for the B200 kernels in aria_b200/csrc.  Only the
 * test-suite, __graft_entry__.smoke() and the CPU-baseline leg of bench.py may
 * load it; the product library never links it and has no CPU fallback.
 *
 * Parity status: UNPINNED against executed reference output.  The reference is
 * Rust (crate `aria` 3.6.0) and no Rust toolchain exists in this build
 * environment, and the reference ships no tests, fixtures or golden vectors for
 * this path.  The packer semantics below are restated line by line from the
 * reference source and cross-checked against two further independent
 * restatements (numpy twin in q4_oracle_np.py, exact-rational pure Python in
 * tests/golden/make_golden.py) plus hand-derived known answers.
 *
 * Reference lines followed (paths inside the lold3344/ARIA project):
 *   src/transformer_cuda.rs:548-575   quantize_q4_0 (18-byte blocks)
 *   src/transformer_cuda.rs:3214-3218 push_q4!: f16 weights -> f32 (exact) -> packer
 *   src/transformer_cuda.rs:3322-3333 cpu_matmul (row-major, i-p-j, f32)
 *   src/transformer_cuda.rs:1318-1321 LM-head dot products in `step`
 * Third-party semantics restated (crate pinned in Cargo.lock):
 *   half 2.7.1  f16::from_f32  -> IEEE-754 binary16, round-to-nearest-even,
 *                                 overflow to +-Inf, quiet NaN kept
 *   Rust core   f32::max       -> IEEE maxNum (a NaN operand is ignored)
 *   Rust core   f32::round     -> half away from zero
 *   Rust core   `f32 as i32`   -> saturating, NaN -> 0
 *   Rust release profile       -> i32 `+` wraps (overflow-checks off)
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define Q4O_BLOCK 32
#define Q4O_BLOCK_BYTES 18

/* ---------------------------------------------------------------- f16 <-> f32 */

/* IEEE binary32 -> binary16 with round-to-nearest-even (the conversion that
 * half 2.7.1's f16::from_f32 performs, in software or via F16C). */
uint16_t q4o_f32_to_f16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const uint32_t exp32 = (bits >> 23) & 0xFFu;
    uint32_t mant = bits & 0x7FFFFFu;

    if (exp32 == 0xFFu) { /* Inf or NaN: keep the top mantissa bits, force quiet */
        if (mant == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7C00u | 0x0200u | (mant >> 13));
    }
    const int e = (int)exp32 - 127 + 15; /* re-biased exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7C00u); /* too large: Inf */
    if (e <= 0) {
        /* result is a binary16 subnormal (or zero): shift the full significand */
        const int shift = 14 - e; /* >= 14 */
        if (shift > 24) return sign;  /* below half the smallest subnormal */
        mant |= 0x800000u;           /* implicit leading one */
        uint32_t q = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q += 1u;
        return (uint16_t)(sign | q); /* a carry into the exponent is correct */
    }
    uint32_t q = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1u; /* may carry to Inf */
    return (uint16_t)(sign | q);
}

/* binary16 -> binary32, exact. */
float q4o_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t m = (uint32_t)h & 0x3FFu;
    uint32_t out;
    if (e == 0x1Fu) {
        out = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        out = sign | ((e - 15u + 127u) << 23) | (m << 13);
    } else if (m == 0) {
        out = sign;
    } else { /* subnormal: normalise */
        int ee = -1;
        do { m <<= 1; ee++; } while ((m & 0x400u) == 0);
        m &= 0x3FFu;
        out = sign | ((uint32_t)(127 - 15 - ee) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

/* ---------------------------------------------------------------- packer */

/* Rust `(x as i32)`: saturating conversion, NaN -> 0. */
static int32_t rust_f32_as_i32(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

/* One 32-element block -> 18 bytes.  Follows transformer_cuda.rs:554-573. */
static void pack_block(const float* src, size_t len, uint8_t* out) {
    float abs_max = 0.0f; /* fold(0f32, f32::max) over |x| */
    for (size_t i = 0; i < len; i++) abs_max = fmaxf(abs_max, fabsf(src[i]));
    const float scale = (abs_max > 0.0f) ? abs_max / 7.0f : 1.0f;
    const uint16_t scale_bits = q4o_f32_to_f16(scale);
    out[0] = (uint8_t)(scale_bits & 0xFFu); /* to_le_bytes */
    out[1] = (uint8_t)(scale_bits >> 8);
    uint8_t* nib = out + 2;
    memset(nib, 0, 16);
    for (int i = 0; i < Q4O_BLOCK; i++) {
        const float val = ((size_t)i < len) ? src[i] : 0.0f; /* short tail padded with 0.0 */
        const float r = roundf(val / scale);                  /* f32 scale, not the f16 one */
        /* i32 add wraps in release builds; unreachable in practice since |val/scale| <= 7 */
        const int32_t q_wide = (int32_t)((uint32_t)rust_f32_as_i32(r) + 8u);
        const uint8_t q = (uint8_t)(q_wide < 0 ? 0 : (q_wide > 15 ? 15 : q_wide));
        if ((i & 1) == 0) nib[i / 2] = q;             /* element 2j -> low nibble of byte j */
        else nib[i / 2] |= (uint8_t)(q << 4);         /* element 2j+1 -> high nibble */
    }
}

size_t q4o_packed_bytes(size_t n) { return (n + Q4O_BLOCK - 1) / Q4O_BLOCK * Q4O_BLOCK_BYTES; }

/* quantize_q4_0(&[f32]) -> Vec<u8>  (transformer_cuda.rs:549-575) */
void q4o_quantize_q4_0(const float* data, size_t n, uint8_t* out) {
    const size_t nb = (n + Q4O_BLOCK - 1) / Q4O_BLOCK;
    for (size_t b = 0; b < nb; b++) {
        const size_t start = b * Q4O_BLOCK;
        const size_t end = (start + Q4O_BLOCK < n) ? start + Q4O_BLOCK : n;
        pack_block(data + start, end - start, out + b * Q4O_BLOCK_BYTES);
    }
}

/* push_q4! path: f16 weights are widened to f32 (exact) and then packed. */
void q4o_quantize_q4_0_f16(const uint16_t* data, size_t n, uint8_t* out) {
    const size_t nb = (n + Q4O_BLOCK - 1) / Q4O_BLOCK;
    for (size_t b = 0; b < nb; b++) {
        float tmp[Q4O_BLOCK];
        const size_t start = b * Q4O_BLOCK;
        const size_t end = (start + Q4O_BLOCK < n) ? start + Q4O_BLOCK : n;
        for (size_t i = start; i < end; i++) tmp[i - start] = q4o_f16_to_f32(data[i]);
        pack_block(tmp, end - start, out + b * Q4O_BLOCK_BYTES);
    }
}

/* Inverse implied by transformer_cuda.rs:560-570: w = (q - 8) * f32(scale_f16).
 * The reference has no dequantiser of its own. */
void q4o_dequantize_q4_0(const uint8_t* blocks, size_t n, float* out) {
    for (size_t i = 0; i < n; i++) {
        const uint8_t* blk = blocks + (i / Q4O_BLOCK) * Q4O_BLOCK_BYTES;
        const float s = q4o_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const int j = (int)(i % Q4O_BLOCK);
        const uint8_t byte = blk[2 + j / 2];
        const int q = (j & 1) ? (byte >> 4) : (byte & 0xF);
        out[i] = (float)(q - 8) * s;
    }
}

/* ---------------------------------------------------------------- matmul */

/* Parity reference: y[m][n] = alpha * sum_k x[m][k] * W(k,n) (+ bias[n]) + beta*y0,
 * computed in double from the exactly dequantised weights.
 * layout 0 (KN): W stored flat as w[k][n], blocks along n   (w_qkv/w_out/w_ff1/w_ff2,
 *                transformer_cuda.rs:263-270, used by gemm(..,false,false) at :1583)
 * layout 1 (NK): W stored flat as w[n][k], blocks along k   (tied LM head `embed`,
 *                used by gemm(..,false,true) at :1864)
 * x is f16 bits [M][ldx]; y (f64) is [M][N] dense. */
int q4o_matmul_ref_f64(const uint8_t* blocks, int layout, int K, int N,
                       const uint16_t* x, int M, int ldx, const uint16_t* bias,
                       double alpha, double* y) {
    const size_t nel = (size_t)K * (size_t)N;
    float* w = (float*)malloc(nel * sizeof(float));
    if (!w) return -1;
    q4o_dequantize_q4_0(blocks, nel, w);
    for (int m = 0; m < M; m++) {
        for (int n = 0; n < N; n++) {
            double acc = 0.0;
            for (int k = 0; k < K; k++) {
                const double wk = (layout == 0) ? w[(size_t)k * N + n] : w[(size_t)n * K + k];
                acc += (double)q4o_f16_to_f32(x[(size_t)m * ldx + k]) * wk;
            }
            acc *= alpha;
            if (bias) acc += (double)q4o_f16_to_f32(bias[n]);
            y[(size_t)m * N + n] = acc;
        }
    }
    free(w);
    return 0;
}

/* cpu_matmul (transformer_cuda.rs:3322-3333), faithful: f32, i-p-j loop order,
 * no reassociation (built with -ffp-contract=off, no fast-math). c must be zeroed. */
void q4o_cpu_matmul_f32(const float* a, const float* b, int m, int k, int n, float* c) {
    for (int i = 0; i < m; i++)
        for (int p = 0; p < k; p++) {
            const float av = a[(size_t)i * k + p];
            const float* brow = b + (size_t)p * n;
            float* crow = c + (size_t)i * n;
            for (int j = 0; j < n; j++) crow[j] += av * brow[j];
        }
}

/* LM-head form of `step` (transformer_cuda.rs:1318-1321): logits[v] = dot(x, embed[v]). */
void q4o_cpu_matmul_t_f32(const float* a, const float* b, int m, int k, int n, float* c) {
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            float s = 0.0f;
            const float* arow = a + (size_t)i * k;
            const float* brow = b + (size_t)j * k;
            for (int p = 0; p < k; p++) s += arow[p] * brow[p];
            c[(size_t)i * n + j] = s;
        }
}

/* ---------------------------------------------------------------- CPU baseline */

/* The reference's CPU arithmetic for one Q4_0 projection: dequantise the packed
 * blocks to f32, widen the f16 activations, then cpu_matmul (KN) or the
 * dot-product form (NK).  `threads` > 1 splits rows of the output (OpenMP),
 * which the serial reference does not do; 1 reproduces it.  w_scratch must
 * hold K*N floats, x_scratch M*K floats.  y is f32 [M][N]. */
void q4o_baseline_projection(const uint8_t* blocks, int layout, int K, int N,
                             const uint16_t* x, int M, float* y,
                             float* w_scratch, float* x_scratch, int threads) {
    const size_t nel = (size_t)K * (size_t)N;
    const size_t nb = nel / Q4O_BLOCK;
#ifdef _OPENMP
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
    for (long long b = 0; b < (long long)nb; b++)
        q4o_dequantize_q4_0(blocks + (size_t)b * Q4O_BLOCK_BYTES, Q4O_BLOCK, w_scratch + (size_t)b * Q4O_BLOCK);
    for (size_t i = 0; i < (size_t)M * K; i++) x_scratch[i] = q4o_f16_to_f32(x[i]);
    memset(y, 0, (size_t)M * N * sizeof(float));
    if (layout == 0) {
        /* split the output columns across threads; each keeps the i-p-j order */
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
        {
            const int t = omp_get_thread_num(), nt = omp_get_num_threads();
#else
        {
            const int t = 0, nt = 1;
#endif
            const int j0 = (int)((long long)N * t / nt), j1 = (int)((long long)N * (t + 1) / nt);
            for (int i = 0; i < M; i++)
                for (int p = 0; p < K; p++) {
                    const float av = x_scratch[(size_t)i * K + p];
                    const float* brow = w_scratch + (size_t)p * N;
                    float* crow = y + (size_t)i * N;
                    for (int j = j0; j < j1; j++) crow[j] += av * brow[j];
                }
        }
    } else {
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
        for (int j = 0; j < N; j++)
            for (int i = 0; i < M; i++) {
                float s = 0.0f;
                const float* arow = x_scratch + (size_t)i * K;
                const float* brow = w_scratch + (size_t)j * K;
                for (int p = 0; p < K; p++) s += arow[p] * brow[p];
                y[(size_t)i * N + j] = s;
            }
    }
}

int q4o_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
