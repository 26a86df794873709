/*
 * tcg_oracle.c -- CPU oracle for the tensor-core GEMM path (TEST INFRASTRUCTURE).
 *
 * Plain-C restatement of the reference's host-side data generation, naive
 * GEMMs, quantisation and accuracy metrics (MattJBorowski1991/TensorCorePTX,
 * src/data.cu, src/data_int8.cu, src/data_int4.cu).  Used only by tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs as the checker.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, so float expressions are
 * evaluated exactly as written, one rounding per operation, as the reference's
 * host code is compiled without FMA contraction).
 */
#include "tcg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* IEEE binary16 conversions, written from the IEEE 754 definition.         */
/* ------------------------------------------------------------------------ */

uint16_t oracle_f32_to_f16(float x)
{
    uint32_t u;
    memcpy(&u, &x, sizeof u);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t exp = (u >> 23) & 0xFFu;
    uint32_t man = u & 0x7FFFFFu;
    if (exp == 0xFFu) /* inf / nan (nan keeps a quiet payload bit) */
        return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31)
        return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        /* result is subnormal (or zero): m = full_mantissa >> (14 - e) */
        if (e < -10)
            return (uint16_t)sign;
        uint32_t full = man | 0x800000u;
        int shift = 14 - e;
        uint32_t m = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1u)))
            m++; /* may carry into the smallest normal: still correct */
        return (uint16_t)(sign | m);
    }
    uint32_t m = man >> 13;
    uint32_t rem = man & 0x1FFFu;
    uint32_t h = sign | ((uint32_t)e << 10) | m;
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u)))
        h++; /* carry propagates into the exponent, up to infinity */
    return (uint16_t)h;
}

float oracle_f16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {
            int s = 0;
            while (!(man & 0x400u)) {
                man <<= 1;
                s++;
            }
            man &= 0x3FFu;
            u = sign | ((uint32_t)(127 - 14 - s) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((exp - 15u + 127u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* ------------------------------------------------------------------------ */
/* Seeded generators.  They consume glibc rand() in exactly the reference's  */
/* order so that outputs are bit-identical to its known answers.            */
/* ------------------------------------------------------------------------ */

/* src/data.cu:6-14: srand(42); per batch all of A then all of B; each value
 * (float)rand()/RAND_MAX*0.1f-0.05f rounded to binary16. */
void oracle_generate_fp16(uint16_t* A, uint16_t* B, int M, int N, int K, int batches)
{
    srand(42);
    for (int b = 0; b < batches; ++b) {
        for (long i = 0; i < (long)M * K; ++i)
            A[(long)b * M * K + i] = oracle_f32_to_f16((float)rand() / RAND_MAX * 0.1f - 0.05f);
        for (long i = 0; i < (long)K * N; ++i)
            B[(long)b * K * N + i] = oracle_f32_to_f16((float)rand() / RAND_MAX * 0.1f - 0.05f);
    }
}

/* src/data_int8.cu:6-14: srand(42); values rand()%255-127 in [-127,127]. */
void oracle_generate_int8(int8_t* A, int8_t* BT, int M, int N, int K, int batches)
{
    srand(42);
    for (int b = 0; b < batches; ++b) {
        for (long i = 0; i < (long)M * K; ++i)
            A[(long)b * M * K + i] = (int8_t)(rand() % 255 - 127);
        for (long i = 0; i < (long)N * K; ++i)
            BT[(long)b * N * K + i] = (int8_t)(rand() % 255 - 127);
    }
}

static int8_t pack_pair(int8_t lo, int8_t hi)
{
    return (int8_t)((lo & 0x0F) | ((hi & 0x0F) << 4));
}

static int8_t nib_lo(int8_t p) { return (int8_t)((int8_t)(p << 4) >> 4); }
static int8_t nib_hi(int8_t p) { return (int8_t)(p >> 4); }

/* src/data_int4.cu:26-42: srand(42); per packed byte draw lo then hi, each
 * rand()%15-7 in [-7,7]; byte = lo | hi<<4. */
void oracle_generate_int4_packed(int8_t* A, int8_t* BT, int M, int N, int K, int batches)
{
    srand(42);
    long ra = (long)M * (K / 2), rb = (long)N * (K / 2);
    for (int b = 0; b < batches; ++b) {
        for (long i = 0; i < ra; ++i) {
            int8_t lo = (int8_t)((rand() % 15) - 7);
            int8_t hi = (int8_t)((rand() % 15) - 7);
            A[(long)b * ra + i] = pack_pair(lo, hi);
        }
        for (long i = 0; i < rb; ++i) {
            int8_t lo = (int8_t)((rand() % 15) - 7);
            int8_t hi = (int8_t)((rand() % 15) - 7);
            BT[(long)b * rb + i] = pack_pair(lo, hi);
        }
    }
}

/* Box-Muller draw, src/data_int8.cu:56-60 (same as src/data_int4.cu:88-92). */
static float box_muller(void)
{
    float u1 = ((float)rand() + 1.f) / ((float)RAND_MAX + 2.f);
    float u2 = (float)rand() / ((float)RAND_MAX + 1.f);
    return sqrtf(-2.f * logf(u1)) * cosf(2.f * 3.14159265f * u2);
}

void oracle_generate_fp32_normal(float* A, float* BT, int M, int N, int K, int batches)
{
    srand(43);
    for (int b = 0; b < batches; ++b) {
        for (long i = 0; i < (long)M * K; ++i)
            A[(long)b * M * K + i] = box_muller();
        for (long i = 0; i < (long)N * K; ++i)
            BT[(long)b * N * K + i] = box_muller();
    }
}

/* ------------------------------------------------------------------------ */
/* GEMMs.  C rows [row0, row0+rows) of one batch; C is written at its full  */
/* M x N position (C + m*N).                                                */
/* ------------------------------------------------------------------------ */

void oracle_gemm_f16_f32acc(const uint16_t* A, const uint16_t* B, float* C,
                            int M, int N, int K, int row0, int rows)
{
    (void)M;
    /* convert B once per call; same products and k order as the reference */
    float* Bf = (float*)malloc(sizeof(float) * (size_t)K * N);
    for (long i = 0; i < (long)K * N; ++i)
        Bf[i] = oracle_f16_to_f32(B[i]);
    float* arow = (float*)malloc(sizeof(float) * (size_t)K);
    for (int m = row0; m < row0 + rows; ++m) {
        for (int k = 0; k < K; ++k)
            arow[k] = oracle_f16_to_f32(A[(long)m * K + k]);
        for (int n = 0; n < N; ++n) {
            float acc = 0.f;
            for (int k = 0; k < K; ++k)
                acc += arow[k] * Bf[(long)k * N + n];
            C[(long)m * N + n] = acc;
        }
    }
    free(arow);
    free(Bf);
}

void oracle_gemm_f16_f64(const uint16_t* A, const uint16_t* B, double* C,
                         int M, int N, int K, int b_kn, int row0, int rows)
{
    (void)M;
    /* binary16 -> float lookup; each product is formed in double and summed
     * in increasing k for every output element */
    float* lut = (float*)malloc(sizeof(float) * 65536);
    for (uint32_t h = 0; h < 65536; ++h)
        lut[h] = oracle_f16_to_f32((uint16_t)h);
    double* acc = (double*)malloc(sizeof(double) * (size_t)N);
    for (int m = row0; m < row0 + rows; ++m) {
        const uint16_t* a = A + (long)m * K;
        if (b_kn) {
            for (int n = 0; n < N; ++n)
                acc[n] = 0.0;
            for (int k = 0; k < K; ++k) {
                const double av = lut[a[k]];
                const uint16_t* b = B + (long)k * N;
                for (int n = 0; n < N; ++n)
                    acc[n] += av * (double)lut[b[n]];
            }
        } else {
            for (int n = 0; n < N; ++n) {
                const uint16_t* b = B + (long)n * K;
                double s = 0.0;
                for (int k = 0; k < K; ++k)
                    s += (double)lut[a[k]] * (double)lut[b[k]];
                acc[n] = s;
            }
        }
        for (int n = 0; n < N; ++n)
            C[(long)m * N + n] = acc[n];
    }
    free(acc);
    free(lut);
}

double oracle_f8_to_f64(uint8_t v, int fmt)
{
    const int sign = (v >> 7) & 1;
    int e, m;
    double val;
    if (fmt == 0) { /* e4m3 */
        e = (v >> 3) & 0xF;
        m = v & 0x7;
        if (e == 0xF && m == 0x7)
            return NAN;
        val = e == 0 ? ldexp((double)m / 8.0, -6) : ldexp(1.0 + (double)m / 8.0, e - 7);
    } else { /* e5m2 */
        e = (v >> 2) & 0x1F;
        m = v & 0x3;
        if (e == 0x1F)
            return m ? NAN : (sign ? -INFINITY : INFINITY);
        val = e == 0 ? ldexp((double)m / 4.0, -14) : ldexp(1.0 + (double)m / 4.0, e - 15);
    }
    return sign ? -val : val;
}

void oracle_gemm_f8_f64(const uint8_t* A, const uint8_t* B, double* C, int M, int N, int K,
                        int a_fmt, int b_fmt, int b_kn, int row0, int rows)
{
    (void)M;
    double la[256], lb[256];
    for (int i = 0; i < 256; ++i) {
        la[i] = oracle_f8_to_f64((uint8_t)i, a_fmt);
        lb[i] = oracle_f8_to_f64((uint8_t)i, b_fmt);
    }
    for (int m = row0; m < row0 + rows; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k)
                acc += la[A[(long)m * K + k]] * lb[b_kn ? B[(long)k * N + n] : B[(long)n * K + k]];
            C[(long)m * N + n] = acc;
        }
}

/* int32 accumulation as in the reference; done in uint32 so that a wrap
 * (impossible for |a|,|b| <= 128 and K <= 2^17) is defined behaviour. */
void oracle_gemm_s8(const int8_t* A, const int8_t* BT, int32_t* C,
                    int M, int N, int K, int row0, int rows)
{
    (void)M;
    for (int m = row0; m < row0 + rows; ++m) {
        const int8_t* a = A + (long)m * K;
        for (int n = 0; n < N; ++n) {
            const int8_t* b = BT + (long)n * K;
            uint32_t acc = 0;
            for (int k = 0; k < K; ++k)
                acc += (uint32_t)((int32_t)a[k] * (int32_t)b[k]);
            C[(long)m * N + n] = (int32_t)acc;
        }
    }
}

void oracle_gemm_s8_kn(const int8_t* A, const int8_t* B, int32_t* C,
                       int M, int N, int K, int row0, int rows)
{
    (void)M;
    int8_t* bt = (int8_t*)malloc((size_t)K * N);
    for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n)
            bt[(long)n * K + k] = B[(long)k * N + n];
    oracle_gemm_s8(A, bt, C, M, N, K, row0, rows);
    free(bt);
}

void oracle_unpack_s4(const int8_t* packed, int8_t* out, long n_packed_bytes)
{
    for (long i = 0; i < n_packed_bytes; ++i) {
        out[2 * i] = nib_lo(packed[i]);
        out[2 * i + 1] = nib_hi(packed[i]);
    }
}

void oracle_gemm_s4(const int8_t* Ap, const int8_t* BTp, int32_t* C,
                    int M, int N, int K, int row0, int rows)
{
    (void)M;
    long kb = K / 2;
    for (int m = row0; m < row0 + rows; ++m) {
        const int8_t* a = Ap + (long)m * kb;
        for (int n = 0; n < N; ++n) {
            const int8_t* b = BTp + (long)n * kb;
            uint32_t acc = 0;
            for (long k = 0; k < kb; ++k) {
                acc += (uint32_t)((int32_t)nib_lo(a[k]) * (int32_t)nib_lo(b[k]));
                acc += (uint32_t)((int32_t)nib_hi(a[k]) * (int32_t)nib_hi(b[k]));
            }
            C[(long)m * N + n] = (int32_t)acc;
        }
    }
}

void oracle_gemm_f32(const float* A, const float* BT, float* C,
                     int M, int N, int K, int row0, int rows)
{
    (void)M;
    for (int m = row0; m < row0 + rows; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k)
                acc += (double)A[(long)m * K + k] * (double)BT[(long)n * K + k];
            C[(long)m * N + n] = (float)acc;
        }
}

/* ------------------------------------------------------------------------ */
/* Quantisation.                                                            */
/* ------------------------------------------------------------------------ */

static int8_t round_half_away(float q)
{
    return (int8_t)(int)(q >= 0.f ? q + 0.5f : q - 0.5f);
}

float oracle_quantize_absmax_s8(const float* src, int8_t* dst, long n)
{
    float absmax = 0.f;
    for (long i = 0; i < n; ++i) {
        float v = src[i] < 0.f ? -src[i] : src[i];
        if (v > absmax)
            absmax = v;
    }
    float scale = absmax / 127.f;
    float inv = (scale > 0.f) ? (1.f / scale) : 0.f;
    for (long i = 0; i < n; ++i) {
        float q = src[i] * inv;
        if (q > 127.f) q = 127.f;
        if (q < -127.f) q = -127.f;
        dst[i] = round_half_away(q);
    }
    return scale;
}

float oracle_quantize_absmax_s4(const float* src, int8_t* dst_packed, int rows, int cols_k)
{
    long n = (long)rows * cols_k;
    float absmax = 0.f;
    for (long i = 0; i < n; ++i) {
        float v = src[i] < 0.f ? -src[i] : src[i];
        if (v > absmax)
            absmax = v;
    }
    float scale = absmax / 7.f;
    float inv = (scale > 0.f) ? (1.f / scale) : 0.f;
    for (int r = 0; r < rows; ++r)
        for (int k = 0; k < cols_k; k += 2) {
            float q0 = src[(long)r * cols_k + k] * inv;
            float q1 = src[(long)r * cols_k + k + 1] * inv;
            if (q0 > 7.f) q0 = 7.f;
            if (q0 < -7.f) q0 = -7.f;
            if (q1 > 7.f) q1 = 7.f;
            if (q1 < -7.f) q1 = -7.f;
            dst_packed[(long)r * (cols_k / 2) + k / 2] = pack_pair(round_half_away(q0), round_half_away(q1));
        }
    return scale;
}

void oracle_dequantize(const int32_t* src, float* dst, long n, float scale_a, float scale_bt)
{
    float combined = scale_a * scale_bt;
    for (long i = 0; i < n; ++i)
        dst[i] = (float)src[i] * combined;
}

/* ------------------------------------------------------------------------ */
/* Accuracy metrics.                                                        */
/* ------------------------------------------------------------------------ */

oracle_acc_f32 oracle_measure_accuracy(const float* ref, const float* out, int M, int N, float pass_tol)
{
    double sse = 0, sum_rel = 0, max_abs = 0;
    long n = (long)M * N;
    for (long i = 0; i < n; ++i) {
        double diff = fabs((double)(ref[i] - out[i]));
        max_abs = fmax(max_abs, diff);
        sse += diff * diff;
        sum_rel += diff / (fabs((double)ref[i]) + 1e-6);
    }
    oracle_acc_f32 r;
    r.max_abs_err = (float)max_abs;
    r.rmse = (float)sqrt(sse / (double)n);
    r.real_err_pct = (float)(sum_rel / (double)n * 100.0);
    r.pass = r.max_abs_err < pass_tol;
    return r;
}

oracle_acc_i32 oracle_measure_accuracy_i32(const int32_t* ref, const int32_t* out, int M, int N)
{
    int64_t max_abs = 0;
    double sse = 0.0;
    long max_i = 0, n = (long)M * N;
    for (long i = 0; i < n; ++i) {
        int64_t d = (int64_t)ref[i] - (int64_t)out[i];
        int64_t ad = d < 0 ? -d : d;
        if (ad > max_abs) {
            max_abs = ad;
            max_i = i;
        }
        sse += (double)d * (double)d;
    }
    oracle_acc_i32 r;
    r.max_abs_err = (int32_t)max_abs;
    r.rmse = (float)sqrt(sse / (double)n);
    r.max_row = (int)(max_i / N);
    r.max_col = (int)(max_i % N);
    r.ref_at_max = ref[max_i];
    r.out_at_max = out[max_i];
    r.pass = (max_abs == 0);
    return r;
}

oracle_acc_quant oracle_measure_accuracy_quant(const float* ref, const float* out, int M, int N, float pass_tol)
{
    double max_abs = 0.0, sse = 0.0, sum_rel = 0.0, sig_sq = 0.0;
    long n = (long)M * N;
    for (long i = 0; i < n; ++i) {
        double d = (double)ref[i] - (double)out[i];
        double ad = d < 0.0 ? -d : d;
        if (ad > max_abs)
            max_abs = ad;
        sse += d * d;
        sig_sq += (double)ref[i] * (double)ref[i];
        sum_rel += ad / ((double)(ref[i] < 0.f ? -ref[i] : ref[i]) + 1e-6);
    }
    oracle_acc_quant r;
    r.max_abs_err = (float)max_abs;
    r.rmse = (float)sqrt(sse / (double)n);
    r.real_err_pct = (float)(sum_rel / (double)n * 100.0);
    r.snr_db = (sse > 0.0) ? (float)(10.0 * log10(sig_sq / sse)) : 999.f;
    r.pass = (r.max_abs_err < pass_tol);
    return r;
}
