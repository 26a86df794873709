/* cpu_blocked.c -- cache-blocked, multi-threaded CPU GEMMs: the host-core
 * baseline reported beside the B200 numbers (baseline and test infrastructure,
 * never on the product path).
 *
 * The reference's own CPU GEMMs are naive triple loops, one thread
 * (src/data.cu:16-24 cpu_gemm_fp16, src/data_int8.cu:18-26 cpu_gemm_int8,
 * src/data_int4.cu:46-61 cpu_gemm_int4).  These compute the same products
 * with the work a tuned host GEMM does: threads over output tiles, K split
 * into chunks that stay in the core's L2, and an AVX2 register-blocked inner
 * kernel (int8: 2 x 4 dot products of 16 sign-extended bytes per step with
 * vpmaddwd, exact int32; fp16: operands widened to fp32 once, then FMA rows
 * of C in i-k-j order).  Integer results are exact (equal to the reference's
 * cpu_gemm_int8 / cpu_gemm_int4); the fp16 one sums in another order than the
 * reference's loop and is within the fp16 tolerance of an fp64 GEMM.
 *
 * Layouts follow the reference: A M x K row-major; int8/int4 B given as BT
 * (N x K, K contiguous); int4 packed two per byte along K, low nibble = even k
 * (src/data_int4.h:4-6); fp16 B is K x N row-major; C M x N row-major.
 */
#include <immintrin.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- a minimal parallel-for: `threads` workers take indices [0, n) in
 * order from a shared counter (dynamic scheduling). */
typedef void (*body_fn)(long i, void* ctx);
typedef struct {
    long n;
    long next;
    pthread_mutex_t mu;
    body_fn fn;
    void* ctx;
} pfor_t;

static void* pfor_worker(void* arg)
{
    pfor_t* p = (pfor_t*)arg;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        const long i = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (i >= p->n) return NULL;
        p->fn(i, p->ctx);
    }
}

static void parallel_for(long n, int threads, body_fn fn, void* ctx)
{
    pfor_t p;
    p.n = n;
    p.next = 0;
    p.fn = fn;
    p.ctx = ctx;
    pthread_mutex_init(&p.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    int started = 0;
    for (int t = 1; t < threads; ++t)
        if (pthread_create(&tid[started], NULL, pfor_worker, &p) == 0) ++started;
    pfor_worker(&p);
    for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
    pthread_mutex_destroy(&p.mu);
}

#define TILE_M 64
#define TILE_N 64
#define TILE_K 2048

static int32_t hsum8(__m256i v)
{
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}

/* C[i][j] += sum_{k < kc} a[i][k] * b[j][k] for the 2 x 4 block at a, b
 * (row strides lda / ldb bytes); kc a multiple of 16. */
static void micro_2x4(const int8_t* a, const int8_t* b, long lda, long ldb, int kc, int32_t* c, long ldc)
{
    __m256i acc[8];
    for (int i = 0; i < 8; ++i) acc[i] = _mm256_setzero_si256();
    for (int k = 0; k < kc; k += 16) {
        const __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + k)));
        const __m256i a1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + lda + k)));
        for (int j = 0; j < 4; ++j) {
            const __m256i bj = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + j * ldb + k)));
            acc[j] = _mm256_add_epi32(acc[j], _mm256_madd_epi16(a0, bj));
            acc[4 + j] = _mm256_add_epi32(acc[4 + j], _mm256_madd_epi16(a1, bj));
        }
    }
    for (int j = 0; j < 4; ++j) {
        c[j] += hsum8(acc[j]);
        c[ldc + j] += hsum8(acc[4 + j]);
    }
}

static int32_t dot_s8(const int8_t* a, const int8_t* b, int n)
{
    int32_t s = 0;
    for (int k = 0; k < n; ++k) s += (int32_t)a[k] * (int32_t)b[k];
    return s;
}

/* One output tile, all of K in chunks of TILE_K. */
static void tile_s8(const int8_t* A, const int8_t* BT, int32_t* C, int N, int K, int i0, int i1, int j0, int j1)
{
    for (int i = i0; i < i1; ++i) memset(C + (long)i * N + j0, 0, sizeof(int32_t) * (size_t)(j1 - j0));
    const int kv = K & ~15;
    for (int k0 = 0; k0 < kv; k0 += TILE_K) {
        const int kc = (kv - k0) < TILE_K ? (kv - k0) : TILE_K;
        int i = i0;
        for (; i + 2 <= i1; i += 2) {
            int j = j0;
            for (; j + 4 <= j1; j += 4)
                micro_2x4(A + (long)i * K + k0, BT + (long)j * K + k0, K, K, kc, C + (long)i * N + j, N);
            for (; j < j1; ++j)
                for (int r = 0; r < 2; ++r)
                    C[(long)(i + r) * N + j] += dot_s8(A + (long)(i + r) * K + k0, BT + (long)j * K + k0, kc);
        }
        for (; i < i1; ++i)
            for (int j = j0; j < j1; ++j) C[(long)i * N + j] += dot_s8(A + (long)i * K + k0, BT + (long)j * K + k0, kc);
    }
    if (kv < K)
        for (int i = i0; i < i1; ++i)
            for (int j = j0; j < j1; ++j) C[(long)i * N + j] += dot_s8(A + (long)i * K + kv, BT + (long)j * K + kv, K - kv);
}

typedef struct {
    const int8_t* A;
    const int8_t* BT;
    int32_t* C;
    int M, N, K, tn;
} s8_ctx;

static void s8_tile_body(long t, void* v)
{
    const s8_ctx* c = (const s8_ctx*)v;
    const int i0 = (int)(t / c->tn) * TILE_M, j0 = (int)(t % c->tn) * TILE_N;
    const int i1 = i0 + TILE_M < c->M ? i0 + TILE_M : c->M, j1 = j0 + TILE_N < c->N ? j0 + TILE_N : c->N;
    tile_s8(c->A, c->BT, c->C, c->N, c->K, i0, i1, j0, j1);
}

void cpu_blocked_gemm_s8(const int8_t* A, const int8_t* BT, int32_t* C, int M, int N, int K, int threads)
{
    s8_ctx c = {A, BT, C, M, N, K, (N + TILE_N - 1) / TILE_N};
    parallel_for((long)((M + TILE_M - 1) / TILE_M) * c.tn, threads, s8_tile_body, &c);
}

/* Packed int4 rows (K/2 bytes each) widened to int8, low nibble first. */
typedef struct {
    const int8_t* in;
    int8_t* out;
    int K;
} widen_ctx;

static void widen_body(long r, void* v)
{
    const widen_ctx* c = (const widen_ctx*)v;
    const long half = c->K / 2;
    for (long k = 0; k < half; ++k) {
        const int8_t x = c->in[r * half + k];
        c->out[r * c->K + 2 * k] = (int8_t)((int8_t)(x << 4) >> 4);
        c->out[r * c->K + 2 * k + 1] = (int8_t)(x >> 4);
    }
}

static void widen_rows(const int8_t* in, int8_t* out, long rows, int K, int threads)
{
    widen_ctx c = {in, out, K};
    parallel_for(rows, threads, widen_body, &c);
}

/* int4: both operands widened once (part of the timed work), then the int8
 * kernel.  Returns 0, or -1 when the scratch cannot be allocated. */
int cpu_blocked_gemm_s4(const int8_t* A_packed, const int8_t* BT_packed, int32_t* C, int M, int N, int K,
                        int threads)
{
    int8_t* a8 = (int8_t*)malloc((size_t)M * K);
    int8_t* b8 = (int8_t*)malloc((size_t)N * K);
    if (!a8 || !b8) {
        free(a8);
        free(b8);
        return -1;
    }
    widen_rows(A_packed, a8, M, K, threads);
    widen_rows(BT_packed, b8, N, K, threads);
    cpu_blocked_gemm_s8(a8, b8, C, M, N, K, threads);
    free(a8);
    free(b8);
    return 0;
}

/* fp16 (IEEE half bits) -> fp32, exact. */
static float half_to_float(uint16_t h)
{
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0x1F) {
        bits = s | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = s | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = s;
    } else {  /* subnormal: normalise */
        e = 113;
        while (!(m & 0x400u)) {
            m <<= 1;
            --e;
        }
        bits = s | (e << 23) | ((m & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

typedef struct {
    const uint16_t* src;
    float* dst;
    long n;
} cvt_ctx;

static void cvt_body(long blk, void* v)
{
    const cvt_ctx* c = (const cvt_ctx*)v;
    const long x1 = (blk + 1) * 65536 < c->n ? (blk + 1) * 65536 : c->n;
    for (long x = blk * 65536; x < x1; ++x) c->dst[x] = half_to_float(c->src[x]);
}

static void widen_half(const uint16_t* src, float* dst, long n, int threads)
{
    cvt_ctx c = {src, dst, n};
    parallel_for((n + 65535) / 65536, threads, cvt_body, &c);
}

typedef struct {
    const float* af;
    const float* bf;
    float* C;
    int M, N, K, tn;
} f16_ctx;

#define F16_BM 32
#define F16_BN 256
#define F16_BK 256

static void f16_tile_body(long t, void* v)
{
    const f16_ctx* p = (const f16_ctx*)v;
    const int M = p->M, N = p->N, K = p->K;
    const int i0 = (int)(t / p->tn) * F16_BM, j0 = (int)(t % p->tn) * F16_BN;
    const int i1 = i0 + F16_BM < M ? i0 + F16_BM : M, j1 = j0 + F16_BN < N ? j0 + F16_BN : N;
    for (int i = i0; i < i1; ++i) memset(p->C + (long)i * N + j0, 0, sizeof(float) * (size_t)(j1 - j0));
    for (int k0 = 0; k0 < K; k0 += F16_BK) {
        const int k1 = k0 + F16_BK < K ? k0 + F16_BK : K;
        for (int i = i0; i < i1; ++i) {
            float* c = p->C + (long)i * N;
            for (int k = k0; k < k1; ++k) {
                const float a = p->af[(long)i * K + k];
                const float* b = p->bf + (long)k * N;
                for (int j = j0; j < j1; ++j) c[j] += a * b[j];
            }
        }
    }
}

/* fp16 inputs, fp32 accumulation and output: C = A (M x K) * B (K x N). */
int cpu_blocked_gemm_f16(const uint16_t* A, const uint16_t* B, float* C, int M, int N, int K, int threads)
{
    float* af = (float*)malloc(sizeof(float) * (size_t)M * K);
    float* bf = (float*)malloc(sizeof(float) * (size_t)K * N);
    if (!af || !bf) {
        free(af);
        free(bf);
        return -1;
    }
    widen_half(A, af, (long)M * K, threads);
    widen_half(B, bf, (long)K * N, threads);
    f16_ctx c = {af, bf, C, M, N, K, (N + F16_BN - 1) / F16_BN};
    parallel_for((long)((M + F16_BM - 1) / F16_BM) * c.tn, threads, f16_tile_body, &c);
    free(af);
    free(bf);
    return 0;
}
