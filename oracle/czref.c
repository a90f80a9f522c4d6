/* czref — CPU restatement of colizig's block-FP8 MoE expert path.
 * TEST INFRASTRUCTURE ONLY (parity oracle + timed CPU baseline); see czref.h
 * for the list of reference functions each routine restates.
 *
 * Build: oracle/Makefile  (gcc -O3 -mavx2 -mfma -ffp-contract=off).  Without
 * AVX2 the scalar branches compute the identical values lane by lane.
 */
#define _GNU_SOURCE
#include "czref.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define CZ_AVX2 1
#else
#define CZ_AVX2 0
#endif

#define BLOCK 128          /* fp8.zig:13 */
#define LANES 8            /* AVX2 f32 vector width of the reference box */
#define UNROLL 4           /* matmul.zig:58 */
#define MAX_DEQUANT_ROW 8192 /* fp8.zig:17 */
#define MIN_WORK (96u * 1024u) /* parallel.zig:21 */

size_t czref_nblk(size_t x) { return (x + BLOCK - 1) / BLOCK; } /* fp8.zig:19-21 */

/* ---- exp: restatement of Zig's @exp(f32) -------------------------------
 * x = k*ln2 + r with |r| <= ln2/2 (Cody-Waite: LN2_HI has 42 fractional bits
 * so k*LN2_HI is exact), exp(r) = sum_{n<=13} r^n/n! by Horner in double,
 * 2^k applied exactly, then one rounding to f32.  Constants are ln2 and 1/n!
 * rounded to double. */
static const double CZ_LOG2E = 0x1.71547652b82fep+0;
static const double CZ_LN2_HI = 0x1.62e42fefa3800p-1;
static const double CZ_LN2_LO = 0x1.ef35793c76730p-45;
static const double CZ_INV_FACT[14] = {
    0x1.0000000000000p+0, 0x1.0000000000000p+0, 0x1.0000000000000p-1, 0x1.5555555555555p-3,
    0x1.5555555555555p-5, 0x1.1111111111111p-7, 0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
    0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26,
    0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};

float czref_expf(float x) {
    if (x != x) return x;
    if (x > 100.0f) return INFINITY;
    if (x < -110.0f) return 0.0f;
    const double xd = (double)x;
    const double kd = rint(xd * CZ_LOG2E);
    double r = fma(-kd, CZ_LN2_HI, xd);
    r = fma(-kd, CZ_LN2_LO, r);
    double p = CZ_INV_FACT[13];
    for (int n = 12; n >= 0; --n) p = fma(p, r, CZ_INV_FACT[n]);
    return (float)ldexp(p, (int)kd);
}

void czref_expf_n(const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = czref_expf(x[i]);
}

/* activation.zig:8-20 */
float czref_sigmoid(float x) {
    if (x >= 0.0f) {
        const float z = czref_expf(-x);
        return 1.0f / (1.0f + z);
    }
    const float z = czref_expf(x);
    return z / (1.0f + z);
}

float czref_silu(float x) { return x * czref_sigmoid(x); }

/* ---- E4M3 ------------------------------------------------------------ */

/* pow2f: m * 2^k evaluated in f64, narrowed (fp8.zig:55-64). */
static float pow2f(float m, int k) {
    double r = m;
    if (k >= 0)
        for (int i = 0; i < k; ++i) r *= 2.0;
    else
        for (int i = 0; i > k; --i) r *= 0.5;
    return (float)r;
}

/* decodeE4M3 (fp8.zig:40-51). */
static float decode_e4m3(uint8_t byte) {
    const float sign = (byte & 0x80) ? -1.0f : 1.0f;
    const uint32_t ex = (byte >> 3) & 0x0f;
    const uint32_t mant = byte & 0x07;
    if (ex == 0) {
        if (mant == 0) return sign * 0.0f;
        return sign * pow2f((float)mant / 8.0f, 1 - 7);
    }
    if (ex == 0x0f && mant == 0x07) {
        uint32_t bits = 0x7fc00000u;
        float nan;
        memcpy(&nan, &bits, 4);
        return sign * nan;
    }
    const float m = 1.0f + (float)mant / 8.0f;
    return sign * pow2f(m, (int)ex - 7);
}

static float g_lut[256];
static pthread_once_t g_lut_once = PTHREAD_ONCE_INIT;
static void lut_init(void) {
    for (int b = 0; b < 256; ++b) g_lut[b] = decode_e4m3((uint8_t)b);
}
void czref_e4m3_lut(float out[256]) {
    pthread_once(&g_lut_once, lut_init);
    memcpy(out, g_lut, sizeof g_lut);
}

/* decodeLane for one lane (fp8.zig:80-106): arithmetic bit build, then * sc. */
static inline float decode_lane1(uint8_t byte, float sc) {
    const uint32_t b = byte;
    const uint32_t sign32 = (b >> 7) << 31;
    const uint32_t ex = (b >> 3) & 0x0f;
    const uint32_t mant = b & 0x07;
    const uint32_t normal_bits = sign32 | ((ex + 120) << 23) | (mant << 20);
    const float mant_f = (float)mant;
    const float sub = mant_f * 0x1p-9f;
    uint32_t subn_bits;
    memcpy(&subn_bits, &sub, 4);
    subn_bits |= sign32;
    uint32_t bits = (ex == 0) ? subn_bits : normal_bits;
    if (ex == 15 && mant == 7) bits = 0x7fc00000u;
    float v;
    memcpy(&v, &bits, 4);
    return v * sc;
}

#if CZ_AVX2
static inline __m256 decode_lane8(const uint8_t* p, __m256 sc) {
    const __m256i b = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)p));
    const __m256i sign32 = _mm256_slli_epi32(_mm256_srli_epi32(b, 7), 31);
    const __m256i ex = _mm256_and_si256(_mm256_srli_epi32(b, 3), _mm256_set1_epi32(0x0f));
    const __m256i mant = _mm256_and_si256(b, _mm256_set1_epi32(0x07));
    const __m256i normal_bits = _mm256_or_si256(
        _mm256_or_si256(sign32, _mm256_slli_epi32(_mm256_add_epi32(ex, _mm256_set1_epi32(120)), 23)),
        _mm256_slli_epi32(mant, 20));
    const __m256 mant_f = _mm256_cvtepi32_ps(mant);
    const __m256i subn_bits =
        _mm256_or_si256(_mm256_castps_si256(_mm256_mul_ps(mant_f, _mm256_set1_ps(0x1p-9f))), sign32);
    const __m256i is_sub = _mm256_cmpeq_epi32(ex, _mm256_setzero_si256());
    __m256i bits = _mm256_blendv_epi8(normal_bits, subn_bits, is_sub);
    const __m256i is_nan = _mm256_and_si256(_mm256_cmpeq_epi32(ex, _mm256_set1_epi32(15)),
                                            _mm256_cmpeq_epi32(mant, _mm256_set1_epi32(7)));
    bits = _mm256_blendv_epi8(bits, _mm256_set1_epi32(0x7fc00000), is_nan);
    return _mm256_mul_ps(_mm256_castsi256_ps(bits), sc);
}

/* @reduce(.Add, v): lanes summed 0..7 in order. */
static inline float reduce_ordered(__m256 v) {
    float t[8];
    _mm256_storeu_ps(t, v);
    float s = t[0];
    for (int l = 1; l < 8; ++l) s += t[l];
    return s;
}
#endif

/* dequantRow (fp8.zig:123-130). */
void czref_dequant_row(float* out, const uint8_t* w, const float* scale_row, size_t n) {
    pthread_once(&g_lut_once, lut_init);
    size_t i = 0;
    for (; i + LANES <= n; i += LANES) {
        const float sc = scale_row[i / BLOCK];
#if CZ_AVX2
        _mm256_storeu_ps(out + i, decode_lane8(w + i, _mm256_set1_ps(sc)));
#else
        for (int l = 0; l < LANES; ++l) out[i + l] = decode_lane1(w[i + l], sc);
#endif
    }
    for (; i < n; ++i) out[i] = g_lut[w[i]] * scale_row[i / BLOCK];
}

/* dotFp8Row (fp8.zig:137-160): two @mulAdd chains of 8 lanes. */
float czref_dot_fp8_row(const float* x, const uint8_t* w, const float* scale_row, size_t n) {
    pthread_once(&g_lut_once, lut_init);
    size_t i = 0;
#if CZ_AVX2
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    for (; i + 2 * LANES <= n; i += 2 * LANES) {
        const __m256 w0 = decode_lane8(w + i, _mm256_set1_ps(scale_row[i / BLOCK]));
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), w0, acc0);
        const __m256 w1 = decode_lane8(w + i + LANES, _mm256_set1_ps(scale_row[(i + LANES) / BLOCK]));
        acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i + LANES), w1, acc1);
    }
    for (; i + LANES <= n; i += LANES) {
        const __m256 wv = decode_lane8(w + i, _mm256_set1_ps(scale_row[i / BLOCK]));
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), wv, acc0);
    }
    float sum = reduce_ordered(_mm256_add_ps(acc0, acc1));
#else
    float acc0[LANES] = {0}, acc1[LANES] = {0};
    for (; i + 2 * LANES <= n; i += 2 * LANES) {
        const float sc0 = scale_row[i / BLOCK], sc1 = scale_row[(i + LANES) / BLOCK];
        for (int l = 0; l < LANES; ++l) acc0[l] = fmaf(x[i + l], decode_lane1(w[i + l], sc0), acc0[l]);
        for (int l = 0; l < LANES; ++l)
            acc1[l] = fmaf(x[i + LANES + l], decode_lane1(w[i + LANES + l], sc1), acc1[l]);
    }
    for (; i + LANES <= n; i += LANES) {
        const float sc = scale_row[i / BLOCK];
        for (int l = 0; l < LANES; ++l) acc0[l] = fmaf(x[i + l], decode_lane1(w[i + l], sc), acc0[l]);
    }
    float sum = acc0[0] + acc1[0];
    for (int l = 1; l < LANES; ++l) sum += acc0[l] + acc1[l];
#endif
    for (; i < n; ++i) sum += x[i] * (g_lut[w[i]] * scale_row[i / BLOCK]);
    return sum;
}

/* dotF32 (matmul.zig:60-82): 4 @mulAdd chains x 8 lanes, total = ((a0+a1)+a2)+a3,
 * ordered lane reduce, then a scalar @mulAdd tail. */
float czref_dot_f32(const float* a, const float* b, size_t n) {
    size_t i = 0;
#if CZ_AVX2
    __m256 acc[UNROLL];
    for (int k = 0; k < UNROLL; ++k) acc[k] = _mm256_setzero_ps();
    for (; i + UNROLL * LANES <= n; i += UNROLL * LANES)
        for (int k = 0; k < UNROLL; ++k)
            acc[k] = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + k * LANES), _mm256_loadu_ps(b + i + k * LANES),
                                     acc[k]);
    for (; i + LANES <= n; i += LANES)
        acc[0] = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc[0]);
    __m256 total = _mm256_setzero_ps();
    for (int k = 0; k < UNROLL; ++k) total = _mm256_add_ps(total, acc[k]);
    float sum = reduce_ordered(total);
#else
    float acc[UNROLL][LANES];
    memset(acc, 0, sizeof acc);
    for (; i + UNROLL * LANES <= n; i += UNROLL * LANES)
        for (int k = 0; k < UNROLL; ++k)
            for (int l = 0; l < LANES; ++l)
                acc[k][l] = fmaf(a[i + k * LANES + l], b[i + k * LANES + l], acc[k][l]);
    for (; i + LANES <= n; i += LANES)
        for (int l = 0; l < LANES; ++l) acc[0][l] = fmaf(a[i + l], b[i + l], acc[0][l]);
    float total[LANES] = {0};
    for (int k = 0; k < UNROLL; ++k)
        for (int l = 0; l < LANES; ++l) total[l] += acc[k][l];
    float sum = total[0];
    for (int l = 1; l < LANES; ++l) sum += total[l];
#endif
    for (; i < n; ++i) sum = fmaf(a[i], b[i], sum);
    return sum;
}

/* ---- parallel.chunks (parallel.zig:50-76) ------------------------------
 * A persistent pool of (threads - 1) workers plus the calling thread.  `body`
 * runs on contiguous ranges [lo, hi) of size ceil(n / tasks). */
typedef void (*chunk_body)(void* ctx, size_t lo, size_t hi);

static struct {
    pthread_mutex_t mu;
    pthread_cond_t cv_work;
    pthread_cond_t cv_done;
    int max_tasks;
    int nworkers;
    pthread_t* th;
    unsigned gen;
    chunk_body fn;
    void* ctx;
    size_t n, csize, nchunks;
    atomic_size_t next;
    atomic_size_t done;
} g_pool = {.mu = PTHREAD_MUTEX_INITIALIZER,
            .cv_work = PTHREAD_COND_INITIALIZER,
            .cv_done = PTHREAD_COND_INITIALIZER,
            .max_tasks = 1};

static __thread int t_in_worker = 0;

static void run_chunks(void) {
    for (;;) {
        const size_t c = atomic_fetch_add(&g_pool.next, 1);
        if (c >= g_pool.nchunks) break;
        const size_t lo = c * g_pool.csize;
        size_t hi = lo + g_pool.csize;
        if (hi > g_pool.n) hi = g_pool.n;
        t_in_worker = 1;
        g_pool.fn(g_pool.ctx, lo, hi);
        t_in_worker = 0;
        if (atomic_fetch_add(&g_pool.done, 1) + 1 == g_pool.nchunks) {
            pthread_mutex_lock(&g_pool.mu);
            pthread_cond_broadcast(&g_pool.cv_done);
            pthread_mutex_unlock(&g_pool.mu);
        }
    }
}

static void* worker_main(void* arg) {
    (void)arg;
    unsigned seen = 0;
    pthread_mutex_lock(&g_pool.mu);
    for (;;) {
        while (g_pool.gen == seen) pthread_cond_wait(&g_pool.cv_work, &g_pool.mu);
        seen = g_pool.gen;
        if (g_pool.fn == NULL) break; /* shutdown */
        pthread_mutex_unlock(&g_pool.mu);
        run_chunks();
        pthread_mutex_lock(&g_pool.mu);
    }
    pthread_mutex_unlock(&g_pool.mu);
    return NULL;
}

static void pool_stop(void) {
    if (g_pool.nworkers == 0) return;
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = NULL;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv_work);
    pthread_mutex_unlock(&g_pool.mu);
    for (int i = 0; i < g_pool.nworkers; ++i) pthread_join(g_pool.th[i], NULL);
    free(g_pool.th);
    g_pool.th = NULL;
    g_pool.nworkers = 0;
}

void czref_set_threads(int n) {
    pool_stop();
    g_pool.max_tasks = n > 1 ? n : 1;
    if (g_pool.max_tasks > 1) {
        g_pool.th = (pthread_t*)calloc((size_t)g_pool.max_tasks - 1, sizeof(pthread_t));
        for (int i = 0; i < g_pool.max_tasks - 1; ++i) {
            if (pthread_create(&g_pool.th[i], NULL, worker_main, NULL) != 0) break;
            g_pool.nworkers++;
        }
    }
}

int czref_get_threads(void) { return g_pool.max_tasks; }

static void chunks(size_t n, size_t work, void* ctx, chunk_body body) {
    if (n == 0) return;
    if (g_pool.max_tasks <= 1) {
        body(ctx, 0, n);
        return;
    }
    const size_t tasks = (size_t)g_pool.max_tasks < n ? (size_t)g_pool.max_tasks : n;
    if (tasks <= 1 || work < MIN_WORK || t_in_worker) {
        body(ctx, 0, n);
        return;
    }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = body;
    g_pool.ctx = ctx;
    g_pool.n = n;
    g_pool.csize = (n + tasks - 1) / tasks;
    g_pool.nchunks = (n + g_pool.csize - 1) / g_pool.csize;
    atomic_store(&g_pool.next, 0);
    atomic_store(&g_pool.done, 0);
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv_work);
    pthread_mutex_unlock(&g_pool.mu);
    run_chunks();
    pthread_mutex_lock(&g_pool.mu);
    while (atomic_load(&g_pool.done) < g_pool.nchunks) pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
}

/* ---- matmuls -------------------------------------------------------------- */

typedef struct {
    float* y;
    const float* x;
    const float* w;
    size_t S, I, O;
} mm_ctx;

static void mm_body(void* p, size_t o0, size_t o1) {
    const mm_ctx* c = (const mm_ctx*)p;
    for (size_t o = o0; o < o1; ++o) {
        const float* wr = c->w + o * c->I;
        for (size_t s = 0; s < c->S; ++s) c->y[s * c->O + o] = czref_dot_f32(c->x + s * c->I, wr, c->I);
    }
}

/* matmul.zig:21-33 */
void czref_matmul_f32(float* y, const float* x, const float* w, size_t S, size_t I, size_t O) {
    mm_ctx c = {y, x, w, S, I, O};
    chunks(O, O * I * S, &c, mm_body);
}

/* bf16ToF32 (matmul.zig:108-110): bf16 is the top half of an f32. */
static inline float bf16_f32(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* dotBf16 (matmul.zig:84-106): dotF32's 4 FMA chains x 8 lanes, each weight lane
 * widened exactly (bits << 16), then the same ordered reduction and FMA tail. */
float czref_dot_bf16(const float* a, const uint16_t* b, size_t n) {
    size_t i = 0;
#if CZ_AVX2
    __m256 acc[UNROLL];
    for (int k = 0; k < UNROLL; ++k) acc[k] = _mm256_setzero_ps();
#define CZ_WIDEN(p) _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(_mm_loadu_si128((const __m128i*)(p))), 16))
    for (; i + UNROLL * LANES <= n; i += UNROLL * LANES)
        for (int k = 0; k < UNROLL; ++k)
            acc[k] = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + k * LANES), CZ_WIDEN(b + i + k * LANES), acc[k]);
    for (; i + LANES <= n; i += LANES) acc[0] = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), CZ_WIDEN(b + i), acc[0]);
#undef CZ_WIDEN
    __m256 total = _mm256_setzero_ps();
    for (int k = 0; k < UNROLL; ++k) total = _mm256_add_ps(total, acc[k]);
    float sum = reduce_ordered(total);
#else
    float acc[UNROLL][LANES];
    memset(acc, 0, sizeof acc);
    for (; i + UNROLL * LANES <= n; i += UNROLL * LANES)
        for (int k = 0; k < UNROLL; ++k)
            for (int l = 0; l < LANES; ++l)
                acc[k][l] = fmaf(a[i + k * LANES + l], bf16_f32(b[i + k * LANES + l]), acc[k][l]);
    for (; i + LANES <= n; i += LANES)
        for (int l = 0; l < LANES; ++l) acc[0][l] = fmaf(a[i + l], bf16_f32(b[i + l]), acc[0][l]);
    float total[LANES] = {0};
    for (int k = 0; k < UNROLL; ++k)
        for (int l = 0; l < LANES; ++l) total[l] += acc[k][l];
    float sum = total[0];
    for (int l = 1; l < LANES; ++l) sum += total[l];
#endif
    for (; i < n; ++i) sum = fmaf(a[i], bf16_f32(b[i]), sum);
    return sum;
}

typedef struct {
    float* y;
    const float* x;
    const uint16_t* w;
    size_t S, I, O;
} mmb_ctx;

static void mmb_body(void* p, size_t o0, size_t o1) {
    const mmb_ctx* c = (const mmb_ctx*)p;
    for (size_t o = o0; o < o1; ++o) {
        const uint16_t* wr = c->w + o * c->I;
        for (size_t s = 0; s < c->S; ++s) c->y[s * c->O + o] = czref_dot_bf16(c->x + s * c->I, wr, c->I);
    }
}

/* matmulBf16 (matmul.zig:36-48): y[S,O] = x[S,I] @ w[O,I]^T, fan-out over O rows. */
void czref_matmul_bf16(float* y, const float* x, const uint16_t* w, size_t S, size_t I, size_t O) {
    mmb_ctx c = {y, x, w, S, I, O};
    chunks(O, O * I * S, &c, mmb_body);
}

typedef struct {
    float* y;
    const float* x;
    const uint8_t* w;
    const float* scales;
    size_t S, I, O, nbi;
} fp8_ctx;

static void fp8_decode_body(void* p, size_t o0, size_t o1) {
    const fp8_ctx* c = (const fp8_ctx*)p;
    for (size_t o = o0; o < o1; ++o)
        c->y[o] = czref_dot_fp8_row(c->x, c->w + o * c->I, c->scales + (o / BLOCK) * c->nbi, c->I);
}

static void fp8_prefill_body(void* p, size_t o0, size_t o1) {
    const fp8_ctx* c = (const fp8_ctx*)p;
    float rowbuf[MAX_DEQUANT_ROW];
    for (size_t o = o0; o < o1; ++o) {
        czref_dequant_row(rowbuf, c->w + o * c->I, c->scales + (o / BLOCK) * c->nbi, c->I);
        for (size_t s = 0; s < c->S; ++s) c->y[s * c->O + o] = czref_dot_f32(c->x + s * c->I, rowbuf, c->I);
    }
}

/* matmulFp8Cpu (fp8.zig:215-257). */
void czref_matmul_fp8(float* y, const float* x, const uint8_t* w, const float* scales, size_t S, size_t I,
                      size_t O) {
    fp8_ctx c = {y, x, w, scales, S, I, O, czref_nblk(I)};
    if (S == 1) {
        chunks(O, O * I, &c, fp8_decode_body);
        return;
    }
    if (I > MAX_DEQUANT_ROW) return; /* asserted by the reference (fp8.zig:178) */
    chunks(O, O * I * S, &c, fp8_prefill_body);
}

/* rmsnorm.zig:32-40 rms: f64 sum of squares, mean narrowed to f32, then
 * r = 1/sqrt(mean + eps) and out = v * r * w (two f32 multiplies). */
void czref_rms(float* out, const float* x, const float* w, size_t n, float eps) {
    double ss = 0;
    for (size_t i = 0; i < n; ++i) ss += (double)x[i] * x[i];
    const float mean = (float)(ss / (double)n);
    const float r = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * r * w[i];
}

/* ---- MoE layer (moe.zig) ----------------------------------------------- */

/* route (moe.zig:435-463).  `logits` is [E] scratch. */
static void route(const czref_layer* L, const czref_dims* d, const float* xs, float* logits, uint32_t* idx,
                  float* gates) {
    const size_t E = d->experts, K = d->topk;
    czref_matmul_f32(logits, xs, L->router, 1, d->hidden, E);
    float mx = logits[0];
    for (size_t e = 0; e < E; ++e) mx = fmaxf(mx, logits[e]); /* @max: NaN-ignoring */
    double all = 0;
    for (size_t e = 0; e < E; ++e) {
        logits[e] = czref_expf(logits[e] - mx);
        all += logits[e];
    }
    double top = 0;
    for (size_t z = 0; z < K; ++z) {
        size_t best = 0;
        float bv = -1.0f;
        for (size_t e = 0; e < E; ++e) {
            int chosen = 0;
            for (size_t j = 0; j < z; ++j) chosen = chosen || (idx[j] == e);
            if (!chosen && logits[e] > bv) {
                bv = logits[e];
                best = e;
            }
        }
        idx[z] = (uint32_t)best;
        top += logits[best];
    }
    const double den = d->norm_topk ? top : all;
    for (size_t z = 0; z < K; ++z) gates[z] = (float)((double)logits[idx[z]] / den);
}

void czref_route(const czref_layer* L, const czref_dims* d, const float* xs, uint32_t* idx, float* gates) {
    float* logits = (float*)malloc(d->experts * sizeof(float));
    route(L, d, xs, logits, idx, gates);
    free(logits);
}

typedef struct {
    float *logits, *sg, *su, *sh, *shared, *eg, *eu, *eh, *eo;
    uint32_t* idx;
    float* gates;
    uint32_t *r_idx, *ord;
    float *r_gate, *xb, *bg, *bu, *bo;
} scratch;

static int has_shared(const czref_dims* d) { return d->shared_inter != 0; }

/* addSharedExpert (moe.zig:467-479): block-FP8 shared projections, or the
 * reference's own BF16 NativeMatrix projections (matmulBf16) when given. */
static void add_shared(const czref_layer* L, const czref_dims* d, const float* xs, float* ys, scratch* sc) {
    if (!has_shared(d)) return;
    const size_t H = d->hidden, SI = d->shared_inter;
    if (L->sh_gate_bf16) {
        czref_matmul_bf16(sc->sg, xs, L->sh_gate_bf16, 1, H, SI);
        czref_matmul_bf16(sc->su, xs, L->sh_up_bf16, 1, H, SI);
    } else {
        czref_matmul_fp8(sc->sg, xs, L->sh_gate_w, L->sh_gate_s, 1, H, SI);
        czref_matmul_fp8(sc->su, xs, L->sh_up_w, L->sh_up_s, 1, H, SI);
    }
    for (size_t j = 0; j < SI; ++j) sc->sh[j] = czref_silu(sc->sg[j]) * sc->su[j];
    if (L->sh_gate_bf16)
        czref_matmul_bf16(sc->shared, sc->sh, L->sh_down_bf16, 1, SI, H);
    else
        czref_matmul_fp8(sc->shared, sc->sh, L->sh_down_w, L->sh_down_s, 1, SI, H);
    float sgate = 0;
    for (size_t dd = 0; dd < H; ++dd) sgate += xs[dd] * L->sh_gate[dd];
    sgate = czref_sigmoid(sgate);
    for (size_t dd = 0; dd < H; ++dd) ys[dd] += sgate * sc->shared[dd];
}

/* evalExpertBody (moe.zig:557-572): one expert per z, output row scaled by its gate. */
typedef struct {
    const czref_layer* L;
    const czref_dims* d;
    const float* xs;
    scratch* sc;
} eval_ctx;

static void eval_body(void* p, size_t z0, size_t z1) {
    const eval_ctx* c = (const eval_ctx*)p;
    const size_t H = c->d->hidden, I = c->d->inter;
    for (size_t z = z0; z < z1; ++z) {
        const uint32_t e = c->sc->idx[z];
        float* eg = c->sc->eg + z * I;
        float* eu = c->sc->eu + z * I;
        float* eh = c->sc->eh + z * I;
        float* eo = c->sc->eo + z * H;
        czref_matmul_fp8(eg, c->xs, c->L->gate_w[e], c->L->gate_s[e], 1, H, I);
        czref_matmul_fp8(eu, c->xs, c->L->up_w[e], c->L->up_s[e], 1, H, I);
        for (size_t j = 0; j < I; ++j) eh[j] = czref_silu(eg[j]) * eu[j];
        czref_matmul_fp8(eo, eh, c->L->down_w[e], c->L->down_s[e], 1, I, H);
        const float g = c->sc->gates[z];
        for (size_t dd = 0; dd < H; ++dd) eo[dd] *= g;
    }
}

/* forwardDense (moe.zig:481-539).  With no GPU and a cache holding every expert,
 * the reference fans the K experts out over threads (par = true); the result is
 * bit-identical to its serial loop. */
static void forward_dense(const czref_layer* L, const czref_dims* d, const float* x, size_t S, float* out,
                          scratch* sc, uint32_t* idx_out, float* gates_out) {
    const size_t H = d->hidden, K = d->topk, I = d->inter;
    for (size_t s = 0; s < S; ++s) {
        const float* xs = x + s * H;
        float* ys = out + s * H;
        memset(ys, 0, H * sizeof(float));
        route(L, d, xs, sc->logits, sc->idx, sc->gates);
        if (idx_out) memcpy(idx_out + s * K, sc->idx, K * sizeof(uint32_t));
        if (gates_out) memcpy(gates_out + s * K, sc->gates, K * sizeof(float));
        eval_ctx c = {L, d, xs, sc};
        chunks(K, K * 3 * I * H, &c, eval_body);
        for (size_t z = 0; z < K; ++z) {
            const float* eo = sc->eo + z * H;
            for (size_t dd = 0; dd < H; ++dd) ys[dd] += eo[dd];
        }
        add_shared(L, d, xs, ys, sc);
    }
}

/* forwardGrouped (moe.zig:597-665).  The reference orders the (token, slot)
 * pairs with std.sort.pdq by expert id; pairs of one expert never share a token,
 * so the order inside a group does not change any output.  A stable counting
 * order (ascending expert, then token, then slot) is used here. */
static void forward_grouped(const czref_layer* L, const czref_dims* d, const float* x, size_t S, float* out,
                            scratch* sc, uint32_t* idx_out, float* gates_out) {
    const size_t H = d->hidden, K = d->topk, I = d->inter, E = d->experts;
    for (size_t s = 0; s < S; ++s) {
        const float* xs = x + s * H;
        float* ys = out + s * H;
        memset(ys, 0, H * sizeof(float));
        route(L, d, xs, sc->logits, sc->idx, sc->gates);
        for (size_t z = 0; z < K; ++z) {
            sc->r_idx[s * K + z] = sc->idx[z];
            sc->r_gate[s * K + z] = sc->gates[z];
        }
        add_shared(L, d, xs, ys, sc);
    }
    if (idx_out) memcpy(idx_out, sc->r_idx, S * K * sizeof(uint32_t));
    if (gates_out) memcpy(gates_out, sc->r_gate, S * K * sizeof(float));

    const size_t M = S * K;
    size_t* cnt = (size_t*)calloc(E + 1, sizeof(size_t));
    for (size_t i = 0; i < M; ++i) cnt[sc->r_idx[i] + 1]++;
    for (size_t e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
    for (size_t i = 0; i < M; ++i) sc->ord[cnt[sc->r_idx[i]]++] = (uint32_t)i;
    free(cnt);

    size_t p = 0;
    while (p < M) {
        const uint32_t eid = sc->r_idx[sc->ord[p]];
        size_t q = p;
        while (q < M && sc->r_idx[sc->ord[q]] == eid) q++;
        const size_t n = q - p;
        for (size_t k = 0; k < n; ++k) {
            const size_t tok = sc->ord[p + k] / K;
            memcpy(sc->xb + k * H, x + tok * H, H * sizeof(float));
        }
        czref_matmul_fp8(sc->bg, sc->xb, L->gate_w[eid], L->gate_s[eid], n, H, I);
        czref_matmul_fp8(sc->bu, sc->xb, L->up_w[eid], L->up_s[eid], n, H, I);
        for (size_t j = 0; j < n * I; ++j) sc->bg[j] = czref_silu(sc->bg[j]) * sc->bu[j];
        czref_matmul_fp8(sc->bo, sc->bg, L->down_w[eid], L->down_s[eid], n, I, H);
        for (size_t k = 0; k < n; ++k) {
            const uint32_t slot = sc->ord[p + k];
            const size_t tok = slot / K;
            const float g = sc->r_gate[slot];
            float* ys = out + tok * H;
            const float* eo = sc->bo + k * H;
            for (size_t dd = 0; dd < H; ++dd) ys[dd] += g * eo[dd];
        }
        p = q;
    }
}

int czref_moe_forward(const czref_layer* L, const czref_dims* d, const float* x, size_t S, float* out,
                      uint32_t* idx_out, float* gates_out) {
    if (!L || !d || !x || !out || S == 0 || d->topk == 0 || d->topk > d->experts || d->hidden == 0 ||
        d->inter == 0)
        return -1;
    if (d->topk > 64) return -1;
    const size_t H = d->hidden, K = d->topk, I = d->inter, E = d->experts, SI = d->shared_inter;
    const size_t T = S;
    scratch sc;
    sc.logits = (float*)malloc(E * sizeof(float));
    sc.sg = (float*)malloc((SI + 1) * sizeof(float));
    sc.su = (float*)malloc((SI + 1) * sizeof(float));
    sc.sh = (float*)malloc((SI + 1) * sizeof(float));
    sc.shared = (float*)malloc(H * sizeof(float));
    sc.eg = (float*)malloc(K * I * sizeof(float));
    sc.eu = (float*)malloc(K * I * sizeof(float));
    sc.eh = (float*)malloc(K * I * sizeof(float));
    sc.eo = (float*)malloc(K * H * sizeof(float));
    sc.idx = (uint32_t*)malloc(K * sizeof(uint32_t));
    sc.gates = (float*)malloc(K * sizeof(float));
    sc.r_idx = (uint32_t*)malloc(T * K * sizeof(uint32_t));
    sc.ord = (uint32_t*)malloc(T * K * sizeof(uint32_t));
    sc.r_gate = (float*)malloc(T * K * sizeof(float));
    /* The reference sizes these [max_tokens, *] (moe.zig:353-361), which holds
     * because a token never picks an expert twice.  When every logit is NaN the
     * reference picks id 0 in every round (moe.zig:447-460) and one group gets
     * S*K rows, overflowing that scratch; S*K rows keep the restatement defined. */
    sc.xb = (float*)malloc(T * K * H * sizeof(float));
    sc.bg = (float*)malloc(T * K * I * sizeof(float));
    sc.bu = (float*)malloc(T * K * I * sizeof(float));
    sc.bo = (float*)malloc(T * K * H * sizeof(float));
    if (S == 1)
        forward_dense(L, d, x, S, out, &sc, idx_out, gates_out);
    else
        forward_grouped(L, d, x, S, out, &sc, idx_out, gates_out);
    free(sc.logits);
    free(sc.sg);
    free(sc.su);
    free(sc.sh);
    free(sc.shared);
    free(sc.eg);
    free(sc.eu);
    free(sc.eh);
    free(sc.eo);
    free(sc.idx);
    free(sc.gates);
    free(sc.r_idx);
    free(sc.ord);
    free(sc.r_gate);
    free(sc.xb);
    free(sc.bg);
    free(sc.bu);
    free(sc.bo);
    return 0;
}
