/*
 * TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's CPU GEMV path,
 * used as the timed CPU baseline (bench.py --impl reference, cpu_baseline)
 * and as a second checker.  Never linked into libcudalab_gemv.so.
 *
 * It performs the reference's two CPU steps (cudalab/int4gemv_correctness.py:
 * 220-221 and cudalab/qgemv_quantize.py:67-70):
 *   1. dequantise the whole weight matrix to fp32
 *      (int4: unpack(W_packed) * fp16 scale, cudalab/int4gemv_quantize.py:137-149;
 *       int8: W_q * fp32 scale[n]),
 *   2. y = fp16(W_dequant @ fp32(x)) with fp32 accumulation,
 * each parallelised over rows with POSIX threads (the reference's torch CPU
 * kernels are multi-threaded too).
 *
 * binary16 <-> binary32 conversions are written out from the IEEE-754
 * definitions (exact decode; round-to-nearest-even encode).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

static float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal: m * 2^-24, exact in binary32 */
            float v = (float)m * (1.0f / 16777216.0f);
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) /* rounds to >= 65520: overflow to inf */
        return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) { /* below 2^-14: subnormal half (or zero) */
        float a;
        memcpy(&a, &ax, 4);
        /* a * 2^24 is exact; nearbyintf rounds half to even in the default mode */
        const float q = nearbyintf(a * 16777216.0f);
        return (uint16_t)(sign | (uint16_t)q);
    }
    /* normal: keep 10 mantissa bits, round to nearest even on the 13 dropped */
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t e = (ax >> 23) - 112u;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u; /* carry may bump exponent */
    return (uint16_t)(sign | h);
}

/* ---- row-parallel driver ---- */
typedef struct {
    int kind; /* 4 = int4 dequant, 8 = int8 dequant, 0 = mv */
    const void* W;
    const void* scale;
    const float* xf;
    float* work;
    uint16_t* y;
    int64_t N, K, r0, r1;
} Job;

static void dequant_rows(const Job* j) {
    const int64_t K = j->K;
    for (int64_t n = j->r0; n < j->r1; ++n) {
        float* dr = j->work + n * K;
        if (j->kind == 4) {
            const uint8_t* wr = (const uint8_t*)j->W + n * (K / 2);
            const uint16_t* sr = (const uint16_t*)j->scale + n * (K / 128);
            for (int64_t g = 0; g < K / 128; ++g) {
                const float s = h2f(sr[g]);
                for (int64_t b = g * 64; b < g * 64 + 64; ++b) {
                    const int v = wr[b];
                    const int lo = (v & 0xF) >= 8 ? (v & 0xF) - 16 : (v & 0xF);
                    const int hi = (v >> 4) >= 8 ? (v >> 4) - 16 : (v >> 4);
                    dr[2 * b] = (float)lo * s;
                    dr[2 * b + 1] = (float)hi * s;
                }
            }
        } else {
            const int8_t* wr = (const int8_t*)j->W + n * K;
            const float s = ((const float*)j->scale)[n];
            for (int64_t k = 0; k < K; ++k) dr[k] = (float)wr[k] * s;
        }
    }
}

static void mv_rows(const Job* j) {
    const int64_t K = j->K;
    for (int64_t n = j->r0; n < j->r1; ++n) {
        const float* dr = j->work + n * K;
        float acc = 0.f;
        for (int64_t k = 0; k < K; ++k) acc += dr[k] * j->xf[k];
        j->y[n] = f2h(acc);
    }
}

static void* worker(void* arg) {
    const Job* j = (const Job*)arg;
    if (j->kind == 0) mv_rows(j); else dequant_rows(j);
    return NULL;
}

static int run_parallel(Job proto, int threads) {
    enum { kMaxThreads = 512 };
    pthread_t tid[kMaxThreads];
    Job jobs[kMaxThreads];
    if (threads < 1) threads = 1;
    if (threads > kMaxThreads) threads = kMaxThreads;
    if (threads > proto.N) threads = (int)proto.N;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        jobs[t] = proto;
        jobs[t].r0 = proto.N * t / threads;
        jobs[t].r1 = proto.N * (t + 1) / threads;
        if (t == 0) continue;
        if (pthread_create(&tid[t], NULL, worker, &jobs[t]) != 0) {
            worker(&jobs[t]); /* run inline when no thread can be created */
            tid[t] = 0;
        } else {
            ++started;
        }
    }
    worker(&jobs[0]);
    for (int t = 1; t < threads; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
    (void)started;
    return 0;
}

static int gemv_common(int kind, const void* W, const void* scale, const uint16_t* x,
                       uint16_t* y, int64_t N, int64_t K, float* work, int threads) {
    Job p;
    memset(&p, 0, sizeof(p));
    p.kind = kind; p.W = W; p.scale = scale; p.work = work; p.y = y; p.N = N; p.K = K;
    run_parallel(p, threads);                 /* step 1: materialise W_dequant */
    float* xf = work + N * K;                 /* caller sized work as N*K + K floats */
    for (int64_t k = 0; k < K; ++k) xf[k] = h2f(x[k]);
    p.kind = 0; p.xf = xf;
    run_parallel(p, threads);                 /* step 2: fp32 mv, fp16 out */
    return 0;
}

/* INT4: W_packed uint8 [N, K/2], scale fp16 bits [N, K/128], x fp16 bits [K];
 * work: N*K + K floats supplied by the caller. */
int oracle_int4_gemv(const uint8_t* Wp, const uint16_t* scale, const uint16_t* x, uint16_t* y,
                     int64_t N, int64_t K, float* work, int threads) {
    if (N <= 0 || K <= 0 || (K % 128) != 0 || !work) return 1;
    return gemv_common(4, Wp, scale, x, y, N, K, work, threads);
}

/* INT8: W_q int8 [N, K], scale fp32 [N], x fp16 bits [K]; work N*K + K floats. */
int oracle_int8_gemv(const int8_t* Wq, const float* scale, const uint16_t* x, uint16_t* y,
                     int64_t N, int64_t K, float* work, int threads) {
    if (N <= 0 || K <= 0 || !work) return 1;
    return gemv_common(8, Wq, scale, x, y, N, K, work, threads);
}

int oracle_max_threads(void) {
    const long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* Exposed for the conversion self-test. */
float oracle_h2f(uint16_t h) { return h2f(h); }
uint16_t oracle_f2h(float f) { return f2h(f); }
