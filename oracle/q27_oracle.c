/*
 * q27_oracle.c -- CPU restatement of the q27 attention hot path. TEST INFRASTRUCTURE ONLY:
 * loaded by the test-suite, the smoke check and the benchmark's CPU-baseline leg, never by
 * the product path (see q27_oracle.h for the citation of each function and for how the
 * restatement is pinned to the reference).
 */
#include "q27_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int q27o_version(void) { return 1; }

/* ------------------------------------------------------------------ conversions ---- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float q27o_half_to_float(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0) {
        if (m == 0) return u2f(s);
        /* subnormal: m * 2^-24 */
        float v = (float)m * (1.0f / 16777216.0f);
        return s ? -v : v;
    }
    if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
    return u2f(s | ((e + 112) << 23) | (m << 13));
}

uint16_t q27o_float_to_half(float f) {
    uint32_t u = f2u(f);
    uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(s | 0x7e00u);          /* NaN */
    if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);         /* >= 65520 -> inf */
    if (a < 0x33000001u) return s;                                /* <= 2^-25 -> 0 (ties to even) */
    int e = (int)(a >> 23) - 127;
    uint32_t m = (a & 0x7fffffu) | 0x800000u; /* 24-bit significand */
    int shift;                                /* bits dropped from m */
    uint32_t base;
    if (e < -14) { shift = 13 + (-14 - e); base = 0; }            /* subnormal result */
    else { shift = 13; base = (uint32_t)(e + 15) << 10; }
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (e >= -14) q &= 0x3ffu;
    uint32_t r = base + q;
    if (rem > half || (rem == half && (r & 1u))) r++;             /* carries propagate into exp */
    return (uint16_t)(s | r);
}

float q27o_e4m3_to_float(uint8_t v) {
    int s = v >> 7, e = (v >> 3) & 0xf, m = v & 7;
    float r;
    if (e == 0xf && m == 7) return u2f(0x7fc00000u | ((uint32_t)s << 31));
    if (e == 0) r = (float)m * (1.0f / 512.0f);                   /* m/8 * 2^-6 */
    else r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -r : r;
}

uint8_t q27o_float_to_e4m3(float f) {
    uint32_t u = f2u(f);
    uint8_t s = (uint8_t)((u >> 24) & 0x80u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint8_t)(s | 0x7f);              /* NaN */
    float x = u2f(a);
    if (x >= 448.0f) return (uint8_t)(s | 0x7e);                  /* satfinite (inf too) */
    /* quantum: 2^-9 below 2^-6, else 2^(e-3) */
    int e;
    (void)frexpf(x, &e);            /* x = f * 2^e, f in [0.5,1) -> floor(log2 x) = e-1 */
    int ex = e - 1;
    if (ex < -6) ex = -6;
    float q = ldexpf(1.0f, ex - 3);
    float t = x / q;                /* exact: power-of-two scaling */
    float fl = floorf(t), d = t - fl;
    int n = (int)fl;
    if (d > 0.5f || (d == 0.5f && (n & 1))) n++;
    /* n in [0,16]; rebuild */
    float y = (float)n * q;
    if (y >= 448.0f) return (uint8_t)(s | 0x7e);
    if (y == 0.0f) return s;
    (void)frexpf(y, &e);
    ex = e - 1;
    if (ex < -6) return (uint8_t)(s | (uint8_t)(int)(y * 512.0f)); /* subnormal: m = y/2^-9 */
    int m = (int)((y / ldexpf(1.0f, ex) - 1.0f) * 8.0f);
    return (uint8_t)(s | ((ex + 7) << 3) | m);
}

float q27o_round_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return f;
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    u &= 0xffff0000u;
    return u2f(u);
}

void q27o_float_to_half_n(const float* x, int64_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = q27o_float_to_half(x[i]);
}
void q27o_float_to_e4m3_n(const float* x, int64_t n, uint8_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = q27o_float_to_e4m3(x[i]);
}
void q27o_round_bf16_n(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) x[i] = q27o_round_bf16(x[i]);
}

/* ------------------------------------------------------------------- turbo3 -------- */

static const float T3_CENTROIDS[8] = {-0.190207f, -0.118786f, -0.066822f, -0.021663f,
                                      0.021663f,  0.066822f,  0.118786f,  0.190207f};
/* sign diagonals as bit masks: bit j set <=> element j is -1 */
static const uint32_t T3_S1_NEG[4] = {0xE46A0359u, 0x42F85949u, 0xA4C63BBBu, 0x49F250A9u};
static const uint32_t T3_S2_NEG[4] = {0x16ACEE90u, 0x3F628FDCu, 0xB7A5357Au, 0xBEA56562u};
static const float T3_INV_SQRT_128 = 0.08838834764831845f;
static float T3_S1[128], T3_S2[128];
static int t3_tables_ready = 0;

/* turbo5: the 32-level table and its 31 decision thresholds are odd-symmetric
 * (c[31-i] = -c[i], T[30-i] = -T[i], T[15] = 0); the positive halves are stated here and
 * mirrored at start-up (src/turbo5.cuh:63-80 lists all 63 numbers). */
static const float T5_CENTROIDS_POS[16] = {
    0.00582388f, 0.01750547f, 0.02928998f, 0.04125080f, 0.05346908f, 0.06603809f,
    0.07906913f, 0.09270022f, 0.10710939f, 0.12253633f, 0.13932019f, 0.15797059f,
    0.17931595f, 0.20486116f, 0.23786362f, 0.28821075f};
static const float T5_THRESH_POS[15] = {
    0.01166468f, 0.02339773f, 0.03527039f, 0.04735994f, 0.05975358f,
    0.07255360f, 0.08588468f, 0.09990481f, 0.11482286f, 0.13092826f,
    0.14864540f, 0.16864327f, 0.19208856f, 0.22136238f, 0.26303717f};
static float T5_CENTROIDS[32], T5_THRESH[31];

static void t3_init(void) {
    if (t3_tables_ready) return;
    for (int j = 0; j < 128; j++) {
        T3_S1[j] = (T3_S1_NEG[j >> 5] >> (j & 31)) & 1u ? -1.f : 1.f;
        T3_S2[j] = (T3_S2_NEG[j >> 5] >> (j & 31)) & 1u ? -1.f : 1.f;
    }
    for (int i = 0; i < 16; i++) {
        T5_CENTROIDS[16 + i] = T5_CENTROIDS_POS[i];
        T5_CENTROIDS[15 - i] = -T5_CENTROIDS_POS[i];
    }
    T5_THRESH[15] = 0.f;
    for (int i = 0; i < 15; i++) {
        T5_THRESH[16 + i] = T5_THRESH_POS[i];
        T5_THRESH[14 - i] = -T5_THRESH_POS[i];
    }
    t3_tables_ready = 1;
}
__attribute__((constructor)) static void t3_ctor(void) { t3_init(); }

const float* q27o_t3_centroids(void) { return T3_CENTROIDS; }
const float* q27o_t3_s1(void) { t3_init(); return T3_S1; }
const float* q27o_t3_s2(void) { t3_init(); return T3_S2; }

int q27o_t3_nearest(float v) {
    if (v < -0.154496f) return 0;
    if (v < -0.092804f) return 1;
    if (v < -0.044243f) return 2;
    if (v < 0.000000f) return 3;
    if (v < 0.044243f) return 4;
    if (v < 0.092804f) return 5;
    if (v < 0.154496f) return 6;
    return 7;
}

static void t3_butterfly(float* x) {
    for (int h = 1; h < 128; h *= 2)
        for (int i = 0; i < 128; i += h * 2)
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
}

void q27o_t3_fwht(float* x) {
    t3_init();
    for (int i = 0; i < 128; i++) x[i] *= T3_S1[i];
    t3_butterfly(x);
    for (int i = 0; i < 128; i++) x[i] *= T3_INV_SQRT_128 * T3_S2[i];
}

void q27o_t3_fwht_inv(float* x) {
    t3_init();
    for (int i = 0; i < 128; i++) x[i] *= T3_S2[i];
    t3_butterfly(x);
    for (int i = 0; i < 128; i++) x[i] *= T3_INV_SQRT_128 * T3_S1[i];
}

void q27o_t3_quant(const float* x, uint8_t* blk) {
    float buf[128], nsq = 0.f;
    for (int j = 0; j < 128; j++) { buf[j] = x[j]; nsq += buf[j] * buf[j]; }
    float gn = sqrtf(nsq), inv = gn > 1e-10f ? 1.f / gn : 0.f;
    for (int j = 0; j < 128; j++) buf[j] *= inv;
    q27o_t3_fwht(buf);
    uint8_t* qs = blk + 2;
    uint8_t* signs = blk + 34;
    memset(qs, 0, 32);
    memset(signs, 0, 16);
    float rsq = 0.f;
    for (int j = 0; j < 128; j++) {
        int idx = q27o_t3_nearest(buf[j]);
        qs[j / 4] |= (uint8_t)((idx & 3) << ((j % 4) * 2));
        if (idx & 4) signs[j / 8] |= (uint8_t)(1 << (j % 8));
        rsq += T3_CENTROIDS[idx] * T3_CENTROIDS[idx];
    }
    float rn = sqrtf(rsq), corr = rn > 1e-10f ? gn / rn : gn;
    uint16_t h = q27o_float_to_half(corr);
    memcpy(blk, &h, 2);
}

void q27o_t3_dequant(const uint8_t* blk, float* y) {
    uint16_t h;
    memcpy(&h, blk, 2);
    float norm = q27o_half_to_float(h);
    const uint8_t* qs = blk + 2;
    const uint8_t* signs = blk + 34;
    for (int j = 0; j < 128; j++) {
        uint8_t l = (qs[j / 4] >> ((j % 4) * 2)) & 3;
        uint8_t hb = (signs[j / 8] >> (j % 8)) & 1;
        y[j] = T3_CENTROIDS[l | (hb << 2)] * norm;
    }
}

/* ------------------------------------------------------------------- turbo5 -------- */

const float* q27o_t5_centroids(void) { t3_init(); return T5_CENTROIDS; }
const float* q27o_t5_thresholds(void) { t3_init(); return T5_THRESH; }

int q27o_t5_nearest(float v) {
    int idx = 0;
    for (int i = 0; i < 31; i++) idx += v >= T5_THRESH[i];
    return idx;
}

/* sum of 128 floats: serially, or as the halving tree r[j] += r[j+s], s = 64, 32 .. 1 */
static float sum128(const float* v, int tree) {
    if (!tree) {
        float s = 0.f;
        for (int j = 0; j < 128; j++) s += v[j];
        return s;
    }
    float r[128];
    memcpy(r, v, sizeof r);
    for (int s = 64; s > 0; s >>= 1)
        for (int j = 0; j < s; j++) r[j] += r[j + s];
    return r[0];
}

void q27o_t5_quant(const float* x, uint8_t* blk, int tree) {
    t3_init();
    float buf[128], sq[128];
    for (int j = 0; j < 128; j++) { buf[j] = x[j]; sq[j] = x[j] * x[j]; }
    float gn = sqrtf(sum128(sq, tree)), inv = gn > 1e-10f ? 1.f / gn : 0.f;
    for (int j = 0; j < 128; j++) buf[j] *= inv;
    q27o_t3_fwht(buf);
    uint8_t* qs = blk + 2;
    uint8_t* hi = blk + 66;
    memset(qs, 0, 64);
    memset(hi, 0, 16);
    for (int j = 0; j < 128; j++) {
        int idx = q27o_t5_nearest(buf[j]);
        qs[j / 2] |= (uint8_t)((idx & 15) << ((j % 2) * 4));
        if (idx & 16) hi[j / 8] |= (uint8_t)(1 << (j % 8));
        sq[j] = T5_CENTROIDS[idx] * T5_CENTROIDS[idx];
    }
    float rn = sqrtf(sum128(sq, tree)), corr = rn > 1e-10f ? gn / rn : gn;
    uint16_t h = q27o_float_to_half(corr);
    memcpy(blk, &h, 2);
}

void q27o_t5_dequant(const uint8_t* blk, float* y) {
    t3_init();
    uint16_t h;
    memcpy(&h, blk, 2);
    float norm = q27o_half_to_float(h);
    const uint8_t* qs = blk + 2;
    const uint8_t* hi = blk + 66;
    for (int j = 0; j < 128; j++) {
        uint8_t l = (qs[j / 2] >> ((j % 2) * 4)) & 15;
        uint8_t hb = (hi[j / 8] >> (j % 8)) & 1;
        y[j] = T5_CENTROIDS[l | (hb << 4)] * norm;
    }
}

/* ------------------------------------------------------------------ int8-g64 ------- */

void q27o_i8_quant(const float* x, uint8_t* blk) {
    int8_t* qs = (int8_t*)blk;
    for (int g = 0; g < 2; g++) {
        float amax = 0.f;
        for (int j = 0; j < 64; j++) amax = fmaxf(amax, fabsf(x[g * 64 + j]));
        uint16_t sh = q27o_float_to_half(amax / 127.0f);
        float sw = q27o_half_to_float(sh);                /* the ROUNDED scale */
        float inv = sw > 0.f ? 1.0f / sw : 0.f;
        memcpy(blk + 128 + 2 * g, &sh, 2);
        for (int j = 0; j < 64; j++) {
            int q = (int)rintf(x[g * 64 + j] * inv);      /* nearest even, as __float2int_rn */
            q = q < -127 ? -127 : q > 127 ? 127 : q;
            qs[g * 64 + j] = (int8_t)(sw > 0.f ? q : 0);
        }
    }
}

void q27o_i8_dequant(const uint8_t* blk, float* y) {
    const int8_t* qs = (const int8_t*)blk;
    for (int g = 0; g < 2; g++) {
        uint16_t sh;
        memcpy(&sh, blk + 128 + 2 * g, 2);
        float sc = q27o_half_to_float(sh);
        for (int j = 0; j < 64; j++) y[g * 64 + j] = (float)qs[g * 64 + j] * sc;
    }
}

static int nthr(int n) {
#ifdef _OPENMP
    if (n <= 0) n = omp_get_max_threads();
    return n;
#else
    (void)n;
    return 1;
#endif
}

void q27o_t3_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int nthreads) {
    t3_init();
    int nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t g = 0; g < ngroups; g++) q27o_t3_quant(x + g * 128, blocks + g * 50);
}

void q27o_t5_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int tree,
                          int nthreads) {
    t3_init();
    int nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t g = 0; g < ngroups; g++)
        q27o_t5_quant(x + g * 128, blocks + g * Q27O_T5_BLOCK, tree);
}

void q27o_i8_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int nthreads) {
    int nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t g = 0; g < ngroups; g++) q27o_i8_quant(x + g * 128, blocks + g * Q27O_I8_BLOCK);
}

void q27o_wht_groups(float* x, int64_t ngroups, int inverse, int nthreads) {
    t3_init();
    int nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t g = 0; g < ngroups; g++) {
        if (inverse) q27o_t3_fwht_inv(x + g * 128);
        else q27o_t3_fwht(x + g * 128);
    }
}

/* storage format of one side of a kind: the K side varies, the V side of every kind from
 * turbo3 up is turbo3 (src/cuda_common.h:47-53) */
enum { RF_F16, RF_FP8, RF_T3, RF_T5, RF_I8, RF_BAD };
static int side_fmt(int kvk, int is_v) {
    switch (kvk) {
    case Q27O_KV_F16: return RF_F16;
    case Q27O_KV_FP8: return RF_FP8;
    case Q27O_KV_T3: return RF_T3;
    case Q27O_KV_T3V: return is_v ? RF_T3 : RF_F16;
    case Q27O_KV_T5K: return is_v ? RF_T3 : RF_T5;
    case Q27O_KV_I8G64: return is_v ? RF_T3 : RF_I8;
    default: return RF_BAD;
    }
}

static int64_t fmt_row_bytes(int fmt, int n_kv) {
    switch (fmt) {
    case RF_F16: return (int64_t)n_kv * Q27O_HD * 2;
    case RF_FP8: return (int64_t)n_kv * Q27O_HD;
    case RF_T3: return (int64_t)n_kv * 2 * Q27O_T3_BLOCK;
    case RF_T5: return (int64_t)n_kv * 2 * Q27O_T5_BLOCK;
    case RF_I8: return (int64_t)n_kv * 2 * Q27O_I8_BLOCK;
    default: return -1;
    }
}

int64_t q27o_row_bytes_side(int kvk, int n_kv, int is_v) {
    return fmt_row_bytes(side_fmt(kvk, is_v), n_kv);
}
int64_t q27o_row_bytes(int kvk, int n_kv) { return q27o_row_bytes_side(kvk, n_kv, 0); }

/* one (row, head) slice of 256 dims -> fp32 */
static void deq_head(const uint8_t* cache, int fmt, int64_t row, int n_kv, int kvh, float* y) {
    if (fmt == RF_F16) {
        const uint16_t* p = (const uint16_t*)cache + ((size_t)row * n_kv + kvh) * Q27O_HD;
        for (int i = 0; i < Q27O_HD; i++) y[i] = q27o_half_to_float(p[i]);
    } else if (fmt == RF_FP8) {
        const uint8_t* p = cache + ((size_t)row * n_kv + kvh) * Q27O_HD;
        for (int i = 0; i < Q27O_HD; i++) y[i] = q27o_e4m3_to_float(p[i]);
    } else if (fmt == RF_T3) {
        const uint8_t* p = cache + ((size_t)row * n_kv + kvh) * 2 * Q27O_T3_BLOCK;
        q27o_t3_dequant(p, y);
        q27o_t3_dequant(p + Q27O_T3_BLOCK, y + 128);
    } else if (fmt == RF_T5) {
        const uint8_t* p = cache + ((size_t)row * n_kv + kvh) * 2 * Q27O_T5_BLOCK;
        q27o_t5_dequant(p, y);
        q27o_t5_dequant(p + Q27O_T5_BLOCK, y + 128);
    } else {
        const uint8_t* p = cache + ((size_t)row * n_kv + kvh) * 2 * Q27O_I8_BLOCK;
        q27o_i8_dequant(p, y);
        q27o_i8_dequant(p + Q27O_I8_BLOCK, y + 128);
    }
}

int q27o_kv_dequant_side(const void* cache, int kvk, int is_v, int64_t rows, int n_kv,
                         float* out, int nthreads) {
    const int fmt = side_fmt(kvk, is_v);
    if (fmt == RF_BAD) return 1;
    t3_init();
    int nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int h = 0; h < n_kv; h++)
            deq_head((const uint8_t*)cache, fmt, r, n_kv, h,
                     out + ((size_t)r * n_kv + h) * Q27O_HD);
    return 0;
}

int q27o_kv_dequant(const void* cache, int kvk, int64_t rows, int n_kv, float* out,
                    int nthreads) {
    return q27o_kv_dequant_side(cache, kvk, 0, rows, n_kv, out, nthreads);
}

/* ------------------------------------------------------------------ attention ------ */

/* One (query vector, kv head) over rows [lo, hi): exact two-pass softmax in double.
 * Returns m (window max score), l = sum exp(s-m), acc[256] = sum exp(s-m) v. */
static void attn_window(const float* qv, const uint8_t* kc, const uint8_t* vc, int kvk,
                        int n_kv, int kvh, double scale, int64_t lo, int64_t hi, double* m_out,
                        double* l_out, double* acc) {
    for (int i = 0; i < Q27O_HD; i++) acc[i] = 0.0;
    if (hi <= lo) { *m_out = -DBL_MAX; *l_out = 0.0; return; }
    int64_t n = hi - lo;
    double* sc = (double*)malloc((size_t)n * sizeof(double));
    float row[Q27O_HD];
    double mx = -1e300;
    for (int64_t p = lo; p < hi; p++) {
        deq_head(kc, side_fmt(kvk, 0), p, n_kv, kvh, row);
        double d = 0;
        for (int i = 0; i < Q27O_HD; i++) d += (double)qv[i] * (double)row[i];
        d *= scale;
        sc[p - lo] = d;
        if (d > mx) mx = d;
    }
    double lsum = 0;
    for (int64_t p = 0; p < n; p++) { sc[p] = exp(sc[p] - mx); lsum += sc[p]; }
    for (int64_t p = lo; p < hi; p++) {
        deq_head(vc, side_fmt(kvk, 1), p, n_kv, kvh, row);
        double w = sc[p - lo];
        for (int i = 0; i < Q27O_HD; i++) acc[i] += w * (double)row[i];
    }
    free(sc);
    *m_out = mx;
    *l_out = lsum;
}

int q27o_attn_partial(const float* q, int64_t q_lane_stride, int q_stride, const void* kcache,
                      const void* vcache, int kvk, const int* pos, int ntok, int n_q, int n_kv,
                      float scale, int64_t lo, int64_t hi, float* part, int nthreads) {
    if (q27o_row_bytes(kvk, n_kv) < 0 || n_q % n_kv) return 1;
    t3_init();
    int gqa = n_q / n_kv, nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int w = 0; w < ntok * n_q; w++) {
        int t = w / n_q, h = w % n_q;
        int64_t wl = lo < 0 ? 0 : lo, wh = hi;
        if (wh > (int64_t)pos[t] + 1) wh = (int64_t)pos[t] + 1;
        double m, l, acc[Q27O_HD];
        attn_window(q + (size_t)t * q_lane_stride + (size_t)h * q_stride, (const uint8_t*)kcache,
                    (const uint8_t*)vcache, kvk, n_kv, h / gqa, (double)scale, wl, wh, &m, &l,
                    acc);
        float* dst = part + (size_t)w * Q27O_FD_ST;
        dst[0] = (wh <= wl) ? -FLT_MAX : (float)m;
        dst[1] = (float)l;
        for (int i = 0; i < Q27O_HD; i++) dst[2 + i] = (float)acc[i];
    }
    return 0;
}

int q27o_attn_decode(const float* q, int64_t q_lane_stride, int q_stride, const void* kcache,
                     const void* vcache, int kvk, const int* pos, int ntok, int n_q, int n_kv,
                     float scale, float* out, int nthreads) {
    if (q27o_row_bytes(kvk, n_kv) < 0 || n_q % n_kv) return 1;
    t3_init();
    int gqa = n_q / n_kv, nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int w = 0; w < ntok * n_q; w++) {
        int t = w / n_q, h = w % n_q;
        double m, l, acc[Q27O_HD];
        attn_window(q + (size_t)t * q_lane_stride + (size_t)h * q_stride, (const uint8_t*)kcache,
                    (const uint8_t*)vcache, kvk, n_kv, h / gqa, (double)scale, 0,
                    (int64_t)pos[t] + 1, &m, &l, acc);
        float* dst = out + (size_t)t * n_q * Q27O_HD + (size_t)h * Q27O_HD;
        for (int i = 0; i < Q27O_HD; i++) dst[i] = (float)(acc[i] / l);
    }
    return 0;
}

int q27o_merge_partials(const float* parts, int nparts, int64_t npairs, float* out,
                        int normalise) {
#pragma omp parallel for schedule(static)
    for (int64_t w = 0; w < npairs; w++) {
        double mg = -DBL_MAX;
        for (int s = 0; s < nparts; s++) {
            float ms = parts[((size_t)s * npairs + w) * Q27O_FD_ST];
            if (ms != -FLT_MAX && (double)ms > mg) mg = ms;
        }
        double lg = 0, acc[Q27O_HD];
        for (int i = 0; i < Q27O_HD; i++) acc[i] = 0;
        for (int s = 0; s < nparts; s++) {
            const float* pp = parts + ((size_t)s * npairs + w) * Q27O_FD_ST;
            if (pp[0] == -FLT_MAX) continue;
            double e = exp((double)pp[0] - mg);
            lg += (double)pp[1] * e;
            for (int i = 0; i < Q27O_HD; i++) acc[i] += (double)pp[2 + i] * e;
        }
        if (normalise) {
            float* dst = out + (size_t)w * Q27O_HD;
            for (int i = 0; i < Q27O_HD; i++) dst[i] = (float)(lg > 0 ? acc[i] / lg : 0.0);
        } else {
            float* dst = out + (size_t)w * Q27O_FD_ST;
            dst[0] = mg == -DBL_MAX ? -FLT_MAX : (float)mg;
            dst[1] = (float)lg;
            for (int i = 0; i < Q27O_HD; i++) dst[2 + i] = (float)acc[i];
        }
    }
    return 0;
}

int q27o_attn_prefill(const float* qT, int q_stride, int q_row, const void* kcache,
                      const void* vcache, int kvk, int base_pos, int t0, int SB, int n_q,
                      int n_kv, float scale, float* outT, int out_row, int nthreads) {
    if (q27o_row_bytes(kvk, n_kv) < 0 || n_q % n_kv) return 1;
    t3_init();
    int gqa = n_q / n_kv, nt = nthr(nthreads);
    (void)nt;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int w = 0; w < SB * n_q; w++) {
        int t = t0 + w / n_q, h = w % n_q;
        double m, l, acc[Q27O_HD];
        attn_window(qT + (size_t)t * q_row + (size_t)h * q_stride, (const uint8_t*)kcache,
                    (const uint8_t*)vcache, kvk, n_kv, h / gqa, (double)scale, 0,
                    (int64_t)base_pos + t + 1, &m, &l, acc);
        float* dst = outT + (size_t)t * out_row + (size_t)h * Q27O_HD;
        for (int i = 0; i < Q27O_HD; i++) dst[i] = (float)(acc[i] / l);
    }
    return 0;
}

/* ---------------------------------------------------------------- generators ------- */

uint64_t q27o_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

void q27o_randn(float* out, int64_t n, uint64_t seed, int nthreads) {
    int nt = nthr(nthreads);
    (void)nt;
    const uint64_t key = q27o_splitmix64(seed ^ 0x5851F42D4C957F2Dull);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (n + 1) / 2; i++) {
        uint64_t r = q27o_splitmix64(key + (uint64_t)i * 0x2545F4914F6CDD1Dull);
        /* two 32-bit uniforms in (0,1] and [0,1) */
        double u1 = ((double)(uint32_t)(r >> 32) + 1.0) * (1.0 / 4294967296.0);
        double u2 = (double)(uint32_t)r * (1.0 / 4294967296.0);
        double rad = sqrt(-2.0 * log(u1)), ang = 6.283185307179586476925 * u2;
        out[2 * i] = (float)(rad * cos(ang));
        if (2 * i + 1 < n) out[2 * i + 1] = (float)(rad * sin(ang));
    }
}
