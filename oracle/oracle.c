/*
 * oracle.c -- CPU restatement of OuroborOS's quantized-weight matmul path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h for the contract and the list of
 * reference functions each routine follows). Built by oracle/Makefile with
 * -O2 -ffp-contract=off; never linked into the product library.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------ */
/* generators                                                          */
/* ------------------------------------------------------------------ */

/* ouro-wgpu/tests/l1_parity.rs:7-15: st = st*6364136223846793005 + 1442695040888963407 */
uint64_t orc_lcg_step(uint64_t *st) {
    *st = *st * 6364136223846793005ULL + 1442695040888963407ULL;
    return *st;
}

/* l1_parity.rs:7-15: one byte per step, (st >> 33) as u8 */
void orc_lcg_bytes(uint64_t seed, uint8_t *out, size_t n) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; i++) out[i] = (uint8_t)(orc_lcg_step(&st) >> 33);
}

/* uniform on (0, 1] from the top 24 bits of one LCG step */
static double u01(uint64_t *st) {
    return (double)((orc_lcg_step(st) >> 40) + 1) * (1.0 / 16777216.0);
}

/* Box-Muller pairs on (0,1] uniforms, rounded once to fp32. */
void orc_normals(uint64_t seed, float *out, size_t n) {
    uint64_t st = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        double r = sqrt(-2.0 * log(u01(&st)));
        double t = two_pi * u01(&st);
        out[i] = (float)(r * cos(t));
        if (i + 1 < n) out[i + 1] = (float)(r * sin(t));
    }
}

/* iid ternary with p(-1, 0, +1) = (.25, .5, .25): two bits of one step */
void orc_ternary(uint64_t seed, int8_t *w, size_t n) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; i++) {
        unsigned v = (unsigned)(orc_lcg_step(&st) >> 62);
        w[i] = (int8_t)(v == 0 ? -1 : (v == 3 ? 1 : 0));
    }
}

/* iid signs with p = .5 */
void orc_signs(uint64_t seed, int8_t *w, size_t n) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; i++) w[i] = (orc_lcg_step(&st) >> 63) ? 1 : -1;
}

/* Multiply a seeded fraction `frac` of positions by `mult` (C3's 1% x20 outliers). */
void orc_outliers(uint64_t seed, float *x, size_t n, double frac, float mult) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; i++)
        if (u01(&st) <= frac) x[i] = x[i] * mult;
}

/* fp16(|N(0, sigma)|) group scales (C3) */
void orc_group_scales(uint64_t seed, uint16_t *scales, size_t n, float sigma) {
    float *tmp = (float *)malloc(n * sizeof(float));
    orc_normals(seed, tmp, n);
    for (size_t i = 0; i < n; i++) scales[i] = orc_f32_to_f16(fabsf(tmp[i]) * sigma);
    free(tmp);
}

/* ------------------------------------------------------------------ */
/* f16                                                                 */
/* ------------------------------------------------------------------ */

/* cluster/src/infer/dequant.rs:21-47 (subnormals and infinities handled) */
float orc_f16_to_f32(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u;
    int32_t exp = (bits >> 10) & 0x1f;
    uint32_t frac = bits & 0x3ffu;
    uint32_t out;
    if (exp == 0) {
        if (frac == 0) {
            out = sign << 31;
        } else {
            int32_t e = -1;
            uint32_t f = frac;
            while ((f & 0x400u) == 0) {
                f <<= 1;
                e += 1;
            }
            f &= 0x3ffu;
            uint32_t exp32 = (uint32_t)(127 - 15 - e);
            out = (sign << 31) | (exp32 << 23) | (f << 13);
        }
    } else if (exp == 0x1f) {
        out = (sign << 31) | (0xffu << 23) | (frac << 13);
    } else {
        out = (sign << 31) | ((uint32_t)(exp + 127 - 15) << 23) | (frac << 13);
    }
    float r;
    memcpy(&r, &out, 4);
    return r;
}

/* f32 -> f16, round to nearest even (generators only; not on the compute path) */
uint16_t orc_f32_to_f16(float v) {
    uint32_t x;
    memcpy(&x, &v, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (absx < 0x38800000u) {                                   /* subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign;
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 112;
    uint32_t m = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ */
/* packers                                                             */
/* ------------------------------------------------------------------ */

void orc_pack_tern2(const int8_t *w, int M, int K, uint8_t *packed) {
    size_t rb = (size_t)K / 4;
    memset(packed, 0, (size_t)M * rb);
    for (int m = 0; m < M; m++)
        for (int k = 0; k < K; k++) {
            unsigned c = (unsigned)(w[(size_t)m * K + k] + 1);
            packed[(size_t)m * rb + k / 4] |= (uint8_t)(c << (2 * (k % 4)));
        }
}

void orc_pack_sign1(const int8_t *w, int M, int K, uint8_t *packed) {
    size_t rb = (size_t)K / 8;
    memset(packed, 0, (size_t)M * rb);
    for (int m = 0; m < M; m++)
        for (int k = 0; k < K; k++)
            if (w[(size_t)m * K + k] > 0) packed[(size_t)m * rb + k / 8] |= (uint8_t)(1u << (k % 8));
}

/* absmean scale of a ternary tensor W_fp = w * base: mean |W_fp| (double sum, one rounding) */
float orc_absmean_scale(const int8_t *w, size_t n, float base) {
    double s = 0.0;
    for (size_t i = 0; i < n; i++) s += fabs((double)w[i] * (double)base);
    return (float)(s / (double)n);
}

/* ------------------------------------------------------------------ */
/* Hadamard (cluster/src/infer/hadamard.rs)                            */
/* ------------------------------------------------------------------ */

/* hadamard.rs:15-31: butterflies with h = 1, 2, 4, ...; lo <- a+b, hi <- a-b */
void orc_wht_inplace(float *x, size_t n) {
    for (size_t h = 1; h < n; h *= 2)
        for (size_t c = 0; c < n; c += 2 * h)
            for (size_t i = c; i < c + h; i++) {
                float a = x[i], b = x[i + h];
                x[i] = a + b;
                x[i + h] = a - b;
            }
}

/* hadamard.rs:33-37 */
static int check_rot(size_t n, size_t block) {
    if (block == 0 || (block & (block - 1)) != 0) return -1;
    if (n % block != 0) return -1;
    return 0;
}

/* hadamard.rs:41-53: v *= s; WHT per block; v *= 1/sqrt(block) */
int orc_rotate_fwd(float *x, const float *signs, size_t n, size_t block) {
    if (check_rot(n, block)) return -1;
    float scale = 1.0f / sqrtf((float)block);
    if (signs)
        for (size_t i = 0; i < n; i++) x[i] = x[i] * signs[i];
    for (size_t b = 0; b < n; b += block) orc_wht_inplace(x + b, block);
    for (size_t i = 0; i < n; i++) x[i] = x[i] * scale;
    return 0;
}

/* hadamard.rs:57-66: WHT per block; v *= s * scale (s*scale first) */
int orc_rotate_inv(float *x, const float *signs, size_t n, size_t block) {
    if (check_rot(n, block)) return -1;
    float scale = 1.0f / sqrtf((float)block);
    for (size_t b = 0; b < n; b += block) orc_wht_inplace(x + b, block);
    for (size_t i = 0; i < n; i++) x[i] = x[i] * ((signs ? signs[i] : 1.0f) * scale);
    return 0;
}

/* ------------------------------------------------------------------ */
/* activation quantisation (kernel K1; parity unpinned, fixed here)     */
/* ------------------------------------------------------------------ */

int orc_quantize_act(const float *x, int B, int K, const float *signs, int had_block, int8_t *q,
                     float *s_x, float *x_rot) {
    if (B < 0 || K <= 0) return -1;
    float *row = (float *)malloc((size_t)K * sizeof(float));
    for (int b = 0; b < B; b++) {
        memcpy(row, x + (size_t)b * K, (size_t)K * sizeof(float));
        if (had_block > 0) {
            if (orc_rotate_fwd(row, signs, (size_t)K, (size_t)had_block)) {
                free(row);
                return -1;
            }
        }
        if (x_rot) memcpy(x_rot + (size_t)b * K, row, (size_t)K * sizeof(float));
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = fmaxf(amax, fabsf(row[k]));
        float s = amax / 127.0f;
        s_x[b] = s;
        for (int k = 0; k < K; k++) {
            int v = 0;
            if (s != 0.0f) {
                float r = rintf(row[k] / s);
                r = fminf(fmaxf(r, -127.0f), 127.0f);
                v = (int)r;
            }
            q[(size_t)b * K + k] = (int8_t)v;
        }
    }
    free(row);
    return 0;
}

/* ------------------------------------------------------------------ */
/* int8-activation GEMM                                                 */
/* ------------------------------------------------------------------ */

static int32_t tern_row_dot(const uint8_t *prow, int K, const int8_t *q) {
    int32_t acc = 0;
    for (int k = 0; k < K; k++) {
        int c = (prow[k >> 2] >> (2 * (k & 3))) & 3;
        acc += (c - 1) * (int32_t)q[k];
    }
    return acc;
}

static void tern_rows(const uint8_t *packed, int r0, int r1, int M, int K, float w_scale,
                      const int8_t *q, const float *s_x, int B, int32_t *acc, float *y) {
    size_t rb = (size_t)K / 4;
    for (int b = 0; b < B; b++)
        for (int m = r0; m < r1; m++) {
            int32_t a = tern_row_dot(packed + (size_t)m * rb, K, q + (size_t)b * K);
            if (acc) acc[(size_t)b * M + m] = a;
            y[(size_t)b * M + m] = ((float)a * w_scale) * s_x[b];
        }
}

int orc_gemm_tern2(const uint8_t *packed, int M, int K, float w_scale, const int8_t *q,
                   const float *s_x, int B, int32_t *acc, float *y) {
    if (M < 0 || K <= 0 || K % 4 || B < 0) return -1;
    tern_rows(packed, 0, M, M, K, w_scale, q, s_x, B, acc, y);
    return 0;
}

static void sign_rows(const uint8_t *packed, const uint16_t *scales, int r0, int r1, int M,
                      int K, const int8_t *q, const float *s_x, int B, int32_t *acc_g, float *y) {
    size_t rb = (size_t)K / 8;
    int G = K / 128;
    for (int b = 0; b < B; b++) {
        const int8_t *qb = q + (size_t)b * K;
        for (int m = r0; m < r1; m++) {
            const uint8_t *prow = packed + (size_t)m * rb;
            float sum = 0.0f;
            for (int g = 0; g < G; g++) {
                int32_t a = 0;
                for (int k = g * 128; k < g * 128 + 128; k++) {
                    int bit = (prow[k >> 3] >> (k & 7)) & 1;
                    a += (bit ? 1 : -1) * (int32_t)qb[k];
                }
                if (acc_g) acc_g[((size_t)b * M + m) * G + g] = a;
                float t = (float)a * orc_f16_to_f32(scales[(size_t)m * G + g]);
                sum = sum + t;
            }
            y[(size_t)b * M + m] = sum * s_x[b];
        }
    }
}

int orc_gemm_sign1(const uint8_t *packed, const uint16_t *scales, int M, int K, const int8_t *q,
                   const float *s_x, int B, int32_t *acc_g, float *y) {
    if (M < 0 || K <= 0 || K % 128 || B < 0) return -1;
    sign_rows(packed, scales, 0, M, M, K, q, s_x, B, acc_g, y);
    return 0;
}

/* ---- threaded variants: rows chunked as ceil(out/nt) like ops.rs:104-105 ---- */

typedef struct {
    int kind; /* 0 tern, 1 sign, 2 tl1 sse, 3 tq1, 4 f16, 5 bf16, 6 tl1 sse K columns (B = k) */
    const uint8_t *packed;
    const uint16_t *scales;
    int r0, r1, M, K, B;
    float w_scale;
    const int8_t *q;
    const float *s_x;
    const float *xf;
    float *y;
} mt_job;

static void tl1_rows_sse(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                         float *y);
static void tq1_rows(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                     float *y);
static void tl1_rows_sse_k(const uint8_t *payload, int r0, int r1, int in_len, int out_len,
                           const float *x, int k, float *y);
static void half_rows(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                      float *y, int bf16);

static void *mt_worker(void *p) {
    mt_job *j = (mt_job *)p;
    switch (j->kind) {
        case 0:
            tern_rows(j->packed, j->r0, j->r1, j->M, j->K, j->w_scale, j->q, j->s_x, j->B, NULL,
                      j->y);
            break;
        case 1:
            sign_rows(j->packed, j->scales, j->r0, j->r1, j->M, j->K, j->q, j->s_x, j->B, NULL,
                      j->y);
            break;
        case 2:
            tl1_rows_sse(j->packed, j->r0, j->r1, j->K, j->xf, j->y);
            break;
        case 3:
            tq1_rows(j->packed, j->r0, j->r1, j->K, j->xf, j->y);
            break;
        case 4:
        case 5:
            half_rows(j->packed, j->r0, j->r1, j->K, j->xf, j->y, j->kind == 5);
            break;
        case 6:
            tl1_rows_sse_k(j->packed, j->r0, j->r1, j->K, j->M, j->xf, j->B, j->y);
            break;
    }
    return NULL;
}

int orc_hw_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static int run_mt(mt_job proto, int M, int threads) {
    if (threads <= 0) threads = orc_hw_threads();
    int nt = threads < M ? threads : M;
    if (nt < 1) nt = 1;
    int chunk = (M + nt - 1) / nt;
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nt);
    mt_job *jobs = (mt_job *)malloc(sizeof(mt_job) * (size_t)nt);
    int started = 0;
    for (int t = 0; t < nt; t++) {
        jobs[t] = proto;
        jobs[t].r0 = t * chunk;
        jobs[t].r1 = (t + 1) * chunk < M ? (t + 1) * chunk : M;
        if (jobs[t].r0 >= jobs[t].r1) continue;
        if (pthread_create(&tid[started], NULL, mt_worker, &jobs[t]) != 0) {
            mt_worker(&jobs[t]);
            continue;
        }
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
    return 0;
}

int orc_gemm_tern2_mt(const uint8_t *packed, int M, int K, float w_scale, const int8_t *q,
                      const float *s_x, int B, float *y, int threads) {
    if (M < 0 || K <= 0 || K % 4 || B < 0) return -1;
    mt_job j = {0};
    j.kind = 0, j.packed = packed, j.M = M, j.K = K, j.B = B, j.w_scale = w_scale, j.q = q,
    j.s_x = s_x, j.y = y;
    return run_mt(j, M, threads);
}

int orc_gemm_sign1_mt(const uint8_t *packed, const uint16_t *scales, int M, int K,
                      const int8_t *q, const float *s_x, int B, float *y, int threads) {
    if (M < 0 || K <= 0 || K % 128 || B < 0) return -1;
    mt_job j = {0};
    j.kind = 1, j.packed = packed, j.scales = scales, j.M = M, j.K = K, j.B = B, j.q = q,
    j.s_x = s_x, j.y = y;
    return run_mt(j, M, threads);
}

/* ------------------------------------------------------------------ */
/* the reference's own formats                                         */
/* ------------------------------------------------------------------ */

static const uint8_t POW3[6] = {1, 3, 9, 27, 81, 243};

/* dequant.rs:134-138 / 57-61: q = byte*3^n (mod 256); xi = (q*3)>>8; trit = xi - 1 */
static inline int digit(uint8_t byte, int n) {
    uint8_t q = (uint8_t)(byte * POW3[n]);
    return (int)(((uint16_t)q * 3) >> 8);
}

/* dequant.rs:50-80: qs[48] | qh[4] | f16 d; order qs[0..32] x5, qs[32..48] x5, qh x4 */
void orc_tq1_block(const uint8_t *bytes, float *out) {
    const uint8_t *qs = bytes, *qh = bytes + 48;
    float d = orc_f16_to_f32((uint16_t)(bytes[52] | (bytes[53] << 8)));
    int o = 0;
    for (int n = 0; n < 5; n++)
        for (int m = 0; m < 32; m++) out[o++] = ((float)digit(qs[m], n) - 1.0f) * d;
    for (int n = 0; n < 5; n++)
        for (int m = 32; m < 48; m++) out[o++] = ((float)digit(qs[m], n) - 1.0f) * d;
    for (int n = 0; n < 4; n++)
        for (int m = 0; m < 4; m++) out[o++] = ((float)digit(qh[m], n) - 1.0f) * d;
}

/* dequant.rs:146-171: qs[24] | qh[2] | f16 d; elements n*16+m, 80+n*8+m, 120+n*2+h */
void orc_tl1_group(const uint8_t *bytes, float *out) {
    float d = orc_f16_to_f32((uint16_t)(bytes[26] | (bytes[27] << 8)));
    const uint8_t *qs = bytes, *qh = bytes + 24;
    int o = 0;
    for (int n = 0; n < 5; n++)
        for (int m = 0; m < 16; m++) out[o++] = (float)(digit(qs[m], n) - 1) * d;
    for (int n = 0; n < 5; n++)
        for (int m = 0; m < 8; m++) out[o++] = (float)(digit(qs[16 + m], n) - 1) * d;
    for (int n = 0; n < 4; n++)
        for (int m = 0; m < 2; m++) out[o++] = (float)(digit(qh[m], n) - 1) * d;
}

/* ops.rs:324-363 (tl1_rows_scalar): one running fp32 sum per row, mul then add */
int orc_matvec_tl1_scalar(const uint8_t *payload, int out_len, int in_len, const float *x,
                          float *y) {
    if (in_len % 128) return -1;
    int gpr = in_len / 128;
    for (int row = 0; row < out_len; row++) {
        size_t row_base = (size_t)row * gpr * 28;
        float sum = 0.0f;
        for (int g = 0; g < gpr; g++) {
            const uint8_t *gb = payload + row_base + (size_t)g * 28;
            float d = orc_f16_to_f32((uint16_t)(gb[26] | (gb[27] << 8)));
            const float *xg = x + (size_t)g * 128;
            for (int n = 0; n < 5; n++)
                for (int m = 0; m < 16; m++) {
                    float t = (float)(digit(gb[m], n) - 1) * d;
                    sum = sum + t * xg[n * 16 + m];
                }
            for (int n = 0; n < 5; n++)
                for (int m = 0; m < 8; m++) {
                    float t = (float)(digit(gb[16 + m], n) - 1) * d;
                    sum = sum + t * xg[80 + n * 8 + m];
                }
            for (int n = 0; n < 4; n++)
                for (int m = 0; m < 2; m++) {
                    float t = (float)(digit(gb[24 + m], n) - 1) * d;
                    sum = sum + t * xg[120 + n * 2 + m];
                }
        }
        y[row] = sum;
    }
    return 0;
}

/*
 * ops.rs:499-584 (tl1_rows_avx2, SSE4.1): per group a 4-lane accumulator fed by
 * digits8 (decode 8 trits, (t*d)*x, add) for qs[0..8], qs[8..16], qs[16..24]
 * per stage n; the qh tail is added to the row sum in scalar order, then
 * hsum(acc) is added per group.
 */
#if defined(__x86_64__)
__attribute__((target("sse4.1"))) static inline __m128 digits8(const uint8_t *p, int pn,
                                                               __m128 d, const float *xp,
                                                               __m128 acc) {
    __m128i b = _mm_loadl_epi64((const __m128i *)p);
    __m128i w = _mm_unpacklo_epi8(b, _mm_setzero_si128());
    __m128i q = _mm_mullo_epi16(w, _mm_set1_epi16((short)pn));
    q = _mm_and_si128(q, _mm_set1_epi16(0xFF));
    q = _mm_mullo_epi16(q, _mm_set1_epi16(3));
    q = _mm_srli_epi16(q, 8);
    q = _mm_sub_epi16(q, _mm_set1_epi16(1));
    __m128 flo = _mm_cvtepi32_ps(_mm_cvtepi16_epi32(q));
    __m128 fhi = _mm_cvtepi32_ps(_mm_cvtepi16_epi32(_mm_unpackhi_epi64(q, q)));
    acc = _mm_add_ps(_mm_mul_ps(_mm_mul_ps(flo, d), _mm_loadu_ps(xp)), acc);
    return _mm_add_ps(_mm_mul_ps(_mm_mul_ps(fhi, d), _mm_loadu_ps(xp + 4)), acc);
}

__attribute__((target("sse4.1"))) static inline float hsum4(__m128 v) {
    __m128 s = _mm_add_ps(v, _mm_movehl_ps(v, v));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
    return _mm_cvtss_f32(s);
}

__attribute__((target("sse4.1"))) static void tl1_rows_sse(const uint8_t *payload, int r0,
                                                           int r1, int in_len, const float *x,
                                                           float *y) {
    int gpr = in_len / 128;
    for (int row = r0; row < r1; row++) {
        size_t row_base = (size_t)row * gpr * 28;
        float sum = 0.0f;
        for (int g = 0; g < gpr; g++) {
            const uint8_t *qs = payload + row_base + (size_t)g * 28;
            float d = orc_f16_to_f32((uint16_t)(qs[26] | (qs[27] << 8)));
            __m128 dv = _mm_set1_ps(d);
            const float *xp = x + (size_t)g * 128;
            __m128 acc = _mm_setzero_ps();
            for (int n = 0; n < 5; n++) {
                int pn = POW3[n];
                acc = digits8(qs, pn, dv, xp + n * 16, acc);
                acc = digits8(qs + 8, pn, dv, xp + n * 16 + 8, acc);
                acc = digits8(qs + 16, pn, dv, xp + 80 + n * 8, acc);
            }
            const uint8_t *qh = qs + 24;
            for (int n = 0; n < 4; n++)
                for (int m = 0; m < 2; m++) {
                    float t = (float)(digit(qh[m], n) - 1) * d;
                    sum = sum + t * xp[120 + n * 2 + m];
                }
            sum = sum + hsum4(acc);
        }
        y[row] = sum;
    }
}
#else
static void tl1_rows_sse(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                         float *y) {
    size_t rb = (size_t)in_len / 128 * 28;
    orc_matvec_tl1_scalar(payload + (size_t)r0 * rb, r1 - r0, in_len, x, y + r0);
}
#endif

int orc_matvec_tl1_sse(const uint8_t *payload, int out_len, int in_len, const float *x,
                       float *y, int threads) {
    if (in_len % 128) return -1;
    mt_job j = {0};
    j.kind = 2, j.packed = payload, j.M = out_len, j.K = in_len, j.xf = x, j.y = y;
    return run_mt(j, out_len, threads);
}

/*
 * ops.rs:244-286 (tl1_rows_scalar_k): per row, per group, per column c the
 * running sum continues from the previous group's value in the scalar order of
 * tl1_rows_scalar. Output is [k][out_len] (y[c*out_len + r], ops.rs:158-161).
 */
int orc_matmul_tl1_scalar(const uint8_t *payload, int out_len, int in_len, const float *x,
                          int k, float *y) {
    if (in_len % 128 || k < 0) return -1;
    int gpr = in_len / 128;
    float *sums = (float *)calloc((size_t)(k > 0 ? k : 1), sizeof(float));
    for (int row = 0; row < out_len; row++) {
        size_t row_base = (size_t)row * gpr * 28;
        for (int c = 0; c < k; c++) sums[c] = 0.0f;
        for (int g = 0; g < gpr; g++) {
            const uint8_t *gb = payload + row_base + (size_t)g * 28;
            float d = orc_f16_to_f32((uint16_t)(gb[26] | (gb[27] << 8)));
            for (int c = 0; c < k; c++) {
                const float *xc = x + (size_t)c * in_len + (size_t)g * 128;
                float acc = sums[c];
                for (int n = 0; n < 5; n++) {
                    for (int m = 0; m < 16; m++) {
                        float t = (float)(digit(gb[m], n) - 1) * d;
                        acc = acc + t * xc[n * 16 + m];
                    }
                    for (int m = 0; m < 8; m++) {
                        float t = (float)(digit(gb[16 + m], n) - 1) * d;
                        acc = acc + t * xc[80 + n * 8 + m];
                    }
                }
                for (int n = 0; n < 4; n++)
                    for (int m = 0; m < 2; m++) {
                        float t = (float)(digit(gb[24 + m], n) - 1) * d;
                        acc = acc + t * xc[120 + n * 2 + m];
                    }
                sums[c] = acc;
            }
        }
        for (int c = 0; c < k; c++) y[(size_t)c * out_len + row] = sums[c];
    }
    free(sums);
    return 0;
}

/*
 * ops.rs:162-215 with tl1_rows_avx2_k (ops.rs:381-481), the x86 K-column path
 * of matmul_tl1: each stage n of a group is decoded once (qs[0..8], qs[8..16],
 * qs[16..24] -> 4-lane halves lo/hi) and fed to every column. Per column two
 * 4-lane accumulators run over the whole row and take (t*d)*x in the order
 * lo0, hi0, lo1, hi1, lo2, hi2; the qh tail goes to a scalar per-column sum
 * that starts at zero (the scratch row); at the end of the row
 * y = tail + (hsum(lo) + hsum(hi)). Output [k][out_len] (y[c*out_len + r]).
 * This order differs from matvec_tl1's (one accumulator per group), so the two
 * agree only within the reference's own test tolerance (ops.rs:721-750).
 */
#if defined(__x86_64__)
__attribute__((target("sse4.1"))) static inline void decode8_halves(const uint8_t *p, int pn,
                                                                    __m128 *lo, __m128 *hi) {
    __m128i b = _mm_loadl_epi64((const __m128i *)p);
    __m128i w = _mm_unpacklo_epi8(b, _mm_setzero_si128());
    __m128i q = _mm_mullo_epi16(w, _mm_set1_epi16((short)pn));
    q = _mm_and_si128(q, _mm_set1_epi16(0xFF));
    q = _mm_mullo_epi16(q, _mm_set1_epi16(3));
    q = _mm_srli_epi16(q, 8);
    q = _mm_sub_epi16(q, _mm_set1_epi16(1));
    *lo = _mm_cvtepi32_ps(_mm_cvtepi16_epi32(q));
    *hi = _mm_cvtepi32_ps(_mm_cvtepi16_epi32(_mm_unpackhi_epi64(q, q)));
}

__attribute__((target("sse4.1"))) static inline __m128 mac4(__m128 t, __m128 d, const float *xp,
                                                            __m128 acc) {
    return _mm_add_ps(_mm_mul_ps(_mm_mul_ps(t, d), _mm_loadu_ps(xp)), acc);
}

__attribute__((target("sse4.1"))) static void tl1_rows_sse_k(const uint8_t *payload, int r0,
                                                             int r1, int in_len, int out_len,
                                                             const float *x, int k, float *y) {
    if (k <= 0) return;
    int gpr = in_len / 128;
    __m128 *acc = (__m128 *)aligned_alloc(16, sizeof(__m128) * 2 * (size_t)k);
    float *tail = (float *)malloc(sizeof(float) * (size_t)k);
    for (int row = r0; row < r1; row++) {
        size_t row_base = (size_t)row * gpr * 28;
        for (int c = 0; c < 2 * k; c++) acc[c] = _mm_setzero_ps();
        for (int c = 0; c < k; c++) tail[c] = 0.0f;
        for (int g = 0; g < gpr; g++) {
            const uint8_t *qs = payload + row_base + (size_t)g * 28;
            float d = orc_f16_to_f32((uint16_t)(qs[26] | (qs[27] << 8)));
            __m128 dv = _mm_set1_ps(d);
            size_t xg = (size_t)g * 128;
            for (int n = 0; n < 5; n++) {
                __m128 lo0, hi0, lo1, hi1, lo2, hi2;
                decode8_halves(qs, POW3[n], &lo0, &hi0);
                decode8_halves(qs + 8, POW3[n], &lo1, &hi1);
                decode8_halves(qs + 16, POW3[n], &lo2, &hi2);
                for (int c = 0; c < k; c++) {
                    const float *xp = x + (size_t)c * in_len + xg;
                    __m128 a = acc[2 * c], b = acc[2 * c + 1];
                    a = mac4(lo0, dv, xp + n * 16, a);
                    b = mac4(hi0, dv, xp + n * 16 + 4, b);
                    a = mac4(lo1, dv, xp + n * 16 + 8, a);
                    b = mac4(hi1, dv, xp + n * 16 + 12, b);
                    a = mac4(lo2, dv, xp + 80 + n * 8, a);
                    b = mac4(hi2, dv, xp + 80 + n * 8 + 4, b);
                    acc[2 * c] = a;
                    acc[2 * c + 1] = b;
                }
            }
            const uint8_t *qh = qs + 24;
            for (int n = 0; n < 4; n++)
                for (int m = 0; m < 2; m++) {
                    float t = (float)(digit(qh[m], n) - 1) * d;
                    for (int c = 0; c < k; c++)
                        tail[c] = tail[c] + t * x[(size_t)c * in_len + xg + 120 + n * 2 + m];
                }
        }
        for (int c = 0; c < k; c++)
            y[(size_t)c * out_len + row] = tail[c] + (hsum4(acc[2 * c]) + hsum4(acc[2 * c + 1]));
    }
    free(acc);
    free(tail);
}
#else
/* elsewhere the reference runs tl1_rows_scalar_k (ops.rs:244-286) */
static void tl1_rows_sse_k(const uint8_t *payload, int r0, int r1, int in_len, int out_len,
                           const float *x, int k, float *y) {
    int gpr = in_len / 128;
    for (int row = r0; row < r1; row++) {
        size_t row_base = (size_t)row * gpr * 28;
        for (int c = 0; c < k; c++) {
            const float *xc = x + (size_t)c * in_len;
            float acc = 0.0f;
            for (int g = 0; g < gpr; g++) {
                const uint8_t *gb = payload + row_base + (size_t)g * 28;
                float d = orc_f16_to_f32((uint16_t)(gb[26] | (gb[27] << 8)));
                const float *xg = xc + (size_t)g * 128;
                for (int n = 0; n < 5; n++) {
                    for (int m = 0; m < 16; m++)
                        acc = acc + (float)(digit(gb[m], n) - 1) * d * xg[n * 16 + m];
                    for (int m = 0; m < 8; m++)
                        acc = acc + (float)(digit(gb[16 + m], n) - 1) * d * xg[80 + n * 8 + m];
                }
                for (int n = 0; n < 4; n++)
                    for (int m = 0; m < 2; m++)
                        acc = acc + (float)(digit(gb[24 + m], n) - 1) * d * xg[120 + n * 2 + m];
            }
            y[(size_t)c * out_len + row] = acc;
        }
    }
}
#endif

int orc_matmul_tl1_sse(const uint8_t *payload, int out_len, int in_len, const float *x, int k,
                       float *y, int threads) {
    if (in_len % 128 || k < 0 || out_len < 0) return -1;
    if (k == 0 || out_len == 0) return 0;
    mt_job j = {0};
    j.kind = 6, j.packed = payload, j.M = out_len, j.K = in_len, j.B = k, j.xf = x, j.y = y;
    return run_mt(j, out_len, threads);
}

/* ops.rs:101-128 with dequant_tq1_row (dequant.rs:96-105) then dot (ops.rs:53-60) */
static void tq1_rows(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                     float *y) {
    size_t rb = (size_t)in_len / 256 * 54;
    float *row = (float *)malloc((size_t)in_len * sizeof(float));
    for (int r = r0; r < r1; r++) {
        for (size_t b = 0; b < rb / 54; b++)
            orc_tq1_block(payload + (size_t)r * rb + b * 54, row + b * 256);
        float s = 0.0f;
        for (int i = 0; i < in_len; i++) s = s + row[i] * x[i];
        y[r] = s;
    }
    free(row);
}

int orc_matvec_tq1(const uint8_t *payload, int out_len, int in_len, const float *x, float *y,
                   int threads) {
    if (in_len % 256) return -1;
    mt_job j = {0};
    j.kind = 3, j.packed = payload, j.M = out_len, j.K = in_len, j.xf = x, j.y = y;
    return run_mt(j, out_len, threads);
}

/* bf16_to_f32 (dequant.rs, test_bf16_known_values dequant.rs:680-690): the
 * top 16 bits of an f32 */
float orc_bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

/* matvec_f16 (ops.rs:131-153) and matvec_bf16 (ops.rs:600-620): each row one
 * fp32 chain in element order, s = s + f32(w) * x[i] with the product and
 * the sum rounded separately (this file is built with -ffp-contract=off). */
static void half_rows(const uint8_t *payload, int r0, int r1, int in_len, const float *x,
                      float *y, int bf16) {
    for (int r = r0; r < r1; r++) {
        const uint8_t *w = payload + (size_t)r * in_len * 2;
        float s = 0.0f;
        for (int i = 0; i < in_len; i++) {
            uint16_t bits = (uint16_t)(w[2 * i] | (w[2 * i + 1] << 8));
            float wf = bf16 ? orc_bf16_to_f32(bits) : orc_f16_to_f32(bits);
            s = s + wf * x[i];
        }
        y[r] = s;
    }
}

int orc_matvec_half(const uint8_t *payload, int out_len, int in_len, const float *x, float *y,
                    int bf16, int threads) {
    mt_job j = {0};
    j.kind = bf16 ? 5 : 4, j.packed = payload, j.M = out_len, j.K = in_len, j.xf = x, j.y = y;
    return run_mt(j, out_len, threads);
}

/* finite_argmax (infer/mod.rs:70-83): NaN skipped, the first maximum wins,
 * 0 when every value is NaN */
int orc_finite_argmax(const float *l, int n) {
    int best = 0, found = 0;
    for (int i = 0; i < n; i++) {
        if (l[i] != l[i]) continue;
        if (!found || l[i] > l[best]) {
            best = i;
            found = 1;
        }
    }
    return best;
}

/* ---- the decode step's host ops (ops.rs:11-60, infer/mod.rs:338-365), fp32 ---- */

/* rmsnorm (ops.rs:12-17): ms = (sum of v*v in element order) / n,
 * inv = 1 / sqrt(ms + eps), y = (x * inv) * w */
void orc_rmsnorm(const float *x, const float *w, int n, float eps, float *y) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss = ss + x[i] * x[i];
    float ms = ss / (float)n;
    float inv = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * inv * w[i];
}

/* rope_neox (ops.rs:21-33), in place over the first `rot` values of one head:
 * theta_i = 1 / base^(2i / rot), angle = t * theta_i, pairs (i, i + rot/2) */
void orc_rope_neox(float *v, long long t, int rot, float base) {
    int half = rot / 2;
    for (int i = 0; i < half; i++) {
        float theta = 1.0f / powf(base, (float)(2 * i) / (float)rot);
        float ang = (float)t * theta;
        float c = cosf(ang), s = sinf(ang);
        float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * c - x1 * s;
        v[i + half] = x1 * c + x0 * s;
    }
}

/* silu (ops.rs:34-36): x / (1 + exp(-x)) */
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* the FFN activation of run_layer (infer/mod.rs:330): silu(gate) * up */
void orc_swiglu(const float *gate, const float *up, int n, float *out) {
    for (int i = 0; i < n; i++) out[i] = orc_silu(gate[i]) * up[i];
}

/* softmax (ops.rs:39-50), in place: m = max (NaN ignored, as f32::max),
 * e = exp(x - m) summed in order, then each times 1 / sum */
void orc_softmax(float *v, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = fmaxf(m, v[i]);
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        v[i] = expf(v[i] - m);
        s = s + v[i];
    }
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) v[i] = v[i] * inv;
}

/* dot (ops.rs:53-60): one running sum in element order */
float orc_dot(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s = s + a[i] * b[i];
    return s;
}

/* attend (infer/mod.rs:338-365): causal GQA over positions 0..seq-1 of one
 * sequence. k, v: [seq][n_kv * hd]; q, out: [n_head * hd]. Per head: scores =
 * dot(q, k_t) * (1 / sqrt(hd)), softmax, out += w_t * v_t for t ascending. */
int orc_attend(const float *q, const float *k, const float *v, int seq, int n_head, int n_kv,
               int hd, float *out) {
    if (seq < 1 || n_kv < 1 || n_head % n_kv || hd < 1) return -1;
    int groups = n_head / n_kv, kv_dim = n_kv * hd;
    float scale = 1.0f / sqrtf((float)hd);
    float *sc = (float *)malloc(sizeof(float) * (size_t)seq);
    if (!sc) return -1;
    for (int i = 0; i < n_head * hd; i++) out[i] = 0.0f;
    for (int h = 0; h < n_head; h++) {
        const float *qh = q + (size_t)h * hd;
        int kvh = h / groups;
        for (int t = 0; t < seq; t++)
            sc[t] = orc_dot(qh, k + (size_t)t * kv_dim + (size_t)kvh * hd, hd) * scale;
        orc_softmax(sc, seq);
        float *o = out + (size_t)h * hd;
        for (int t = 0; t < seq; t++) {
            const float *vt = v + (size_t)t * kv_dim + (size_t)kvh * hd;
            for (int i = 0; i < hd; i++) o[i] = o[i] + sc[t] * vt[i];
        }
    }
    free(sc);
    return 0;
}
