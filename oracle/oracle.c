/*
 * oracle.c -- CPU restatement of the Chaos decode-step layer (TEST INFRASTRUCTURE).
 *
 * Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU legs. See
 * oracle.h for what is restated from where. Build: oracle/Makefile (gcc, OpenMP,
 * -ffp-contract=off so that no multiply-add is fused unless written as fmaf).
 *
 * ARITHMETIC CONTRACT (shared with bigtea_b200/csrc; every item is exact IEEE-754
 * single precision with round-to-nearest-even unless stated):
 *  C1 f16: f32->f16 rounds to nearest even, f16->f32 exact.
 *  C2 dequant: Q4_K y = (d*sc)*q - (dmin*m); Q6_K y = (d*sc)*q  (gguf-py order).
 *  C3 Q8_K activations: per 256 values, amax/first-occurrence signed max mx,
 *     iscale = -127/mx, q = min(127, rint(iscale*x)), d = 1/iscale, bsums over 16.
 *  C4 K-quant row dot: per superblock an exact int32 sum, then
 *     Q4_K sb = (float)sumi*(dw*dx) - (float)summ*(dminw*dx), Q6_K sb = (float)sumi*(dw*dx);
 *     row = ((0 + sb0) + sb1) + ... in superblock order.
 *  C5 P2 reduction (norms, router dot, softmax sum): lane l of 32 accumulates elements
 *     l, l+32, ... in order (fmaf for products), then an xor butterfly 16,8,4,2,1.
 *  C6 RMSNorm: mean = P2(x*x)/n; s = 1/sqrt(mean+eps); y = (x*s)*w.
 *  C7 exp: or_exp below (Cody-Waite reduction by ln2, degree-7 Taylor, Horner in fmaf).
 *  C8 attention: q rounded to f16; s = fmaf-sequential dot over d, times scale;
 *     keys in chunks of `chunk` (128); per chunk m = max s, p = exp(s-m), l = P3 sum (32-lane
 *     butterflies per 32 keys, warps summed in order from 0), acc = fmaf-sequential p*v;
 *     combine chunks in order: f = exp(m_c - M), L = fmaf(l_c,f,L), O = fmaf(acc_c,f,O),
 *     out = O/L.
 *  C9 RoPE: NeoX pairs (i, i+n_rot/2); theta_0 = pos, theta_{i+1} = theta_i*powf(base,-2/n_rot);
 *     cos/sin from libm on the host (a table); x0' = x0*c - x1*s, x1' = x0*s + x1*c.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_err[512];
static void set_err(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg); }
const char *or_last_error(void) { return g_err; }
void or_set_error_text(const char *msg) { set_err(msg); }

int or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* ------------------------------------------------------------------ C1 f16 */
uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t e8 = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (e8 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    int e = (int)e8 - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t h = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            /* subnormal: renormalise */
            int sh = 0;
            while (!(m & 0x400u)) {
                m <<= 1;
                sh++;
            }
            m &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ------------------------------------------------------------------ C7 exp */
static float pow2i(int n) { /* 2^n for n in [-126, 127] */
    uint32_t bits = (uint32_t)(n + 127) << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

float or_exp(float x) {
    if (!(x < 88.72283935546875f)) return (x != x) ? x : INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    float n = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187045e-06f, r);
    float p = 1.98412698e-4f; /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-3f); /* 1/720 */
    p = fmaf(p, r, 8.33333333e-3f); /* 1/120 */
    p = fmaf(p, r, 4.16666667e-2f); /* 1/24 */
    p = fmaf(p, r, 1.66666667e-1f); /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return (p * pow2i(127)) * pow2i(ni - 127);
    if (ni < -126) return (p * pow2i(ni + 64)) * pow2i(-64);
    return p * pow2i(ni);
}

float or_silu(float x) { return x / (1.0f + or_exp(-x)); }

/* ------------------------------------------------------------------ formats */
int64_t or_row_bytes(int type, int64_t n) {
    switch (type) {
    case OR_F32: return n * 4;
    case OR_F16: return n * 2;
    case OR_Q4_K: return (n % 256) ? -1 : n / 256 * 144;
    case OR_Q6_K: return (n % 256) ? -1 : n / 256 * 210;
    default: return -1;
    }
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* get_scale_min_k4: 6-bit scale and min of sub-block j from the 12 packed bytes */
static inline void q4k_scale_min(const uint8_t *s, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dequant_q4k_block(const uint8_t *b, float *y) {
    float d = or_f16_to_f32(rd16(b));
    float dmin = or_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qs = b + 16;
    for (int g = 0; g < 4; g++) {
        int s0, m0, s1, m1;
        q4k_scale_min(sc, 2 * g, &s0, &m0);
        q4k_scale_min(sc, 2 * g + 1, &s1, &m1);
        float d0 = d * (float)s0, mm0 = dmin * (float)m0;
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            y[64 * g + l] = d0 * (float)(qs[32 * g + l] & 0xF) - mm0;
            y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - mm1;
        }
    }
}

/* Q6_K value i of a block as a signed 6-bit integer in [-32, 31] */
static inline int q6k_value(const uint8_t *b, int i) {
    const uint8_t *ql = b, *qh = b + 128;
    int n = i / 128, r = i % 128, quad = r / 32, l = r % 32;
    int lo;
    if (quad == 0) lo = ql[64 * n + l] & 0xF;
    else if (quad == 1) lo = ql[64 * n + 32 + l] & 0xF;
    else if (quad == 2) lo = ql[64 * n + l] >> 4;
    else lo = ql[64 * n + 32 + l] >> 4;
    int hi = (qh[32 * n + l] >> (2 * quad)) & 3;
    return (lo | (hi << 4)) - 32;
}

static void dequant_q6k_block(const uint8_t *b, float *y) {
    float d = or_f16_to_f32(rd16(b + 208));
    const int8_t *sc = (const int8_t *)(b + 192);
    for (int i = 0; i < 256; i++) y[i] = (d * (float)sc[i / 16]) * (float)q6k_value(b, i);
}

int or_dequant(int type, const void *src, int64_t n, float *dst) {
    const uint8_t *s = (const uint8_t *)src;
    switch (type) {
    case OR_F32: memcpy(dst, src, (size_t)n * 4); return 0;
    case OR_F16:
        for (int64_t i = 0; i < n; i++) dst[i] = or_f16_to_f32(rd16(s + 2 * i));
        return 0;
    case OR_Q4_K:
        if (n % 256) return -1;
        for (int64_t b = 0; b < n / 256; b++) dequant_q4k_block(s + 144 * b, dst + 256 * b);
        return 0;
    case OR_Q6_K:
        if (n % 256) return -1;
        for (int64_t b = 0; b < n / 256; b++) dequant_q6k_block(s + 210 * b, dst + 256 * b);
        return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------ C3 Q8_K */
void or_quantize_q8k(const float *x, int64_t n, or_block_q8k *y) {
    for (int64_t b = 0; b < n / 256; b++) {
        const float *xb = x + 256 * b;
        or_block_q8k *yb = y + b;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < 256; j++) {
            float ax = fabsf(xb[j]);
            if (ax > amax) {
                amax = ax;
                mx = xb[j];
            }
        }
        if (amax == 0.0f) {
            yb->d = 0.0f;
            memset(yb->qs, 0, 256);
            memset(yb->bsums, 0, sizeof yb->bsums);
            continue;
        }
        float iscale = -127.0f / mx;
        for (int j = 0; j < 256; j++) {
            int v = (int)rintf(iscale * xb[j]);
            yb->qs[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int j = 0; j < 16; j++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += yb->qs[16 * j + i];
            yb->bsums[j] = (int16_t)s;
        }
        yb->d = 1.0f / iscale;
    }
}

/* ------------------------------------------------------------------ C4 dots */
/* The integer part of a K-quant dot is exact, so the blocks are first unpacked to signed bytes
 * (as ggml's generic dot does into aux8) and the integer sums run over plain arrays; the float
 * combination keeps the contract's order. or_gemv runs the AVX2 form below (the same integers);
 * these plain dots are its check (or_gemv_scalar_dots). */
static void unpack_q4k(const uint8_t *blk, int8_t q[256], int sc[8], int mn[8]) {
    const uint8_t *qs = blk + 16;
    for (int g = 0; g < 4; g++) {
        q4k_scale_min(blk + 4, 2 * g, &sc[2 * g], &mn[2 * g]);
        q4k_scale_min(blk + 4, 2 * g + 1, &sc[2 * g + 1], &mn[2 * g + 1]);
        for (int l = 0; l < 32; l++) {
            q[64 * g + l] = (int8_t)(qs[32 * g + l] & 0xF);
            q[64 * g + 32 + l] = (int8_t)(qs[32 * g + l] >> 4);
        }
    }
}

static void unpack_q6k(const uint8_t *blk, int8_t q[256]) {
    const uint8_t *ql = blk, *qh = blk + 128;
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            const uint8_t a = ql[64 * n + l], b = ql[64 * n + 32 + l], h = qh[32 * n + l];
            q[128 * n + l] = (int8_t)(((a & 0xF) | (((h >> 0) & 3) << 4)) - 32);
            q[128 * n + 32 + l] = (int8_t)(((b & 0xF) | (((h >> 2) & 3) << 4)) - 32);
            q[128 * n + 64 + l] = (int8_t)(((a >> 4) | (((h >> 4) & 3) << 4)) - 32);
            q[128 * n + 96 + l] = (int8_t)(((b >> 4) | (((h >> 6) & 3) << 4)) - 32);
        }
}

static inline int32_t idot(const int8_t *a, const int8_t *b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

static float dot_q4k_row(const uint8_t *row, const or_block_q8k *a, int nsb) {
    float acc = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 144 * b;
        const or_block_q8k *ab = a + b;
        int8_t q[256];
        int sc[8], mn[8];
        unpack_q4k(blk, q, sc, mn);
        float dw = or_f16_to_f32(rd16(blk)), dminw = or_f16_to_f32(rd16(blk + 2));
        int32_t sumi = 0, summ = 0;
        for (int j = 0; j < 8; j++) {
            sumi += sc[j] * idot(q + 32 * j, ab->qs + 32 * j, 32);
            summ += mn[j] * (ab->bsums[2 * j] + ab->bsums[2 * j + 1]);
        }
        float t1 = dw * ab->d;
        float t2 = (float)sumi * t1;
        float t3 = dminw * ab->d;
        float t4 = (float)summ * t3;
        acc = acc + (t2 - t4);
    }
    return acc;
}

static float dot_q6k_row(const uint8_t *row, const or_block_q8k *a, int nsb) {
    float acc = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 210 * b;
        const or_block_q8k *ab = a + b;
        const int8_t *sc = (const int8_t *)(blk + 192);
        int8_t q[256];
        unpack_q6k(blk, q);
        float dw = or_f16_to_f32(rd16(blk + 208));
        int32_t sumi = 0;
        for (int s = 0; s < 16; s++) sumi += sc[s] * idot(q + 16 * s, ab->qs + 16 * s, 16);
        acc = acc + (float)sumi * (dw * ab->d);
    }
    return acc;
}

static void butterfly32(float v[32]) {
    for (int o = 16; o >= 1; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ o];
        memcpy(v, t, sizeof t);
    }
}

float or_dot_p2(const float *a, const float *b, int n) {
    float lane[32];
    for (int l = 0; l < 32; l++) {
        float acc = 0.0f;
        for (int i = l; i < n; i += 32) acc = fmaf(a[i], b[i], acc);
        lane[l] = acc;
    }
    butterfly32(lane);
    return lane[0];
}

float or_sumsq_p2(const float *x, int n) { return or_dot_p2(x, x, n); }

static float sum_p2(const float *x, int n) {
    float lane[32];
    for (int l = 0; l < 32; l++) {
        float acc = 0.0f;
        for (int i = l; i < n; i += 32) acc = acc + x[i];
        lane[l] = acc;
    }
    butterfly32(lane);
    return lane[0];
}

static float dot_q4k_row_avx2(const uint8_t *row, const or_block_q8k *a, int nsb);
static float dot_q6k_row_avx2(const uint8_t *row, const or_block_q8k *a, int nsb);

int or_gemv(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y) {
    const uint8_t *w = (const uint8_t *)W;
    if (type == OR_F32) {
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++) y[r] = or_dot_p2((const float *)(w + r * cols * 4), x, (int)cols);
        return 0;
    }
    if ((type != OR_Q4_K && type != OR_Q6_K) || cols % 256) return -1;
    int nsb = (int)(cols / 256);
    or_block_q8k *a = (or_block_q8k *)malloc(sizeof(or_block_q8k) * (size_t)nsb);
    or_quantize_q8k(x, cols, a);
    int64_t rb = or_row_bytes(type, cols);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        y[r] = (type == OR_Q4_K) ? dot_q4k_row_avx2(w + r * rb, a, nsb) : dot_q6k_row_avx2(w + r * rb, a, nsb);
    free(a);
    return 0;
}

/* ------------------------------------------------------------------ C6 norm */
void or_rmsnorm(const float *x, const float *w, int n, float eps, float *y) {
    float mean = or_sumsq_p2(x, n) / (float)n;
    float s = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] * s) * w[i];
}

/* ------------------------------------------------------------------ C9 rope */
void or_rope_table(int n_pos, int n_rot, float base, float *cs) {
    float theta_scale = powf(base, -2.0f / (float)n_rot);
    for (int p = 0; p < n_pos; p++) {
        float theta = (float)p;
        float *row = cs + (size_t)p * n_rot;
        for (int i = 0; i < n_rot / 2; i++) {
            row[2 * i] = cosf(theta);
            row[2 * i + 1] = sinf(theta);
            theta *= theta_scale;
        }
    }
}

void or_rope_neox(float *x, int n_rot, const float *cs) {
    int h = n_rot / 2;
    for (int i = 0; i < h; i++) {
        float c = cs[2 * i], s = cs[2 * i + 1];
        float x0 = x[i], x1 = x[i + h];
        float a = x0 * c, b = x1 * s, e = x0 * s, f = x1 * c;
        x[i] = a - b;
        x[i + h] = e + f;
    }
}

/* ------------------------------------------------------------------ router */
void or_softmax(const float *logits, int n, float *probs) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = logits[i] > m ? logits[i] : m;
    for (int i = 0; i < n; i++) probs[i] = or_exp(logits[i] - m);
    float s = sum_p2(probs, n);
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) probs[i] = probs[i] * inv;
}

/* f32::total_cmp as a signed integer key */
static inline int32_t total_key(float f) {
    int32_t b;
    memcpy(&b, &f, 4);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return b;
}

void or_route(const float *probs, int n, int k, int32_t *ids, float *weights) {
    /* stable sort descending by total_cmp == rank by (key desc, index asc) */
    int taken = 0;
    int32_t *order = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    for (int i = 0; i < n; i++) order[i] = i;
    for (int i = 1; i < n; i++) { /* insertion sort: stable */
        int32_t v = order[i];
        int j = i - 1;
        while (j >= 0 && total_key(probs[order[j]]) < total_key(probs[v])) {
            order[j + 1] = order[j];
            j--;
        }
        order[j + 1] = v;
    }
    if (k > n) k = n;
    float total = 0.0f;
    for (int i = 0; i < k; i++) {
        ids[i] = order[i];
        weights[i] = probs[order[i]];
        total = total + weights[i];
        taken++;
    }
    if (total > 0.0f)
        for (int i = 0; i < taken; i++) weights[i] = weights[i] / total;
    free(order);
}

uint32_t or_argmax(const float *logits, int64_t n) {
    if (n <= 0) return 0;
    int64_t best = 0;
    int32_t bk = total_key(logits[0]);
    for (int64_t i = 1; i < n; i++) {
        int32_t k = total_key(logits[i]);
        if (k >= bk) { /* max_by keeps the last of equal maxima */
            bk = k;
            best = i;
        }
    }
    return (uint32_t)best;
}

/* ------------------------------------------------------------------ C8 attention */
/* f16 -> f32 by F16C (vcvtph2ps): exact for every finite value and infinity, as or_f16_to_f32;
 * a signalling NaN comes out quiet, which changes no non-NaN result. */
#include <immintrin.h>
/* 8x8 transpose of eight f32 vectors (r[i] lane j -> r[j] lane i) */
static inline void transpose8(__m256 r[8]) {
    __m256 t0 = _mm256_unpacklo_ps(r[0], r[1]), t1 = _mm256_unpackhi_ps(r[0], r[1]);
    __m256 t2 = _mm256_unpacklo_ps(r[2], r[3]), t3 = _mm256_unpackhi_ps(r[2], r[3]);
    __m256 t4 = _mm256_unpacklo_ps(r[4], r[5]), t5 = _mm256_unpackhi_ps(r[4], r[5]);
    __m256 t6 = _mm256_unpacklo_ps(r[6], r[7]), t7 = _mm256_unpackhi_ps(r[6], r[7]);
    __m256 u0 = _mm256_shuffle_ps(t0, t2, 0x44), u1 = _mm256_shuffle_ps(t0, t2, 0xEE);
    __m256 u2 = _mm256_shuffle_ps(t1, t3, 0x44), u3 = _mm256_shuffle_ps(t1, t3, 0xEE);
    __m256 u4 = _mm256_shuffle_ps(t4, t6, 0x44), u5 = _mm256_shuffle_ps(t4, t6, 0xEE);
    __m256 u6 = _mm256_shuffle_ps(t5, t7, 0x44), u7 = _mm256_shuffle_ps(t5, t7, 0xEE);
    r[0] = _mm256_permute2f128_ps(u0, u4, 0x20);
    r[1] = _mm256_permute2f128_ps(u1, u5, 0x20);
    r[2] = _mm256_permute2f128_ps(u2, u6, 0x20);
    r[3] = _mm256_permute2f128_ps(u3, u7, 0x20);
    r[4] = _mm256_permute2f128_ps(u0, u4, 0x31);
    r[5] = _mm256_permute2f128_ps(u1, u5, 0x31);
    r[6] = _mm256_permute2f128_ps(u2, u6, 0x31);
    r[7] = _mm256_permute2f128_ps(u3, u7, 0x31);
}

/* The K-quant row dots with AVX2 integer arithmetic, as ggml's x86 path computes them: the
 * unsigned weight values times the signed Q8_K values by _mm256_maddubs_epi16 (no pair sum
 * saturates: |15·128·2| and |63·128·2| are below 2^15), widened by _mm256_madd_epi16 and scaled
 * per sub-block in int32. The integer sums are exact, so they equal dot_q4k_row's and
 * dot_q6k_row's; the float combination is the same code in the same order. */
static inline int32_t hsum_epi32(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}

static float dot_q4k_row_avx2(const uint8_t *row, const or_block_q8k *a, int nsb) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), ones = _mm256_set1_epi16(1);
    float acc = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 144 * b;
        const or_block_q8k *ab = a + b;
        int sc[8], mn[8];
        for (int j = 0; j < 8; j++) q4k_scale_min(blk + 4, j, &sc[j], &mn[j]);
        __m256i vs = _mm256_setzero_si256();
        for (int g = 0; g < 4; g++) {
            const __m256i w = _mm256_loadu_si256((const __m256i *)(blk + 16 + 32 * g));
            const __m256i lo = _mm256_and_si256(w, m4), hi = _mm256_and_si256(_mm256_srli_epi16(w, 4), m4);
            const __m256i a0 = _mm256_loadu_si256((const __m256i *)(ab->qs + 64 * g));
            const __m256i a1 = _mm256_loadu_si256((const __m256i *)(ab->qs + 64 * g + 32));
            const __m256i d0 = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, a0), ones);
            const __m256i d1 = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, a1), ones);
            vs = _mm256_add_epi32(vs, _mm256_mullo_epi32(d0, _mm256_set1_epi32(sc[2 * g])));
            vs = _mm256_add_epi32(vs, _mm256_mullo_epi32(d1, _mm256_set1_epi32(sc[2 * g + 1])));
        }
        const int32_t sumi = hsum_epi32(vs);
        int32_t summ = 0;
        for (int j = 0; j < 8; j++) summ += mn[j] * (ab->bsums[2 * j] + ab->bsums[2 * j + 1]);
        float dw = or_f16_to_f32(rd16(blk)), dminw = or_f16_to_f32(rd16(blk + 2));
        float t1 = dw * ab->d;
        float t2 = (float)sumi * t1;
        float t3 = dminw * ab->d;
        float t4 = (float)summ * t3;
        acc = acc + (t2 - t4);
    }
    return acc;
}

static float dot_q6k_row_avx2(const uint8_t *row, const or_block_q8k *a, int nsb) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), m3 = _mm256_set1_epi8(0x03), ones = _mm256_set1_epi16(1);
    float acc = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 210 * b;
        const or_block_q8k *ab = a + b;
        const int8_t *sc = (const int8_t *)(blk + 192);
        __m256i vs = _mm256_setzero_si256();
        for (int n = 0; n < 2; n++) {
            const __m256i la = _mm256_loadu_si256((const __m256i *)(blk + 64 * n));
            const __m256i lb = _mm256_loadu_si256((const __m256i *)(blk + 64 * n + 32));
            const __m256i h = _mm256_loadu_si256((const __m256i *)(blk + 128 + 32 * n));
            /* the unsigned 6-bit values q + 32 of values 128n + 32k + l, l = 0..31 */
            __m256i u[4];
            u[0] = _mm256_or_si256(_mm256_and_si256(la, m4), _mm256_slli_epi16(_mm256_and_si256(h, m3), 4));
            u[1] = _mm256_or_si256(_mm256_and_si256(lb, m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 2), m3), 4));
            u[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(la, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 4), m3), 4));
            u[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(lb, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 6), m3), 4));
            for (int k = 0; k < 4; k++) {
                const __m256i av = _mm256_loadu_si256((const __m256i *)(ab->qs + 128 * n + 32 * k));
                const __m256i d = _mm256_madd_epi16(_mm256_maddubs_epi16(u[k], av), ones);
                /* lanes 0-3: sub-block 8n + 2k (values l < 16), lanes 4-7: sub-block 8n + 2k + 1 */
                const int s0 = sc[8 * n + 2 * k], s1 = sc[8 * n + 2 * k + 1];
                vs = _mm256_add_epi32(vs, _mm256_mullo_epi32(d, _mm256_setr_epi32(s0, s0, s0, s0, s1, s1, s1, s1)));
            }
        }
        int32_t corr = 0;  /* the -32 offset: 32 * sum_s sc_s * (sum of the sub-block's 16 activations) */
        for (int s2 = 0; s2 < 16; s2++) corr += sc[s2] * ab->bsums[s2];
        const int32_t sumi = hsum_epi32(vs) - 32 * corr;
        float dw = or_f16_to_f32(rd16(blk + 208));
        acc = acc + (float)sumi * (dw * ab->d);
    }
    return acc;
}

int or_gemv_scalar_dots(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y) {
    /* or_gemv with the plain C dots: the check that the AVX2 dots give the same bits */
    if ((type != OR_Q4_K && type != OR_Q6_K) || cols % 256) return -1;
    const int nsb = (int)(cols / 256);
    or_block_q8k *a = (or_block_q8k *)malloc(sizeof(or_block_q8k) * (size_t)nsb);
    or_quantize_q8k(x, cols, a);
    const int64_t rb = or_row_bytes(type, cols);
    for (int64_t r = 0; r < rows; r++)
        y[r] = (type == OR_Q4_K) ? dot_q4k_row((const uint8_t *)W + r * rb, a, nsb)
                                 : dot_q6k_row((const uint8_t *)W + r * rb, a, nsb);
    free(a);
    return 0;
}

void or_attn_head(const float *q, const uint16_t *k, const uint16_t *v, int64_t ld, int nk,
                  int head_dim, float scale, int chunk, float *out) {
    float qf[512];
    for (int d = 0; d < head_dim; d++) qf[d] = or_f16_to_f32(or_f32_to_f16(q[d]));
    int nc = (nk + chunk - 1) / chunk;
    float *mc = (float *)malloc(sizeof(float) * (size_t)nc);
    float *lc = (float *)malloc(sizeof(float) * (size_t)nc);
    float *ac = (float *)calloc((size_t)nc * head_dim, sizeof(float));
    float *s = (float *)malloc(sizeof(float) * (size_t)chunk);
    float *p = (float *)malloc(sizeof(float) * (size_t)chunk);
    for (int c = 0; c < nc; c++) {
        int base = c * chunk, cnt = nk - base < chunk ? nk - base : chunk;
        float m = -INFINITY;
        /* eight keys at a time: each key's dot is its own in-order fmaf chain over d (one lane
         * of a fused multiply-add), the eight chains only run side by side */
        for (int j0 = 0; j0 < cnt; j0 += 8) {
            const int nj = cnt - j0 < 8 ? cnt - j0 : 8;
            __m256 acc = _mm256_setzero_ps();
            for (int d0 = 0; d0 < head_dim; d0 += 8) {
                __m256 r[8];
                for (int jj = 0; jj < 8; jj++) {
                    const uint16_t *kr = k + (int64_t)(base + j0 + (jj < nj ? jj : 0)) * ld + d0;
                    r[jj] = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)kr));
                }
                transpose8(r); /* r[e] = element d0 + e of the eight keys */
                for (int e = 0; e < 8; e++) acc = _mm256_fmadd_ps(_mm256_set1_ps(qf[d0 + e]), r[e], acc);
            }
            float av[8];
            _mm256_storeu_ps(av, acc);
            for (int jj = 0; jj < nj; jj++) {
                s[j0 + jj] = av[jj] * scale;
                m = s[j0 + jj] > m ? s[j0 + jj] : m;
            }
        }
        for (int j = 0; j < chunk; j++) p[j] = j < cnt ? or_exp(s[j] - m) : 0.0f;
        float l = 0.0f;
        for (int w = 0; w < chunk / 32; w++) {
            float lane[32];
            memcpy(lane, p + 32 * w, sizeof lane);
            butterfly32(lane);
            l = l + lane[0];
        }
        float *a = ac + (size_t)c * head_dim;
        if (head_dim == 128) { /* the 128 sums in 16 registers across the keys: the same chains */
            __m256 acc8[16];
            for (int i = 0; i < 16; i++) acc8[i] = _mm256_setzero_ps();
            for (int j = 0; j < cnt; j++) { /* a[d] = fmaf(p_j, v_jd, a[d]) in key order */
                const uint16_t *vr = v + (int64_t)(base + j) * ld;
                const __m256 pj = _mm256_set1_ps(p[j]);
                for (int i = 0; i < 16; i++)
                    acc8[i] = _mm256_fmadd_ps(pj, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(vr + 8 * i))), acc8[i]);
            }
            for (int i = 0; i < 16; i++) _mm256_storeu_ps(a + 8 * i, acc8[i]);
        } else {
            for (int j = 0; j < cnt; j++) { /* a[d] = fmaf(p_j, v_jd, a[d]) in key order */
                const uint16_t *vr = v + (int64_t)(base + j) * ld;
                const __m256 pj = _mm256_set1_ps(p[j]);
                for (int d0 = 0; d0 < head_dim; d0 += 8) {
                    const __m256 vv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(vr + d0)));
                    _mm256_storeu_ps(a + d0, _mm256_fmadd_ps(pj, vv, _mm256_loadu_ps(a + d0)));
                }
            }
        }
        mc[c] = m;
        lc[c] = l;
    }
    float M = -INFINITY;
    for (int c = 0; c < nc; c++) M = mc[c] > M ? mc[c] : M;
    float L = 0.0f;
    for (int d = 0; d < head_dim; d++) out[d] = 0.0f;
    for (int c = 0; c < nc; c++) {
        float f = or_exp(mc[c] - M);
        L = fmaf(lc[c], f, L);
        for (int d = 0; d < head_dim; d++) out[d] = fmaf(ac[(size_t)c * head_dim + d], f, out[d]);
    }
    for (int d = 0; d < head_dim; d++) out[d] = out[d] / L;
    free(mc);
    free(lc);
    free(ac);
    free(s);
    free(p);
}

/* ------------------------------------------------------------------ ggml-cpu's generic algorithms
 * A second set of numerics, chosen per op by the bits of or_config.numerics (OR_NUM_*), that
 * restates the scalar ("generic", no SIMD) code paths of ggml's CPU backend for the calls the
 * reference makes on this path. It is not what the device computes: it measures how far the
 * arithmetic contract above lies from ggml's own results on the same model and tokens.
 * ggml is llama.cpp's tensor library (MIT), unpinned in the reference (git HEAD, CI); these are
 * restatements of its published algorithms, cited by function:
 *  - rms_norm (ggml_compute_forward_rms_norm_f32; call site graph.rs:705): sum of the f32
 *    squares in ggml_float (double), in order; mean = (float)(sum / n); scale = 1.0f /
 *    sqrtf(mean + eps); y = x * scale, then ggml_mul by the weight;
 *  - mul_mat of a K-quant matrix (graph.rs:690): activations to Q8_K (quantize_row_q8_K_ref, the
 *    contract's C3), then ggml_vec_dot_q{4,6}_K_q8_K_generic: eight int32 lanes per superblock
 *    (lane l collects positions l mod 8), float lanes sums[l] += d * aux32[l] over superblocks,
 *    the Q4_K min term subtracted from a separate float sumf per superblock, lanes added at end;
 *  - mul_mat of an F32 matrix (the router): ggml_vec_dot_f32 generic, products in f32, sum in
 *    double, in order;
 *  - soft_max_ext(logits, no mask, scale 1, max_bias 0) (graph.rs:1616-1630): max in order,
 *    val = expf(x - max) (libm), sum in double, y = val * (float)(1.0 / sum);
 *  - silu (graph.rs:731): x / (1.0f + expf(-x)) (libm), then ggml_mul by up and ggml_scale by
 *    the route weight;
 *  - flash_attn_ext (graph.rs:1220-1247; ggml_compute_forward_flash_attn_ext_f16_one_chunk): q
 *    converted to f16; per key in order: s = ggml_vec_dot_f16 (f16 products in f32, summed in
 *    double) * scale; online softmax: a new maximum M rescales the accumulator by
 *    ms = expf(Mold - M) (ggml_vec_scale_f16), else vs = expf(s - M); the value row is added
 *    with weight vs (ggml_vec_mad_f16: y = f16(f32(y) + f32(v) * vs)); S = S * ms + vs; at the
 *    end out = f32(acc) * (1.0f / S). With f16 values ggml keeps that accumulator in f16 (the
 *    VKQ16 buffer); OR_NUM_ATTN_F32V keeps it in f32 instead, the accumulation of ggml's
 *    f32-value branch, to show how much of the distance the f16 accumulator accounts for.
 * Multiplications and additions are separately rounded (ggml's generic C is compiled as ISO C,
 * where GCC does not contract them). OR_NUM_FMA contracts the multiply-adds of the K-quant dot
 * lanes and of the attention accumulator into fmaf, as a GNU-C build of the same generic code
 * would: another build of ggml, to show how far two builds of ggml lie from each other. */
static float gg_sumsq_scale(const float *x, int n, float eps) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    return 1.0f / sqrtf(mean + eps);
}

static void gg_rmsnorm(const float *x, const float *w, int n, float eps, float *y) {
    const float sc = gg_sumsq_scale(x, n, eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] * sc) * w[i];
}

static float gg_dot_q4k_row(const uint8_t *row, const or_block_q8k *a, int nsb, int fma) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sumf = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 144 * b;
        const or_block_q8k *ab = a + b;
        int8_t q[256];
        int sc[8], mn[8];
        unpack_q4k(blk, q, sc, mn);
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; j++)         /* sub-blocks of 32 */
            for (int k = 0; k < 4; k++)     /* four groups of 8 */
                for (int l = 0; l < 8; l++) aux32[l] += sc[j] * (q[32 * j + 8 * k + l] * ab->qs[32 * j + 8 * k + l]);
        int32_t summ = 0;
        for (int j = 0; j < 16; j++) summ += ab->bsums[j] * mn[j / 2];
        const float d = or_f16_to_f32(rd16(blk)) * ab->d;
        for (int l = 0; l < 8; l++) sums[l] = fma ? fmaf(d, (float)aux32[l], sums[l]) : sums[l] + d * (float)aux32[l];
        const float dmin = or_f16_to_f32(rd16(blk + 2)) * ab->d;
        sumf = fma ? fmaf(-dmin, (float)summ, sumf) : sumf - dmin * (float)summ;
    }
    for (int l = 0; l < 8; l++) sumf += sums[l];
    return sumf;
}

static float gg_dot_q6k_row(const uint8_t *row, const or_block_q8k *a, int nsb, int fma) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sumf = 0.0f;
    for (int b = 0; b < nsb; b++) {
        const uint8_t *blk = row + 210 * b;
        const or_block_q8k *ab = a + b;
        const int8_t *sc = (const int8_t *)(blk + 192);
        int8_t q[256];
        unpack_q6k(blk, q);
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 16; j++)        /* sub-blocks of 16 */
            for (int k = 0; k < 2; k++)
                for (int l = 0; l < 8; l++) aux32[l] += sc[j] * (q[16 * j + 8 * k + l] * ab->qs[16 * j + 8 * k + l]);
        const float d = or_f16_to_f32(rd16(blk + 208)) * ab->d;
        for (int l = 0; l < 8; l++) sums[l] = fma ? fmaf(d, (float)aux32[l], sums[l]) : sums[l] + d * (float)aux32[l];
    }
    for (int l = 0; l < 8; l++) sumf += sums[l];
    return sumf;
}

static float gg_dot_f32(const float *a, const float *b, int n) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)(a[i] * b[i]);
    return (float)sum;
}

static int gg_gemv(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y, int fma) {
    const uint8_t *w = (const uint8_t *)W;
    if (type == OR_F32) {
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++) y[r] = gg_dot_f32((const float *)(w + r * cols * 4), x, (int)cols);
        return 0;
    }
    if ((type != OR_Q4_K && type != OR_Q6_K) || cols % 256) return -1;
    const int nsb = (int)(cols / 256);
    or_block_q8k *a = (or_block_q8k *)malloc(sizeof(or_block_q8k) * (size_t)nsb);
    or_quantize_q8k(x, cols, a);
    const int64_t rb = or_row_bytes(type, cols);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        y[r] = (type == OR_Q4_K) ? gg_dot_q4k_row(w + r * rb, a, nsb, fma) : gg_dot_q6k_row(w + r * rb, a, nsb, fma);
    free(a);
    return 0;
}

static void gg_softmax(const float *x, int n, float *y) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
        const float v = expf(x[i] - mx);
        sum += (double)v;
        y[i] = v;
    }
    const float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; i++) y[i] *= inv;
}

static float gg_silu(float x) { return x / (1.0f + expf(-x)); }

static void gg_attn_head(const float *q, const uint16_t *k, const uint16_t *v, int64_t ld, int nk, int head_dim,
                         float scale, int f32_acc, int fma, float *out) {
    float qf[512], acc32[512];
    uint16_t acc16[512];
    for (int d = 0; d < head_dim; d++) {
        qf[d] = or_f16_to_f32(or_f32_to_f16(q[d]));
        acc32[d] = 0.0f;
        acc16[d] = 0;
    }
    float S = 0.0f, M = -INFINITY;
    for (int j = 0; j < nk; j++) {
        const uint16_t *kr = k + (int64_t)j * ld, *vr = v + (int64_t)j * ld;
        double dot = 0.0;
        for (int d = 0; d < head_dim; d++) dot += (double)(or_f16_to_f32(kr[d]) * qf[d]);
        float s = (float)dot;
        s = s * scale;
        s += 0.0f; /* the causal mask: 0 for every visible key */
        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        if (s > M) {
            M = s;
            ms = expf(Mold - M);
            for (int d = 0; d < head_dim; d++) {
                if (f32_acc) acc32[d] *= ms;
                else acc16[d] = or_f32_to_f16(or_f16_to_f32(acc16[d]) * ms);
            }
        } else {
            vs = expf(s - M);
        }
        for (int d = 0; d < head_dim; d++) {
            const float a0 = f32_acc ? acc32[d] : or_f16_to_f32(acc16[d]), vv = or_f16_to_f32(vr[d]);
            const float a1 = fma ? fmaf(vv, vs, a0) : a0 + vv * vs;
            if (f32_acc) acc32[d] = a1;
            else acc16[d] = or_f32_to_f16(a1);
        }
        S = S * ms + vs;
    }
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
    for (int d = 0; d < head_dim; d++) out[d] = (f32_acc ? acc32[d] : or_f16_to_f32(acc16[d])) * S_inv;
}

/* the per-op dispatch the model uses: each op takes ggml's algorithm when its bit is set */
static int num_gemv(int mode, int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y) {
    const int bit = type == OR_F32 ? OR_NUM_FDOT : OR_NUM_QDOT;
    return (mode & bit) ? gg_gemv(type, W, rows, cols, x, y, (mode & OR_NUM_FMA) != 0)
                        : or_gemv(type, W, rows, cols, x, y);
}
static void num_rmsnorm(int mode, const float *x, const float *w, int n, float eps, float *y) {
    if (mode & OR_NUM_NORM) gg_rmsnorm(x, w, n, eps, y);
    else or_rmsnorm(x, w, n, eps, y);
}
static void num_softmax(int mode, const float *x, int n, float *y) {
    if (mode & OR_NUM_SOFTMAX) gg_softmax(x, n, y);
    else or_softmax(x, n, y);
}
static float num_silu(int mode, float x) { return (mode & OR_NUM_SILU) ? gg_silu(x) : or_silu(x); }

/* single ops of the ggml mode, for the tests' independent numpy restatement */
void or_ggml_rmsnorm(const float *x, const float *w, int n, float eps, float *y) { gg_rmsnorm(x, w, n, eps, y); }
int or_ggml_gemv(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y) {
    return gg_gemv(type, W, rows, cols, x, y, 0);
}
void or_ggml_softmax(const float *x, int n, float *y) { gg_softmax(x, n, y); }
void or_ggml_attn_head(const float *q, const uint16_t *k, const uint16_t *v, int64_t ld, int nk, int head_dim,
                       float scale, int f32_acc, float *out) {
    gg_attn_head(q, k, v, ld, nk, head_dim, scale, f32_acc, 0, out);
}

/* ------------------------------------------------------------------ model */
typedef struct {
    int type;
    int64_t ne[4];
    const uint8_t *data;
} tref;

typedef struct {
    tref attn_norm, q, k, v, q_norm, k_norm, o, ffn_norm, gate_inp, gate, up, down;
    tref gate_bias; /* optional ffn_gate_inp.bias: data NULL when absent */
    /* optional shared expert (ffn_{gate,up,down}_shexp; data NULL when absent), added
     * unweighted to the routed sum before the residual as llama.cpp's deepseek2 graph does */
    tref gate_sh, up_sh, down_sh;
} layer_w;

struct or_model {
    or_config c;
    tref embd, out_norm, out;
    layer_w *L;
    float *rope; /* [max_positions][n_rot] */
    /* debug captures of the last forward */
    int dbg_tokens;
    int32_t *dbg_ids;   /* [n_layer][T][k] */
    float *dbg_w;       /* [n_layer][T][k] */
    float *dbg_hidden;  /* [T][E] */
    float *dbg_gap;     /* [n_layer][T]: the K-th largest router probability minus the (K+1)-th */
    /* when set: route() is replaced by that model's choice for the same layer and token in its
     * last forward (the weights still come from this model's own probabilities), so that two
     * numerics can be compared without the discontinuity of a different expert set */
    const struct or_model *route_from;
};

struct or_kv {
    const or_model *m;
    int len;
    int kvw;
    uint16_t **k, **v; /* per layer [max_positions][kvw] */
};

static int find_tensor(const or_tensor *ts, int n, const char *name, tref *out, int required) {
    for (int i = 0; i < n; i++) {
        if (strcmp(ts[i].name, name) == 0) {
            out->type = ts[i].type;
            memcpy(out->ne, ts[i].ne, sizeof out->ne);
            out->data = (const uint8_t *)ts[i].data;
            return 0;
        }
    }
    out->data = NULL;
    if (required) {
        char msg[256];
        snprintf(msg, sizeof msg, "missing tensor %s", name);
        set_err(msg);
        return -1;
    }
    return 0;
}

or_model *or_model_new(const or_config *cfg, const or_tensor *ts, int n) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->c = *cfg;
    if (m->c.expert_workers <= 0) m->c.expert_workers = 4;
    if (m->c.attn_chunk <= 0) m->c.attn_chunk = 128;
    if (m->c.n_rot <= 0) m->c.n_rot = m->c.head_dim;
    int bad = 0;
    bad |= find_tensor(ts, n, "token_embd.weight", &m->embd, 1);
    bad |= find_tensor(ts, n, "output_norm.weight", &m->out_norm, 1);
    find_tensor(ts, n, "output.weight", &m->out, 0);
    if (!m->out.data) m->out = m->embd;
    m->L = (layer_w *)calloc((size_t)cfg->n_layer, sizeof(layer_w));
    char nm[128];
#define GETW(field, suffix)                                              \
    snprintf(nm, sizeof nm, "blk.%d.%s", il, suffix);                    \
    bad |= find_tensor(ts, n, nm, &m->L[il].field, 1);
    for (int il = 0; il < cfg->n_layer; il++) {
        GETW(attn_norm, "attn_norm.weight");
        GETW(q, "attn_q.weight");
        GETW(k, "attn_k.weight");
        GETW(v, "attn_v.weight");
        GETW(q_norm, "attn_q_norm.weight");
        GETW(k_norm, "attn_k_norm.weight");
        GETW(o, "attn_output.weight");
        GETW(ffn_norm, "ffn_norm.weight");
        GETW(gate_inp, "ffn_gate_inp.weight");
        snprintf(nm, sizeof nm, "blk.%d.ffn_gate_inp.bias", il);
        find_tensor(ts, n, nm, &m->L[il].gate_bias, 0);
        snprintf(nm, sizeof nm, "blk.%d.ffn_gate_shexp.weight", il);
        find_tensor(ts, n, nm, &m->L[il].gate_sh, 0);
        snprintf(nm, sizeof nm, "blk.%d.ffn_up_shexp.weight", il);
        find_tensor(ts, n, nm, &m->L[il].up_sh, 0);
        snprintf(nm, sizeof nm, "blk.%d.ffn_down_shexp.weight", il);
        find_tensor(ts, n, nm, &m->L[il].down_sh, 0);
        if ((m->L[il].gate_sh.data != NULL) != (m->L[il].down_sh.data != NULL) ||
            (m->L[il].gate_sh.data != NULL) != (m->L[il].up_sh.data != NULL)) {
            set_err("a shared expert needs its gate, up and down tensors");
            bad = 1;
        }
        GETW(gate, "ffn_gate_exps.weight");
        GETW(up, "ffn_up_exps.weight");
        GETW(down, "ffn_down_exps.weight");
    }
#undef GETW
    if (bad) {
        or_model_free(m);
        return NULL;
    }
    m->rope = (float *)malloc(sizeof(float) * (size_t)m->c.max_positions * m->c.n_rot);
    or_rope_table(m->c.max_positions, m->c.n_rot, m->c.rope_base, m->rope);
    return m;
}

void or_model_free(or_model *m) {
    if (!m) return;
    free(m->L);
    free(m->rope);
    free(m->dbg_ids);
    free(m->dbg_w);
    free(m->dbg_hidden);
    free(m->dbg_gap);
    free(m);
}

void or_model_route_from(or_model *m, const or_model *src) { m->route_from = src; }

int or_debug_route_gap(const or_model *m, int layer, int t, float *gap) {
    if (!m->dbg_gap || t >= m->dbg_tokens || layer >= m->c.n_layer) return -1;
    *gap = m->dbg_gap[(size_t)layer * m->dbg_tokens + t];
    return 0;
}

or_kv *or_kv_new(const or_model *m) {
    or_kv *kv = (or_kv *)calloc(1, sizeof(or_kv));
    kv->m = m;
    kv->kvw = m->c.n_head_kv * m->c.head_dim;
    kv->k = (uint16_t **)calloc((size_t)m->c.n_layer, sizeof(uint16_t *));
    kv->v = (uint16_t **)calloc((size_t)m->c.n_layer, sizeof(uint16_t *));
    for (int l = 0; l < m->c.n_layer; l++) {
        kv->k[l] = (uint16_t *)calloc((size_t)m->c.max_positions * kv->kvw, 2);
        kv->v[l] = (uint16_t *)calloc((size_t)m->c.max_positions * kv->kvw, 2);
    }
    return kv;
}

void or_kv_free(or_kv *kv) {
    if (!kv) return;
    for (int l = 0; l < kv->m->c.n_layer; l++) {
        free(kv->k[l]);
        free(kv->v[l]);
    }
    free(kv->k);
    free(kv->v);
    free(kv);
}

int or_kv_len(const or_kv *kv) { return kv->len; }
void or_kv_set_len(or_kv *kv, int n) { kv->len = n; }

void or_kv_read(const or_kv *kv, int layer, int n_pos, uint16_t *k, uint16_t *v) {
    memcpy(k, kv->k[layer], (size_t)n_pos * kv->kvw * 2);
    memcpy(v, kv->v[layer], (size_t)n_pos * kv->kvw * 2);
}

void or_kv_write(or_kv *kv, int layer, int n_pos, const uint16_t *k, const uint16_t *v) {
    memcpy(kv->k[layer], k, (size_t)n_pos * kv->kvw * 2);
    memcpy(kv->v[layer], v, (size_t)n_pos * kv->kvw * 2);
}

static const uint8_t *expert_slice(const tref *t, int e, int64_t rows, int64_t cols) {
    return t->data + (int64_t)e * rows * or_row_bytes(t->type, cols);
}

int or_forward(or_model *m, or_kv *kv, const int32_t *tokens, int T, int pos_start, float *logits) {
    const or_config *c = &m->c;
    const int E = c->n_embd, H = c->n_head, HK = c->n_head_kv, D = c->head_dim;
    const int NE = c->n_expert, K = c->n_expert_used, F = c->n_ff_exp;
    const int QW = H * D, KW = HK * D;
    const int mode = c->numerics;
    if (T <= 0) { set_err("no tokens"); return -1; }
    if (pos_start != kv->len) { set_err("pos_start must equal the cache length"); return -1; }
    if (pos_start + T > c->max_positions) { set_err("context exceeds max_positions"); return -1; }
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= c->n_vocab) { set_err("token id out of range"); return -1; }

    free(m->dbg_ids);
    free(m->dbg_w);
    free(m->dbg_hidden);
    free(m->dbg_gap);
    m->dbg_gap = (float *)calloc((size_t)c->n_layer * T, sizeof(float));
    m->dbg_tokens = T;
    m->dbg_ids = (int32_t *)calloc((size_t)c->n_layer * T * K, sizeof(int32_t));
    m->dbg_w = (float *)calloc((size_t)c->n_layer * T * K, sizeof(float));
    m->dbg_hidden = (float *)calloc((size_t)T * E, sizeof(float));

    float *x = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *xn = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *q = (float *)malloc(sizeof(float) * (size_t)T * QW);
    float *kk = (float *)malloc(sizeof(float) * (size_t)T * KW);
    float *vv = (float *)malloc(sizeof(float) * (size_t)T * KW);
    float *att = (float *)malloc(sizeof(float) * (size_t)T * QW);
    float *ao = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *ffin = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *rl = (float *)malloc(sizeof(float) * (size_t)NE);
    float *pr = (float *)malloc(sizeof(float) * (size_t)NE);
    float *g = (float *)malloc(sizeof(float) * (size_t)F);
    float *u = (float *)malloc(sizeof(float) * (size_t)F);
    float *o = (float *)malloc(sizeof(float) * (size_t)E);
    float *eo = (float *)malloc(sizeof(float) * (size_t)K * E);
    float *sum = (float *)malloc(sizeof(float) * (size_t)E);
    float *tot = (float *)malloc(sizeof(float) * (size_t)E);
    int FS = 0; /* the widest shared expert of the model */
    for (int il = 0; il < c->n_layer; il++)
        if (m->L[il].gate_sh.data && (int)m->L[il].gate_sh.ne[1] > FS) FS = (int)m->L[il].gate_sh.ne[1];
    float *gsh = (float *)malloc(sizeof(float) * (size_t)(FS > 0 ? FS : 1));
    float *ush = (float *)malloc(sizeof(float) * (size_t)(FS > 0 ? FS : 1));
    float *sh = (float *)malloc(sizeof(float) * (size_t)E);
    int32_t ids[64];
    float wts[64];

    /* embedding: get_rows dequantises the token's row (stream.rs:2192-2231) */
    int64_t erb = or_row_bytes(m->embd.type, E);
    for (int t = 0; t < T; t++) or_dequant(m->embd.type, m->embd.data + (int64_t)tokens[t] * erb, E, x + (size_t)t * E);

    const float scale = 1.0f / sqrtf((float)D);
    for (int il = 0; il < c->n_layer; il++) {
        const layer_w *w = &m->L[il];
        /* phase 1: attn norm, q/k/v, q/k head norms, rope (stream.rs:2265-2474) */
        for (int t = 0; t < T; t++) {
            float *xt = x + (size_t)t * E, *xnt = xn + (size_t)t * E;
            num_rmsnorm(mode, xt, (const float *)w->attn_norm.data, E, c->rms_eps, xnt);
            num_gemv(mode, w->q.type, w->q.data, QW, E, xnt, q + (size_t)t * QW);
            num_gemv(mode, w->k.type, w->k.data, KW, E, xnt, kk + (size_t)t * KW);
            num_gemv(mode, w->v.type, w->v.data, KW, E, xnt, vv + (size_t)t * KW);
            const float *cs = m->rope + (size_t)(pos_start + t) * c->n_rot;
            for (int h = 0; h < H; h++) {
                float *qh = q + (size_t)t * QW + h * D;
                num_rmsnorm(mode, qh, (const float *)w->q_norm.data, D, c->rms_eps, qh);
                or_rope_neox(qh, c->n_rot, cs);
            }
            for (int h = 0; h < HK; h++) {
                float *kh = kk + (size_t)t * KW + h * D;
                num_rmsnorm(mode, kh, (const float *)w->k_norm.data, D, c->rms_eps, kh);
                or_rope_neox(kh, c->n_rot, cs);
            }
            /* KvCache::push: f32 -> f16 (kv.rs:184-192) */
            uint16_t *kd = kv->k[il] + (size_t)(pos_start + t) * KW;
            uint16_t *vd = kv->v[il] + (size_t)(pos_start + t) * KW;
            for (int i = 0; i < KW; i++) {
                kd[i] = or_f32_to_f16(kk[(size_t)t * KW + i]);
                vd[i] = or_f32_to_f16(vv[(size_t)t * KW + i]);
            }
        }
        /* phase 2: attention over the history, causal (stream.rs:2554-2703) */
#pragma omp parallel for collapse(2) schedule(dynamic)
        for (int t = 0; t < T; t++)
            for (int h = 0; h < H; h++) {
                int g2 = h / (H / HK);
                if (mode & (OR_NUM_ATTN | OR_NUM_ATTN_F32V))
                    gg_attn_head(q + (size_t)t * QW + h * D, kv->k[il] + g2 * D, kv->v[il] + g2 * D, KW,
                                 pos_start + t + 1, D, scale, (mode & OR_NUM_ATTN_F32V) != 0, (mode & OR_NUM_FMA) != 0,
                                 att + (size_t)t * QW + h * D);
                else
                    or_attn_head(q + (size_t)t * QW + h * D, kv->k[il] + g2 * D, kv->v[il] + g2 * D, KW,
                                 pos_start + t + 1, D, scale, c->attn_chunk, att + (size_t)t * QW + h * D);
            }
        for (int t = 0; t < T; t++) {
            num_gemv(mode, w->o.type, w->o.data, E, QW, att + (size_t)t * QW, ao + (size_t)t * E);
            for (int i = 0; i < E; i++) ffin[(size_t)t * E + i] = x[(size_t)t * E + i] + ao[(size_t)t * E + i];
        }
        /* phase 3: ffn norm, router, softmax (stream.rs:2784-2831) and experts */
        for (int t = 0; t < T; t++) {
            float *fi = ffin + (size_t)t * E, *fn = xn + (size_t)t * E;
            num_rmsnorm(mode, fi, (const float *)w->ffn_norm.data, E, c->rms_eps, fn);
            num_gemv(mode, OR_F32, w->gate_inp.data, NE, E, fn, rl);
            if (w->gate_bias.data) /* ggml_add of the router bias: one f32 add per logit */
                for (int i = 0; i < NE; i++) rl[i] = rl[i] + ((const float *)w->gate_bias.data)[i];
            num_softmax(mode, rl, NE, pr);
            or_route(pr, NE, K, ids, wts);
            {
                float next = -INFINITY; /* the largest probability route() did not take */
                for (int e = 0; e < NE; e++) {
                    int taken = 0;
                    for (int i = 0; i < K; i++) taken |= ids[i] == e;
                    if (!taken && pr[e] > next) next = pr[e];
                }
                m->dbg_gap[(size_t)il * T + t] = pr[ids[K - 1]] - next;
            }
            if (m->route_from && m->route_from->dbg_ids && m->route_from->dbg_tokens == T) {
                float total = 0.0f;
                for (int i = 0; i < K; i++) {
                    ids[i] = m->route_from->dbg_ids[((size_t)il * T + t) * K + i];
                    wts[i] = pr[ids[i]];
                    total = total + wts[i];
                }
                if (total > 0.0f)
                    for (int i = 0; i < K; i++) wts[i] = wts[i] / total;
            }
            memcpy(m->dbg_ids + ((size_t)il * T + t) * K, ids, sizeof(int32_t) * K);
            memcpy(m->dbg_w + ((size_t)il * T + t) * K, wts, sizeof(float) * K);
            /* ascending expert order (BTreeMap in expert_ffn_block, stream.rs:916-926) */
            int32_t sid[64];
            float sw[64];
            for (int i = 0; i < K; i++) {
                sid[i] = ids[i];
                sw[i] = wts[i];
            }
            for (int i = 1; i < K; i++)
                for (int j = i; j > 0 && sid[j - 1] > sid[j]; j--) {
                    int32_t ti = sid[j];
                    sid[j] = sid[j - 1];
                    sid[j - 1] = ti;
                    float tw = sw[j];
                    sw[j] = sw[j - 1];
                    sw[j - 1] = tw;
                }
            for (int i = 0; i < K; i++) {
                int e = sid[i];
                num_gemv(mode, w->gate.type, expert_slice(&w->gate, e, F, E), F, E, fn, g);
                num_gemv(mode, w->up.type, expert_slice(&w->up, e, F, E), F, E, fn, u);
                for (int j = 0; j < F; j++) g[j] = num_silu(mode, g[j]) * u[j];
                num_gemv(mode, w->down.type, expert_slice(&w->down, e, E, F), E, F, g, o);
                for (int j = 0; j < E; j++) eo[(size_t)i * E + j] = o[j] * sw[i];
            }
            if (T == 1) {
                /* expert_ffn_single: chunks of ceil(K/workers), each summed in order by
                 * ggml_add, then partials added to a zero vector (stream.rs:1232-1284) */
                int workers = c->expert_workers < K ? c->expert_workers : K;
                if (workers < 1) workers = 1;
                int chunk = (K + workers - 1) / workers;
                for (int j = 0; j < E; j++) sum[j] = 0.0f;
                for (int s0 = 0; s0 < K; s0 += chunk) {
                    for (int j = 0; j < E; j++) tot[j] = eo[(size_t)s0 * E + j];
                    for (int i = s0 + 1; i < K && i < s0 + chunk; i++)
                        for (int j = 0; j < E; j++) tot[j] = tot[j] + eo[(size_t)i * E + j];
                    if (workers <= 1) memcpy(sum, tot, sizeof(float) * E);
                    else
                        for (int j = 0; j < E; j++) sum[j] = sum[j] + tot[j];
                }
            } else {
                /* expert_ffn_block: accum[t] += w * out, ascending experts (stream.rs:1051-1058) */
                for (int j = 0; j < E; j++) sum[j] = 0.0f;
                for (int i = 0; i < K; i++)
                    for (int j = 0; j < E; j++) sum[j] = sum[j] + eo[(size_t)i * E + j];
            }
            if (w->gate_sh.data) {
                /* shared expert: down(silu(gate x) * up x), then x = (moe + shexp) + ffn_inp */
                const int fs = (int)w->gate_sh.ne[1];
                num_gemv(mode, w->gate_sh.type, w->gate_sh.data, fs, E, fn, gsh);
                num_gemv(mode, w->up_sh.type, w->up_sh.data, fs, E, fn, ush);
                for (int j = 0; j < fs; j++) gsh[j] = num_silu(mode, gsh[j]) * ush[j];
                num_gemv(mode, w->down_sh.type, w->down_sh.data, E, fs, gsh, sh);
                for (int j = 0; j < E; j++) x[(size_t)t * E + j] = (sum[j] + sh[j]) + fi[j];
            } else {
                for (int j = 0; j < E; j++) x[(size_t)t * E + j] = fi[j] + sum[j];
            }
        }
    }
    kv->len += T;
    memcpy(m->dbg_hidden, x, sizeof(float) * (size_t)T * E);

    /* output head on the last position (stream.rs:2853-2914) */
    num_rmsnorm(mode, x + (size_t)(T - 1) * E, (const float *)m->out_norm.data, E, c->rms_eps, xn);
    num_gemv(mode, m->out.type, m->out.data, c->n_vocab, E, xn, logits);

    free(x); free(xn); free(q); free(kk); free(vv); free(att); free(ao); free(ffin);
    free(rl); free(pr); free(g); free(u); free(o); free(eo); free(sum); free(tot);
    free(gsh); free(ush); free(sh);
    return 0;
}

int or_debug_topk(const or_model *m, int layer, int t, int32_t *ids, float *weights) {
    if (!m->dbg_ids || t >= m->dbg_tokens || layer >= m->c.n_layer) return -1;
    int K = m->c.n_expert_used;
    memcpy(ids, m->dbg_ids + ((size_t)layer * m->dbg_tokens + t) * K, sizeof(int32_t) * K);
    memcpy(weights, m->dbg_w + ((size_t)layer * m->dbg_tokens + t) * K, sizeof(float) * K);
    return 0;
}

int or_debug_hidden(const or_model *m, int t, float *out) {
    if (!m->dbg_hidden || t >= m->dbg_tokens) return -1;
    memcpy(out, m->dbg_hidden + (size_t)t * m->c.n_embd, sizeof(float) * m->c.n_embd);
    return 0;
}

/* ------------------------------------------------------------------ seeded synthetic weights
 * The synthetic-weight generator the tests and the bench's CPU arm use, restated here so that
 * the CPU arm builds the same model bytes without loading the product library. Each
 * 256-element block of a tensor is a function of (seed, tensor id, element index) only:
 * values are an Irwin-Hall(4) approximation of N(mean, sigma) from one splitmix64 hash per
 * element, quantised by a simple K-quant quantiser (per 32-value sub-block min/max with 6-bit
 * scales and mins for Q4_K; per 16-value sub-block absolute max with int8 scales for Q6_K).
 * tests/test_oracle.py checks the bytes against the product's bt_synth_tensor. */
static uint64_t sy_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static float sy_value(uint64_t key, uint64_t idx, float mean, float scale) {
    uint64_t h = sy_mix(key + idx * 0xD1B54A32D192ED03ull);
    int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) + (int)(h >> 48);
    float z = (float)(s - 131070) * scale;
    return mean + z;
}

static int sy_clamp(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void sy_q4k(const float *x, uint8_t *out) {
    float scl[8], mns[8];
    for (int j = 0; j < 8; j++) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int l = 1; l < 32; l++) {
            float v = x[32 * j + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.0f) lo = 0.0f;
        scl[j] = (hi - lo) / 15.0f;
        mns[j] = -lo;
    }
    float ms = 0.0f, mm = 0.0f;
    for (int j = 0; j < 8; j++) {
        if (scl[j] > ms) ms = scl[j];
        if (mns[j] > mm) mm = mns[j];
    }
    uint16_t dh = or_f32_to_f16(ms / 63.0f), dmh = or_f32_to_f16(mm / 63.0f);
    float df = or_f16_to_f32(dh), dmf = or_f16_to_f32(dmh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = df > 0.0f ? sy_clamp((int)rintf(scl[j] / df), 0, 63) : 0;
        m[j] = dmf > 0.0f ? sy_clamp((int)rintf(mns[j] / dmf), 0, 63) : 0;
    }
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(dmh & 0xff);
    out[3] = (uint8_t)(dmh >> 8);
    for (int j = 0; j < 4; j++) { /* the 12 packed scale bytes of the Q4_K format */
        out[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        out[8 + j] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        out[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    for (int g = 0; g < 4; g++) {
        float d0 = df * (float)sc[2 * g], m0 = dmf * (float)m[2 * g];
        float d1 = df * (float)sc[2 * g + 1], m1 = dmf * (float)m[2 * g + 1];
        for (int l = 0; l < 32; l++) {
            int q0 = d0 > 0.0f ? sy_clamp((int)rintf((x[64 * g + l] + m0) / d0), 0, 15) : 0;
            int q1 = d1 > 0.0f ? sy_clamp((int)rintf((x[64 * g + 32 + l] + m1) / d1), 0, 15) : 0;
            out[16 + 32 * g + l] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

static void sy_q6k(const float *x, uint8_t *out) {
    float ds[16];
    for (int s = 0; s < 16; s++) {
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 16; i++) {
            float v = x[16 * s + i];
            if (fabsf(v) > amax) {
                amax = fabsf(v);
                mx = v;
            }
        }
        ds[s] = amax == 0.0f ? 0.0f : mx / -32.0f;
    }
    float amax = 0.0f, smax = 0.0f;
    for (int s = 0; s < 16; s++)
        if (fabsf(ds[s]) > amax) {
            amax = fabsf(ds[s]);
            smax = ds[s];
        }
    int L[256];
    int8_t sc[16];
    uint16_t dh = 0;
    if (amax == 0.0f) {
        for (int i = 0; i < 256; i++) L[i] = 32;
        memset(sc, 0, sizeof sc);
    } else {
        float iscale = -128.0f / smax;
        dh = or_f32_to_f16(1.0f / iscale);
        float df = or_f16_to_f32(dh);
        for (int s = 0; s < 16; s++) {
            sc[s] = (int8_t)sy_clamp((int)rintf(iscale * ds[s]), -128, 127);
            float den = df * (float)sc[s];
            for (int i = 0; i < 16; i++)
                L[16 * s + i] = (den != 0.0f ? sy_clamp((int)rintf(x[16 * s + i] / den), -32, 31) : 0) + 32;
        }
    }
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            int a = L[128 * n + l], b = L[128 * n + 32 + l], c = L[128 * n + 64 + l], d = L[128 * n + 96 + l];
            out[64 * n + l] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
            out[64 * n + 32 + l] = (uint8_t)((b & 0xF) | ((d & 0xF) << 4));
            out[128 + 32 * n + l] = (uint8_t)((a >> 4) | ((b >> 4) << 2) | ((c >> 4) << 4) | ((d >> 4) << 6));
        }
    memcpy(out + 192, sc, 16);
    out[208] = (uint8_t)(dh & 0xff);
    out[209] = (uint8_t)(dh >> 8);
}

uint64_t or_tensor_id(const char *name) { /* FNV-1a, 64-bit */
    uint64_t h = 1469598103934665603ull;
    for (; *name; name++) {
        h ^= (uint8_t)*name;
        h *= 1099511628211ull;
    }
    return h;
}

int or_synth_tensor(int type, int64_t rows, int64_t cols, uint64_t seed, uint64_t tensor_id, float mean,
                    float sigma, void *out) {
    const int64_t n = rows * cols;
    if (type != OR_F32 && type != OR_F16 && type != OR_Q4_K && type != OR_Q6_K) return -1;
    if ((type == OR_Q4_K || type == OR_Q6_K) && cols % 256) return -1;
    const uint64_t key = sy_mix(seed ^ sy_mix(tensor_id));
    const float scale = sigma * 2.64296052e-05f; /* sigma * sqrt(3) / 65536 */
    const int eb = type == OR_F32 ? 4 : type == OR_F16 ? 2 : 0;
    const int bb = type == OR_Q4_K ? 144 : type == OR_Q6_K ? 210 : 256 * eb;
    const int64_t nblk = (n + 255) / 256;
    uint8_t *o = (uint8_t *)out;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nblk; i++) {
        float x[256];
        uint8_t blk[1024];
        for (int k = 0; k < 256; k++) x[k] = sy_value(key, (uint64_t)i * 256u + (uint64_t)k, mean, scale);
        if (type == OR_Q4_K) sy_q4k(x, blk);
        else if (type == OR_Q6_K) sy_q6k(x, blk);
        else if (type == OR_F32) memcpy(blk, x, sizeof x);
        else
            for (int k = 0; k < 256; k++) {
                uint16_t h = or_f32_to_f16(x[k]);
                blk[2 * k] = (uint8_t)(h & 0xff);
                blk[2 * k + 1] = (uint8_t)(h >> 8);
            }
        int64_t left = n - i * 256;
        int nb = (eb && left < 256) ? (int)left * eb : bb;
        memcpy(o + (eb ? i * 256 * eb : i * bb), blk, (size_t)nb);
    }
    return 0;
}

/* ------------------------------------------------------------------ host memory bandwidth
 * A STREAM-style copy of `bytes` over `threads` OpenMP threads, best of `reps`: GB/s counting
 * the bytes read and written (the figure the CPU decode's bandwidth ceiling is quoted on). */
double or_copy_gbs(int64_t bytes, int threads, int reps) {
    const int64_t n = bytes / 8;
    double *a = (double *)malloc((size_t)n * 8), *b = (double *)malloc((size_t)n * 8);
    if (!a || !b) {
        free(a);
        free(b);
        return 0.0;
    }
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        a[i] = (double)i;
        b[i] = 0.0;
    }
    double best = 0.0;
    for (int r = 0; r < reps; r++) {
#ifdef _OPENMP
        double t0 = omp_get_wtime();
#else
        double t0 = 0.0;
#endif
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) b[i] = a[i];
#ifdef _OPENMP
        double dt = omp_get_wtime() - t0;
#else
        double dt = 1.0;
#endif
        double gbs = 2.0 * (double)n * 8.0 / dt / 1e9;
        if (gbs > best) best = gbs;
    }
    volatile double sink = b[n / 2];
    (void)sink;
    free(a);
    free(b);
    return best;
}
