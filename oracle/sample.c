/*
 * sample.c -- CPU restatement of Chaos's token sampler, core/arch/src/sample.rs (TEST INFRASTRUCTURE).
 *
 * Loaded only through liboracle.so by tests/. Every function follows the Rust function it names,
 * statement by statement, in f32 with round-to-nearest-even and no fused operations (the
 * Makefile's -ffp-contract=off), so that a device implementation can be held to it bit for bit.
 *
 * Where the reference's result is not fixed by its source, this restatement fixes it (the same
 * rules bind the device sampler):
 *  S1 exp, ln and pow are this library's (C7 or_exp; S5 or_ln and S6 or_pow below), not libm's.
 *     Rust's f32::exp/ln/powf call the platform libm; the two agree to a few ulp.
 *  S2 sort_unstable_by has no tie order. Here ties are broken by the smaller token id (the main
 *     descending sort of logits) or the earlier candidate (typical_p's two sorts).
 *  S3 f32::powi (DRY) is square-and-multiply: r = 1; for each bit of the exponent from the
 *     lowest, r *= a if the bit is set, then a *= a (the compiler runtime's __powisf2).
 *  S4 log2 (mirostat) is or_ln(x) * 1.44269502 (f32).
 *  S5 ln x = e ln2 + 2 atanh(s), s = (m-1)/(m+1), m in [sqrt(1/2), sqrt(2)), the series to s^11.
 *  S6 pow x^y = exp(y ln x) (C7, S5), with the IEEE special cases for x = 0, 1, inf and NaN.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

const char *or_last_error(void);
void or_set_error_text(const char *msg);

/* ------------------------------------------------------------------ S5 ln, S6 pow */
static const float LN2_HI = 0.693145751953125f;          /* 16 significant bits: e * LN2_HI is exact */
static const float LN2_LO = 1.428606765330187045e-06f;   /* ln 2 - LN2_HI */

static float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* ln x = e ln2 + ln m, m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s) with s = (m-1)/(m+1),
 * 2 atanh(s) = 2s (1 + s^2/3 + s^4/5 + ... + s^10/11), the series in Horner form with fmaf. */
float or_ln(float x) {
    if (x != x) return x;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (x == INFINITY) return x;
    int e = 0;
    uint32_t u = f_bits(x);
    if ((u >> 23) == 0) {            /* subnormal: scale by 2^23 (exact) */
        x = x * 8388608.0f;
        u = f_bits(x);
        e = -23;
    }
    e += (int)((u >> 23) & 0xffu) - 127;
    float m = bits_f((u & 0x7fffffu) | 0x3f800000u); /* [1, 2) */
    if (m > 1.41421353816986083984375f) {
        m = m * 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float z = s * s;
    float p = 9.09090936e-2f;        /* 1/11 */
    p = fmaf(p, z, 1.11111112e-1f);  /* 1/9 */
    p = fmaf(p, z, 1.42857149e-1f);  /* 1/7 */
    p = fmaf(p, z, 2.00000003e-1f);  /* 1/5 */
    p = fmaf(p, z, 3.33333343e-1f);  /* 1/3 */
    p = fmaf(p, z, 1.0f);
    float lnm = (s + s) * p;
    float fe = (float)e;
    return fe * LN2_HI + fmaf(fe, LN2_LO, lnm);
}

/* x^y for the sampler's operands (x >= 0): exp(y ln x) with the IEEE special cases */
float or_pow(float x, float y) {
    if (y == 0.0f || x == 1.0f) return 1.0f;
    if (x != x || y != y) return NAN;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return y > 0.0f ? 0.0f : INFINITY;
    if (x == INFINITY) return y > 0.0f ? INFINITY : 0.0f;
    return or_exp(y * or_ln(x));
}

/* S3 */
static float powi_f(float a, int b) {
    int recip = b < 0;
    unsigned k = recip ? (unsigned)(-(long)b) : (unsigned)b;
    float r = 1.0f;
    for (;;) {
        if (k & 1u) r *= a;
        k >>= 1;
        if (k == 0) break;
        a *= a;
    }
    return recip ? 1.0f / r : r;
}

/* S4 */
static float log2_f(float x) { return or_ln(x) * 1.44269502162933349609375f; }

/* f32::total_cmp as an unsigned key */
static uint32_t total_key(float f) {
    uint32_t u = f_bits(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static float clampf_rs(float v, float lo, float hi) { /* f32::clamp: NaN stays NaN */
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

/* ------------------------------------------------------------------ config and RNG */
void or_sampler_config_default(or_sampler_config *c) {
    memset(c, 0, sizeof *c);
    c->adaptive_p = -1.0f;
    c->adaptive_decay = 0.95f;
    c->temperature = 0.0f;
    c->top_k = 0;
    c->top_p = 1.0f;
    c->min_p = 0.0f;
    c->repeat_penalty = 1.0f;
    c->repeat_last_n = 64;
    c->dry_multiplier = 0.0f;
    c->dry_base = 1.75f;
    c->dry_allowed_length = 2;
    c->dry_penalty_last_n = 0;
    c->typical_p = 1.0f;
    c->top_n_sigma = 0.0f;
    c->dynatemp_range = 0.0f;
    c->dynatemp_exponent = 1.0f;
    c->xtc_probability = 0.0f;
    c->xtc_threshold = 0.1f;
    c->mirostat = 0;
    c->mirostat_tau = 5.0f;
    c->mirostat_eta = 0.1f;
    c->ignore_eos = 0;
    c->eos = -1;
    c->chain = NULL;
    c->seed = 0;
}

void or_sampler_config_llamacpp(or_sampler_config *c) {
    or_sampler_config_default(c);
    c->temperature = 0.8f;
    c->top_k = 40;
    c->top_p = 0.95f;
    c->min_p = 0.05f;
    c->repeat_penalty = 1.1f;
}

void or_sampler_init(const or_sampler_config *c, or_sampler_state *st) {
    st->rng = c->seed + 0x9E3779B97F4A7C15ull;
    float decay = clampf_rs(c->adaptive_decay, 0.0f, 0.99f);
    float ap = c->adaptive_p;
    float apmax = (ap != ap || ap < 0.0f) ? 0.0f : ap; /* f32::max(adaptive_p, 0) */
    st->ap_weighted = apmax / (1.0f - decay);
    st->ap_total = 1.0f / (1.0f - decay);
    st->mu = 2.0f * c->mirostat_tau;
}

/* SplitMix64, 24 bits */
float or_sampler_next_f32(or_sampler_state *st) {
    st->rng += 0x9E3779B97F4A7C15ull;
    uint64_t z = st->rng;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)(uint32_t)(z >> 40) / 16777216.0f;
}

static int is_greedy(const or_sampler_config *c) {
    return c->temperature <= 0.0f && c->repeat_penalty == 1.0f && c->frequency_penalty == 0.0f &&
           c->presence_penalty == 0.0f && c->n_bias == 0 && !c->ignore_eos && c->mirostat == 0 &&
           c->dry_multiplier == 0.0f && c->adaptive_p < 0.0f && c->n_suppress == 0;
}

/* argmax with max_by(total_cmp): the last maximum wins (sample.rs:928-935) */
static int64_t argmax_last(const float *v, int64_t n) {
    int64_t best = 0;
    uint32_t bk = total_key(v[0]);
    for (int64_t i = 1; i < n; i++) {
        uint32_t k = total_key(v[i]);
        if (k >= bk) {
            bk = k;
            best = i;
        }
    }
    return best;
}

/* ------------------------------------------------------------------ stages */
static float sum_f(const float *v, int64_t n) {
    float t = 0.0f;
    for (int64_t i = 0; i < n; i++) t += v[i];
    return t;
}

static void renormalise(float *v, int64_t n) { /* sample.rs:1060-1068 */
    float total = sum_f(v, n);
    if (total > 0.0f)
        for (int64_t i = 0; i < n; i++) v[i] = v[i] / total;
}

static void softmax_c(float *v, int64_t n) { /* sample.rs:1010-1026: the first entry is the max */
    if (n == 0) return;
    float max = v[0];
    float total = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        v[i] = or_exp(v[i] - max);
        total += v[i];
    }
    if (total > 0.0f)
        for (int64_t i = 0; i < n; i++) v[i] = v[i] / total;
}

void or_stage_temperature(float *v, int64_t n, float temperature) { /* sample.rs:755-770 */
    if (fabsf(temperature - 1.0f) <= FLT_EPSILON) return;
    float t = temperature;
    if (t != t || t < 1e-6f) t = 1e-6f; /* f32::max(temperature, 1e-6) */
    float inv = 1.0f / t;
    for (int64_t i = 0; i < n; i++) v[i] = or_pow(v[i], inv);
    float total = sum_f(v, n);
    if (total > 0.0f)
        for (int64_t i = 0; i < n; i++) v[i] = v[i] / total;
}

static float entropy_of(const float *v, int64_t n) {
    float s = 0.0f;
    for (int64_t i = 0; i < n; i++)
        if (v[i] > 0.0f) s += v[i] * or_ln(v[i]);
    return -s;
}

typedef struct {
    uint64_t key;
    int64_t idx;
} kidx;

static int cmp_kidx(const void *a, const void *b) {
    uint64_t x = ((const kidx *)a)->key, y = ((const kidx *)b)->key;
    return x < y ? -1 : x > y;
}

int64_t or_stage_typical_p(uint32_t *ids, float *v, int64_t n, float typical_p) { /* sample.rs:782-818 */
    if (typical_p >= 1.0f || n < 2) return n;
    float entropy = entropy_of(v, n);
    kidx *sc = malloc((size_t)n * sizeof *sc);
    for (int64_t i = 0; i < n; i++) {
        float lp = v[i];
        if (lp != lp || lp < 1e-30f) lp = 1e-30f; /* f32::max(p, 1e-30) */
        float score = fabsf(-or_ln(lp) - entropy);
        sc[i].key = ((uint64_t)total_key(score) << 32) | (uint64_t)(uint32_t)i; /* S2: earlier first */
        sc[i].idx = i;
    }
    qsort(sc, (size_t)n, sizeof *sc, cmp_kidx);
    float cum = 0.0f;
    int64_t keep = 0;
    for (int64_t j = 0; j < n; j++) {
        cum += v[sc[j].idx];
        keep++;
        if (cum >= typical_p) break;
    }
    /* kept, re-sorted descending by probability (S2: the earlier candidate first) */
    kidx *kp = malloc((size_t)keep * sizeof *kp);
    for (int64_t j = 0; j < keep; j++) {
        int64_t i = sc[j].idx;
        kp[j].key = ((uint64_t)(~total_key(v[i])) << 32) | (uint64_t)(uint32_t)i;
        kp[j].idx = i;
    }
    qsort(kp, (size_t)keep, sizeof *kp, cmp_kidx);
    uint32_t *nid = malloc((size_t)keep * sizeof *nid);
    float *nv = malloc((size_t)keep * sizeof *nv);
    for (int64_t j = 0; j < keep; j++) {
        nid[j] = ids[kp[j].idx];
        nv[j] = v[kp[j].idx];
    }
    memcpy(ids, nid, (size_t)keep * sizeof *nid);
    memcpy(v, nv, (size_t)keep * sizeof *nv);
    free(sc);
    free(kp);
    free(nid);
    free(nv);
    return keep;
}

int64_t or_stage_top_n_sigma(uint32_t *ids, float *v, int64_t n, float nsig) { /* sample.rs:820-857 */
    if (nsig <= 0.0f || n < 2) return n;
    float max = -INFINITY;
    for (int64_t i = 0; i < n; i++) max = fmaxf(max, v[i]);
    if (!isfinite(max)) return n;
    int64_t cnt = 0;
    float sum = 0.0f;
    for (int64_t i = 0; i < n; i++)
        if (isfinite(v[i])) {
            sum += v[i];
            cnt++;
        }
    if (cnt < 2) return n;
    float mean = sum / (float)cnt;
    float var = 0.0f;
    for (int64_t i = 0; i < n; i++)
        if (isfinite(v[i])) var += (v[i] - mean) * (v[i] - mean);
    var = var / (float)cnt;
    float sigma = sqrtf(var);
    if (sigma <= 0.0f) return n;
    float floor_ = max - nsig * sigma;
    int64_t k = 0;
    for (int64_t i = 0; i < n; i++)
        if (v[i] >= floor_) {
            ids[k] = ids[i];
            v[k] = v[i];
            k++;
        }
    return k;
}

int64_t or_stage_xtc(uint32_t *ids, float *v, int64_t n, float probability, float threshold, float roll) {
    /* sample.rs:859-868 */
    if (probability <= 0.0f || roll >= probability || n < 2) return n;
    int64_t above = 0;
    while (above < n && v[above] >= threshold) above++;
    if (above < 2) return n;
    int64_t drop = above - 1;
    memmove(ids, ids + drop, (size_t)(n - drop) * sizeof *ids);
    memmove(v, v + drop, (size_t)(n - drop) * sizeof *v);
    return n - drop;
}

float or_dynamic_temperature(const float *v, int64_t n, float temperature, float range, float exponent) {
    /* sample.rs:878-915 */
    float lo = temperature - range;
    if (lo != lo || lo < 0.0f) lo = 0.0f; /* f32::max(.., 0) */
    float hi = temperature + range;
    if (n < 2) return temperature;
    float entropy = entropy_of(v, n);
    float max_entropy = or_ln((float)n);
    if (max_entropy <= 0.0f) return temperature;
    float normalised = clampf_rs(entropy / max_entropy, 0.0f, 1.0f);
    float ex = exponent;
    if (ex != ex || ex < 1e-6f) ex = 1e-6f;
    return lo + (hi - lo) * or_pow(normalised, ex);
}

int64_t or_stage_top_p(uint32_t *ids, float *v, int64_t n, float top_p) { /* sample.rs:1028-1045 */
    (void)ids;
    if (top_p >= 1.0f) return n;
    float acc = 0.0f;
    int64_t keep = n;
    for (int64_t i = 0; i < n; i++) {
        acc += v[i];
        if (acc >= top_p) {
            keep = i + 1;
            break;
        }
    }
    if (keep < 1) keep = 1;
    if (keep > n) keep = n;
    renormalise(v, keep);
    return keep;
}

int64_t or_stage_min_p(uint32_t *ids, float *v, int64_t n, float min_p) { /* sample.rs:1047-1058 */
    (void)ids;
    if (min_p <= 0.0f || n == 0) return n;
    float floor_ = min_p * v[0];
    int64_t keep = 0;
    while (keep < n && v[keep] >= floor_) keep++;
    if (keep < 1) keep = 1;
    renormalise(v, keep);
    return keep;
}

void or_stage_penalties(const uint32_t *ids, float *v, int64_t n, const uint32_t *history, int64_t nh,
                        float repeat, float frequency, float presence, uint32_t last_n) {
    /* sample.rs:967-1008 */
    if (last_n == 0 || nh == 0) return;
    if (repeat == 1.0f && frequency == 0.0f && presence == 0.0f) return;
    int64_t w0 = nh > (int64_t)last_n ? nh - (int64_t)last_n : 0;
    for (int64_t i = 0; i < n; i++) {
        uint32_t count = 0;
        for (int64_t j = w0; j < nh; j++) count += history[j] == ids[i];
        if (!count) continue;
        if (repeat != 1.0f) v[i] = v[i] > 0.0f ? v[i] / repeat : v[i] * repeat;
        v[i] = v[i] - ((float)count * frequency + presence);
    }
}

void or_stage_dry(const uint32_t *ids, float *v, int64_t n, const uint32_t *history, int64_t nh,
                  float multiplier, float base, uint32_t allowed, uint32_t penalty_last_n,
                  const uint32_t *breakers, uint32_t nb) {
    /* sample.rs:682-753 */
    if (multiplier <= 0.0f || nh < 2) return;
    const uint32_t *w = history;
    int64_t wn = nh;
    if (!(penalty_last_n == 0 || (int64_t)penalty_last_n >= nh)) {
        w = history + (nh - penalty_last_n);
        wn = penalty_last_n;
    }
    if (wn < 2) return;
#define IS_BREAKER(t) ({ int hit_ = 0; for (uint32_t b_ = 0; b_ < nb; b_++) hit_ |= breakers[b_] == (t); hit_; })
    uint32_t last = w[wn - 1];
    if (IS_BREAKER(last)) return;
    uint32_t *pid = malloc((size_t)wn * sizeof *pid);
    float *pval = malloc((size_t)wn * sizeof *pval);
    int64_t np = 0;
    for (int64_t i = 0; i < wn - 1; i++) {
        if (w[i] != last) continue;
        int64_t len = 1;
        while (len <= i && len < wn && w[i - len] == w[wn - 1 - len] && !IS_BREAKER(w[i - len])) len++;
        if (len < (int64_t)allowed) continue;
        uint32_t next = w[i + 1];
        float penalty = multiplier * powi_f(base, (int)(len - (int64_t)allowed));
        int64_t k = 0;
        while (k < np && pid[k] != next) k++;
        if (k == np) {
            pid[np] = next;
            pval[np] = 0.0f;
            np++;
        }
        if (penalty > pval[k]) pval[k] = penalty;
    }
#undef IS_BREAKER
    for (int64_t i = 0; i < n && np; i++)
        for (int64_t k = 0; k < np; k++)
            if (pid[k] == ids[i]) {
                v[i] = v[i] - pval[k];
                break;
            }
    free(pid);
    free(pval);
}

/* ------------------------------------------------------------------ Sampler::sample */
static int cmp_u64(const void *a, const void *b) {
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? -1 : x > y;
}

static int64_t draw(or_sampler_state *st, const float *v, int64_t n, int *found) {
    float r = or_sampler_next_f32(st);
    float acc = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        acc += v[i];
        if (r < acc) {
            *found = 1;
            return i;
        }
    }
    *found = 0;
    return n - 1; /* the last candidate; -1 when there is none */
}

int64_t or_sample(const or_sampler_config *c, or_sampler_state *st, const float *logits, int64_t nv,
                  const uint32_t *history, int64_t nh) {
    if (nv <= 0) return 0;
    if (c->chain)
        for (uint32_t k = 0; k < c->n_chain; k++)
            if (c->chain[k] < OR_STAGE_TOP_K || c->chain[k] > OR_STAGE_TEMPERATURE) {
                or_set_error_text("unknown sampler stage");
                return -1;
            }
    if (is_greedy(c)) return argmax_last(logits, nv);

    uint32_t *ids = malloc((size_t)nv * sizeof *ids);
    float *v = malloc((size_t)nv * sizeof *v);
    for (int64_t i = 0; i < nv; i++) {
        ids[i] = (uint32_t)i;
        v[i] = logits[i];
    }
    for (uint32_t k = 0; k < c->n_bias; k++)
        if (c->bias_ids[k] < (uint64_t)nv) v[c->bias_ids[k]] = v[c->bias_ids[k]] + c->bias_values[k];
    if (c->ignore_eos && c->eos >= 0 && c->eos < nv) v[c->eos] = -INFINITY;
    for (uint32_t k = 0; k < c->n_suppress; k++)
        if (c->suppress_ids[k] < (uint64_t)nv) v[c->suppress_ids[k]] = -INFINITY;
    or_stage_penalties(ids, v, nv, history, nh, c->repeat_penalty, c->frequency_penalty, c->presence_penalty,
                       c->repeat_last_n);
    or_stage_dry(ids, v, nv, history, nh, c->dry_multiplier, c->dry_base, c->dry_allowed_length,
                 c->dry_penalty_last_n, c->dry_breakers, c->n_dry_breakers);

    int64_t out;
    if (c->temperature <= 0.0f && c->mirostat == 0 && c->adaptive_p < 0.0f) {
        out = argmax_last(v, nv);
        goto done;
    }
    {
        /* the sort: descending total_cmp, ties by the smaller id (S2) */
        uint64_t *key = malloc((size_t)nv * sizeof *key);
        for (int64_t i = 0; i < nv; i++) key[i] = ((uint64_t)(~total_key(v[i])) << 32) | ids[i];
        qsort(key, (size_t)nv, sizeof *key, cmp_u64);
        float *sv = malloc((size_t)nv * sizeof *sv);
        for (int64_t i = 0; i < nv; i++) {
            ids[i] = (uint32_t)key[i];
            sv[i] = v[ids[i]];
        }
        memcpy(v, sv, (size_t)nv * sizeof *v);
        free(sv);
        free(key);
    }
    int64_t n = or_stage_top_n_sigma(ids, v, nv, c->top_n_sigma);
    if (c->top_k > 0 && (int64_t)c->top_k < n) n = c->top_k;
    softmax_c(v, n);

    if (c->mirostat > 0) { /* sample.rs:421-455 */
        float cut = or_pow(2.0f, -st->mu);
        int64_t kept = 0;
        for (int64_t i = 0; i < n; i++) kept += v[i] >= cut;
        if (kept < 1) kept = 1;
        if (kept < n) n = kept;
        float temp = c->temperature <= 0.0f ? 1.0f : c->temperature;
        or_stage_temperature(v, n, temp);
        int found;
        int64_t i = draw(st, v, n, &found);
        uint32_t cid = i >= 0 ? ids[i] : 0;
        float cp = i >= 0 ? v[i] : 1.0f;
        float pm = cp;
        if (pm != pm || pm < 1e-30f) pm = 1e-30f;
        float observed = -log2_f(pm);
        st->mu = st->mu - c->mirostat_eta * (observed - c->mirostat_tau);
        st->mu = clampf_rs(st->mu, 0.0f, 100.0f);
        out = cid;
        goto done_id;
    }

    {
        static const int32_t dflt[6] = {OR_STAGE_TOP_K, OR_STAGE_TYPICAL_P, OR_STAGE_TOP_P,
                                        OR_STAGE_MIN_P, OR_STAGE_XTC, OR_STAGE_TEMPERATURE};
        const int32_t *chain = c->chain ? c->chain : dflt;
        uint32_t nc = c->chain ? c->n_chain : 6;
        for (uint32_t k = 0; k < nc; k++) {
            switch (chain[k]) {
            case OR_STAGE_TOP_K:
                if (c->top_k > 0 && n > (int64_t)c->top_k) n = c->top_k;
                break;
            case OR_STAGE_TYPICAL_P: n = or_stage_typical_p(ids, v, n, c->typical_p); break;
            case OR_STAGE_TOP_P: n = or_stage_top_p(ids, v, n, c->top_p); break;
            case OR_STAGE_MIN_P: n = or_stage_min_p(ids, v, n, c->min_p); break;
            case OR_STAGE_XTC:
                if (c->xtc_probability > 0.0f) {
                    float roll = or_sampler_next_f32(st);
                    n = or_stage_xtc(ids, v, n, c->xtc_probability, c->xtc_threshold, roll);
                }
                break;
            case OR_STAGE_TEMPERATURE: {
                float temp = c->dynatemp_range > 0.0f
                                 ? or_dynamic_temperature(v, n, c->temperature, c->dynatemp_range, c->dynatemp_exponent)
                                 : c->temperature;
                or_stage_temperature(v, n, temp);
                break;
            }
            }
        }
    }

    if (c->adaptive_p >= 0.0f) { /* sample.rs:374-419 */
        float target = clampf_rs(c->adaptive_p, 0.0f, 1.0f);
        float mean = st->ap_total == 0.0f ? target : st->ap_weighted / st->ap_total;
        float adapted = clampf_rs(2.0f * target - mean, 0.0f, 1.0f);
        float *orig = malloc((size_t)(n > 0 ? n : 1) * sizeof *orig);
        memcpy(orig, v, (size_t)n * sizeof *v);
        for (int64_t i = 0; i < n; i++) {
            if (v[i] == -INFINITY) continue;
            float dist = fabsf((v[i] - adapted) / 0.3f);
            v[i] = 5.0f - 10.0f * dist * dist / (1.0f + dist);
        }
        softmax_c(v, n);
        int found;
        int64_t idx = draw(st, v, n, &found);
        if (idx < 0) idx = 0;
        float decay = clampf_rs(c->adaptive_decay, 0.0f, 0.99f);
        float o = (n > 0 && idx < n) ? orig[idx] : 0.0f;
        st->ap_weighted = o + decay * st->ap_weighted;
        st->ap_total = 1.0f + decay * st->ap_total;
        out = (n > 0 && idx < n) ? ids[idx] : 0;
        free(orig);
        goto done_id;
    }

    {
        int found;
        int64_t i = draw(st, v, n, &found);
        out = i >= 0 ? ids[i] : 0;
    }
done_id:
done:
    free(ids);
    free(v);
    return out;
}
