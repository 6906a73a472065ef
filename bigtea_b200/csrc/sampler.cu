// The token sampler on the device: Chaos's Sampler::sample (core/arch/src/sample.rs:474-680).
//
// Three launches per call, all on the engine stream:
//  1. samp_prepare_kernel, one CTA per sequence: copies the logits row, applies the logit bias,
//     ignore_eos, the infill suppression, the repeat/frequency/presence penalties and DRY
//     (sample.rs:491-575), and takes the (penalised) argmax when the configuration is greedy
//     (sample.rs:478-480, 576-595). Otherwise it writes sort keys.
//  2. One radix sort of (sequence, descending total_cmp order) keys with token ids as values
//     (sample.rs:599): a stable sort, so that equal logits keep ascending ids.
//  3. samp_chain_kernel, one CTA per sequence: top_n_sigma, top_k, the softmax, mirostat or the
//     stage chain, adaptive-p and the final draw (sample.rs:601-679).
//
// The arithmetic is the oracle's, bit for bit: every sum the reference accumulates in candidate
// order is accumulated in that order (staged through shared memory, added by one thread);
// elementwise work (exp, pow, divisions) runs on all threads, since each element's value does not
// depend on the order. exp is C7 (bt::bt_exp); ln and pow are S5/S6 below; ties in the sorts go to
// the smaller token id or the earlier candidate. The library is built with --fmad=false, so no
// multiply-add is fused unless written as fmaf.
#include <cub/device/device_radix_sort.cuh>

#include "bt_common.cuh"
#include "sampler.cuh"

namespace {

constexpr int ST = 1024;  // threads per CTA
constexpr int CH = 1024;  // elements per serial-sum chunk

__device__ __forceinline__ float f_nan() { return __int_as_float(0x7fc00000); }
__device__ __forceinline__ float f_inf() { return __int_as_float(0x7f800000); }

// f32::total_cmp as an unsigned key, and back
__device__ __forceinline__ uint32_t total_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// S5: ln x = e ln2 + 2 atanh((m-1)/(m+1)), m in [sqrt(1/2), sqrt(2)), the atanh series to s^11
__device__ float samp_ln(float x) {
    if (x != x) return x;
    if (x < 0.0f) return f_nan();
    if (x == 0.0f) return -f_inf();
    if (x == f_inf()) return x;
    int e = 0;
    uint32_t u = __float_as_uint(x);
    if ((u >> 23) == 0) {
        x = x * 8388608.0f;
        u = __float_as_uint(x);
        e = -23;
    }
    e += (int)((u >> 23) & 0xffu) - 127;
    float m = __uint_as_float((u & 0x7fffffu) | 0x3f800000u);
    if (m > 1.41421353816986083984375f) {
        m = m * 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float z = s * s;
    float p = 9.09090936e-2f;
    p = fmaf(p, z, 1.11111112e-1f);
    p = fmaf(p, z, 1.42857149e-1f);
    p = fmaf(p, z, 2.00000003e-1f);
    p = fmaf(p, z, 3.33333343e-1f);
    p = fmaf(p, z, 1.0f);
    float lnm = (s + s) * p;
    float fe = (float)e;
    return fe * 0.693145751953125f + fmaf(fe, 1.428606765330187045e-06f, lnm);
}

// S6: x^y = exp(y ln x), with the IEEE special cases
__device__ float samp_pow(float x, float y) {
    if (y == 0.0f || x == 1.0f) return 1.0f;
    if (x != x || y != y) return f_nan();
    if (x < 0.0f) return f_nan();
    if (x == 0.0f) return y > 0.0f ? 0.0f : f_inf();
    if (x == f_inf()) return y > 0.0f ? f_inf() : 0.0f;
    return bt::bt_exp(y * samp_ln(x));
}

// f32::powi as square-and-multiply
__device__ float samp_powi(float a, int b) {
    bool recip = b < 0;
    unsigned k = recip ? (unsigned)(-(long long)b) : (unsigned)b;
    float r = 1.0f;
    for (;;) {
        if (k & 1u) r = r * a;
        k >>= 1;
        if (k == 0) break;
        a = a * a;
    }
    return recip ? 1.0f / r : r;
}

__device__ __forceinline__ float clamp_rs(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

// SplitMix64, 24 bits (sample.rs:462-472)
__device__ __forceinline__ float next_f32(unsigned long long &st) {
    st += 0x9E3779B97F4A7C15ull;
    unsigned long long z = st;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)(uint32_t)(z >> 40) / 16777216.0f;
}

// ------------------------------------------------------------------ block helpers
struct Smem {
    float buf[CH];
    uint32_t ibuf[CH];
    unsigned char use[CH];
    unsigned long long skey[SAMP_TYPICAL_MAX];
    unsigned long long red_u[ST / 32];
    float red_f[ST / 32];
    float fval;
    int ival;
    unsigned long long rng;
    float mu, apw, apt;
};

// (key << 32 | index) maximum over the block: the last maximum wins
__device__ unsigned long long blk_max_u64(Smem &S, unsigned long long x) {
    for (int o = 16; o; o >>= 1) {
        unsigned long long y = __shfl_xor_sync(0xffffffffu, x, o);
        x = y > x ? y : x;
    }
    if ((threadIdx.x & 31) == 0) S.red_u[threadIdx.x >> 5] = x;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = S.red_u[0];
        for (int w = 1; w < ST / 32; w++) m = S.red_u[w] > m ? S.red_u[w] : m;
        S.red_u[0] = m;
    }
    __syncthreads();
    unsigned long long r = S.red_u[0];
    __syncthreads();
    return r;
}

__device__ int blk_argmax_last(Smem &S, const float *a, int n) {
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < n; i += ST) {
        unsigned long long k = ((unsigned long long)total_key(a[i]) << 32) | (uint32_t)i;
        best = k > best ? k : best;
    }
    return (int)(uint32_t)blk_max_u64(S, best);
}

// the sum of term(a[i]) over the i that term accepts, added in index order by one thread
template <class Term> __device__ float blk_serial_sum(Smem &S, const float *a, int n, Term term) {
    float t = 0.0f;
    for (int base = 0; base < n; base += CH) {
        const int m = min(CH, n - base);
        for (int j = threadIdx.x; j < m; j += ST) {
            bool u = true;
            S.buf[j] = term(a[base + j], u);
            S.use[j] = u;
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int j = 0; j < m; j++)
                if (S.use[j]) t = t + S.buf[j];
        __syncthreads();
    }
    if (threadIdx.x == 0) S.fval = t;
    __syncthreads();
    const float r = S.fval;
    __syncthreads();
    return r;
}

__device__ float blk_sum(Smem &S, const float *a, int n) {
    return blk_serial_sum(S, a, n, [](float x, bool &) { return x; });
}

// the first i whose running sum acc (in index order) meets the test: mode 0 acc >= target,
// mode 1 target < acc; -1 when none does
__device__ int blk_walk(Smem &S, const float *a, int n, float target, int mode) {
    float acc = 0.0f;
    if (threadIdx.x == 0) S.ival = -1;
    __syncthreads();
    for (int base = 0; base < n; base += CH) {
        const int m = min(CH, n - base);
        for (int j = threadIdx.x; j < m; j += ST) S.buf[j] = a[base + j];
        __syncthreads();
        if (threadIdx.x == 0)
            for (int j = 0; j < m; j++) {
                acc = acc + S.buf[j];
                if (mode == 0 ? acc >= target : target < acc) {
                    S.ival = base + j;
                    break;
                }
            }
        __syncthreads();
        const int hit = S.ival;
        __syncthreads();
        if (hit >= 0) break;
    }
    const int r = S.ival;
    __syncthreads();
    return r;
}

// take_while(a[i] >= floor).count()
__device__ int blk_prefix_ge(Smem &S, const float *a, int n, float fl) {
    if (threadIdx.x == 0) S.ival = n;
    __syncthreads();
    int first = n;
    for (int i = threadIdx.x; i < n; i += ST)
        if (!(a[i] >= fl)) {
            first = i;
            break;
        }
    if (first < n) atomicMin(&S.ival, first);
    __syncthreads();
    const int r = S.ival;
    __syncthreads();
    return r;
}

// the number of i with a[i] >= cut
__device__ int blk_count_ge(Smem &S, const float *a, int n, float cut) {
    if (threadIdx.x == 0) S.ival = 0;
    __syncthreads();
    int c = 0;
    for (int i = threadIdx.x; i < n; i += ST) c += a[i] >= cut;
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(&S.ival, c);
    __syncthreads();
    const int r = S.ival;
    __syncthreads();
    return r;
}

// fold(-inf, f32::max): NaN is skipped
__device__ float blk_fmax(Smem &S, const float *a, int n) {
    float m = -f_inf();
    for (int i = threadIdx.x; i < n; i += ST) m = fmaxf(m, a[i]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) S.red_f[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = S.red_f[0];
        for (int w = 1; w < ST / 32; w++) r = fmaxf(r, S.red_f[w]);
        S.fval = r;
    }
    __syncthreads();
    const float r = S.fval;
    __syncthreads();
    return r;
}

__device__ void blk_scale(float *a, int n, float total) {
    for (int i = threadIdx.x; i < n; i += ST) a[i] = a[i] / total;
    __syncthreads();
}

// softmax (sample.rs:1010-1026): the first entry is taken as the maximum
__device__ void blk_softmax(Smem &S, float *a, int n) {
    if (n == 0) return;
    const float mx = a[0];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += ST) a[i] = bt::bt_exp(a[i] - mx);
    __syncthreads();
    const float total = blk_sum(S, a, n);
    if (total > 0.0f) blk_scale(a, n, total);
}

__device__ void blk_renormalise(Smem &S, float *a, int n) {
    const float total = blk_sum(S, a, n);
    if (total > 0.0f) blk_scale(a, n, total);
}

// apply_temperature (sample.rs:755-770)
__device__ void blk_temperature(Smem &S, float *a, int n, float t) {
    if (fabsf(t - 1.0f) <= 1.1920928955078125e-07f) return;
    float tt = t;
    if (tt != tt || tt < 1e-6f) tt = 1e-6f;
    const float inv = 1.0f / tt;
    for (int i = threadIdx.x; i < n; i += ST) a[i] = samp_pow(a[i], inv);
    __syncthreads();
    blk_renormalise(S, a, n);
}

__device__ float blk_entropy(Smem &S, const float *a, int n) {
    return -blk_serial_sum(S, a, n, [](float x, bool &u) {
        u = x > 0.0f;
        return u ? x * samp_ln(x) : 0.0f;
    });
}

// dynamic_temperature (sample.rs:878-915)
__device__ float blk_dyntemp(Smem &S, const float *a, int n, float t, float range, float ex) {
    float lo = t - range;
    if (lo != lo || lo < 0.0f) lo = 0.0f;
    const float hi = t + range;
    if (n < 2) return t;
    const float entropy = blk_entropy(S, a, n);
    const float max_entropy = samp_ln((float)n);
    if (max_entropy <= 0.0f) return t;
    const float norm = clamp_rs(entropy / max_entropy, 0.0f, 1.0f);
    float e = ex;
    if (e != e || e < 1e-6f) e = 1e-6f;
    return lo + (hi - lo) * samp_pow(norm, e);
}

// ascending bitonic sort of P (a power of two, <= SAMP_TYPICAL_MAX) distinct keys
__device__ void blk_bitonic(unsigned long long *k, int P) {
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < P; i += ST) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const unsigned long long x = k[i], y = k[j];
                    if ((x > y) == up) {
                        k[i] = y;
                        k[j] = x;
                    }
                }
            }
            __syncthreads();
        }
}

// typical_p (sample.rs:782-818) on a[0..n), n <= SAMP_TYPICAL_MAX; returns the new length
__device__ int blk_typical(Smem &S, float *a, uint32_t *id, int n, float typical_p) {
    const float entropy = blk_entropy(S, a, n);
    int P = 2;
    while (P < n) P <<= 1;
    for (int i = threadIdx.x; i < P; i += ST) {
        if (i < n) {
            float lp = a[i];
            if (lp != lp || lp < 1e-30f) lp = 1e-30f;
            const float score = fabsf(-samp_ln(lp) - entropy);
            S.skey[i] = ((unsigned long long)total_key(score) << 32) | (uint32_t)i;
        } else {
            S.skey[i] = ~0ull;
        }
    }
    __syncthreads();
    blk_bitonic(S.skey, P);
    if (threadIdx.x == 0) {
        float cum = 0.0f;
        int keep = 0;
        for (int j = 0; j < n; j++) {
            cum = cum + a[(uint32_t)S.skey[j]];
            keep++;
            if (cum >= typical_p) break;
        }
        S.ival = keep;
    }
    __syncthreads();
    const int keep = S.ival;
    __syncthreads();
    for (int j = threadIdx.x; j < P; j += ST) {
        if (j < keep) {
            const uint32_t i = (uint32_t)S.skey[j];
            S.skey[j] = ((unsigned long long)(~total_key(a[i])) << 32) | i;
        } else {
            S.skey[j] = ~0ull;
        }
    }
    __syncthreads();
    blk_bitonic(S.skey, P);
    for (int j = threadIdx.x; j < keep; j += ST) {
        const uint32_t i = (uint32_t)S.skey[j];
        S.skey[j] = ((unsigned long long)id[i] << 32) | __float_as_uint(a[i]);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < keep; j += ST) {
        a[j] = __uint_as_float((uint32_t)S.skey[j]);
        id[j] = (uint32_t)(S.skey[j] >> 32);
    }
    __syncthreads();
    return keep;
}

// retain(a[i] >= floor), keeping the order (top_n_sigma, sample.rs:856)
__device__ int blk_retain_ge(Smem &S, float *a, uint32_t *id, int n, float fl) {
    int w = 0;
    for (int base = 0; base < n; base += CH) {
        const int m = min(CH, n - base);
        for (int j = threadIdx.x; j < m; j += ST) {
            S.buf[j] = a[base + j];
            S.ibuf[j] = id[base + j];
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int j = 0; j < m; j++)
                if (S.buf[j] >= fl) {
                    a[w] = S.buf[j];
                    id[w] = S.ibuf[j];
                    w++;
                }
        __syncthreads();
    }
    if (threadIdx.x == 0) S.ival = w;
    __syncthreads();
    const int r = S.ival;
    __syncthreads();
    return r;
}

// a random number drawn by thread 0, seen by all
__device__ float blk_next(Smem &S) {
    if (threadIdx.x == 0) S.fval = next_f32(S.rng);
    __syncthreads();
    const float r = S.fval;
    __syncthreads();
    return r;
}

// ------------------------------------------------------------------ kernels
__global__ void __launch_bounds__(ST) samp_prepare_kernel(SampParams P, SampLists L, const float *logits, int V,
                                                          float *work, float *drypen, unsigned long long *keys,
                                                          uint32_t *ids, uint32_t *tok, int *status) {
    __shared__ Smem S;
    const int s = blockIdx.x;
    const float *row = logits + (size_t)s * V;
    float *w = work + (size_t)s * V;
    if (P.greedy) {  // is_greedy: argmax of the raw logits (sample.rs:478-480)
        const int i = blk_argmax_last(S, row, V);
        if (threadIdx.x == 0) {
            tok[s] = (uint32_t)i;
            status[s] = SAMP_DONE_ARGMAX;
        }
        return;
    }
    for (int i = threadIdx.x; i < V; i += ST) w[i] = row[i];
    __syncthreads();
    if (threadIdx.x == 0) {  // sample.rs:487-515, in list order
        for (int k = 0; k < P.n_bias; k++) {
            const uint32_t t = L.bias_ids[k];
            if (t < (uint32_t)V) w[t] = w[t] + L.bias_values[k];
        }
        if (P.ignore_eos && P.eos >= 0 && P.eos < V) w[P.eos] = -f_inf();
        for (int k = 0; k < P.n_suppress; k++) {
            const uint32_t t = L.suppress_ids[k];
            if (t < (uint32_t)V) w[t] = -f_inf();
        }
    }
    __syncthreads();
    const uint32_t *hist = L.hist + L.hist_off[s];
    const int nh = (int)(L.hist_off[s + 1] - L.hist_off[s]);
    // penalties (sample.rs:967-1008): one thread per distinct token of the window
    if (P.repeat_last_n != 0 && nh > 0 &&
        !(P.repeat_penalty == 1.0f && P.frequency_penalty == 0.0f && P.presence_penalty == 0.0f)) {
        const int w0 = nh > (int)P.repeat_last_n ? nh - (int)P.repeat_last_n : 0;
        const uint32_t *win = hist + w0;
        const int wn = nh - w0;
        for (int j = threadIdx.x; j < wn; j += ST) {
            const uint32_t t = win[j];
            bool first = t < (uint32_t)V;
            for (int k = 0; k < j && first; k++) first = win[k] != t;
            if (!first) continue;
            uint32_t count = 0;
            for (int k = j; k < wn; k++) count += win[k] == t;
            float x = w[t];
            if (P.repeat_penalty != 1.0f) x = x > 0.0f ? x / P.repeat_penalty : x * P.repeat_penalty;
            w[t] = x - ((float)count * P.frequency_penalty + P.presence_penalty);
        }
    }
    __syncthreads();
    // DRY (sample.rs:682-753): the largest penalty per continuation, through an int max on the
    // penalty's bits (positive floats order as their bits)
    if (P.dry_multiplier > 0.0f && nh >= 2) {
        const uint32_t *win = hist;
        int wn = nh;
        if (!(P.dry_penalty_last_n == 0 || (int)P.dry_penalty_last_n >= nh)) {
            win = hist + (nh - (int)P.dry_penalty_last_n);
            wn = (int)P.dry_penalty_last_n;
        }
        auto breaker = [&](uint32_t t) {
            for (int b = 0; b < P.n_breakers; b++)
                if (L.breakers[b] == t) return true;
            return false;
        };
        if (wn >= 2 && !breaker(win[wn - 1])) {
            const uint32_t last = win[wn - 1];
            int *pen = reinterpret_cast<int *>(drypen + (size_t)s * V);
            for (int pass = 0; pass < 2; pass++) {
                for (int i = threadIdx.x; i < wn - 1; i += ST) {
                    if (win[i] != last) continue;
                    int len = 1;
                    while (len <= i && len < wn && win[i - len] == win[wn - 1 - len] && !breaker(win[i - len])) len++;
                    if (len < (int)P.dry_allowed_length) continue;
                    const uint32_t next = win[i + 1];
                    if (next >= (uint32_t)V) continue;
                    if (pass == 0) {
                        const float p = P.dry_multiplier * samp_powi(P.dry_base, len - (int)P.dry_allowed_length);
                        if (p > 0.0f) atomicMax(pen + next, __float_as_int(p));
                    } else {
                        const int old = atomicExch(pen + next, 0);
                        if (old) w[next] = w[next] - __int_as_float(old);
                    }
                }
                __syncthreads();
            }
        }
    }
    __syncthreads();
    if (P.temperature <= 0.0f && P.mirostat == 0 && P.adaptive_p < 0.0f) {  // sample.rs:588-595
        const int i = blk_argmax_last(S, w, V);
        if (threadIdx.x == 0) {
            tok[s] = (uint32_t)i;
            status[s] = SAMP_DONE_ARGMAX;
        }
        return;
    }
    const unsigned long long hi = (unsigned long long)s << 32;
    for (int i = threadIdx.x; i < V; i += ST) {
        keys[(size_t)s * V + i] = hi | (uint32_t)(~total_key(w[i]));
        ids[(size_t)s * V + i] = (uint32_t)i;
    }
    if (threadIdx.x == 0) status[s] = SAMP_OK;
}

__global__ void __launch_bounds__(ST) samp_chain_kernel(SampParams P, const unsigned long long *keys,
                                                        const uint32_t *sorted_ids, int V, float *work,
                                                        uint32_t *idw, float *orig, SampState *state, uint32_t *tok,
                                                        int *status) {
    __shared__ Smem S;
    const int s = blockIdx.x;
    if (status[s] != SAMP_OK) return;
    float *v = work + (size_t)s * V;
    uint32_t *cid = idw + (size_t)s * V;
    float *og = orig + (size_t)s * V;
    for (int i = threadIdx.x; i < V; i += ST) {
        v[i] = key_float(~(uint32_t)keys[(size_t)s * V + i]);
        cid[i] = sorted_ids[(size_t)s * V + i];
    }
    if (threadIdx.x == 0) {
        S.rng = state[s].rng;
        S.mu = state[s].mu;
        S.apw = state[s].ap_weighted;
        S.apt = state[s].ap_total;
    }
    __syncthreads();
    int n = V;
    // top_n_sigma (sample.rs:820-857), on the sorted logits
    if (P.top_n_sigma > 0.0f && n >= 2) {
        const float mx = blk_fmax(S, v, n);
        if (isfinite(mx)) {
            int cnt = 0;
            {
                if (threadIdx.x == 0) S.ival = 0;
                __syncthreads();
                int c = 0;
                for (int i = threadIdx.x; i < n; i += ST) c += isfinite(v[i]) ? 1 : 0;
                for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
                if ((threadIdx.x & 31) == 0 && c) atomicAdd(&S.ival, c);
                __syncthreads();
                cnt = S.ival;
                __syncthreads();
            }
            if (cnt >= 2) {
                const float sum = blk_serial_sum(S, v, n, [](float x, bool &u) {
                    u = isfinite(x);
                    return x;
                });
                const float mean = sum / (float)cnt;
                float var = blk_serial_sum(S, v, n, [mean](float x, bool &u) {
                    u = isfinite(x);
                    return (x - mean) * (x - mean);
                });
                var = var / (float)cnt;
                const float sigma = sqrtf(var);
                if (sigma > 0.0f) n = blk_retain_ge(S, v, cid, n, mx - P.top_n_sigma * sigma);
            }
        }
    }
    if (P.top_k > 0 && (int)P.top_k < n) n = (int)P.top_k;
    blk_softmax(S, v, n);

    if (P.mirostat > 0) {  // sample.rs:421-455
        if (threadIdx.x == 0) S.fval = samp_pow(2.0f, -S.mu);
        __syncthreads();
        const float cut = S.fval;
        __syncthreads();
        int kept = blk_count_ge(S, v, n, cut);
        if (kept < 1) kept = 1;
        if (kept < n) n = kept;
        blk_temperature(S, v, n, P.temperature <= 0.0f ? 1.0f : P.temperature);
        const float r = blk_next(S);
        int i = blk_walk(S, v, n, r, 1);
        if (i < 0) i = n - 1;
        if (threadIdx.x == 0) {
            const uint32_t id = i >= 0 ? cid[i] : 0u;
            float pm = i >= 0 ? v[i] : 1.0f;
            if (pm != pm || pm < 1e-30f) pm = 1e-30f;
            const float observed = -(samp_ln(pm) * 1.44269502162933349609375f);
            float mu = S.mu - P.mirostat_eta * (observed - P.mirostat_tau);
            S.mu = clamp_rs(mu, 0.0f, 100.0f);
            tok[s] = id;
        }
    } else {
        int off = 0;  // XTC drops a prefix: the candidates are v[off .. off + n)
        for (int k = 0; k < P.n_chain; k++) {
            switch (P.chain[k]) {
            case 0:  // TopK
                if (P.top_k > 0 && n > (int)P.top_k) n = (int)P.top_k;
                break;
            case 1:  // TypicalP
                if (P.typical_p < 1.0f && n >= 2) {
                    if (n > SAMP_TYPICAL_MAX) {
                        if (threadIdx.x == 0) status[s] = SAMP_ERR_TYPICAL_TOO_MANY;
                        return;
                    }
                    n = blk_typical(S, v + off, cid + off, n, P.typical_p);
                }
                break;
            case 2:  // TopP
                if (P.top_p < 1.0f) {
                    const int i = blk_walk(S, v + off, n, P.top_p, 0);
                    int keep = i >= 0 ? i + 1 : n;
                    if (keep < 1) keep = 1;
                    if (keep > n) keep = n;
                    n = keep;
                    blk_renormalise(S, v + off, n);
                }
                break;
            case 3:  // MinP
                if (P.min_p > 0.0f && n > 0) {
                    const float fl = P.min_p * v[off];
                    int keep = blk_prefix_ge(S, v + off, n, fl);
                    if (keep < 1) keep = 1;
                    n = keep;
                    blk_renormalise(S, v + off, n);
                }
                break;
            case 4:  // Xtc
                if (P.xtc_probability > 0.0f) {
                    const float roll = blk_next(S);
                    if (!(roll >= P.xtc_probability) && n >= 2) {
                        const int above = blk_prefix_ge(S, v + off, n, P.xtc_threshold);
                        if (above >= 2) {
                            off += above - 1;
                            n -= above - 1;
                        }
                    }
                }
                break;
            case 5: {  // Temperature
                const float t = P.dynatemp_range > 0.0f
                                    ? blk_dyntemp(S, v + off, n, P.temperature, P.dynatemp_range, P.dynatemp_exponent)
                                    : P.temperature;
                blk_temperature(S, v + off, n, t);
                break;
            }
            }
        }
        float *a = v + off;
        uint32_t *ai = cid + off;
        if (P.adaptive_p >= 0.0f) {  // sample.rs:374-419
            if (threadIdx.x == 0) {
                const float target = clamp_rs(P.adaptive_p, 0.0f, 1.0f);
                const float mean = S.apt == 0.0f ? target : S.apw / S.apt;
                S.fval = clamp_rs(2.0f * target - mean, 0.0f, 1.0f);
            }
            __syncthreads();
            const float adapted = S.fval;
            __syncthreads();
            for (int i = threadIdx.x; i < n; i += ST) {
                const float p = a[i];
                og[i] = p;
                if (p == -f_inf()) continue;
                const float dist = fabsf((p - adapted) / 0.3f);
                a[i] = 5.0f - 10.0f * dist * dist / (1.0f + dist);
            }
            __syncthreads();
            blk_softmax(S, a, n);
            const float r = blk_next(S);
            int idx = blk_walk(S, a, n, r, 1);
            if (idx < 0) idx = n - 1;
            if (idx < 0) idx = 0;
            if (threadIdx.x == 0) {
                const float decay = clamp_rs(P.adaptive_decay, 0.0f, 0.99f);
                const float o = (n > 0 && idx < n) ? og[idx] : 0.0f;
                S.apw = o + decay * S.apw;
                S.apt = 1.0f + decay * S.apt;
                tok[s] = (n > 0 && idx < n) ? ai[idx] : 0u;
            }
        } else {
            const float r = blk_next(S);
            int i = blk_walk(S, a, n, r, 1);
            if (i < 0) i = n - 1;
            if (threadIdx.x == 0) tok[s] = i >= 0 ? ai[i] : 0u;
        }
    }
    if (threadIdx.x == 0) {
        state[s].rng = S.rng;
        state[s].mu = S.mu;
        state[s].ap_weighted = S.apw;
        state[s].ap_total = S.apt;
    }
}

struct Carve {
    size_t off = 0;
    template <typename T> size_t take(size_t count) {
        const size_t at = (off + 255) & ~(size_t)255;
        off = at + count * sizeof(T);
        return at;
    }
};

int end_bit_for(int n_seqs) {
    int b = 0;
    while ((1 << b) < n_seqs) b++;
    return 32 + b;
}

size_t sort_temp_bytes(int n_seqs, int V) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const unsigned long long *)nullptr, (unsigned long long *)nullptr,
                                    (const uint32_t *)nullptr, (uint32_t *)nullptr, n_seqs * V, 0,
                                    end_bit_for(n_seqs));
    return bytes;
}

}  // namespace

size_t sampler_scratch_bytes(int n_seqs, int V) {
    const size_t n = (size_t)n_seqs * V;
    Carve c;
    c.take<float>(n);               // work
    c.take<float>(n);               // DRY penalties, then the adaptive-p originals
    c.take<unsigned long long>(n);  // keys in
    c.take<unsigned long long>(n);  // keys out
    c.take<uint32_t>(n);            // ids in, then the chain's candidate ids
    c.take<uint32_t>(n);            // ids out
    c.take<char>(sort_temp_bytes(n_seqs, V));
    return c.off + 256;
}

cudaError_t sampler_launch(cudaStream_t st, const SampParams &P, const SampLists &L, const float *logits, int V,
                           int n_seqs, void *scratch, size_t scratch_bytes, SampState *state, uint32_t *tok,
                           int *status) {
    const size_t n = (size_t)n_seqs * V;
    if (scratch_bytes < sampler_scratch_bytes(n_seqs, V)) return cudaErrorInvalidValue;
    char *base = static_cast<char *>(scratch);
    Carve c;
    float *work = reinterpret_cast<float *>(base + c.take<float>(n));
    float *aux = reinterpret_cast<float *>(base + c.take<float>(n));
    auto *kin = reinterpret_cast<unsigned long long *>(base + c.take<unsigned long long>(n));
    auto *kout = reinterpret_cast<unsigned long long *>(base + c.take<unsigned long long>(n));
    auto *iin = reinterpret_cast<uint32_t *>(base + c.take<uint32_t>(n));
    auto *iout = reinterpret_cast<uint32_t *>(base + c.take<uint32_t>(n));
    size_t tbytes = sort_temp_bytes(n_seqs, V);
    void *temp = base + c.take<char>(tbytes);
    cudaError_t e;
    if (P.dry_multiplier > 0.0f && (e = cudaMemsetAsync(aux, 0, n * sizeof(float), st)) != cudaSuccess) return e;
    samp_prepare_kernel<<<n_seqs, ST, 0, st>>>(P, L, logits, V, work, aux, kin, iin, tok, status);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const bool argmax_only = P.greedy || (P.temperature <= 0.0f && P.mirostat == 0 && P.adaptive_p < 0.0f);
    if (argmax_only) return cudaSuccess;
    if ((e = cub::DeviceRadixSort::SortPairs(temp, tbytes, kin, kout, iin, iout, (int)n, 0, end_bit_for(n_seqs),
                                             st)) != cudaSuccess)
        return e;
    samp_chain_kernel<<<n_seqs, ST, 0, st>>>(P, kout, iout, V, work, iin, aux, state, tok, status);
    return cudaGetLastError();
}
