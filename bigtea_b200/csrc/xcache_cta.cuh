// xcache_cta.cuh -- one layer's expert-cache lookup by one CTA, and the slot copies by many, as
// device functions: the lookup kernel (xcache.cu) and the persistent decode step
// (step_kernel.cu) both run them.
//
// The decisions are ExpertCachePolicy's (expert_cache.h). The host handles a layer's distinct
// experts in order; here the hits go first, in parallel, then the misses in order. That is the
// same result: the layer's resident entries are pinned before any of them is handled, so no
// miss can evict a hit's slot or be compared with a hit's use count, and a hit's bookkeeping
// (its use count, its slot's last use, all at the layer's tick) does not depend on the order.
#pragma once
#include <stdint.h>

#include "bt_common.cuh"
#include "xcache_dev.cuh"

namespace bt {

// shared-memory scratch of a lookup: XC_SCRATCH_BYTES from a 16-byte aligned buffer
struct XcScratch {
    int *dist;           // [XC_MAX_SEL] distinct experts in order of first selection
    int *slot;           // [XC_MAX_SEL] their slots (-1 = miss, until handled)
    unsigned char *seen; // [XC_MAX_NE]
    int *i32;            // [32] nd, scan, victim, nc, hits, reduction slots
    unsigned long long *u64;  // [16] tick, reduction values
};
constexpr int XC_SCRATCH_BYTES = XC_MAX_SEL * 8 + XC_MAX_NE + 32 * 4 + 16 * 8;

__device__ __forceinline__ XcScratch xc_scratch(void *buf) {
    XcScratch sc;
    uint8_t *p = reinterpret_cast<uint8_t *>(buf);
    sc.u64 = reinterpret_cast<unsigned long long *>(p);
    sc.i32 = reinterpret_cast<int *>(p + 16 * 8);
    sc.dist = sc.i32 + 32;
    sc.slot = sc.dist + XC_MAX_SEL;
    sc.seen = reinterpret_cast<unsigned char *>(sc.slot + XC_MAX_SEL);
    return sc;
}

__device__ __forceinline__ unsigned long long xc_rand(unsigned long long &rng) {  // xorshift64
    unsigned long long x = rng;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    rng = x;
    return x;
}

// the least-used of a sample of admitted entries (fewest uses, the first met on ties); entries
// the current layer uses are skipped; stale keys are dropped as they are met
static __device__ __noinline__ int xc_weakest(const XcDev &x, int &n_keys, unsigned long long &rng, unsigned long long tick,
                                       int sample) {
    int best = -1;
    unsigned best_uses = 0;
    int tries = 0;
    while (tries < sample * 2 && n_keys > 0) {
        tries++;
        const int i = (int)(xc_rand(rng) % (unsigned long long)n_keys);
        const int key = x.keys[i];
        const int s = x.slot_of[key];
        if (s < 0) {
            x.keys[i] = x.keys[n_keys - 1];
            n_keys--;
            continue;
        }
        if (x.inuse[s] == tick) continue;
        const unsigned uses = x.freq[key];
        if (best < 0 || uses < best_uses) {
            best = s;
            best_uses = uses;
        }
    }
    return best;
}

// One layer's lookup by every thread of one CTA (blockDim.x a multiple of 32, at most 256).
// sel: n_tok tokens' k_per selected experts, token t's at sel + t * sel_stride. Writes each
// distinct expert's slot to slot_row[expert] (a cache slot, or cap + i: a bounce slot served
// once) and the slots to fill to copies; returns their number to every thread.
static __device__ __noinline__ int xc_lookup_cta(const XcDev &x, int layer, const int *sel, int n_tok, int k_per,
                                          int sel_stride, int *slot_row, const uint8_t *host_layer, uint8_t *pool,
                                          long long stride, long long bytes, int n_bounce, XcCopy *copies,
                                          int *n_copies, int *err, XcScratch sc) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nwarps = nth >> 5;
    for (int i = tid; i < x.NE; i += nth) sc.seen[i] = 0;
    __syncthreads();
    if (tid == 0) {
        int nd = 0;
        bool bad = false;
        for (int t = 0; t < n_tok; t++)
            for (int k = 0; k < k_per; k++) {  // distinct experts in order of first selection
                const int e = sel[t * sel_stride + k];
                if (e < 0 || e >= x.NE || nd >= XC_MAX_SEL) {
                    bad = true;
                    continue;
                }
                if (!sc.seen[e]) {
                    sc.seen[e] = 1;
                    sc.dist[nd++] = e;
                }
            }
        if (bad) atomicOr(err, ERR_BAD_INDEX);
        sc.i32[0] = nd;
        sc.i32[4] = 0;  // hits
        sc.u64[0] = x.st[XC_TICK] + 1;
    }
    __syncthreads();
    const int nd = sc.i32[0];
    const unsigned long long tick = sc.u64[0];
    // the resident entries, in parallel: pinned for the layer, one use each, their last use
    for (int i = tid; i < nd; i += nth) {
        const int key = layer * x.NE + sc.dist[i];
        const int s = x.slot_of[key];
        sc.slot[i] = s;
        if (s >= 0) {
            x.inuse[s] = tick;
            x.last[s] = tick;
            x.freq[key]++;
            slot_row[sc.dist[i]] = s;
            atomicAdd(&sc.i32[4], 1);
        }
    }
    __syncthreads();
    // the misses in order (thread 0), with the CTA searching an LRU victim when one is needed
    unsigned long long rng = 0, misses = 0, evictions = 0, admissions = 0, bypasses = 0, copied = 0;
    int n_free = 0, n_keys = 0, nc = 0, bounce = 0;
    if (tid == 0) {
        rng = x.st[XC_RNG];
        n_free = x.ctr[XC_NFREE];
        n_keys = x.ctr[XC_NKEYS];
    }
    for (int i = 0; i < nd; i++) {
        if (sc.slot[i] >= 0) continue;  // a hit (uniform: every thread reads the same entry)
        int s = -1, key = 0;
        if (tid == 0) {
            key = layer * x.NE + sc.dist[i];
            x.freq[key]++;
            sc.i32[1] = 0;
            sc.i32[2] = -1;
            if (n_free > 0) {
                s = x.free_list[--n_free];
            } else if (x.policy == 0) {
                sc.i32[1] = 1;  // LRU: the CTA searches the victim
            } else {
                int v = xc_weakest(x, n_keys, rng, tick, 8);
                if (v >= 0 && x.freq[key] <= x.freq[x.key_of[v]]) v = -1;  // the incumbent stays
                sc.i32[2] = v;
            }
        }
        __syncthreads();
        if (sc.i32[1]) {  // argmin of (last use, slot) over the slots this layer does not use
            unsigned long long bv = ~0ull;
            int bs = -1;
            for (int c = tid; c < x.cap; c += nth) {
                if (x.inuse[c] == tick) continue;
                const unsigned long long v = x.last[c];
                if (v < bv) {  // c grows within a thread: the first minimum is kept
                    bv = v;
                    bs = c;
                }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const unsigned long long ov = __shfl_xor_sync(FULL, bv, o);
                const int os = __shfl_xor_sync(FULL, bs, o);
                if (os >= 0 && (bs < 0 || ov < bv || (ov == bv && os < bs))) {
                    bv = ov;
                    bs = os;
                }
            }
            if (lane == 0) {
                sc.u64[8 + warp] = bv;
                sc.i32[16 + warp] = bs;
            }
            __syncthreads();
            if (tid == 0) {
                int v = -1;
                unsigned long long vv = ~0ull;
                for (int w = 0; w < nwarps; w++) {
                    const int ws = sc.i32[16 + w];
                    const unsigned long long wv = sc.u64[8 + w];
                    if (ws >= 0 && (v < 0 || wv < vv || (wv == vv && ws < v))) {
                        v = ws;
                        vv = wv;
                    }
                }
                sc.i32[2] = v;
            }
        }
        if (tid == 0) {
            const int e = sc.dist[i];
            misses++;
            if (s < 0) {  // no free slot: evict the victim, if any
                const int v = sc.i32[2];
                if (v >= 0) {
                    x.slot_of[x.key_of[v]] = -1;
                    x.key_of[v] = -1;
                    evictions++;
                    s = v;
                }
            }
            bool ok = true;
            if (s < 0) {  // served once from a bounce slot
                bypasses++;
                if (bounce >= n_bounce) {
                    atomicOr(err, ERR_BAD_INDEX);
                    ok = false;
                } else {
                    s = x.cap + bounce++;
                }
            } else {
                x.slot_of[key] = s;
                x.key_of[s] = key;
                x.last[s] = tick;
                x.inuse[s] = tick;
                if (x.policy == 1) {
                    if (n_keys == x.keycap) {  // full: drop the stale keys, in order
                        int m = 0;
                        for (int q = 0; q < n_keys; q++)
                            if (x.slot_of[x.keys[q]] >= 0) x.keys[m++] = x.keys[q];
                        n_keys = m;
                    }
                    x.keys[n_keys++] = key;
                }
                admissions++;
            }
            if (ok) {
                slot_row[e] = s;
                copies[nc].src = host_layer + (long long)e * stride;
                copies[nc].dst = pool + (long long)s * stride;
                nc++;
                copied += (unsigned long long)bytes;
            }
        }
        __syncthreads();  // the next miss's decision reads state this one wrote
    }
    if (tid == 0) {
        x.st[XC_TICK] = tick;
        x.st[XC_RNG] = rng;
        x.st[XC_HITS] += (unsigned long long)sc.i32[4];
        x.st[XC_MISSES] += misses;
        x.st[XC_EVICTIONS] += evictions;
        x.st[XC_ADMISSIONS] += admissions;
        x.st[XC_BYPASSES] += bypasses;
        x.st[XC_BYTES] += copied;
        x.ctr[XC_NFREE] = n_free;
        x.ctr[XC_NKEYS] = n_keys;
        *n_copies = nc;
        sc.i32[3] = nc;
    }
    __syncthreads();
    return sc.i32[3];
}

// The copies [0, nc) of `bytes` each, 16 bytes per step, split over `nthreads` threads of which
// this is number `rank`: four loads in flight before the stores.
__device__ __forceinline__ void xc_copy_part(const XcCopy *copies, int nc, long long bytes, long long rank,
                                             long long nthreads) {
    const long long per = bytes / 16, total = per * nc;
    for (long long i = rank; i < total; i += nthreads * 4) {
        uint4 v[4];
        long long idx[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            idx[u] = i + (long long)u * nthreads;
            if (idx[u] < total) {
                const long long c = idx[u] / per, o = idx[u] - c * per;
                v[u] = __ldcv(reinterpret_cast<const uint4 *>(copies[c].src) + o);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (idx[u] < total) {
                const long long c = idx[u] / per, o = idx[u] - c * per;
                reinterpret_cast<uint4 *>(copies[c].dst)[o] = v[u];
            }
        }
    }
}

}  // namespace bt
