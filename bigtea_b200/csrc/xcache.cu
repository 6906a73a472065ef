// xcache.cu -- the expert-cache policy on the device: one layer's lookup and the slot copies.
//
// The decisions are ExpertCachePolicy's (expert_cache.h), step for step: the layer's resident
// entries are pinned for the layer, then each distinct expert in order of first selection counts
// one use and either hits, takes a free slot, evicts (LRU: the least recently used slot not
// pinned, the lowest slot on ties; FREQ: the least-used of a sample of 8 admitted entries by
// xorshift64, replaced only when the newcomer has strictly more uses) or is served once from a
// bounce slot. Thread 0 keeps the bookkeeping; the LRU victim search, a scan of every slot, is
// an argmin over the CTA. References: core/arch/src/stream.rs:1314-1379 (admit, weakest),
// core/arch/src/expert_cache.rs.
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "xcache_dev.cuh"

namespace bt {

namespace {

constexpr int XC_THREADS = 256;

__device__ unsigned long long xc_rand(unsigned long long &rng) {  // xorshift64
    unsigned long long x = rng;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    rng = x;
    return x;
}

// the least-used of a sample of admitted entries (fewest uses, the first met on ties); entries
// the current layer uses are skipped; stale keys are dropped as they are met
__device__ int xc_weakest(const XcDev &x, int &n_keys, unsigned long long &rng, unsigned long long tick, int sample) {
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

__global__ void __launch_bounds__(XC_THREADS) xcache_lookup_kernel(XcDev x, int layer, const int *sel, int n_sel,
                                                                   int *slot_row, const uint8_t *host_layer,
                                                                   uint8_t *pool, long long stride, long long bytes,
                                                                   int n_bounce, XcCopy *copies, int *n_copies,
                                                                   int *err) {
    __shared__ int dist[XC_MAX_SEL];
    __shared__ unsigned char seen[XC_MAX_NE];
    __shared__ int nd_s, scan_s, victim_s;
    __shared__ unsigned long long tick_s;  // the layer's tick, for the victim search of every thread
    __shared__ unsigned long long red_v[XC_THREADS / 32];
    __shared__ int red_s[XC_THREADS / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();
    for (int i = tid; i < x.NE; i += XC_THREADS) seen[i] = 0;
    __syncthreads();
    // thread 0 keeps the policy's scalars in registers for the whole layer
    unsigned long long tick = 0, rng = 0, hits = 0, misses = 0, evictions = 0, admissions = 0, bypasses = 0,
                       copied = 0;
    int n_free = 0, n_keys = 0, nc = 0, bounce = 0;
    if (tid == 0) {
        int nd = 0;
        bool bad = false;
        for (int i = 0; i < n_sel; i++) {  // distinct experts in order of first selection
            const int e = sel[i];
            if (e < 0 || e >= x.NE) {
                bad = true;
                continue;
            }
            if (!seen[e]) {
                seen[e] = 1;
                dist[nd++] = e;
            }
        }
        if (bad) atomicOr(err, ERR_BAD_INDEX);
        nd_s = nd;
        tick = x.st[XC_TICK] + 1;
        tick_s = tick;
        rng = x.st[XC_RNG];
        n_free = x.ctr[XC_NFREE];
        n_keys = x.ctr[XC_NKEYS];
        for (int i = 0; i < nd; i++) {  // this layer's resident entries are pinned for the step
            const int s = x.slot_of[layer * x.NE + dist[i]];
            if (s >= 0) x.inuse[s] = tick;
        }
    }
    __syncthreads();
    const int nd = nd_s;
    tick = tick_s;
    for (int i = 0; i < nd; i++) {
        int s = -1;
        bool hit = false;
        int key = 0;
        if (tid == 0) {
            key = layer * x.NE + dist[i];
            x.freq[key]++;
            s = x.slot_of[key];
            scan_s = 0;
            victim_s = -1;
            if (s >= 0) {
                hit = true;
            } else if (n_free > 0) {
                s = x.free_list[--n_free];
            } else if (x.policy == 0) {
                scan_s = 1;  // LRU: the CTA searches the victim
            } else {
                int v = xc_weakest(x, n_keys, rng, tick, 8);
                if (v >= 0 && x.freq[key] <= x.freq[x.key_of[v]]) v = -1;  // the incumbent stays
                victim_s = v;
            }
        }
        __syncthreads();
        if (scan_s) {  // argmin of (last use, slot) over the slots this layer does not use
            unsigned long long bv = ~0ull;
            int bs = -1;
            for (int c = tid; c < x.cap; c += XC_THREADS) {
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
                red_v[warp] = bv;
                red_s[warp] = bs;
            }
            __syncthreads();
            if (tid == 0) {
                int v = -1;
                unsigned long long vv = ~0ull;
                for (int w = 0; w < XC_THREADS / 32; w++)
                    if (red_s[w] >= 0 && (v < 0 || red_v[w] < vv || (red_v[w] == vv && red_s[w] < v))) {
                        v = red_s[w];
                        vv = red_v[w];
                    }
                victim_s = v;
            }
            __syncthreads();
        }
        if (tid == 0) {
            const int e = dist[i];
            bool copy = false;
            if (hit) {
                hits++;
                x.last[s] = tick;
            } else {
                misses++;
                if (s < 0) {  // no free slot: evict the victim, if any
                    const int v = victim_s;
                    if (v >= 0) {
                        x.slot_of[x.key_of[v]] = -1;
                        x.key_of[v] = -1;
                        evictions++;
                        s = v;
                    }
                }
                if (s < 0) {  // served once from a bounce slot
                    bypasses++;
                    if (bounce >= n_bounce) {
                        atomicOr(err, ERR_BAD_INDEX);
                        continue;
                    }
                    s = x.cap + bounce++;
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
                copy = true;
            }
            slot_row[e] = s;
            if (copy) {
                copies[nc].src = host_layer + (long long)e * stride;
                copies[nc].dst = pool + (long long)s * stride;
                nc++;
                copied += (unsigned long long)bytes;
            }
        }
    }
    if (tid == 0) {
        x.st[XC_TICK] = tick;
        x.st[XC_RNG] = rng;
        x.st[XC_HITS] += hits;
        x.st[XC_MISSES] += misses;
        x.st[XC_EVICTIONS] += evictions;
        x.st[XC_ADMISSIONS] += admissions;
        x.st[XC_BYPASSES] += bypasses;
        x.st[XC_BYTES] += copied;
        x.ctr[XC_NFREE] = n_free;
        x.ctr[XC_NKEYS] = n_keys;
        *n_copies = nc;
    }
    pdl_trigger();
}

// every listed slot filled from its host block, 16 bytes per thread and step
__global__ void __launch_bounds__(256) xcache_copy_kernel(const XcCopy *copies, const int *n_copies, long long bytes) {
    pdl_wait();
    const int n = *n_copies;
    const long long per = bytes / 16, total = per * n;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (long long)gridDim.x * 256 * 4) {
        uint4 v[4];
        long long idx[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {  // four loads in flight before the stores
            idx[u] = i + (long long)u * gridDim.x * 256;
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
    pdl_trigger();
}

}  // namespace

cudaError_t launch_xcache_lookup(const XcDev &x, int layer, const int *sel, int n_sel, int *slot_row,
                                 const uint8_t *host_layer, uint8_t *pool, long long stride, long long bytes,
                                 int n_bounce, XcCopy *copies, int *n_copies, int *err, cudaStream_t st) {
    if (n_sel > XC_MAX_SEL || x.NE > XC_MAX_NE) return cudaErrorInvalidValue;
    xcache_lookup_kernel<<<1, XC_THREADS, 0, st>>>(x, layer, sel, n_sel, slot_row, host_layer, pool, stride, bytes,
                                                    n_bounce, copies, n_copies, err);
    return cudaGetLastError();
}

cudaError_t launch_xcache_copy(const XcCopy *copies, const int *n_copies, long long bytes, int grid, cudaStream_t st) {
    if (bytes % 16) return cudaErrorInvalidValue;
    xcache_copy_kernel<<<grid, 256, 0, st>>>(copies, n_copies, bytes);
    return cudaGetLastError();
}

}  // namespace bt
