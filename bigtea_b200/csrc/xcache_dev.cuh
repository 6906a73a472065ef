// xcache_dev.cuh -- the expert-cache policy on the device (xcache.cu).
//
// The same decisions as ExpertCachePolicy (expert_cache.h), on state that lives in device
// memory, so that a step of the per-phase kernels needs no host round trip per layer: after a
// layer's router, one CTA looks the layer's distinct selected experts up (LRU or the
// reference's frequency-gated admission), writes the layer's slot row and a list of copies,
// and a copy kernel fills the missed slots straight from the pinned host copies of the experts.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace bt {

// counters, one u64 each (XcDev::st)
enum { XC_TICK = 0, XC_RNG, XC_HITS, XC_MISSES, XC_EVICTIONS, XC_ADMISSIONS, XC_BYPASSES, XC_BYTES, XC_N };
// small integers (XcDev::ctr)
enum { XC_NFREE = 0, XC_NKEYS, XC_NCTR = 4 };

struct XcDev {
    int policy, cap, NE, keycap;
    int *slot_of;             // [n_layer * NE] -> slot, or -1
    unsigned *freq;           // [n_layer * NE] selections
    int *key_of;              // [cap] -> key, or -1
    unsigned long long *last; // [cap] tick of the slot's last use
    unsigned long long *inuse;// [cap] tick of the layer using the slot
    int *free_list;           // [cap] never-used slots, a stack
    int *keys;                // [keycap] admitted keys (FREQ; may hold stale ones)
    int *ctr;                 // [XC_NCTR]
    unsigned long long *st;   // [XC_N]
};

struct XcCopy {
    const uint8_t *src;  // an expert's gate | up | down block in pinned host memory (device address)
    uint8_t *dst;        // its slot in the pool
};

// One layer: sel[n_sel] the (token, slot) expert ids of the step; slot_row[NE] receives each
// distinct selected expert's slot (a cache slot, or a bounce slot cap + i for an expert served
// once); copies / n_copies the slots to fill; err gets ERR_BAD_INDEX for an id out of range.
cudaError_t launch_xcache_lookup(const XcDev &x, int layer, const int *sel, int n_sel, int *slot_row,
                                 const uint8_t *host_layer, uint8_t *pool, long long stride, long long bytes,
                                 int n_bounce, XcCopy *copies, int *n_copies, int *err, cudaStream_t st);
// the copies of the last lookup: n_copies blocks of `bytes` (a multiple of 16)
cudaError_t launch_xcache_copy(const XcCopy *copies, const int *n_copies, long long bytes, int grid, cudaStream_t st);

constexpr int XC_MAX_SEL = 1024;  // (token, slot) ids one lookup takes
constexpr int XC_MAX_NE = 1024;   // experts per layer the lookup's dedupe covers

}  // namespace bt
