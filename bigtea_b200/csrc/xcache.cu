// xcache.cu -- the expert-cache policy on the device: one layer's lookup and the slot copies.
//
// The decisions are ExpertCachePolicy's (expert_cache.h), step for step: the layer's resident
// entries are pinned for the layer, then each distinct expert in order of first selection counts
// one use and either hits, takes a free slot, evicts (LRU: the least recently used slot not
// pinned, the lowest slot on ties; FREQ: the least-used of a sample of 8 admitted entries by
// xorshift64, replaced only when the newcomer has strictly more uses) or is served once from a
// bounce slot. The lookup and the copies are device functions (xcache_cta.cuh) that the
// persistent decode step runs too. References: core/arch/src/stream.rs:1314-1379 (admit,
// weakest), core/arch/src/expert_cache.rs.
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "xcache_cta.cuh"
#include "xcache_dev.cuh"

namespace bt {

namespace {

constexpr int XC_THREADS = 256;

__global__ void __launch_bounds__(XC_THREADS) xcache_lookup_kernel(XcDev x, int layer, const int *sel, int n_sel,
                                                                   int *slot_row, const uint8_t *host_layer,
                                                                   uint8_t *pool, long long stride, long long bytes,
                                                                   int n_bounce, XcCopy *copies, int *n_copies,
                                                                   int *err) {
    __shared__ __align__(16) uint8_t scratch[XC_SCRATCH_BYTES];
    pdl_wait();
    xc_lookup_cta(x, layer, sel, 1, n_sel, n_sel, slot_row, host_layer, pool, stride, bytes, n_bounce, copies,
                  n_copies, err, xc_scratch(scratch));
    pdl_trigger();
}

// every listed slot filled from its host block
__global__ void __launch_bounds__(256) xcache_copy_kernel(const XcCopy *copies, const int *n_copies, long long bytes) {
    pdl_wait();
    xc_copy_part(copies, *n_copies, bytes, blockIdx.x * 256ll + threadIdx.x, (long long)gridDim.x * 256);
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
