// bt_common.cuh -- arithmetic contract helpers and sm_100a PTX wrappers shared by the kernels.
//
// The arithmetic contract (exactly what the CPU oracle restates; every op is IEEE-754
// binary32 round-to-nearest-even; the library is compiled with --fmad=false so a product
// and a sum are never fused unless written as fmaf):
//   C1 f32->f16 RNE (__float2half_rn); f16->f32 exact.
//   C2 Q4_K value = (d*sc)*q - (dmin*m); Q6_K value = (d*sc)*q.
//   C3 Q8_K activation: first signed max by |x|, iscale = -127/max, q = min(127, rint(iscale*x)),
//      d = 1/iscale, bsums over 16.
//   C4 K-quant row dot: exact int32 per superblock, then one float combination per superblock,
//      summed in superblock order from 0.
//   C5 P2: 32 lanes, lane l takes elements l, l+32, ... in order, xor butterfly 16,8,4,2,1.
//   C6 RMSNorm y = (x * (1/sqrt(P2(x*x)/n + eps))) * w.
//   C7 bt_exp: Cody-Waite ln2 reduction + degree-7 Taylor polynomial in Horner/fmaf form.
//   C8 attention: chunks of 128 keys, per-chunk max/exp/sum/PV, chunks combined in order.
//   C9 RoPE NeoX with a host-computed cos/sin table.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace bt {

constexpr int WARP = 32;
constexpr unsigned FULL = 0xffffffffu;

// error bits a kernel ORs into the engine's device error word
enum : int { ERR_WAIT_TIMEOUT = 1, ERR_BAD_INDEX = 2 };

// ~1 s at the B200's 1.9 GHz SM clock: every spin on an mbarrier gives up after this
constexpr long long WAIT_LIMIT_CYCLES = 2000000000LL;

__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ float pow2i(int n) { return __int_as_float((n + 127) << 23); }

// C7. The same operation sequence as or_exp in the oracle.
__device__ __forceinline__ float bt_exp(float x) {
    if (!(x < 88.72283935546875f)) return (x != x) ? x : __int_as_float(0x7f800000);
    if (x < -103.972084045410156f) return 0.0f;
    float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187045e-06f, r);
    float p = 1.98412698e-4f;
    p = fmaf(p, r, 1.38888889e-3f);
    p = fmaf(p, r, 8.33333333e-3f);
    p = fmaf(p, r, 4.16666667e-2f);
    p = fmaf(p, r, 1.66666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), pow2i(ni - 127));
    if (ni < -126) return __fmul_rn(__fmul_rn(p, pow2i(ni + 64)), pow2i(-64));
    return __fmul_rn(p, pow2i(ni));
}

// f16 x f16 + f32 with one rounding (sm_100 mixed-precision fma on the FMA pipe). Equal to
// fmaf((float)a, (float)b, c): the product of two f16 values is exact in f32.
// Packed pairs of f32 (low half = element 0) and the paired fma of sm_100: each half is one
// fmaf (a single rounding), exactly as the scalar form.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 upk2(f32x2 v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ f32x2 ffma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// (lo, lo) and (hi, hi) of w as two f32x2 of exact f32 values, each half converted twice so the
// pairs need no register moves (FMA pipe)
__device__ __forceinline__ void h2_bcast2(uint32_t w, f32x2 &lo, f32x2 &hi) {
    asm("{\n\t.reg .b16 l, h;\n\t.reg .f32 a, b, c, d;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.f16 a, l, %3;\n\tadd.rn.f32.f16 b, l, %3;\n\tadd.rn.f32.f16 c, h, %3;\n\t"
        "add.rn.f32.f16 d, h, %3;\n\tmov.b64 %0, {a, b};\n\tmov.b64 %1, {c, d};\n\t}"
        : "=l"(lo), "=l"(hi)
        : "r"(w), "f"(-0.0f));
}

__device__ __forceinline__ float fma_f16(uint16_t a, uint16_t b, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}
// f16 -> f32 on the FMA pipe: a + (-0) is exact for every value, signed zeros included.
__device__ __forceinline__ float h2f_fma(uint16_t a) {
    float d;
    asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(a), "f"(-0.0f));
    return d;
}
__device__ __forceinline__ uint16_t lo16(uint32_t w) { return (uint16_t)(w & 0xffffu); }
__device__ __forceinline__ uint16_t hi16(uint32_t w) { return (uint16_t)(w >> 16); }

__device__ __forceinline__ float bt_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, bt_exp(-x))); }

// f32::total_cmp as a signed integer key (core/arch/src/sample.rs:928-935 orders by it)
__device__ __forceinline__ int total_key(float f) {
    int b = __float_as_int(f);
    return b ^ (int)(((unsigned)(b >> 31)) >> 1);
}

__device__ __forceinline__ float butterfly_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// C5 over n elements (lane l: l, l+32, ... in order). Loads are issued 32 at a time ahead of
// the in-order fmaf chain, so the chain waits on one load latency per 32 elements.
__device__ __forceinline__ float warp_sumsq_p2(const float *__restrict__ x, int n, int lane) {
    float acc = 0.0f;
    int i = lane;
    for (; i + 32 * 31 < n; i += 32 * 32) {
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = x[i + 32 * k];
#pragma unroll
        for (int k = 0; k < 32; k++) acc = fmaf(v[k], v[k], acc);
    }
    for (; i < n; i += 32) acc = fmaf(x[i], x[i], acc);
    return butterfly_sum(acc);
}

// C5 dot of a (global, streamed once) and b (any memory).
__device__ __forceinline__ float warp_dot_p2(const float *__restrict__ a, const float *__restrict__ b, int n, int lane) {
    float acc = 0.0f;
    int i = lane;
    for (; i + 32 * 31 < n; i += 32 * 32) {
        float va[32], vb[32];
#pragma unroll
        for (int k = 0; k < 32; k++) {
            va[k] = __ldg(a + i + 32 * k);
            vb[k] = b[i + 32 * k];
        }
#pragma unroll
        for (int k = 0; k < 32; k++) acc = fmaf(va[k], vb[k], acc);
    }
    for (; i < n; i += 32) acc = fmaf(__ldg(a + i), b[i], acc);
    return butterfly_sum(acc);
}

// Start pulling [p, p+bytes) from HBM into L2 without waiting (TMA bulk prefetch).
// p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch a large range in pieces of at most 1 MiB, spread over the calling threads.
__device__ __forceinline__ void prefetch_l2_range(const void *p, unsigned long long bytes, int tid, int nthreads) {
    const unsigned long long piece = 1ull << 20;
    const char *c = reinterpret_cast<const char *>(p);
    unsigned long long n = (bytes + piece - 1) / piece;
    for (unsigned long long k = tid; k < n; k += nthreads) {
        unsigned long long off = k * piece;
        unsigned long long len = bytes - off < piece ? bytes - off : piece;
        prefetch_l2(c + off, (uint32_t)(len & ~15ull));
    }
}

// ---------------------------------------------------------------- PTX: PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- PTX: mbarrier + bulk copies
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and sets ERR_WAIT_TIMEOUT when err is given) if the phase does
// not complete within `limit` SM cycles.
__device__ __forceinline__ bool mbar_wait_l(uint64_t *bar, uint32_t parity, int *err, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) {
            if (err) atomicOr(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    return mbar_wait_l(bar, parity, err, WAIT_LIMIT_CYCLES);
}

// 1-D bulk copy global -> shared (TMA, no tensor map). dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor copy global -> shared through a CUtensorMap (TMA), into this CTA only.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// An L2 policy that marks lines for eviction first: for data streamed once per step (weight
// tiles, KV pages), so that it does not push out what every layer reuses (code, descriptors,
// norm vectors, activations).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// tma_load_2d with an L2 cache policy
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const void *tmap, int x, int y, uint64_t *bar,
                                                 uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

}  // namespace bt
