// step_kernel.cu -- the persistent decode step for sm_100a.
//
// One cooperative kernel (one CTA per SM) runs every layer of a single-token decode step
// for up to STEP_MAX_T sequences: embedding, then per layer the phases
//   QKV (RMSNorm + q/k/v GEMV) | ATTN (q/k head norm, RoPE, f16 KV append, split-K flash
//   decode) | COMBINE (chunk merge) | O (attn_output GEMV + residual) | ROUTER (ffn RMSNorm,
//   F32 router rows) | GATEUP (soft_max + route() in every CTA, expert gate/up GEMV, SiLU)
//   | DOWN (expert down GEMV, the reference's expert sum, residual)
// and finally the output head with a fused argmax and the step's bookkeeping.
//
// At batch 1 a layer moves ~40 MB in a few microseconds, so the step is bound by global round
// trips more than by bandwidth, and the kernel is organised around them:
//  * phases are separated by a one-counter grid barrier (release-add arrival, ld.acquire.gpu
//    polls and no trailing fence; bounded, with a poison bit in the counter that releases every
//    CTA at its next barrier once one CTA has failed);
//  * whatever is static in a phase is requested before the barrier that precedes it: weight
//    tiles into the warps' TMA rings, the K/V pages of a CTA's first attention item, the
//    router rows, the norm vector of the next staging (into shared memory), and the residual
//    rows a CTA adds (into registers, stored to shared memory after the barrier);
//  * the layer descriptors are read into shared memory one layer ahead;
//  * activation staging issues all its loads before the first use (one L2 round trip);
//  * attention items double-buffer their K/V tiles.
// The arithmetic is the contract of bt_common.cuh, operation for operation the same as the
// per-phase kernels of kernels.cu (the tests compare both paths with the CPU oracle bit for bit).
//
// Reference call sites: core/arch/src/stream.rs forward_cached_inner 2106-2915 (per layer:
// 2265-2474 q/k/v, 2545-2552 KvCache::push, 2554-2703 attention, 2723-2726 residual,
// 2784-2831 router, 869-888 route, 1084-1289 experts, 2841-2843 residual, 2853-2914 head).
#include <cuda.h>
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "kernels.cuh"
#include "stage.cuh"
#include "step_kernel.cuh"
#include "xcache_cta.cuh"

namespace bt {

constexpr int STEP_THREADS = 256, STEP_WARPS = 8;
constexpr int RING_SLOTS = 4;
constexpr int PART_ROW = 132;    // floats per (chunk, head) partial: acc[128], m, l, pad
constexpr int ATTN_BUF = 65536;  // one attention item's K and V tiles (128 keys x 128 dims x f16 x 2)
constexpr int LD_WORDS = sizeof(LayerDev) / 4;
// barriers and small tables (1 KB), then two layer descriptors and the head's, then the region
// (1024-byte aligned: the attention tiles' 128-byte swizzle)
constexpr int STEP_HDR_BYTES = 1024 + ((2 * (int)sizeof(LayerDev) + (int)sizeof(QMatDev) + 1023) / 1024) * 1024;
static_assert(LD_WORDS <= 256, "a layer descriptor is copied by one thread per word");
static_assert(sizeof(LayerDev) % 4 == 0, "layer descriptors are copied word by word");
static_assert(STEP_RES == STEP_THREADS, "one residual value per thread");
static_assert(XC_SCRATCH_BYTES <= STEP_CBUF_BYTES, "the cache lookup's scratch fits the combine buffer");

// ------------------------------------------------------------------ shared memory map
struct StepSmem {
    uint8_t *region;     // rings (GEMV phases), K/V tiles (attention) or router rows, STEP_REGION_BYTES
    ActBlock *act;       // activations, STEP_ACT_BYTES
    uint64_t *ring_bar;  // [warp][RING_SLOTS]
    uint64_t *attn_bar;  // [2] one per attention tile buffer
    uint64_t *aux_bar;   // [2] 0: router rows, 1: norm vector
    float *normS;        // [STEP_MAX_T]
    float *misc;         // 64 floats
    int *pos;            // [STEP_MAX_T]
    int *blkn;           // [STEP_MAX_T] the cache block of each token's new position
    int *seq;            // [STEP_MAX_T] each token's sequence
    int *iblk;           // [2][ATTN_CHUNK / 16] page ids of this CTA's first two attention items
    LayerDev *ldesc;     // [2] this layer's and the next layer's descriptors
    QMatDev *outd;       // the output head's descriptor
    int *sel_ids;        // [STEP_MAX_T][MAX_K]
    float *sel_w;        // [STEP_MAX_T][MAX_K]
    int *sel_slot;       // [STEP_MAX_T][MAX_K] the selected experts' cache slots (expert cache)
    float *wv;           // [STEP_WARPS][MAX_K] expert row values of the down phase
    float *cbuf;         // norm vector / router probabilities / combine scratch, STEP_CBUF_BYTES
    float *res;          // [STEP_RES] residual values of this CTA's output rows
};

// ------------------------------------------------------------------ grid barrier
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One monotonic arrival counter, zeroed before each launch: barrier n of a launch completes
// when the counter reaches n * gridDim.x. Thread 0 arrives with a release-add after the CTA's
// __syncthreads and waits with acquire polls: the poll that sees the count complete orders the
// CTA's later reads after every arrival's writes (the adds form one release sequence). The
// wait is bounded: a timeout sets the engine's error word and BAR_POISON in the counter. A CTA
// that finds BAR_POISON leaves, so every CTA leaves at its next barrier; the poll that ends the
// wait brings the poison with it, and no other global read follows the barrier. The error word
// itself is read once, at the first barrier, for an error an earlier launch left.
constexpr unsigned BAR_POISON = 0x80000000u;  // arrivals stay far below bit 31
__device__ __forceinline__ void poison_barrier(unsigned *bar) { atomicOr(bar, BAR_POISON); }

// Arguments by value (the counter, the error word, the wait limit, the drill, this barrier's
// number): a reference would give the caller's variable an address and move it to memory.
// Returns 0 when every CTA arrived, 2 when a thread of this CTA brings a failed wait of its own
// (`bad`: the CTA poisons the barrier and leaves), 1 when the barrier failed or was poisoned.
__device__ __noinline__ int grid_sync(unsigned *bar, int *err, long long limit, int fault_cta, int fault_barrier,
                                     unsigned epoch, bool bad_here, unsigned long long *trace_row) {
    if (__syncthreads_or(bad_here)) return 2;
    // the failure drill: this CTA leaves without arriving, as one that died would
    if (fault_barrier == (int)epoch && fault_cta == (int)blockIdx.x) return 1;
    bool bad = false;
    if (threadIdx.x == 0) {
        if (trace_row) trace_row[blockIdx.x] = global_ns();
        const unsigned target = epoch * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(bar), "r"(1u) : "memory");
        unsigned v = ld_acquire_gpu(bar);
        if (v < target) {
            const long long t0 = clock64();
            while ((v = ld_acquire_gpu(bar)) < target) {
                if (clock64() - t0 > limit) {
                    atomicOr(err, ERR_WAIT_TIMEOUT);
                    poison_barrier(bar);
                    v = BAR_POISON;
                    asm volatile("fence.acq_rel.gpu;" ::: "memory");
                    break;
                }
            }
        }
        bad = v >= BAR_POISON;
        if (epoch == 1) bad |= *reinterpret_cast<volatile int *>(err) != 0;
        if (trace_row && blockIdx.x == 0) trace_row[gridDim.x] = global_ns();
    }
    return __syncthreads_or(bad) ? 1 : 0;
}

// ------------------------------------------------------------------ per-warp TMA ring
// A warp streams its units through `nst` slots of `slot_bytes` in its share of the region.
// Every lane keeps the same counters; lane 0 issues the copies.
struct WarpRing {
    uint8_t *base;
    uint64_t *bars;
    uint32_t par;  // next parity to wait for, one bit per slot
    int nst, slot_bytes, issued, done;

    // A phase's first use of the ring: the region may hold values written by the generic proxy
    // (attention's appended row, normalised router inputs, embedding rows), so the issuing lanes
    // order those before their bulk copies. Within a phase a slot is only read before it is
    // refilled, and the warp's own __syncwarp orders that.
    __device__ void configure(int sbytes) {
        slot_bytes = sbytes;
        nst = (STEP_REGION_BYTES / STEP_WARPS) / sbytes;
        nst = nst > RING_SLOTS ? RING_SLOTS : nst;
        issued = done = 0;
        fence_proxy_async();
    }
    __device__ uint8_t *slot_ptr(int j) const { return base + (size_t)(j % nst) * slot_bytes; }
    __device__ uint64_t *slot_bar(int j) const { return bars + (j % nst); }
    __device__ bool can_issue() const { return issued - done < nst; }
    // wait for unit j (== done); false if the bounded wait ran out, in which case the slot's
    // parity stays, so that a later wait (the failure drain) waits for the same copy
    __device__ bool wait(int j, int *err, long long limit) {
        const int s = j % nst;
        const bool ok = __all_sync(FULL, mbar_wait_l(bars + s, (par >> s) & 1u, err, limit));
        if (ok) par ^= 1u << s;
        return ok;
    }
};

// ------------------------------------------------------------------ unit ranges
// 32-bit unit arithmetic: unit counts stay far below 2^32 / gridDim.x (a 64-bit division is a
// long instruction sequence, and these run per unit)
__device__ __forceinline__ void cta_range(int total, int &u0, int &u1) {
    u0 = (int)((unsigned)blockIdx.x * (unsigned)total / gridDim.x);
    u1 = (int)((unsigned)(blockIdx.x + 1) * (unsigned)total / gridDim.x);
}
__device__ __forceinline__ int warp_units(int u0, int u1, int warp) {
    return (u1 - u0 > warp) ? (int)((u1 - u0 - warp + STEP_WARPS - 1) / STEP_WARPS) : 0;
}

// ------------------------------------------------------------------ shared code
// The step runs each phase once per layer and the whole layer's code does not fit the
// instruction caches, so every instruction a phase executes is fetched again in the next
// layer. Code that several phases run is therefore kept in one non-inlined copy: the K-quant
// slot dots (their loads are explicit shared-memory loads at 32-bit addresses), the Q8_K block
// quantiser and the staging.
__device__ __noinline__ float dot_q4k(uint32_t tile_s, int S, int s, uint32_t act_s) {
    return q4k_dot_s(tile_s, S, s, act_s);
}
__device__ __noinline__ float dot_q6k(uint32_t tile_s, int S, int s, uint32_t act_s) {
    return q6k_dot_s(tile_s, S, s, act_s);
}
// slot s of a tile (tile, S slots) against the activation block at act
__device__ __forceinline__ float slot_dot(bool q4, const uint8_t *tile, int S, int s, const ActBlock *act) {
    return q4 ? dot_q4k(smem_u32(tile), S, s, smem_u32(act)) : dot_q6k(smem_u32(tile), S, s, smem_u32(act));
}

struct F8 {
    float v[8];
};
__device__ __noinline__ void quantize_block_nl(F8 x, uint32_t dst_s, int lane) {
    quantize_block_warp(x.v, reinterpret_cast<ActBlock *>(__cvta_shared_to_generic(dst_s)), lane);
}

// One warp stages nblk 256-value blocks of a row written by other CTAs (C3), the loads of up
// to three blocks issued before the first is quantised.
__device__ __noinline__ void stage_blocks_warp(const float *x, int nblk, uint32_t act_s, int lane) {
    for (int b0 = 0; b0 < nblk; b0 += 3) {
        F8 v[3];
#pragma unroll
        for (int i = 0; i < 3; i++) {
            if (b0 + i < nblk) {
                const float4 *src = reinterpret_cast<const float4 *>(x + (b0 + i) * 256 + lane * 8);
                const float4 a0 = __ldcg(src), a1 = __ldcg(src + 1);
                v[i].v[0] = a0.x; v[i].v[1] = a0.y; v[i].v[2] = a0.z; v[i].v[3] = a0.w;
                v[i].v[4] = a1.x; v[i].v[5] = a1.y; v[i].v[6] = a1.z; v[i].v[7] = a1.w;
            }
        }
#pragma unroll
        for (int i = 0; i < 3; i++)
            if (b0 + i < nblk) quantize_block_nl(v[i], act_s + (uint32_t)((b0 + i) * sizeof(ActBlock)), lane);
    }
}

// ------------------------------------------------------------------ activation staging
__device__ __forceinline__ float4 ld_f4(const float *p, bool global) {
    return global ? __ldcg(reinterpret_cast<const float4 *>(p)) : *reinterpret_cast<const float4 *>(p);
}
__device__ __forceinline__ float ld_f(const float *p, bool global) { return global ? __ldcg(p) : *p; }

// Stage T rows of K values (row stride xs) as Q8_K blocks (C3), in waves of STAGE_B blocks per
// warp. Every load of the first wave is issued before the first use; with `norm` the warps t < T
// load row t lane-strided for the C5 sum of squares (C6) in the same round trip, and the norm
// weights come from `norm_s` (shared memory). `yout` (shared memory, [T][K], optional) receives
// the normalised values. Rows written by other CTAs are read with L1-bypassing loads.
constexpr int STAGE_B = 3;
__device__ __noinline__ void step_stage(const float *x, long long xs, int K, int T, const float *norm_s, float eps,
                                        ActBlock *act, float *normS, float *yout) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool gl = __isGlobal(x), norm = norm_s != nullptr;
    const int nsb = K >> 8, nblk = T * nsb;
    F8 v[STAGE_B];
    auto load_wave = [&](int w0) {
#pragma unroll
        for (int i = 0; i < STAGE_B; i++) {
            const int blk = w0 + warp + i * STEP_WARPS;
            if (blk < nblk) {
                const int t = blk / nsb, b = blk - t * nsb;
                const float *src = x + t * xs + b * 256 + lane * 8;
                const float4 a0 = ld_f4(src, gl), a1 = ld_f4(src + 4, gl);
                v[i].v[0] = a0.x; v[i].v[1] = a0.y; v[i].v[2] = a0.z; v[i].v[3] = a0.w;
                v[i].v[4] = a1.x; v[i].v[5] = a1.y; v[i].v[6] = a1.z; v[i].v[7] = a1.w;
            }
        }
    };
    load_wave(0);
    if (norm) {
        if (warp < T) {
            const float *xt = x + (long long)warp * xs;
            float acc = 0.0f;
            int i = lane;
            for (; i + 32 * 63 < K; i += 32 * 64) {
                float r[64];
#pragma unroll
                for (int k = 0; k < 64; k++) r[k] = ld_f(xt + i + 32 * k, gl);
#pragma unroll
                for (int k = 0; k < 64; k++) acc = fmaf(r[k], r[k], acc);
            }
            for (; i < K; i += 32) {
                const float r = ld_f(xt + i, gl);
                acc = fmaf(r, r, acc);
            }
            acc = butterfly_sum(acc);
            if (lane == 0) normS[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)K), eps)));
        }
        __syncthreads();
    }
    for (int w0 = 0;;) {
#pragma unroll
        for (int i = 0; i < STAGE_B; i++) {
            const int blk = w0 + warp + i * STEP_WARPS;
            if (blk < nblk) {
                if (norm) {
                    const int t = blk / nsb, b = blk - t * nsb;
                    const float s = normS[t];
                    const float4 n0 = *reinterpret_cast<const float4 *>(norm_s + b * 256 + lane * 8);
                    const float4 n1 = *reinterpret_cast<const float4 *>(norm_s + b * 256 + lane * 8 + 4);
                    const float wn[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
                    for (int k = 0; k < 8; k++) v[i].v[k] = __fmul_rn(__fmul_rn(v[i].v[k], s), wn[k]);
                    if (yout) {
                        float4 *d = reinterpret_cast<float4 *>(yout + t * K + b * 256 + lane * 8);
                        d[0] = make_float4(v[i].v[0], v[i].v[1], v[i].v[2], v[i].v[3]);
                        d[1] = make_float4(v[i].v[4], v[i].v[5], v[i].v[6], v[i].v[7]);
                    }
                }
                quantize_block_nl(v[i], smem_u32(act + blk), lane);
            }
        }
        w0 += STAGE_B * STEP_WARPS;
        if (w0 >= nblk) break;
        load_wave(w0);
    }
}

// ------------------------------------------------------------------ GEMV phases
// A "segment list" GEMV over tiles (q|k|v, attn_output, output head).
struct SegList {
    const QMatDev *m[3];
    int out_off[3];
    int n;
    int tile0[3];
    int total;
};

__device__ __forceinline__ SegList make_segs(const QMatDev *a, int oa, const QMatDev *b, int ob, const QMatDev *c,
                                              int oc) {
    SegList s;
    s.n = 0;
    s.total = 0;
    const QMatDev *ms[3] = {a, b, c};
    int os[3] = {oa, ob, oc};
    for (int i = 0; i < 3; i++) {
        if (!ms[i]) continue;
        s.m[s.n] = ms[i];
        s.out_off[s.n] = os[i];
        s.tile0[s.n] = s.total;
        s.total += ms[i]->n_tiles;
        s.n++;
    }
    return s;
}

__device__ __forceinline__ int seg_of(const SegList &s, int u) {
    int si = 0;
    if (s.n > 1 && u >= s.tile0[1]) si = 1;
    if (s.n > 2 && u >= s.tile0[2]) si = 2;
    return si;
}

__device__ __forceinline__ int seglist_max_tile(const SegList &s) {
    int m = 0;
    for (int i = 0; i < s.n; i++) m = s.m[i]->tile_bytes > m ? s.m[i]->tile_bytes : m;
    return m;
}

__device__ void gemv_issue(WarpRing &r, const SegList &s, int u0, int warp, int lane) {
    const int j = r.issued;
    if (lane == 0) {
        const int u = u0 + warp + j * STEP_WARPS;
        const int si = seg_of(s, u);
        const QMatDev &m = *s.m[si];
        const uint8_t *src = m.w + (u - s.tile0[si]) * (long long)m.tile_bytes;
        mbar_arrive_expect_tx(r.slot_bar(j), m.tile_bytes);
        bulk_g2s_hint(r.slot_ptr(j), src, m.tile_bytes, r.slot_bar(j), l2_evict_first_policy());
    }
    r.issued++;
}

__device__ void gemv_preissue(WarpRing &r, const SegList &s, int warp, int lane) {
    int u0, u1;
    cta_range(s.total, u0, u1);
    const int n = warp_units(u0, u1, warp);
    r.configure(seglist_max_tile(s));
    while (r.issued < n && r.can_issue()) gemv_issue(r, s, u0, warp, lane);
}

// Consume every unit of this warp; y[t*ys + off + row] = acc, plus the residual
// res[t*res_ld + off + row - res_row0] (shared memory) when res is given; `amax` folds an argmax
// over the written rows (output head). The segments' parameters are read once into registers.
__device__ __forceinline__ bool gemv_run(WarpRing &r, const SegList &s, const ActBlock *act, int nsbK, int T,
                                         float *y, long long ys, const float *res, int res_row0, int res_ld,
                                         unsigned long long *amax, int *err, long long lim, int warp, int lane,
                                         unsigned long long *cyc = nullptr) {
    long long cw = 0, cc0 = clock64();
    int u0, u1;
    cta_range(s.total, u0, u1);
    const int n = warp_units(u0, u1, warp);
    int sS[3], snsb[3], srpt[3], srows[3], soff[3];
    bool sq4[3];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const QMatDev &m = *s.m[i < s.n ? i : 0];
        sS[i] = m.S;
        snsb[i] = m.nsb;
        srpt[i] = m.rpt;
        srows[i] = m.rows;
        sq4[i] = m.type == T_Q4_K;
        soff[i] = s.out_off[i < s.n ? i : 0];
    }
    unsigned long long best[STEP_MAX_T];
#pragma unroll
    for (int t = 0; t < STEP_MAX_T; t++) best[t] = 0ull;
    bool ok = true;
    for (int j = 0; j < n; j++) {
        while (r.issued < n && r.can_issue()) gemv_issue(r, s, u0, warp, lane);
        const long long w0 = clock64();
        if (!r.wait(j, err, lim)) {
            ok = false;
            break;
        }
        cw += clock64() - w0;
        const int u = u0 + warp + j * STEP_WARPS;
        const int si = seg_of(s, u);
        const int mS = si == 0 ? sS[0] : si == 1 ? sS[1] : sS[2];
        const int mnsb = si == 0 ? snsb[0] : si == 1 ? snsb[1] : snsb[2];
        const int mrpt = si == 0 ? srpt[0] : si == 1 ? srpt[1] : srpt[2];
        const int mrows = si == 0 ? srows[0] : si == 1 ? srows[1] : srows[2];
        const int off = si == 0 ? soff[0] : si == 1 ? soff[1] : soff[2];
        const bool q4 = si == 0 ? sq4[0] : si == 1 ? sq4[1] : sq4[2];
        const uint8_t *tile = r.slot_ptr(j);
        const int tl = u - s.tile0[si];
        const bool active = lane < mS;
        const int rit = active ? lane / mnsb : 0, b = active ? lane - rit * mnsb : 0;
        const int row = tl * mrpt + rit;
        const bool writer = active && b == 0 && row < mrows;
        for (int t = 0; t < T; t++) {
            float v = 0.0f;
            if (active) v = slot_dot(q4, tile, mS, lane, act + t * nsbK + b);
            float acc = 0.0f;
            for (int b2 = 0; b2 < mnsb; b2++) {
                const int srcl = rit * mnsb + b2;
                acc = __fadd_rn(acc, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
            }
            if (writer) {
                const int o = off + row;
                float val = acc;
                if (res) val = __fadd_rn(res[t * res_ld + (o - res_row0)], acc);
                y[t * ys + o] = val;
                if (amax) {
                    const unsigned long long key =
                        ((unsigned long long)((unsigned)total_key(val) ^ 0x80000000u) << 32) | (unsigned)o;
#pragma unroll
                    for (int tt = 0; tt < STEP_MAX_T; tt++)
                        if (tt == t && key > best[tt]) best[tt] = key;
                }
            }
        }
        __syncwarp();
        r.done++;
    }
    if (cyc && lane == 0) {
        atomicMax(cyc, (unsigned long long)cw);
        atomicMax(cyc + 1, (unsigned long long)(clock64() - cc0 - cw));
    }
    if (amax) {
        for (int t = 0; t < T; t++) {
            unsigned long long bv = best[0];
#pragma unroll
            for (int tt = 1; tt < STEP_MAX_T; tt++)
                if (tt == t) bv = best[tt];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const unsigned long long ob = __shfl_xor_sync(FULL, bv, o);
                bv = ob > bv ? ob : bv;
            }
            if (lane == 0 && bv) atomicMax(amax + t, bv);
        }
    }
    return ok;
}

// ------------------------------------------------------------------ expert phases
// unit u of the gate/up phase: units below nr are (token, slot, tile) of the routed experts,
// the rest (token, tile) of the shared expert
template <bool SH, bool XC>
__device__ void gateup_issue(WarpRing &r, const LayerDev &L, const StepSmem &sm, int K, int nr, int u0, int warp,
                             int lane, bool drill, const uint8_t *pool, long long stride) {
    const int j = r.issued;
    if (drill) {  // the failure drill: the slot is counted as requested, but nothing will land
        r.issued++;
        return;
    }
    const int u = u0 + warp + j * STEP_WARPS;
    const bool sh = SH && u >= nr;
    const QMatDev &G = sh ? L.sgate : L.gate, &U = sh ? L.sup : L.up;
    int e = 0, tile;
    if (sh) {
        tile = (u - nr) % G.n_tiles;
    } else {
        const int tk = u / G.n_tiles;
        tile = u - tk * G.n_tiles;
        e = (XC ? sm.sel_slot : sm.sel_ids)[(tk / K) * MAX_K + tk % K];
    }
    uint8_t *dst = r.slot_ptr(j);
    if (lane == 0) mbar_arrive_expect_tx(r.slot_bar(j), G.tile_bytes + U.tile_bytes);
    __syncwarp();
    if (lane < 2) {  // lane 0 the gate tile, lane 1 the up tile
        const QMatDev &m = lane ? U : G;
        // resident: expert e of the matrix; cached: slot e of the pool, gate then up
        const uint8_t *src = XC && !sh ? pool + e * stride + (lane ? G.mat_bytes : 0) : m.w + e * m.mat_bytes;
        bulk_g2s_hint(dst + lane * G.tile_bytes, src + (long long)tile * m.tile_bytes, m.tile_bytes, r.slot_bar(j),
                      l2_evict_first_policy());
    }
    r.issued++;
}

// The down phase's units. A CTA owns the output rows [d0, d1) of T * E; they are cut at token
// boundaries and into pieces of at most maxr rows, and unit i = (piece i / K, expert i % K):
// the piece's rows of one selected expert. A down row of the tiled layout is one tile, so a
// unit is one contiguous copy (one copy per row and expert kept the copy engine far below the
// SM's share of HBM). Piece q -> token t, first row r0 (0..E-1), rows nr, offset of its first
// row in [d0, d1); returns the piece count when q is past the end, -1 otherwise.
__device__ __forceinline__ int down_piece(int d0, int d1, int E, int maxr, int q, int &t, int &r0, int &nr,
                                          int &off) {
    int n = 0;
    for (int tt = d0 / E; tt * E < d1; tt++) {
        const int a = d0 > tt * E ? d0 : tt * E, b = d1 < (tt + 1) * E ? d1 : (tt + 1) * E;
        if (a >= b) continue;
        const int pieces = (b - a + maxr - 1) / maxr;
        if (q < n + pieces) {
            const int k = q - n;
            t = tt;
            r0 = a + k * maxr - tt * E;
            nr = (b - a - k * maxr) < maxr ? (b - a - k * maxr) : maxr;
            off = a + k * maxr - d0;
            return -1;
        }
        n += pieces;
    }
    return n;
}

// each expert's values of the CTA's down rows, [MAX_K][STEP_DOWN_ROWS], after the warps' staged
// products in the activation area
__device__ __forceinline__ float *step_down_part(const StepSmem &sm) {
    return reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(sm.act) +
                                     STEP_WARPS * STEP_MAX_NSB_F * sizeof(ActBlock));
}
static_assert(STEP_WARPS * STEP_MAX_NSB_F * sizeof(ActBlock) + MAX_K * STEP_DOWN_ROWS * 4 <= STEP_ACT_BYTES,
              "the down phase's staged products and row values fit the activation area");

// rows of one down unit's copy: half of a warp's ring share, so two units can be in flight (dtb:
// the largest row of the layer's down matrices)
__device__ __forceinline__ int down_max_rows(int dtb) { return (STEP_REGION_BYTES / STEP_WARPS / 2) / dtb; }
template <bool SH>
__device__ __forceinline__ int down_row_bytes(const LayerDev &L) {
    return SH && L.sdown.tile_bytes > L.down.tile_bytes ? L.sdown.tile_bytes : L.down.tile_bytes;
}

// this warp's j-th down unit (unit warp + j * STEP_WARPS of nk experts per piece; expert index K
// is the shared expert): lane 0 requests it
template <bool SH, bool XC>
__device__ void down_issue(WarpRing &r, const LayerDev &L, const StepSmem &sm, int K, int nk, int E, int d0, int d1,
                           int maxr, int warp, int lane, const uint8_t *pool, long long stride) {
    const int j = r.issued;
    const int i = warp + j * STEP_WARPS, q = i / nk, k = i - q * nk;
    int t, r0, nr, off;
    down_piece(d0, d1, E, maxr, q, t, r0, nr, off);
    if (lane == 0) {
        const bool shx = SH && k == K;
        const QMatDev &m = shx ? L.sdown : L.down;
        const int e = shx ? 0 : (XC ? sm.sel_slot : sm.sel_ids)[t * MAX_K + k];
        // resident: expert e of the matrix; cached: slot e of the pool, after its gate and up
        const uint8_t *src = XC && !shx ? pool + e * stride + L.gate.mat_bytes + L.up.mat_bytes : m.w + e * m.mat_bytes;
        mbar_arrive_expect_tx(r.slot_bar(j), nr * m.tile_bytes);
        bulk_g2s_hint(r.slot_ptr(j), src + (long long)r0 * m.tile_bytes, nr * m.tile_bytes, r.slot_bar(j),
                      l2_evict_first_policy());
    }
    __syncwarp();
    r.issued++;
}

// ------------------------------------------------------------------ attention item helpers
struct AttnItem {
    int t, g, c;
};

// item i of the step's attention work: tokens in order, kv heads, chunks
__device__ __forceinline__ bool attn_item(const StepArgs &p, const int *pos, int i, AttnItem &it) {
    for (int t = 0; t < p.T; t++) {
        const int nc = (pos[t] + ATTN_CHUNK) / ATTN_CHUNK;
        const int cnt = p.HK * nc;
        if (i < cnt) {
            it.t = t;
            it.g = i / nc;
            it.c = i - it.g * nc;
            return true;
        }
        i -= cnt;
    }
    return false;
}

__device__ __forceinline__ int attn_items(const StepArgs &p, const int *pos) {
    int n = 0;
    for (int t = 0; t < p.T; t++) n += p.HK * ((pos[t] + ATTN_CHUNK) / ATTN_CHUNK);
    return n;
}

// The TMA loads of one item's K and V pages into tile buffer `buf`, issued by one warp (lane l
// takes pages l, l+32, ...). `blk_s` holds the item's page ids in shared memory (a CTA's first
// two items, staged once per step), or is null and the ids come from the block table.
__device__ void attn_issue_warp(const StepArgs &p, const CUtensorMap *tmap, const StepSmem &sm, const AttnItem &it,
                                int layer, int buf, const int *blk_s, int lane) {
    const int nk = sm.pos[it.t] + 1, base = it.c * ATTN_CHUNK;
    const int cnt = nk - base < ATTN_CHUNK ? nk - base : ATTN_CHUNK;
    const int npages = (cnt + 15) / 16;
    uint8_t *K0 = sm.region + buf * ATTN_BUF, *K1 = K0 + 16384, *V0 = K0 + 32768, *V1 = K0 + 49152;
    uint64_t *bar = sm.attn_bar + buf;
    if (lane == 0) mbar_arrive_expect_tx(bar, npages * 8192);
    __syncwarp();
    const uint64_t pol = l2_evict_first_policy();
    for (int pg = lane; pg < npages; pg += 32) {
        const int blk = blk_s ? blk_s[pg] : p.block_table[sm.seq[it.t] * p.max_blocks + (base >> 4) + pg];
        const int rowK = (int)(((((long long)layer * p.n_blocks + blk) * 2 + 0) * p.HK + it.g) * 16);
        const int rowV = rowK + p.HK * 16;
        fence_proxy_async();
        tma_load_2d_hint(K0 + pg * 2048, tmap, 0, rowK, bar, pol);
        tma_load_2d_hint(K1 + pg * 2048, tmap, 64, rowK, bar, pol);
        tma_load_2d_hint(V0 + pg * 2048, tmap, 0, rowV, bar, pol);
        tma_load_2d_hint(V1 + pg * 2048, tmap, 64, rowV, bar, pol);
    }
}

// q/k head RMSNorm (C5/C6) and NeoX RoPE (C9) of one head held 4 values per lane
// (lane l: dims l, l+32, l+64, l+96); w holds this lane's norm weights for those dims and cs the
// cos/sin pairs of dims l and l+32.
__device__ __forceinline__ void head_norm_rope(float v[4], const float w[4], const float cs[4], float eps) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) acc = fmaf(v[i], v[i], acc);
    acc = butterfly_sum(acc);
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, 128.0f), eps)));
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __fmul_rn(__fmul_rn(v[i], s), w[i]);
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float c = cs[2 * i], sn = cs[2 * i + 1];
        const float x0 = v[i], x1 = v[i + 2];
        const float a = __fmul_rn(x0, c), b = __fmul_rn(x1, sn), e = __fmul_rn(x0, sn), f = __fmul_rn(x1, c);
        v[i] = __fsub_rn(a, b);
        v[i + 2] = __fadd_rn(e, f);
    }
}

// ------------------------------------------------------------------ attention
// Each half of the CTA (128 threads, warps 4h .. 4h+3, named barrier 1 + h) runs one attention
// item at a time with its own K/V tile buffer and scratch, so a CTA's first two items run
// concurrently.
constexpr int ATTN_SCRATCH = 8192;  // per half: q (D x G f16), p (CH x G f32), reductions, new k/v
static_assert(2 * ATTN_BUF + 2 * ATTN_SCRATCH <= STEP_REGION_BYTES, "attention tiles and scratch fit the region");

__device__ __forceinline__ void half_sync(int h) { asm volatile("bar.sync %0, 128;" ::"r"(1 + h) : "memory"); }
__device__ __forceinline__ bool half_sync_or(int h, bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.or.pred q, %2, 128, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((int)v), "r"(1 + h)
        : "memory");
    return r != 0;
}

// a0 += lo(q) * k, a1 += hi(q) * k with k the low (KHI false) or high half of kw (C8 terms)
template <bool KHI>
__device__ __forceinline__ void fma_qk(uint32_t qw, uint32_t kw, float &a0, float &a1) {
    if constexpr (KHI)
        asm("{\n\t.reg .b16 ql, qh, kl, kh;\n\tmov.b32 {ql, qh}, %2;\n\tmov.b32 {kl, kh}, %3;\n\t"
            "fma.rn.f32.f16 %0, ql, kh, %0;\n\tfma.rn.f32.f16 %1, qh, kh, %1;\n\t}"
            : "+f"(a0), "+f"(a1)
            : "r"(qw), "r"(kw));
    else
        asm("{\n\t.reg .b16 ql, qh, kl, kh;\n\tmov.b32 {ql, qh}, %2;\n\tmov.b32 {kl, kh}, %3;\n\t"
            "fma.rn.f32.f16 %0, ql, kl, %0;\n\tfma.rn.f32.f16 %1, qh, kl, %1;\n\t}"
            : "+f"(a0), "+f"(a1)
            : "r"(qw), "r"(kw));
}
// both halves of w as exact f32 values (FMA pipe)
__device__ __forceinline__ float2 h2f2_fma(uint32_t w) {
    float2 r;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tadd.rn.f32.f16 %0, l, %3;\n\tadd.rn.f32.f16 %1, h, %3;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "r"(w), "f"(-0.0f));
    return r;
}

template <int N>
__device__ __forceinline__ void lds_n(float (&dst)[N], const float *src) {
    if constexpr (N == 4) {
        float4 v = *reinterpret_cast<const float4 *>(src);
        dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
    } else if constexpr (N == 2) {
        float2 v = *reinterpret_cast<const float2 *>(src);
        dst[0] = v.x; dst[1] = v.y;
    } else {
#pragma unroll
        for (int k = 0; k < N; k++) dst[k] = src[k];
    }
}
template <int N>
__device__ __forceinline__ void ldw_n(uint32_t (&dst)[N], const uint32_t *src) {
    if constexpr (N == 4) {
        const uint4 v = *reinterpret_cast<const uint4 *>(src);
        dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
    } else if constexpr (N == 2) {
        const uint2 v = *reinterpret_cast<const uint2 *>(src);
        dst[0] = v.x; dst[1] = v.y;
    } else {
#pragma unroll
        for (int k = 0; k < N; k++) dst[k] = src[k];
    }
}

// One attention item (C8) on half `hf` of the CTA: the K/V tiles are in flight into buffer hf
// (attn_issue). Stages q (f16), appends the new key and value if this is the token's last
// chunk, then scores (thread = key, all G heads, dims in order), the chunk max, exp and P3 sum
// (32-key butterflies, the 4 warp sums in order) and P*V (thread = 2 dims x G/2 heads, keys in
// order).
template <int G>
__device__ bool attn_half(const StepArgs &p, const LayerDev &L, const StepSmem &sm, const AttnItem &it, int layer,
                          int hf, uint32_t &apar, uint32_t &apend, unsigned long long *tp) {
    constexpr int D = 128, HPT = G / 2, CH = ATTN_CHUNK, QWORDS = G / 2;
    const int tid = threadIdx.x & 127, warp = tid >> 5, lane = tid & 31;
    const long long tps = gridDim.x + 1;
    auto PT = [&](int i) {
        if (tp && tid == 0) tp[i * tps + blockIdx.x] = global_ns();
    };
    uint8_t *K0 = sm.region + hf * ATTN_BUF, *K1 = K0 + 16384, *V0 = K0 + 32768, *V1 = K0 + 49152;
    uint8_t *scr = sm.region + 2 * ATTN_BUF + hf * ATTN_SCRATCH;
    uint16_t *qs = reinterpret_cast<uint16_t *>(scr);           // [D][G] f16 bits
    float *ps = reinterpret_cast<float *>(scr + D * G * 2);     // [CH][G]
    float *red = ps + CH * G;                                   // [4][8]
    float *red2 = red + 32;                                     // [4][8]
    float *s_m = red2 + 32, *s_l = s_m + 8;
    __half *kvnew = reinterpret_cast<__half *>(s_l + 8);        // [2][128] the appended key and value
    const int t = it.t, g = it.g, c = it.c;
    const int pos = sm.pos[t], nk = pos + 1, nc = (nk + CH - 1) / CH;
    const int base = c * CH, cnt = nk - base < CH ? nk - base : CH;
    const bool last = c == nc - 1;
    const float *qkv = p.qkv + (long long)t * (p.H * D + 2 * p.HK * D);
    float cs[4];
    {
        const float2 *csrow = reinterpret_cast<const float2 *>(p.rope + (long long)pos * p.n_rot);
        const float2 c0 = __ldg(csrow + lane), c1 = __ldg(csrow + lane + 32);
        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c1.x; cs[3] = c1.y;
    }
    // units: the G q heads, then (last chunk) the new key/value; warp w takes units w, w+4, ...
    const int units = G + (last ? 1 : 0);
    for (int u = warp; u < units; u += 4) {
        float v[4], wn[4];
        if (u < G) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v[i] = __ldcg(qkv + (g * G + u) * D + lane + 32 * i);
                wn[i] = __ldg(L.q_norm + lane + 32 * i);
            }
            head_norm_rope(v, wn, cs, p.eps);
#pragma unroll
            for (int i = 0; i < 4; i++) qs[(lane + 32 * i) * G + u] = __half_as_ushort(__float2half_rn(v[i]));
        } else {
            // KvCache::push of this token's head g: k normed and roped, v as is, both to f16
            float vv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v[i] = __ldcg(qkv + p.H * D + g * D + lane + 32 * i);
                vv[i] = __ldcg(qkv + p.H * D + p.HK * D + g * D + lane + 32 * i);
                wn[i] = __ldg(L.k_norm + lane + 32 * i);
            }
            head_norm_rope(v, wn, cs, p.eps);
            const long long rowK = ((((long long)layer * p.n_blocks + sm.blkn[t]) * 2 + 0) * p.HK + g) * 16 + pos % 16;
            const long long rowV = rowK + (long long)p.HK * 16;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const __half hk = __float2half_rn(v[i]), hv = __float2half_rn(vv[i]);
                p.kv[rowK * D + lane + 32 * i] = hk;
                p.kv[rowV * D + lane + 32 * i] = hv;
                kvnew[lane + 32 * i] = hk;
                kvnew[128 + lane + 32 * i] = hv;
            }
        }
    }
    half_sync(hf);
    PT(0);
    const bool landed = mbar_wait_l(sm.attn_bar + hf, (apar >> hf) & 1u, p.err, p.wait_limit);
    if (landed) {  // else the failure drain waits for the same copies
        apar ^= 1u << hf;
        apend &= ~(1u << hf);
    }
    if (half_sync_or(hf, !landed)) return false;
    PT(1);
    if (last) {  // the new position's row of the tiles is the value just computed
        const int r = pos - base;
        if (tid < 32) {
            const int d0 = tid * 4;  // 4 halves per thread: K then V
            for (int e = 0; e < 4; e++) {
                const int d = d0 + e;
                const int cc = (d & 63) >> 3;
                uint8_t *kt = (d < 64 ? K0 : K1) + r * 128 + ((cc ^ (r & 7)) << 4) + (d & 7) * 2;
                uint8_t *vt = (d < 64 ? V0 : V1) + r * 128 + ((cc ^ (r & 7)) << 4) + (d & 7) * 2;
                *reinterpret_cast<__half *>(kt) = kvnew[d];
                *reinterpret_cast<__half *>(vt) = kvnew[128 + d];
            }
        }
        half_sync(hf);
    }
    // ---- scores: thread = key k, all G heads (pairs of heads per q word)
    const int k = tid;
    const bool valid = k < cnt;
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; h++) sc[h] = 0.0f;
    {
        const uint8_t *krow = K0 + k * 128;
        const int ksw = k & 7;
        const uint32_t *qw = reinterpret_cast<const uint32_t *>(qs);
#pragma unroll 2
        for (int c16 = 0; c16 < 16; c16++) {
            const uint4 w = *reinterpret_cast<const uint4 *>((c16 < 8 ? krow : krow + 16384) + (((c16 & 7) ^ ksw) << 4));
            const uint32_t kw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                uint32_t q[QWORDS];
                ldw_n<QWORDS>(q, qw + (c16 * 8 + e) * QWORDS);
#pragma unroll
                for (int j = 0; j < QWORDS; j++) {
                    if (e & 1)
                        fma_qk<true>(q[j], kw[e >> 1], sc[2 * j], sc[2 * j + 1]);
                    else
                        fma_qk<false>(q[j], kw[e >> 1], sc[2 * j], sc[2 * j + 1]);
                }
            }
        }
    }
    const float NEG_INF = -__int_as_float(0x7f800000);
#pragma unroll
    for (int h = 0; h < G; h++) {
        sc[h] = valid ? __fmul_rn(sc[h], p.scale) : NEG_INF;
        const float m = warp_max(sc[h]);
        if (lane == 0) red[warp * 8 + h] = m;
    }
    half_sync(hf);
    if (tid < G) {
        float m = red[tid];
        for (int w = 1; w < 4; w++) m = fmaxf(m, red[w * 8 + tid]);
        s_m[tid] = m;
    }
    half_sync(hf);
    PT(2);
#pragma unroll
    for (int h = 0; h < G; h++) {
        const float pr = valid ? bt_exp(__fsub_rn(sc[h], s_m[h])) : 0.0f;
        sc[h] = pr;
        const float ws = butterfly_sum(pr);
        if (lane == 0) red2[warp * 8 + h] = ws;
    }
    if constexpr (G % 4 == 0) {
        float4 *prow = reinterpret_cast<float4 *>(ps + k * G);
#pragma unroll
        for (int h4 = 0; h4 < G / 4; h4++) prow[h4] = make_float4(sc[4 * h4], sc[4 * h4 + 1], sc[4 * h4 + 2], sc[4 * h4 + 3]);
    } else {
#pragma unroll
        for (int h = 0; h < G; h++) ps[k * G + h] = sc[h];
    }
    half_sync(hf);
    PT(3);
    if (tid < G) {
        float l = 0.0f;
        for (int w = 0; w < CH / 32; w++) l = __fadd_rn(l, red2[w * 8 + tid]);
        s_l[tid] = l;
    }
    // ---- P*V: thread = dims 2dp, 2dp+1 and heads hq*HPT .. +HPT
    const int dp = tid & 63, hq = tid >> 6;
    float acc0[HPT], acc1[HPT];
#pragma unroll
    for (int h = 0; h < HPT; h++) acc0[h] = acc1[h] = 0.0f;
    {
        const int d = 2 * dp, cc = (d & 63) >> 3;
        const uint8_t *vcol = ((d < 64) ? V0 : V1) + (d & 7) * 2;
        int off[8];
#pragma unroll
        for (int kk = 0; kk < 8; kk++) off[kk] = kk * 128 + ((cc ^ kk) << 4);
        const float *pb0 = ps + hq * HPT;
        // heads in f32x2 pairs when HPT is even: (acc_d[h], acc_d[h+1]) += (p_h, p_h+1) *
        // (v_d, v_d), each v converted twice into both halves of its pair (C8: one fmaf a term)
        constexpr int NPR = HPT % 2 == 0 ? HPT / 2 : 1;
        f32x2 pa0[NPR], pa1[NPR];
#pragma unroll
        for (int j = 0; j < NPR; j++) pa0[j] = pa1[j] = 0ull;
        auto pv_key = [&](const uint8_t *vb, const float *pb, int kk) {
            const uint32_t vw = *reinterpret_cast<const uint32_t *>(vb + off[kk]);
            if constexpr (HPT % 2 == 0) {
                f32x2 vx, vy;
                h2_bcast2(vw, vx, vy);
                if constexpr (NPR % 2 == 0) {  // two head pairs per 16-byte load (row offsets are 16-byte multiples)
                    const ulonglong2 *pq = reinterpret_cast<const ulonglong2 *>(pb + kk * G);
#pragma unroll
                    for (int j2 = 0; j2 < NPR / 2; j2++) {
                        const ulonglong2 w = pq[j2];
                        pa0[2 * j2] = ffma2(w.x, vx, pa0[2 * j2]);
                        pa1[2 * j2] = ffma2(w.x, vy, pa1[2 * j2]);
                        pa0[2 * j2 + 1] = ffma2(w.y, vx, pa0[2 * j2 + 1]);
                        pa1[2 * j2 + 1] = ffma2(w.y, vy, pa1[2 * j2 + 1]);
                    }
                } else {
                    const f32x2 *pp = reinterpret_cast<const f32x2 *>(pb + kk * G);
#pragma unroll
                    for (int j = 0; j < NPR; j++) {
                        const f32x2 pj = pp[j];
                        pa0[j] = ffma2(pj, vx, pa0[j]);
                        pa1[j] = ffma2(pj, vy, pa1[j]);
                    }
                }
            } else {
                const float2 vf = h2f2_fma(vw);
                float pj[HPT];
                lds_n<HPT>(pj, pb + kk * G);
#pragma unroll
                for (int h = 0; h < HPT; h++) {
                    acc0[h] = fmaf(pj[h], vf.x, acc0[h]);
                    acc1[h] = fmaf(pj[h], vf.y, acc1[h]);
                }
            }
        };
        if (cnt == CH) {  // a full chunk: no per-key tests, loads free to run ahead
#pragma unroll 2
            for (int j0 = 0; j0 < CH; j0 += 8) {
#pragma unroll
                for (int kk = 0; kk < 8; kk++) pv_key(vcol + j0 * 128, pb0 + j0 * G, kk);
            }
        } else {
            for (int j0 = 0; j0 < cnt; j0 += 8) {
#pragma unroll
                for (int kk = 0; kk < 8; kk++)
                    if (j0 + kk < cnt) pv_key(vcol + j0 * 128, pb0 + j0 * G, kk);
            }
        }
        if constexpr (HPT % 2 == 0) {
#pragma unroll
            for (int j = 0; j < NPR; j++) {
                const float2 a = upk2(pa0[j]), b = upk2(pa1[j]);
                acc0[2 * j] = a.x;
                acc0[2 * j + 1] = a.y;
                acc1[2 * j] = b.x;
                acc1[2 * j + 1] = b.y;
            }
        }
    }
    half_sync(hf);
    PT(4);
    const int QW = p.H * D;
    const int d = 2 * dp;
    if (nc == 1) {
#pragma unroll
        for (int h = 0; h < HPT; h++) {
            const int head = hq * HPT + h;
            const float f = bt_exp(__fsub_rn(s_m[head], s_m[head]));
            const float Lh = fmaf(s_l[head], f, 0.0f);
            float *o = p.att + (long long)t * QW + (g * G + head) * D + d;
            o[0] = __fdiv_rn(fmaf(acc0[h], f, 0.0f), Lh);
            o[1] = __fdiv_rn(fmaf(acc1[h], f, 0.0f), Lh);
        }
    } else {
        const long long pbase = (((long long)t * p.HK + g) * p.max_chunks) * G * PART_ROW;
#pragma unroll
        for (int h = 0; h < HPT; h++) {
            const int head = hq * HPT + h;
            float *pp = p.part + pbase + ((long long)c * G + head) * PART_ROW;
            *reinterpret_cast<float2 *>(pp + d) = make_float2(acc0[h], acc1[h]);
            if (dp == 0) {
                pp[D] = s_m[head];
                pp[D + 1] = s_l[head];
            }
        }
    }
    half_sync(hf);  // the tiles and scratch are free for this half's next item
    PT(5);
    return true;
}

// One slice of one head's merge of its chunk partials (C8): M = max m_c, f_c = exp(m_c - M),
// L = sum_c l_c f_c and O = sum_c acc_c f_c in chunk order, out = O / L, for the `nd` output
// dimensions starting at `part` (a head's row plus the slice offset; m and l sit at
// `ml[c * cstride]` and one float later). The slice's partials come into `stage` (shared memory,
// STEP_ACT_BYTES) by 16-byte cp.async copies issued from a rolled loop, in the same round trip as
// the m/l loads, so the code stays small (the phase runs from a cold instruction cache every
// layer) and a head split over several CTAs still reads each partial once.
__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ void combine_slice(const float *part, const float *ml, int cstride, int nc, int nd, float *out,
                              float *cbuf, float *stage, float *misc) {
    const int tid = threadIdx.x;
    float *cm = cbuf, *cl = cm + nc, *cf = cl + nc;
    const int vpc = nd / 4;                            // 16-byte vectors per chunk row of the slice
    const int pc = (STEP_ACT_BYTES / 4) / nd;          // chunks per staged piece
    const uint32_t st_s = smem_u32(stage);
    auto issue = [&](int c0) {
        const int n = (nc - c0 < pc ? nc - c0 : pc) * vpc;
#pragma unroll 1
        for (int e = tid; e < n; e += STEP_THREADS) {
            const int c = e / vpc, v = e - c * vpc;
            cp_async16_s(st_s + (uint32_t)e * 16u, part + (long long)(c0 + c) * cstride + 4 * v);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float m0 = 0.0f, l0 = 0.0f;
    const bool has_ml = tid < nc;
    if (has_ml) {
        m0 = __ldcg(ml + (long long)tid * cstride);
        l0 = __ldcg(ml + (long long)tid * cstride + 1);
    }
    issue(0);
    for (int c = tid + STEP_THREADS; c < nc; c += STEP_THREADS) {
        cm[c] = __ldcg(ml + (long long)c * cstride);
        cl[c] = __ldcg(ml + (long long)c * cstride + 1);
    }
    if (has_ml) {
        cm[tid] = m0;
        cl[tid] = l0;
    }
    __syncthreads();
    float M = -__int_as_float(0x7f800000);
#pragma unroll 4
    for (int c = 0; c < nc; c++) M = fmaxf(M, cm[c]);
    for (int c = tid; c < nc; c += STEP_THREADS) cf[c] = bt_exp(__fsub_rn(cm[c], M));
    __syncthreads();
    if (tid == STEP_THREADS - 1) {  // nd <= 128: never one of the dimension threads
        float Lh = 0.0f;
#pragma unroll 4
        for (int c = 0; c < nc; c++) Lh = fmaf(cl[c], cf[c], Lh);
        misc[1] = Lh;
    }
    float O = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < nc; c0 += pc) {
        if (c0) {
            __syncthreads();  // the previous piece has been read
            issue(c0);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        const int n = nc - c0 < pc ? nc - c0 : pc;
        if (tid < nd) {
            const float *col = stage + tid;
#pragma unroll 4
            for (int c = 0; c < n; c++) O = fmaf(col[c * nd], cf[c0 + c], O);
        }
    }
    __syncthreads();
    if (tid < nd) out[tid] = __fdiv_rn(O, misc[1]);
    __syncthreads();
}

// ------------------------------------------------------------------ the failure exit
// Taken by the whole CTA together: every path here comes through a CTA-wide vote or a
// CTA-uniform condition, so no warp leaves while others still wait at a barrier of the CTA.
// With `poison` (this CTA's own wait ran out and already set the error word), the grid barrier
// is poisoned so that every other CTA leaves at its next barrier instead of waiting out its own
// limit. Then the CTA waits, bounded, for its own bulk copies still in flight -- the warps' ring
// slots, the attention tile buffers (apend) and the aux copies (xpend) -- so that none of them
// lands in shared memory after the CTA has gone.
// Everything arrives by value: a reference to the ring or to the shared-memory map would give
// those structs an address and move them out of registers for the whole kernel.
__device__ __noinline__ void step_fail_exit(unsigned *bar, long long limit, uint64_t *ring_bars, uint32_t ring_par,
                                            int ring_nst, int ring_done, int ring_issued, uint64_t *attn_bar,
                                            uint64_t *aux_bar, uint32_t apend, uint32_t apar, uint32_t xpend,
                                            uint32_t xpar, bool poison) {
    const int tid = threadIdx.x;
    if (poison && tid == 0) poison_barrier(bar);
    for (int j = ring_done; j < ring_issued; j++) {  // this warp's ring copies in flight
        const int s = j % ring_nst;
        if (__all_sync(FULL, mbar_wait_l(ring_bars + s, (ring_par >> s) & 1u, nullptr, limit))) ring_par ^= 1u << s;
    }
    const int hf = tid >> 7;
    if ((tid & 127) == 0 && ((apend >> hf) & 1u)) mbar_wait_l(attn_bar + hf, (apar >> hf) & 1u, nullptr, limit);
    if (tid == 0)
        for (int i = 0; i < 2; i++)
            if ((xpend >> i) & 1u) mbar_wait_l(aux_bar + i, (xpar >> i) & 1u, nullptr, limit);
    __syncthreads();
}

// ------------------------------------------------------------------ the kernel
template <int G, bool SH, bool XC>
__global__ void __launch_bounds__(STEP_THREADS, 1)
    decode_step_kernel(const __grid_constant__ StepArgs p, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // offset from the shared array itself (not through an integer), so loads stay ld.shared
    uint8_t *smem = smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023u)) & 1023u);
    StepSmem sm;
    sm.ring_bar = reinterpret_cast<uint64_t *>(smem);  // 8 x 4 x 8 B
    sm.attn_bar = sm.ring_bar + STEP_WARPS * RING_SLOTS;
    sm.aux_bar = sm.attn_bar + 2;
    sm.normS = reinterpret_cast<float *>(smem + 512);
    sm.misc = sm.normS + STEP_MAX_T;
    sm.pos = reinterpret_cast<int *>(sm.misc + 64);
    sm.blkn = sm.pos + STEP_MAX_T;
    sm.seq = sm.blkn + STEP_MAX_T;
    sm.iblk = sm.seq + STEP_MAX_T;
    sm.ldesc = reinterpret_cast<LayerDev *>(smem + 1024);
    sm.outd = reinterpret_cast<QMatDev *>(smem + 1024 + 2 * sizeof(LayerDev));
    sm.region = smem + STEP_HDR_BYTES;
    sm.act = reinterpret_cast<ActBlock *>(sm.region + STEP_REGION_BYTES);
    sm.sel_ids = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(sm.act) + STEP_ACT_BYTES);
    sm.sel_w = reinterpret_cast<float *>(sm.sel_ids + STEP_MAX_T * MAX_K);
    sm.sel_slot = reinterpret_cast<int *>(sm.sel_w + STEP_MAX_T * MAX_K);
    sm.wv = reinterpret_cast<float *>(sm.sel_slot + STEP_MAX_T * MAX_K);
    sm.cbuf = sm.wv + STEP_WARPS * MAX_K;
    sm.res = sm.cbuf + STEP_CBUF_BYTES / 4;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = p.T, E = p.E, QW = p.H * 128, KW = p.HK * 128, K = p.K, F = p.F;
    unsigned epoch = 0;
    auto TR = [&](int layer, int ph) -> unsigned long long * {
        return p.trace ? p.trace + ((long long)layer * STEP_PHASES + ph) * (gridDim.x + 1) : nullptr;
    };
    // cycle counters of the traced step (max over warps), slots 8 + k of the layer's rows
    unsigned long long *cycv = reinterpret_cast<unsigned long long *>(sm.misc + 32);  // [16]
    auto CYC_RESET = [&]() {
        if (p.trace) {
            __syncthreads();
            if (tid < 16) cycv[tid] = 0ull;
            __syncthreads();
        }
    };
    auto CYC_WRITE = [&](int layer, int k, int idx) {  // slot k <- cycles idx (max over warps)
        if (!p.trace) return;
        __syncthreads();
        if (tid == 0) p.trace[((long long)layer * STEP_PHASES + 8 + k) * (gridDim.x + 1) + blockIdx.x] = cycv[idx];
    };
    // a point inside a phase: this CTA's time when all its threads got there
    auto POINT = [&](int layer, int k) {
        if (!p.trace) return;
        __syncthreads();
        if (tid == 0) p.trace[((long long)layer * STEP_PHASES + 8 + k) * (gridDim.x + 1) + blockIdx.x] = global_ns();
    };
    if (p.trace && tid == 0 && blockIdx.x == 0)
        p.trace[((long long)(p.n_layer + 1) * STEP_PHASES) * (gridDim.x + 1)] = global_ns();
    const int nsbE = E / 256, nsbQ = QW / 256, nsbF = F / 256;

    WarpRing ring;
    ring.base = sm.region + (size_t)warp * (STEP_REGION_BYTES / STEP_WARPS);
    ring.bars = sm.ring_bar + warp * RING_SLOTS;
    ring.par = 0;
    ring.configure(4096);
    if (lane == 0) {
        for (int i = 0; i < RING_SLOTS; i++) mbar_init(ring.bars + i, 1);
    }
    if (tid < 4) mbar_init(sm.attn_bar + tid, 1);  // attn_bar[0..1] and aux_bar[0..1]
    if (tid < T) {
        const int seq = p.seq_of[tid], ps = p.dev_len[seq];
        sm.pos[tid] = ps;
        sm.seq[tid] = seq;
        sm.blkn[tid] = p.block_table[seq * p.max_blocks + ps / 16];
    }
    if (tid < LD_WORDS)
        reinterpret_cast<uint32_t *>(sm.ldesc)[tid] = __ldg(reinterpret_cast<const uint32_t *>(p.layers) + tid);
    if (tid == 0) *sm.outd = p.out;
    fence_mbar_init();
    __syncthreads();
    uint32_t apar = 0, xpar = 0;  // next parities of attn_bar[0..1] and aux_bar[0..1]
    // copies in flight that no wait has consumed yet, per attention buffer and aux barrier (what
    // the failure exit waits for); aux 1 (layer 0's attn_norm) is requested below
    uint32_t apend = 0, xpend = 2u;
#define STEP_FAIL(poison)                                                       \
    do {                                                                        \
        step_fail_exit(p.bar, p.wait_limit, ring.bars, ring.par, ring.nst, ring.done, ring.issued, sm.attn_bar, \
                       sm.aux_bar, apend, apar, xpend, xpar, poison);                                    \
        return;                                                                 \
    } while (0)
    {
        // the page ids of this CTA's first two attention items: the same in every layer
        constexpr int PPI = ATTN_CHUNK / 16;
        const int n_it = attn_items(p, sm.pos);
        if (tid < 2 * PPI) {
            const int k = tid / PPI, pg = tid % PPI;
            const int i = blockIdx.x + k * gridDim.x;
            int blk = 0;
            if (i < n_it) {
                AttnItem it;
                attn_item(p, sm.pos, i, it);
                const int nk = sm.pos[it.t] + 1, base = it.c * ATTN_CHUNK;
                if (base + pg * 16 < nk) blk = p.block_table[sm.seq[it.t] * p.max_blocks + (base >> 4) + pg];
            }
            sm.iblk[tid] = blk;
        }
    }
    if (tid == 0) {
        prefetch_tmap(&tmap);
        // layer 0's attn_norm for the first staging
        fence_proxy_async();
        mbar_arrive_expect_tx(sm.aux_bar + 1, E * 4);
        bulk_g2s(sm.cbuf, sm.ldesc[0].attn_norm, E * 4, sm.aux_bar + 1);
    }
    // wait for aux copy i (all threads); false if the bounded wait ran out anywhere in the CTA
    auto wait_aux = [&](int i) -> bool {
        const bool ok = mbar_wait_l(sm.aux_bar + i, (xpar >> i) & 1u, p.err, p.wait_limit);
        if (ok) {
            xpar ^= 1u << i;
            xpend &= ~(1u << i);
        }
        return !__syncthreads_or(!ok);
    };

    // ---- embedding rows (get_rows) for every token, into the region, then layer 0 reads them
    float *x0 = reinterpret_cast<float *>(sm.region);  // [T][E] f32, 16-byte aligned
    {
        const int bb = qk_block_bytes(p.embd_type);
        for (int i = tid; i < T * E; i += STEP_THREADS) {
            const int t = i / E, e = i % E;
            const int tok = p.tokens[t];
            const bool okt = tok >= 0 && tok < p.V;
            const uint8_t *blk = p.embd + ((long long)(okt ? tok : 0) * nsbE + e / 256) * bb;
            const int v = e % 256;
            float yv;
            if (p.embd_type == T_Q4_K) {
                const float dd = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                const float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
                const uint8_t *scb = blk + 4, *qs = blk + 16;
                const int j = v / 32, gi = v / 64, hi = j & 1, l = v % 32;
                int scj, mj;
                if (j < 4) {
                    scj = scb[j] & 63;
                    mj = scb[j + 4] & 63;
                } else {
                    scj = (scb[j + 4] & 0xF) | ((scb[j - 4] >> 6) << 4);
                    mj = (scb[j + 4] >> 4) | ((scb[j] >> 6) << 4);
                }
                const int q = hi ? (qs[32 * gi + l] >> 4) : (qs[32 * gi + l] & 0xF);
                yv = __fsub_rn(__fmul_rn(__fmul_rn(dd, (float)scj), (float)q), __fmul_rn(dmin, (float)mj));
            } else {
                const float dd = f16_bits_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
                const int8_t *scb = reinterpret_cast<const int8_t *>(blk + 192);
                const int n = v / 128, r = v % 128, quad = r / 32, l = r % 32;
                const int lo = quad == 0 ? (blk[64 * n + l] & 0xF)
                                         : quad == 1 ? (blk[64 * n + 32 + l] & 0xF)
                                                     : quad == 2 ? (blk[64 * n + l] >> 4) : (blk[64 * n + 32 + l] >> 4);
                const int hi2 = (blk[128 + 32 * n + l] >> (2 * quad)) & 3;
                yv = __fmul_rn(__fmul_rn(dd, (float)scb[v / 16]), (float)((lo | (hi2 << 4)) - 32));
            }
            yv = okt ? yv : 0.0f;
            x0[i] = yv;
            if (blockIdx.x == 0) p.x[i] = yv;
            if (!okt && e == 0) {
                atomicOr(p.err, ERR_BAD_INDEX);
                poison_barrier(p.bar);
            }
        }
        if (blockIdx.x == 0 && tid < T) p.pos_of[tid] = sm.pos[tid];
        __syncthreads();
    }
    // the rope rows of this step's positions, towards L2
    if (tid < T) prefetch_l2(p.rope + (long long)sm.pos[tid] * p.n_rot, p.n_rot * 4);

    for (int il = 0; il < p.n_layer; il++) {
        const LayerDev &L = sm.ldesc[il & 1];
        bool bad = false;  // this thread's warp saw a bounded wait run out in the current phase
        const bool has_next = il + 1 < p.n_layer;
        // the next layer's descriptor: loaded now, stored to shared memory after the attention
        uint32_t ld_next = 0;
        if (has_next && tid < LD_WORDS) ld_next = __ldg(reinterpret_cast<const uint32_t *>(p.layers + il + 1) + tid);
        // ================= QKV
        const SegList sq = make_segs(&L.q, 0, &L.k, QW, &L.v, QW + KW);
        {
            const float *xs = il == 0 ? x0 : p.x;
            if (!wait_aux(1)) STEP_FAIL(true);  // attn_norm in cbuf
            step_stage(xs, E, E, T, sm.cbuf, p.eps, sm.act, sm.normS, nullptr);
            __syncthreads();
            POINT(il, 0);
            if (il == 0) gemv_preissue(ring, sq, warp, lane);  // the region held the embedding rows
            CYC_RESET();
            bad = !gemv_run(ring, sq, sm.act, nsbE, T, p.qkv, QW + 2 * KW, nullptr, 0, 0, nullptr, p.err, p.wait_limit,
                            warp, lane, p.trace ? cycv : nullptr);
            CYC_WRITE(il, 7, 0);
            CYC_WRITE(il, 8, 1);
        }
        // the K/V pages of this CTA's first two attention items, requested before the barrier
        const int it0 = blockIdx.x;
        const int n_items = attn_items(p, sm.pos);
        __syncthreads();  // every warp is done with its ring slots: the region takes attention tiles
        if (warp < 2) {  // warp k issues item k's pages
            const int i = it0 + warp * gridDim.x;
            if (i < n_items) {
                AttnItem it;
                attn_item(p, sm.pos, i, it);
                attn_issue_warp(p, &tmap, sm, it, il, warp, sm.iblk + warp * (ATTN_CHUNK / 16), lane);
            }
        }
        apend = (it0 < n_items ? 1u : 0u) | (it0 + (int)gridDim.x < n_items ? 2u : 0u);
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 0)))
            STEP_FAIL(gs_ == 2);
        // ================= ATTN: items it0 + k * grid; half hf of the CTA runs k = hf, hf + 2, ...
        {
            const int hf = warp >> 2;
            bool ok = true;
            for (int k = hf;; k += 2) {
                const int i = it0 + k * gridDim.x;
                if (i >= n_items) break;
                AttnItem it;
                attn_item(p, sm.pos, i, it);
                if (k >= 2) {
                    if ((tid & 127) < 32) attn_issue_warp(p, &tmap, sm, it, il, hf, nullptr, lane);
                    apend |= 1u << hf;
                }
                unsigned long long *tp =
                    (p.trace && k == 0) ? p.trace + ((long long)il * STEP_PHASES + 8 + 16) * (gridDim.x + 1) : nullptr;
                if (!attn_half<G>(p, L, sm, it, il, hf, apar, apend, tp)) {
                    ok = false;
                    break;
                }
            }
            if (__syncthreads_or(!ok)) STEP_FAIL(true);
        }
        if (has_next && tid < LD_WORDS) reinterpret_cast<uint32_t *>(sm.ldesc + ((il + 1) & 1))[tid] = ld_next;
        // attn_output tiles are static: request this CTA's first ones now. Its residual rows (x)
        // are final since the last barrier of the previous layer.
        const SegList so = make_segs(&L.o, 0, nullptr, 0, nullptr, 0);
        int o0, o1;
        cta_range(so.total, o0, o1);
        const int orow0 = (int)(o0 * L.o.rpt);
        int orows = (int)(o1 * L.o.rpt) - orow0;
        orows = orow0 + orows > E ? E - orow0 : orows;
        orows = orows < 1 ? 1 : orows;
        float res_pre = 0.0f;
        if (tid < T * orows && orow0 + tid % orows < E)
            res_pre = __ldcg(p.x + (long long)(tid / orows) * E + orow0 + tid % orows);
        __syncthreads();
        gemv_preissue(ring, so, warp, lane);
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 1)))
            STEP_FAIL(gs_ == 2);
        if (tid < T * orows) sm.res[tid] = res_pre;
        // the next layer's small vectors, towards L2
        if (has_next && blockIdx.x < 3) {
            const LayerDev &Ln = sm.ldesc[(il + 1) & 1];
            const float *v = blockIdx.x == 0 ? Ln.attn_norm : blockIdx.x == 1 ? Ln.ffn_norm : Ln.q_norm;
            const int nb = blockIdx.x == 2 ? 128 * 4 : E * 4;
            if (tid * 128 < nb) prefetch_l2(reinterpret_cast<const uint8_t *>(v) + tid * 128, 128);
            if (blockIdx.x == 2 && tid < 4) prefetch_l2(reinterpret_cast<const uint8_t *>(Ln.k_norm) + tid * 128, 128);
        }
        // ================= COMBINE (tokens whose context spans several chunks)
        {
            int multi = 0;
            for (int t = 0; t < T; t++) multi += (sm.pos[t] + 1 > ATTN_CHUNK);
            if (multi) {
                // each head in `split` slices of 128 / split dimensions, as many as the grid covers
                const int split = T * p.H * 4 <= (int)gridDim.x ? 4 : T * p.H * 2 <= (int)gridDim.x ? 2 : 1;
                const int nd = 128 / split;
                const int n_ci = T * p.H * split;
                for (int ci = blockIdx.x; ci < n_ci; ci += gridDim.x) {
                    const int th = ci / split, q = ci - th * split;
                    const int t = th / p.H, hd = th - t * p.H;
                    const int nc = (sm.pos[t] + 1 + ATTN_CHUNK - 1) / ATTN_CHUNK;
                    if (nc == 1) continue;
                    const int g = hd / G, h = hd % G;
                    const float *row =
                        p.part + (((long long)t * p.HK + g) * p.max_chunks) * G * PART_ROW + (long long)h * PART_ROW;
                    combine_slice(row + q * nd, row + 128, G * PART_ROW, nc, nd,
                                  p.att + (long long)t * QW + hd * 128 + q * nd, sm.cbuf,
                                  reinterpret_cast<float *>(sm.act), sm.misc);
                }
                if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                              TR(il, 2)))
                    STEP_FAIL(gs_ == 2);
            }
        }
        // ================= O: ffn_in = x + W_o * att
        step_stage(p.att, QW, QW, T, nullptr, 0.0f, sm.act, nullptr, nullptr);
        __syncthreads();
        POINT(il, 2);
        bad = !gemv_run(ring, so, sm.act, nsbQ, T, p.ffn_in, E, sm.res, orow0, orows, nullptr, p.err, p.wait_limit, warp,
                        lane);
        // this CTA's router rows and the ffn norm vector, requested before the barrier
        const int nrr = (int)blockIdx.x < p.NE ? (p.NE - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        float *rrows = reinterpret_cast<float *>(sm.region);
        float *ynorm = rrows + STEP_ROUTER_ROWS * E;
        __syncthreads();  // every warp is done with its ring slots: the region takes router rows
        if (tid == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(sm.aux_bar + 0, nrr * E * 4);
            for (int k = 0; k < nrr; k++)
                bulk_g2s_hint(rrows + k * E, L.gate_inp + (long long)(blockIdx.x + k * gridDim.x) * E, E * 4,
                              sm.aux_bar + 0, l2_evict_first_policy());
            mbar_arrive_expect_tx(sm.aux_bar + 1, E * 4);
            bulk_g2s(sm.cbuf, L.ffn_norm, E * 4, sm.aux_bar + 1);
        }
        xpend |= 3u;
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 3)))
            STEP_FAIL(gs_ == 2);
        // ================= ROUTER: ffn RMSNorm (staged for the experts too) and router rows
        if (!wait_aux(1)) STEP_FAIL(true);
        step_stage(p.ffn_in, E, E, T, sm.cbuf, p.eps, sm.act, sm.normS, ynorm);
        if (!wait_aux(0)) STEP_FAIL(true);  // its __syncthreads also completes ynorm
        POINT(il, 3);
        for (int q = warp; q < nrr * T; q += STEP_WARPS) {  // (router row k, token t) per warp, C5
            const int k = q / T, t = q % T;
            const float *wr = rrows + k * E, *yt = ynorm + t * E;
            float acc = 0.0f;
#pragma unroll 8
            for (int i = lane; i < E; i += 32) acc = fmaf(wr[i], yt[i], acc);
            acc = butterfly_sum(acc);
            const int row = blockIdx.x + k * gridDim.x;
            if (L.gate_bias) acc = __fadd_rn(acc, L.gate_bias[row]);
            if (lane == 0) p.rlog[(long long)t * p.NE + row] = acc;
        }
        int d0, d1;
        cta_range(T * E, d0, d1);
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 4)))
            STEP_FAIL(gs_ == 2);
        // ================= GATEUP: soft_max + route() in every CTA (C5, C7; stable descending
        // by total_cmp, top K, renormalised), then the experts
        {
            const int NE = p.NE;
            float *prob = sm.cbuf;                                  // [T][NE]
            int *keys = reinterpret_cast<int *>(sm.cbuf + T * NE);  // [T][NE]
            for (int i = tid; i < T * NE; i += STEP_THREADS) prob[i] = __ldcg(p.rlog + i);
            __syncthreads();
            if (warp < T) {
                float *pr = prob + warp * NE;
                float m = -__int_as_float(0x7f800000);
                for (int i = lane; i < NE; i += 32) m = fmaxf(m, pr[i]);
                m = warp_max(m);
                float acc = 0.0f;
                for (int i = lane; i < NE; i += 32) {
                    const float e = bt_exp(__fsub_rn(pr[i], m));
                    pr[i] = e;
                    acc = __fadd_rn(acc, e);
                }
                acc = butterfly_sum(acc);
                const float inv = __fdiv_rn(1.0f, acc);
                for (int i = lane; i < NE; i += 32) {
                    const float v = __fmul_rn(pr[i], inv);
                    pr[i] = v;
                    keys[warp * NE + i] = total_key(v);
                }
            }
            __syncthreads();
            for (int i = tid; i < T * NE; i += STEP_THREADS) {  // rank of every expert, one per thread
                const int t = i / NE, li = i - t * NE;
                const int ki = keys[i];
                const int4 *kr = reinterpret_cast<const int4 *>(keys + t * NE);
                int rank = 0;
#pragma unroll 4
                for (int j4 = 0; j4 < NE / 4; j4++) {
                    const int4 kk = kr[j4];
                    const int j = 4 * j4;
                    rank += (kk.x > ki) | ((kk.x == ki) & (j < li));
                    rank += (kk.y > ki) | ((kk.y == ki) & (j + 1 < li));
                    rank += (kk.z > ki) | ((kk.z == ki) & (j + 2 < li));
                    rank += (kk.w > ki) | ((kk.w == ki) & (j + 3 < li));
                }
                if (rank < K) sm.sel_ids[t * MAX_K + rank] = li;  // by rank for now
            }
            __syncthreads();
            if (warp < T) {  // token t = warp: lane q holds the expert of rank q
                const int t = warp;
                const bool has = lane < K;
                const int id = has ? sm.sel_ids[t * MAX_K + lane] : 0x7fffffff;
                float w = has ? prob[t * NE + id] : 0.0f;
                float total = 0.0f;  // in rank order
                for (int q = 0; q < K; q++) total = __fadd_rn(total, __shfl_sync(FULL, w, q));
                w = total > 0.0f ? __fdiv_rn(w, total) : w;
                if (has && blockIdx.x == 0) {
                    p.dbg_ids[((long long)il * p.TB + t) * K + lane] = id;
                    p.dbg_w[((long long)il * p.TB + t) * K + lane] = w;
                }
                int slot = 0;  // ascending expert ids (distinct)
                for (int q = 0; q < K; q++) slot += __shfl_sync(FULL, id, q) < id;
                __syncwarp();
                if (has) {
                    sm.sel_ids[t * MAX_K + slot] = id;
                    sm.sel_w[t * MAX_K + slot] = w;
                }
            }
            __syncthreads();
        }
        if constexpr (XC) {
            // the expert cache: CTA 0 looks the layer's selections up (the device policy); once
            // every CTA has the slots, each fills its share of the missed ones from the pinned
            // host blocks, and a second barrier orders those copies before the tile requests
            const long long xbytes = L.gate.mat_bytes + L.up.mat_bytes + L.down.mat_bytes;
            if (blockIdx.x == 0)
                xc_lookup_cta(p.xd, il, sm.sel_ids, T, K, MAX_K, p.xc_rows + (long long)il * p.NE, p.xc_host[il],
                              p.xc_pool, p.xc_stride, xbytes, p.xc_bounce, p.xc_copies, p.xc_ncopies, p.err,
                              xc_scratch(sm.cbuf));
            if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, false,
                                          nullptr))
                STEP_FAIL(gs_ == 2);
            const int nc = __ldcg(p.xc_ncopies);
            if (nc > 0) {
                xc_copy_part(p.xc_copies, nc, xbytes, (long long)blockIdx.x * STEP_THREADS + tid,
                             (long long)gridDim.x * STEP_THREADS);
                if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch,
                                              false, nullptr))
                    STEP_FAIL(gs_ == 2);
                // the slots were written through the generic proxy; the tile copies read them
                // through the async proxy
                asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            if (tid < T * K) {
                const int t = tid / K, k = tid - t * K;
                sm.sel_slot[t * MAX_K + k] =
                    __ldcg(p.xc_rows + (long long)il * p.NE + sm.sel_ids[t * MAX_K + k]);
            }
            __syncthreads();
        }
        POINT(il, 4);
        {
            // routed units (token, slot, tile), then the shared expert's (token, tile)
            const int nr = T * K * L.gate.n_tiles, ns = SH ? T * L.sgate.n_tiles : 0;
            int u0, u1;
            cta_range(nr + ns, u0, u1);
            const int n = warp_units(u0, u1, warp);
            const int sgb = SH ? L.sgate.tile_bytes + L.sup.tile_bytes : 0;
            ring.configure(L.gate.tile_bytes + L.up.tile_bytes > sgb ? L.gate.tile_bytes + L.up.tile_bytes : sgb);
            const int nsb = L.gate.nsb;  // gate and up have E columns: the same tile shape throughout
            // both kinds' tile geometry in registers: a unit picks one with selects
            const int rnt = L.gate.n_tiles, rS = L.gate.S, rrpt = L.gate.rpt, rtb = L.gate.tile_bytes;
            const int snt = L.sgate.n_tiles, sS = L.sgate.S, srpt = L.sgate.rpt, stb = L.sgate.tile_bytes;
            const bool rgq4 = L.gate.type == T_Q4_K, ruq4 = L.up.type == T_Q4_K;
            const bool sgq4 = L.sgate.type == T_Q4_K, suq4 = L.sup.type == T_Q4_K;
            const bool drill = p.fault_copy == il + 1 && p.fault_cta == (int)blockIdx.x;
            while (ring.issued < n && ring.can_issue())
                gateup_issue<SH, XC>(ring, L, sm, K, nr, u0, warp, lane, drill, p.xc_pool, p.xc_stride);
            CYC_RESET();
            long long gcw = 0, gc0 = clock64();
            for (int j = 0; j < n; j++) {
                while (ring.issued < n && ring.can_issue())
                    gateup_issue<SH, XC>(ring, L, sm, K, nr, u0, warp, lane, drill, p.xc_pool, p.xc_stride);
                const long long w0 = clock64();
                if (!ring.wait(j, p.err, p.wait_limit)) {
                    bad = true;
                    break;
                }
                gcw += clock64() - w0;
                const int u = u0 + warp + j * STEP_WARPS;
                const bool sh = SH && u >= nr;
                const int gnt = sh ? snt : rnt, gS = sh ? sS : rS, grpt = sh ? srpt : rrpt, gtb = sh ? stb : rtb;
                const bool gq4 = sh ? sgq4 : rgq4, uq4 = sh ? suq4 : ruq4;
                int t, tile, width;
                float *out;
                if (sh) {
                    t = (u - nr) / gnt;
                    tile = (u - nr) - t * gnt;
                    width = p.FS;
                    out = p.shact + (long long)t * p.FS;
                } else {
                    const int tk = u / gnt;
                    tile = u - tk * gnt;
                    t = tk / K;
                    width = F;
                    out = p.act + (long long)tk * F;
                }
                const uint8_t *gt = ring.slot_ptr(j), *ut = gt + gtb;
                const bool active = lane < gS;
                const int rit = active ? lane / nsb : 0, b = active ? lane - rit * nsb : 0;
                const int row = tile * grpt + rit;
                float rowv[2];
#pragma unroll 1
                for (int which = 0; which < 2; which++) {
                    const uint8_t *tl = which ? ut : gt;
                    const bool q4 = which ? uq4 : gq4;
                    float v = 0.0f;
                    if (active) {
                        const ActBlock &ab = sm.act[t * nsbE + b];
                        v = slot_dot(q4, tl, gS, lane, &ab);
                    }
                    float rr = 0.0f;
                    for (int b2 = 0; b2 < nsb; b2++) {
                        const int srcl = rit * nsb + b2;
                        rr = __fadd_rn(rr, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
                    }
                    rowv[which] = rr;
                }
                if (active && b == 0 && row < width) out[row] = __fmul_rn(bt_silu(rowv[0]), rowv[1]);
                __syncwarp();
                ring.done++;
            }
            if (p.trace && lane == 0) {
                atomicMax(cycv + 4, (unsigned long long)gcw);
                atomicMax(cycv + 5, (unsigned long long)(clock64() - gc0 - gcw));
            }
            CYC_WRITE(il, 11, 4);
            CYC_WRITE(il, 12, 5);
            POINT(il, 5);
            // the down rows of this CTA: request the first ones before the barrier
            if (!bad) {  // a warp whose wait ran out keeps its ring as it is, for the failure drain
                const int dtb = down_row_bytes<SH>(L), maxr = down_max_rows(dtb), nk = K + (SH ? 1 : 0);
                int t_, r_, n_, o_;
                const int nt = nk * down_piece(d0, d1, E, maxr, 1 << 30, t_, r_, n_, o_);
                const int dn = nt > warp ? (nt - warp + STEP_WARPS - 1) / STEP_WARPS : 0;
                ring.configure(maxr * dtb);
                while (ring.issued < dn && ring.can_issue())
                    down_issue<SH, XC>(ring, L, sm, K, nk, E, d0, d1, maxr, warp, lane, p.xc_pool, p.xc_stride);
            }
        }
        // the down phase's residual rows (ffn_in, final since the O barrier)
        float dres_pre = 0.0f;
        if (tid < d1 - d0) dres_pre = __ldcg(p.ffn_in + d0 + tid);
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 5)))
            STEP_FAIL(gs_ == 2);
        if (tid < d1 - d0) sm.res[tid] = dres_pre;
        // ================= DOWN: unit (row piece, expert) per warp in turn: the warp stages that
        // expert's SiLU products (C3) and writes its rows' values to shared memory; then one
        // thread per output row adds the experts in the reference's order (the shared expert's
        // value after them, C10), and the residual
        {
            const int dtb = down_row_bytes<SH>(L), maxr = down_max_rows(dtb), nk = K + (SH ? 1 : 0);
            int t_, r_, n_, o_;
            const int nt = nk * down_piece(d0, d1, E, maxr, 1 << 30, t_, r_, n_, o_);
            const int n = nt > warp ? (nt - warp + STEP_WARPS - 1) / STEP_WARPS : 0;
            ActBlock *mine = sm.act + warp * STEP_MAX_NSB_F;  // this warp's expert's products
            float *part = step_down_part(sm);                 // [MAX_K][STEP_DOWN_ROWS] the rows' values
            int staged = -1;                                  // (token, expert) in `mine`
            CYC_RESET();
            long long dcw = 0, dc0 = clock64();
            for (int j = 0; j < n; j++) {
                while (ring.issued < n && ring.can_issue())
                    down_issue<SH, XC>(ring, L, sm, K, nk, E, d0, d1, maxr, warp, lane, p.xc_pool, p.xc_stride);
                const int i = warp + j * STEP_WARPS, q = i / nk, k = i - q * nk;
                int t, r0, nr, off;
                down_piece(d0, d1, E, maxr, q, t, r0, nr, off);
                const bool shx = SH && k == K;
                const int nsbX = shx ? p.FS / 256 : nsbF;
                const int mtb = shx ? L.sdown.tile_bytes : L.down.tile_bytes;
                const bool dq4 = (shx ? L.sdown.type : L.down.type) == T_Q4_K;
                if (t * nk + k != staged) {
                    staged = t * nk + k;
                    __syncwarp();
                    stage_blocks_warp(shx ? p.shact + (long long)t * p.FS : p.act + (long long)(t * K + k) * F, nsbX,
                                      smem_u32(mine), lane);
                    __syncwarp();
                }
                const long long w0 = clock64();
                if (!ring.wait(j, p.err, p.wait_limit)) {
                    bad = true;
                    break;
                }
                dcw += clock64() - w0;
                const uint8_t *tb = ring.slot_ptr(j);
                const int rpp = 32 / nsbX;  // rows per pass of the warp
                for (int rb = 0; rb < nr; rb += rpp) {
                    const int ri = lane / nsbX, b = lane - ri * nsbX, r = rb + ri;
                    const bool valid = ri < rpp && r < nr;
                    float v = 0.0f;
                    if (valid) v = slot_dot(dq4, tb + r * mtb, nsbX, b, mine + b);
                    float acc = 0.0f;
                    for (int b2 = 0; b2 < nsbX; b2++) {
                        const int srcl = ri * nsbX + b2;
                        acc = __fadd_rn(acc, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
                    }
                    if (valid && b == 0) part[k * STEP_DOWN_ROWS + off + r] = acc;
                }
                __syncwarp();
                ring.done++;
            }
            if (p.trace && lane == 0) {
                atomicMax(cycv + 2, (unsigned long long)dcw);
                atomicMax(cycv + 3, (unsigned long long)(clock64() - dc0 - dcw));
            }
            CYC_WRITE(il, 9, 2);
            CYC_WRITE(il, 10, 3);
            POINT(il, 6);
            __syncthreads();
            if (tid < d1 - d0) {
                // expert_ffn_single order: chunks of ceil(K/workers) summed by ggml_add, partials
                // added to a zero vector (stream.rs:1232-1284), then the shared expert and the residual
                int workers = p.workers < K ? p.workers : K;
                if (workers < 1) workers = 1;
                const int wchunk = (K + workers - 1) / workers;
                const int u = d0 + tid, t = u / E;
                const float *w = sm.sel_w + t * MAX_K;
                float sum = 0.0f;
                for (int s0 = 0; s0 < K; s0 += wchunk) {
                    float tot = __fmul_rn(part[s0 * STEP_DOWN_ROWS + tid], w[s0]);
                    for (int q = s0 + 1; q < K && q < s0 + wchunk; q++)
                        tot = __fadd_rn(tot, __fmul_rn(part[q * STEP_DOWN_ROWS + tid], w[q]));
                    sum = workers <= 1 ? tot : __fadd_rn(sum, tot);
                }
                if (SH) sum = __fadd_rn(sum, part[K * STEP_DOWN_ROWS + tid]);
                p.x[u] = __fadd_rn(sum, sm.res[tid]);
            }
        }
        // the next layer's q/k/v tiles (or the output head's) and its norm vector are static:
        // request them now
        __syncthreads();
        if (tid == 0) {
            const float *nv = has_next ? sm.ldesc[(il + 1) & 1].attn_norm : p.out_norm;
            fence_proxy_async();
            mbar_arrive_expect_tx(sm.aux_bar + 1, E * 4);
            bulk_g2s(sm.cbuf, nv, E * 4, sm.aux_bar + 1);
        }
        xpend |= 2u;
        if (bad) {
        } else if (has_next) {  // (a warp whose wait ran out keeps its ring for the drain)
            const LayerDev &Ln = sm.ldesc[(il + 1) & 1];
            const SegList sqn = make_segs(&Ln.q, 0, &Ln.k, QW, &Ln.v, QW + KW);
            gemv_preissue(ring, sqn, warp, lane);
        } else {
            const SegList sout = make_segs(sm.outd, 0, nullptr, 0, nullptr, 0);
            gemv_preissue(ring, sout, warp, lane);
        }
        if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, bad,
                                      TR(il, 6)))
            STEP_FAIL(gs_ == 2);
    }
    // ================= output head with the fused argmax
    bool hbad = false;
    {
        const SegList sout = make_segs(sm.outd, 0, nullptr, 0, nullptr, 0);
        if (!wait_aux(1)) STEP_FAIL(true);  // out_norm in cbuf
        step_stage(p.x, E, E, T, sm.cbuf, p.eps, sm.act, sm.normS, nullptr);
        __syncthreads();
        CYC_RESET();
        hbad = !gemv_run(ring, sout, sm.act, nsbE, T, p.logits, p.V, nullptr, 0, 0, p.amax, p.err, p.wait_limit, warp,
                         lane, p.trace ? cycv : nullptr);
        CYC_WRITE(p.n_layer, 13, 0);
        CYC_WRITE(p.n_layer, 14, 1);
    }
    if (const int gs_ = grid_sync(p.bar, p.err, p.wait_limit, p.fault_cta, p.fault_barrier, ++epoch, hbad,
                                  TR(p.n_layer, 0)))
        STEP_FAIL(gs_ == 2);
    // ================= step end: argmax out, lengths advance, greedy feed-back
    if (blockIdx.x == 0 && tid < T) {
        const int t = tid;
        const unsigned long long packed = p.amax[t];
        p.amax[t] = 0ull;
        const int bi = (int)(packed & 0xffffffffull);
        p.next_token[t] = bi;
        if (p.tokens_buf) p.tokens_buf[t] = bi;
        if (p.gen_out) {
            const int k = p.gen_count[t]++;
            p.gen_out[(long long)k * p.n_out + t] = bi;
        }
        p.dev_len[p.seq_of[t]] += 1;
    }
}

#undef STEP_FAIL

size_t step_smem_bytes(int max_chunks) {
    (void)max_chunks;
    return 1024 + STEP_HDR_BYTES + STEP_REGION_BYTES + STEP_ACT_BYTES + (size_t)STEP_MAX_T * MAX_K * 12 +
           (size_t)STEP_WARPS * MAX_K * 4 + STEP_CBUF_BYTES + (size_t)STEP_RES * 4;
}

cudaError_t init_step_kernel_attributes() {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev))) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
    const void *kerns[] = {(const void *)decode_step_kernel<2, false, false>,
                           (const void *)decode_step_kernel<4, false, false>,
                           (const void *)decode_step_kernel<6, false, false>,
                           (const void *)decode_step_kernel<8, false, false>,
                           (const void *)decode_step_kernel<4, true, false>,
                           (const void *)decode_step_kernel<4, false, true>,
                           (const void *)decode_step_kernel<8, false, true>};
    for (const void *k : kerns) {
        cudaFuncAttributes fa;
        if ((e = cudaFuncGetAttributes(&fa, k))) return e;
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes)))
            return e;
    }
    return cudaSuccess;
}

template <int G, bool SH, bool XC>
static cudaError_t launch_step_g(const StepArgs &a, const CUtensorMap &tmap, int grid, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(STEP_THREADS);
    cfg.dynamicSmemBytes = step_smem_bytes(a.max_chunks);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_step_kernel<G, SH, XC>, a, tmap);
}

cudaError_t launch_decode_step(const StepArgs &a, const CUtensorMap &tmap, int grid, cudaStream_t st) {
    if (a.xc_on && a.FS) return cudaErrorInvalidValue;  // no instantiation carries both
    switch (a.G) {
    case 2: return a.FS || a.xc_on ? cudaErrorInvalidValue : launch_step_g<2, false, false>(a, tmap, grid, st);
    case 4:
        return a.FS      ? launch_step_g<4, true, false>(a, tmap, grid, st)
               : a.xc_on ? launch_step_g<4, false, true>(a, tmap, grid, st)
                         : launch_step_g<4, false, false>(a, tmap, grid, st);
    case 6: return a.FS || a.xc_on ? cudaErrorInvalidValue : launch_step_g<6, false, false>(a, tmap, grid, st);
    case 8:
        return a.FS      ? cudaErrorInvalidValue
               : a.xc_on ? launch_step_g<8, false, true>(a, tmap, grid, st)
                         : launch_step_g<8, false, false>(a, tmap, grid, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace bt
