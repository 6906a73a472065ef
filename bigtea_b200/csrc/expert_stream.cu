// expert_stream.cu -- the single-token expert FFN of many layers in one persistent kernel, for
// measuring the dequant-fused expert GEMV's bandwidth apart from the decode step's latency.
//
// The decode step learns a layer's experts only after that layer's router, so its gate/up
// tiles cannot be requested before then. This kernel runs the same expert arithmetic (the
// C4 K-quant dots, SiLU(gate) * up, the down rows and the reference's expert sum, operation for
// operation the persistent step's GATEUP and DOWN phases) over every layer's selections, which
// it is given up front, as an expert-streaming schedule would have them. Layer s's gate/up and
// layer s-1's down run in the same stage, so one grid-wide dependency per layer (gate/up ->
// down) is waited for a whole stage after the CTA announced it, and the weight stream never
// stops at it:
//
//   * one producer warp per CTA walks the CTA's units in order and requests each into the next
//     free slot of a CTA-wide ring (1-D TMA bulk copies, full/empty mbarrier pairs), as far
//     ahead as the ring holds. Per stage: its gate/up tile pairs of layer s, then its down rows
//     of layer s-1 as one contiguous block per (token, expert) -- a down row of the tiled
//     layout is one tile, so a CTA's rows of one expert are one copy (eight small copies per
//     row, one per expert, held the copy engine to a fraction of the SM's share of HBM);
//   * eight consumer warps take the units round-robin. A stage stages layer s's input as Q8_K
//     (C3) and runs the gate/up units; then each warp, for its down units, stages its expert's
//     SiLU products (three Q8_K blocks) itself and writes each row's dot to shared memory; at
//     the next stage's first CTA barrier one thread per output row adds the experts in the
//     reference's order;
//   * a sync warp waits for the CTA's gate/up units (an mbarrier), arrives at the grid counter
//     (release), polls it until every CTA has arrived (acquire), prefetches the layer's SiLU
//     products into L1 and signals the consumers (an mbarrier), so the grid round trip is off
//     the consumers' path.
//
// Every wait is bounded. A consumer whose wait runs out sets the error word and the counter's
// poison bit; the consumers agree on a failure at their next CTA barrier and stop, the
// producer stops issuing, waits (bounded) for every copy it issued, and the CTA leaves.
//
// Reference: core/arch/src/stream.rs expert_ffn_single 1186-1289 (gate/up, SiLU, down, the
// expert sum in chunks of ceil(K / workers)).
#include <cuda.h>
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "expert_stream.cuh"
#include "kernels.cuh"
#include "stage.cuh"

namespace bt {

namespace {

// NC consumer warps (4 with two CTAs per SM, or 8 with one), then the producer and the sync warp
constexpr int XS_MAX_CONSUMERS = 8;
template <int NC>
constexpr int xs_threads() { return (NC + 2) * 32; }
constexpr int XS_MAX_SLOTS = 32;
constexpr unsigned XS_POISON = 0x80000000u;

// The dots are inlined: the kernel's code fits the instruction cache, and a unit's two gate/up
// dots can then interleave.
__device__ __forceinline__ float xs_slot_dot(bool q4, const uint8_t *tile, int S, int s, const ActBlock *act) {
    return q4 ? q4k_dot_s(smem_u32(tile), S, s, smem_u32(act)) : q6k_dot_s(smem_u32(tile), S, s, smem_u32(act));
}

// named barrier 1 over the consumer warps, with an OR vote
template <int NC>
__device__ __forceinline__ bool consumers_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(NC * 32)
        : "memory");
    return r != 0;
}

// Q8_K staging (C3) of nblk 256-value blocks of x by the consumer warps: each warp's blocks are
// loaded before the first is quantised. The rows were written before an acquire that orders
// these loads (the sync warp's, through the ready mbarrier), or are read-only: plain loads, so
// the lines the sync warp prefetched into L1 serve them.
template <int NC>
__device__ void xs_stage(const float *x, int nblk, ActBlock *act, int warp, int lane) {
    constexpr int B = 3;
    for (int w0 = 0; w0 < nblk; w0 += B * NC) {
        float v[B][8];
#pragma unroll
        for (int i = 0; i < B; i++) {
            const int blk = w0 + warp + i * NC;
            if (blk < nblk) {
                const float4 *src = reinterpret_cast<const float4 *>(x + (long long)blk * 256 + lane * 8);
                const float4 a0 = src[0], a1 = src[1];
                v[i][0] = a0.x; v[i][1] = a0.y; v[i][2] = a0.z; v[i][3] = a0.w;
                v[i][4] = a1.x; v[i][5] = a1.y; v[i][6] = a1.z; v[i][7] = a1.w;
            }
        }
#pragma unroll
        for (int i = 0; i < B; i++) {
            const int blk = w0 + warp + i * NC;
            if (blk < nblk) quantize_block_warp(v[i], act + blk, lane);
        }
    }
}

// the same staging by one warp for nblk blocks, four at a time
__device__ __forceinline__ void xs_stage_warp(const float *x, int nblk, ActBlock *act, int lane) {
    for (int b0 = 0; b0 < nblk; b0 += 4) {
        float v[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (b0 + i < nblk) {
                const float4 *src = reinterpret_cast<const float4 *>(x + (b0 + i) * 256 + lane * 8);
                const float4 a0 = src[0], a1 = src[1];
                v[i][0] = a0.x; v[i][1] = a0.y; v[i][2] = a0.z; v[i][3] = a0.w;
                v[i][4] = a1.x; v[i][5] = a1.y; v[i][6] = a1.z; v[i][7] = a1.w;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (b0 + i < nblk) quantize_block_warp(v[i], act + b0 + i, lane);
    }
}

__device__ __forceinline__ void prefetch_l1(const void *p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// the bytes [0, n) at x into this SM's L1, one 128-byte line per lane and step
__device__ __forceinline__ void prefetch_lines_l1(const void *x, int n, int lane) {
    for (int o = lane * 128; o < n; o += 32 * 128) prefetch_l1(reinterpret_cast<const uint8_t *>(x) + o);
}

// bounded wait on a CTA mbarrier phase that also gives up when `stop` is set
__device__ __forceinline__ bool xs_wait_or_stop(uint64_t *bar, uint32_t par, const int *stop, int *err, long long lim) {
    if (mbar_try_wait(bar, par)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, par)) {
        if (*reinterpret_cast<const volatile int *>(stop)) return false;
        if (clock64() - t0 > lim) {
            atomicOr(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void xs_range(int total, int &u0, int &u1) {
    u0 = (int)((unsigned)blockIdx.x * (unsigned)total / gridDim.x);
    u1 = (int)((unsigned)(blockIdx.x + 1) * (unsigned)total / gridDim.x);
}

struct XsSmem {
    uint64_t *full, *empty;
    uint64_t *gu_done;  // the consumer warps' gate/up units of a stage are done (count NC)
    uint64_t *ready;    // the sync warp saw every CTA's gate/up of a layer (count 1)
    int *stop, *gfail;
    float *wts;   // [T][K] the route weights of the layer whose down rows run
    float *part;  // [K][XS_MAX_ROWS] each expert's value of the CTA's down rows
    ActBlock *act_in;  // [T][E / 256] the gate/up input
    ActBlock *act_dn;  // [XS_MAX_CONSUMERS][F / 256] each warp's expert's SiLU products
    uint8_t *ring;
};

constexpr int XS_MAX_ROWS = 128;  // down rows one CTA owns per layer: T * E / grid

__device__ __forceinline__ XsSmem xs_smem(uint8_t *smem, const ExpertStreamArgs &p) {
    XsSmem sm;
    sm.full = reinterpret_cast<uint64_t *>(smem);
    sm.empty = sm.full + XS_MAX_SLOTS;
    sm.gu_done = sm.empty + XS_MAX_SLOTS;
    sm.ready = sm.gu_done + 1;
    sm.stop = reinterpret_cast<int *>(sm.ready + 1);
    sm.gfail = sm.stop + 1;
    sm.wts = reinterpret_cast<float *>(smem + 1024);  // up to 64 values
    sm.part = reinterpret_cast<float *>(smem + 2048);
    sm.act_in = reinterpret_cast<ActBlock *>(smem + 2048 + MAX_K * XS_MAX_ROWS * 4);
    sm.act_dn = sm.act_in + p.T * (p.E / 256);
    sm.ring = reinterpret_cast<uint8_t *>(sm.act_dn + XS_MAX_CONSUMERS * (p.F / 256));
    return sm;
}

// The CTA's down rows [d0, d1) of T * E, cut at token boundaries and into pieces of at most
// maxr rows; piece q (0-based) -> token t, first row r0 (0..E-1), rows nr, offset of the piece's
// first row in [d0, d1). Returns the piece count when q is past the end.
__device__ __forceinline__ int xs_piece(int d0, int d1, int E, int maxr, int q, int &t, int &r0, int &nr, int &off) {
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

}  // namespace

template <int NC>
__global__ void __maxnreg__(168) expert_stream_kernel(const __grid_constant__ ExpertStreamArgs p) {
    constexpr int XS_CONSUMERS = NC, XS_PRODUCER = NC, XS_SYNC = NC + 1;
    extern __shared__ __align__(1024) uint8_t smem[];
    const XsSmem sm = xs_smem(smem, p);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = p.T, K = p.K, E = p.E, F = p.F, L = p.n_layer, nslot = p.nslot;
    if (tid < nslot) {
        mbar_init(sm.full + tid, 1);
        mbar_init(sm.empty + tid, 1);
    }
    if (tid == 0) {
        *sm.stop = 0;
        *sm.gfail = 0;
        mbar_init(sm.gu_done, XS_CONSUMERS);
        mbar_init(sm.ready, 1);
    }
    fence_mbar_init();
    __syncthreads();
    int d0, d1;
    xs_range(T * E, d0, d1);
    int t_, r_, n_, o_;
    const int nsbF = F / 256;

    if (warp == XS_PRODUCER) {
        // ---------------------------------------------------------------- producer
        // The whole warp walks the units: lane 0 waits for the slot and arms its barrier, then
        // issues the unit's copies (lanes 0 and 1 a gate/up tile pair, lane 0 a down block).
        // Descriptor fields and expert ids are held in registers: the copies' asm statements
        // clobber memory, so anything left in memory would be reloaded per unit.
        const uint64_t pol = l2_evict_first_policy();
        int slot = 0, round = 0, issued = 0;
        bool ok = true;
        for (int s = 0; s <= L && ok; s++) {
            for (int part = 0; part < 2 && ok; part++) {
                const int il = part == 0 ? s : s - 1;
                if (il < 0 || il >= L) continue;
                const LayerDev *Lp = p.layers + il;
                const int *sel = p.sel + il * T * K;
                int n_units, n_tiles = 0, u0 = 0, bytes_a, bytes_b = 0, maxr = 0;
                const uint8_t *wa;
                long long mat_a, mat_b = 0;
                if (part == 0) {
                    int u1;
                    n_tiles = Lp->gate.n_tiles;
                    xs_range(T * K * n_tiles, u0, u1);
                    n_units = u1 - u0;
                    wa = lane == 0 ? Lp->gate.w : Lp->up.w;
                    mat_a = lane == 0 ? Lp->gate.mat_bytes : Lp->up.mat_bytes;
                    bytes_a = lane == 0 ? Lp->gate.tile_bytes : Lp->up.tile_bytes;
                    bytes_b = Lp->gate.tile_bytes + Lp->up.tile_bytes;  // the unit's bytes
                    mat_b = lane == 0 ? 0 : Lp->gate.tile_bytes;        // this lane's offset in the slot
                } else {
                    wa = Lp->down.w;
                    mat_a = Lp->down.mat_bytes;
                    bytes_a = Lp->down.tile_bytes;  // one row
                    maxr = p.slot_bytes / bytes_a;
                    n_units = K * xs_piece(d0, d1, E, maxr, 1 << 30, t_, r_, n_, o_);
                }
                int cur = -1, eid = 0;
                for (int i = 0; i < n_units; i++) {
                    if (round > 0) {  // the consumers' release of this slot's previous unit
                        int okl = 1;
                        if (lane == 0) {
                            const uint32_t par = (uint32_t)((round - 1) & 1);
                            if (!mbar_try_wait(sm.empty + slot, par)) {
                                const long long t0 = clock64();
                                while (!mbar_try_wait(sm.empty + slot, par)) {
                                    if (*reinterpret_cast<volatile int *>(sm.stop)) {
                                        okl = 0;
                                        break;
                                    }
                                    if (clock64() - t0 > p.wait_limit) {
                                        atomicOr(p.err, ERR_WAIT_TIMEOUT);
                                        okl = 0;
                                        break;
                                    }
                                }
                            }
                        }
                        if (!__shfl_sync(FULL, okl, 0)) {
                            ok = false;
                            break;
                        }
                    }
                    uint8_t *dst = sm.ring + slot * p.slot_bytes;
                    if (part == 0) {
                        const int u = u0 + i;
                        const int tk = u / n_tiles, tile = u - tk * n_tiles;
                        if (tk != cur) {
                            cur = tk;
                            eid = sel[tk];
                        }
                        if (lane == 0) mbar_arrive_expect_tx(sm.full + slot, bytes_b);
                        __syncwarp();
                        if (lane < 2)
                            bulk_g2s_hint(dst + mat_b, wa + eid * mat_a + (long long)tile * bytes_a, bytes_a,
                                          sm.full + slot, pol);
                    } else {
                        const int q = i / K, k = i - q * K;
                        xs_piece(d0, d1, E, maxr, q, t_, r_, n_, o_);
                        if (lane == 0) {
                            const int e = sel[t_ * K + k];
                            mbar_arrive_expect_tx(sm.full + slot, n_ * bytes_a);
                            bulk_g2s_hint(dst, wa + e * mat_a + (long long)r_ * bytes_a, n_ * bytes_a, sm.full + slot,
                                          pol);
                        }
                    }
                    __syncwarp();
                    issued++;
                    if (++slot == nslot) {
                        slot = 0;
                        round++;
                    }
                }
            }
        }
        // every copy issued must land before the CTA leaves: the last round of each slot
        if (lane == 0) {
            const int last = issued < nslot ? issued : nslot;
            for (int q = issued - last; q < issued; q++)
                mbar_wait_l(sm.full + q % nslot, (uint32_t)((q / nslot) & 1), p.err, p.wait_limit);
        }
        return;
    }

    if (warp == XS_SYNC) {
        // ---------------------------------------------------------------- sync warp
        // Per layer s: wait for this CTA's gate/up units (gu_done), arrive at the grid counter
        // (release: the consumers' SiLU products, ordered before it by their mbarrier arrivals),
        // poll it until every CTA has arrived (acquire), prefetch layer s's products into L1
        // and tell the consumers (ready). Layer s+1's gate/up input (read-only) is prefetched
        // first.
        for (int s = 0; s < L; s++) {
            if (s + 1 < L) prefetch_lines_l1(p.xin + (long long)(s + 1) * p.xin_stride, T * E * 4, lane);
            int okl = 1;
            if (lane == 0) {
                if (!xs_wait_or_stop(sm.gu_done, (uint32_t)(s & 1), sm.stop, p.err, p.wait_limit)) {
                    okl = 0;
                } else {
                    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p.bar), "r"(1u) : "memory");
                    const unsigned target = (unsigned)(s + 1) * gridDim.x;
                    unsigned v;
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
                    const long long t0 = clock64();
                    while (v < target) {
                        if (clock64() - t0 > p.wait_limit) {
                            atomicOr(p.err, ERR_WAIT_TIMEOUT);
                            atomicOr(p.bar, XS_POISON);
                            v = XS_POISON;
                            break;
                        }
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
                    }
                    okl = v < XS_POISON;
                }
            }
            okl = __shfl_sync(FULL, okl, 0);
            if (okl) prefetch_lines_l1(p.act + (long long)s * T * K * F, T * K * F * 4, lane);
            __syncwarp();
            if (lane == 0) {
                if (!okl) *reinterpret_cast<volatile int *>(sm.gfail) = 1;
                mbar_arrive(sm.ready);
            }
            if (!okl) break;
        }
        return;
    }

    // -------------------------------------------------------------------- consumers
    bool bad = false;
    int j = warp;   // this warp's next unit (CTA-wide unit index)
    int base = 0;   // first unit index of the current part
    const int workers = p.workers < 1 ? 1 : (p.workers < K ? p.workers : K);
    const int wchunk = (K + workers - 1) / workers;
    // the expert sum of layer il's down rows (part[] written by its down units): one thread per
    // row, the reference's order (expert_ffn_single: chunks of ceil(K / workers) summed, partials
    // added to a zero vector), then the (zero) residual
    auto finish_down = [&](int il) {
        for (int r = tid; r < d1 - d0; r += XS_CONSUMERS * 32) {
            const int u = d0 + r, t = u / E;
            const float *w = sm.wts + t * K;
            float sum = 0.0f;
            for (int s0 = 0; s0 < K; s0 += wchunk) {
                float tot = __fmul_rn(sm.part[s0 * XS_MAX_ROWS + r], w[s0]);
                for (int q = s0 + 1; q < K && q < s0 + wchunk; q++)
                    tot = __fadd_rn(tot, __fmul_rn(sm.part[q * XS_MAX_ROWS + r], w[q]));
                sum = workers <= 1 ? tot : __fadd_rn(sum, tot);
            }
            p.out[(long long)il * T * E + u] = __fadd_rn(0.0f, sum);
        }
    };
    bool completed = false;
    for (int s = 0; s <= L; s++) {
        // every warp is done with the previous stage: its down values are complete, the input
        // buffer is free
        if (consumers_sync_or<NC>(bad)) break;
        if (s >= 2) finish_down(s - 2);
        // ---- gate/up of layer s
        if (s < L) {
            const LayerDev &Ld = p.layers[s];
            const int nsb = Ld.gate.nsb, gS = Ld.gate.S, grpt = Ld.gate.rpt, gnt = Ld.gate.n_tiles;
            const bool gq4 = Ld.gate.type == T_Q4_K, uq4 = Ld.up.type == T_Q4_K;
            const int gtb = Ld.gate.tile_bytes;
            int u0, u1;
            xs_range(T * K * gnt, u0, u1);
            xs_stage<NC>(p.xin + (long long)s * p.xin_stride, T * (E / 256), sm.act_in, warp, lane);
            if (consumers_sync_or<NC>(false)) break;
            float *act = p.act + (long long)s * T * K * F;
            for (; j < base + (u1 - u0); j += XS_CONSUMERS) {
                const int slot = j % nslot;
                if (!__all_sync(FULL, mbar_wait_l(sm.full + slot, (uint32_t)((j / nslot) & 1), p.err, p.wait_limit))) {
                    bad = true;
                    break;
                }
                const int u = u0 + (j - base);
                const int tk = u / gnt, tile = u - tk * gnt;
                const int t = tk / K;
                const uint8_t *gt = sm.ring + (size_t)slot * p.slot_bytes, *ut = gt + gtb;
                const bool active = lane < gS;
                const int rit = active ? lane / nsb : 0, b = active ? lane - rit * nsb : 0;
                const int row = tile * grpt + rit;
                float vg = 0.0f, vu = 0.0f;
                if (active) {
                    const ActBlock *ab = sm.act_in + t * (E / 256) + b;
                    vg = xs_slot_dot(gq4, gt, gS, lane, ab);
                    vu = xs_slot_dot(uq4, ut, gS, lane, ab);
                }
                float rg = 0.0f, ru = 0.0f;
                for (int b2 = 0; b2 < nsb; b2++) {
                    const int srcl = rit * nsb + b2 < 32 ? rit * nsb + b2 : 31;
                    rg = __fadd_rn(rg, __shfl_sync(FULL, vg, srcl));
                    ru = __fadd_rn(ru, __shfl_sync(FULL, vu, srcl));
                }
                if (active && b == 0 && row < F) act[(long long)tk * F + row] = __fmul_rn(bt_silu(rg), ru);
                __syncwarp();
                if (lane == 0) mbar_arrive(sm.empty + slot);
            }
            if (bad) j = base + (u1 - u0);  // (the vote before the down units ends the loop)
            __syncwarp();  // the warp's SiLU products, before lane 0's release-arrival
            if (lane == 0) mbar_arrive(sm.gu_done);
            base += u1 - u0;
            while (j < base) j += XS_CONSUMERS;
        }
        // ---- down of layer s - 1: units (piece, expert)
        if (s >= 1) {
            const int il = s - 1;
            const LayerDev &Ld = p.layers[il];
            const int dtb = Ld.down.tile_bytes;
            const bool dq4 = Ld.down.type == T_Q4_K;
            const int maxr = p.slot_bytes / dtb;
            const int n_units = K * xs_piece(d0, d1, E, maxr, 1 << 30, t_, r_, n_, o_);
            // every CTA's gate/up of layer il, seen by the sync warp (normally a stage ago)
            bool gbad = !mbar_wait_l(sm.ready, (uint32_t)(il & 1), p.err, p.wait_limit);
            gbad |= *reinterpret_cast<volatile int *>(sm.gfail) != 0;
            if (tid < T * K) sm.wts[tid] = __ldg(p.wts + il * T * K + tid);
            if (consumers_sync_or<NC>(gbad || bad)) break;
            const float *acts = p.act + (long long)il * T * K * F;
            ActBlock *mine = sm.act_dn + warp * nsbF;
            int staged = -1;  // (token, expert) whose products are in `mine`
            for (; j < base + n_units; j += XS_CONSUMERS) {
                const int i = j - base, q = i / K, k = i - q * K;
                int t, r0, nr, off;
                xs_piece(d0, d1, E, maxr, q, t, r0, nr, off);
                if (t * K + k != staged) {  // this expert's SiLU products as Q8_K (C3), by this warp
                    staged = t * K + k;
                    __syncwarp();
                    xs_stage_warp(acts + (long long)staged * F, nsbF, mine, lane);
                    __syncwarp();
                }
                const int slot = j % nslot;
                if (!__all_sync(FULL, mbar_wait_l(sm.full + slot, (uint32_t)((j / nslot) & 1), p.err, p.wait_limit))) {
                    bad = true;
                    break;
                }
                const uint8_t *tb = sm.ring + (size_t)slot * p.slot_bytes;
                const int rpp = 32 / nsbF;  // rows per pass of the warp
                for (int rb = 0; rb < nr; rb += rpp) {
                    const int ri = lane / nsbF, b = lane - ri * nsbF, r = rb + ri;
                    const bool valid = ri < rpp && r < nr;
                    float v = 0.0f;
                    if (valid) v = xs_slot_dot(dq4, tb + r * dtb, nsbF, b, mine + b);
                    float acc = 0.0f;
                    for (int b2 = 0; b2 < nsbF; b2++) {
                        const int srcl = ri * nsbF + b2;
                        acc = __fadd_rn(acc, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
                    }
                    if (valid && b == 0) sm.part[k * XS_MAX_ROWS + off + r] = acc;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(sm.empty + slot);
            }
            if (bad) j = base + n_units;
            base += n_units;
            while (j < base) j += XS_CONSUMERS;
        }
        completed = s == L;
    }
    // the last layer's expert sums, unless a failure ended the loop (every thread leaves the
    // loop at the same vote, so `completed` is uniform)
    if (completed) {
        if (consumers_sync_or<NC>(bad)) bad = true;
        else finish_down(L - 1);
    }
    // a failure, or the end: tell the producer and the sync warp to stop waiting
    if (bad) atomicOr(p.bar, XS_POISON);
    if (tid == 0) atomicExch(sm.stop, 1);
}

size_t expert_stream_fixed_smem(int T, int E, int K, int F) {
    (void)K;
    return 2048 + (size_t)MAX_K * XS_MAX_ROWS * 4 + (size_t)(T * (E / 256) + XS_MAX_CONSUMERS * (F / 256)) * sizeof(ActBlock);
}

int expert_stream_max_rows() { return XS_MAX_ROWS; }

static size_t xs_smem_bytes(const ExpertStreamArgs &a) {
    return expert_stream_fixed_smem(a.T, a.E, a.K, a.F) + (size_t)a.nslot * a.slot_bytes;
}

template <int NC>
static cudaError_t xs_prepare(const ExpertStreamArgs &a, int *blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(expert_stream_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)xs_smem_bytes(a));
    if (e) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, expert_stream_kernel<NC>, xs_threads<NC>(),
                                                         xs_smem_bytes(a));
}

cudaError_t prepare_expert_stream(const ExpertStreamArgs &a, int *blocks_per_sm) {
    if (a.nslot < 1 || a.nslot > XS_MAX_SLOTS || a.slot_bytes % 16) return cudaErrorInvalidValue;
    if (a.consumers == 4) return xs_prepare<4>(a, blocks_per_sm);
    if (a.consumers == 8) return xs_prepare<8>(a, blocks_per_sm);
    return cudaErrorInvalidValue;
}

int expert_stream_regs() {
    cudaFuncAttributes fa;
    return cudaFuncGetAttributes(&fa, expert_stream_kernel<8>) == cudaSuccess ? fa.numRegs : -1;
}

template <int NC>
static cudaError_t xs_launch(const ExpertStreamArgs &a, int grid, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(xs_threads<NC>());
    cfg.dynamicSmemBytes = xs_smem_bytes(a);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, expert_stream_kernel<NC>, a);
}

cudaError_t launch_expert_stream(const ExpertStreamArgs &a, int grid, cudaStream_t st) {
    if (a.nslot < 1 || a.nslot > XS_MAX_SLOTS || a.slot_bytes % 16) return cudaErrorInvalidValue;
    if (a.consumers == 4) return xs_launch<4>(a, grid, st);
    if (a.consumers == 8) return xs_launch<8>(a, grid, st);
    return cudaErrorInvalidValue;
}

int expert_stream_max_slots() { return XS_MAX_SLOTS; }

}  // namespace bt
