// kernels.cu -- the sm_100a kernels of the decode-step layer.
//
// Reference call sites each kernel replaces (Chaos tree, core/arch/src/stream.rs unless noted):
//   embed_kernel      get_rows on token_embd                           2192-2231
//   kq_rows_kernel    rms_norm+mul then mul_mat (q/k/v, attn_output, output head)
//                                                                      2265-2330, 2669, 2853-2914
//   qkv_post_kernel   q/k head RMSNorm, rope_ext NEOX, KvCache::push  2390-2474, 2545-2552; kv.rs:171-205
//   attn_kernel       flash_attn_ext over the cached history          2554-2703; qwen3.rs:1186-1227
//   router_kernel     ffn_norm, ffn_gate_inp mul_mat, soft_max_ext, route()
//                                                                      2784-2831, 869-888
//   gateup_kernel     per-expert gate/up mul_mat, silu, mul           1168-1172
//   down_kernel       per-expert down mul_mat, scale, the expert sum and the residual add
//                                                                      1173-1176, 1278-1284, 1051-1058, 2841-2843
//   step_end_kernel   argmax (core/arch/src/sample.rs:928-935), KvCache::advance_by (kv.rs:211-213)
#include <cuda.h>
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "kernels.cuh"
#include "stage.cuh"

namespace bt {

// ====================================================================== layout / synthesis
// One thread per (tile-slot, chunk): moves 16 bytes (and the Q6_K d) from GGUF row-major
// bytes into the tiled layout. Rows past the matrix end are zero-filled.
__global__ void repack_kernel(int type, const uint8_t *__restrict__ src, long long rows, long long cols, int rpt,
                              uint8_t *__restrict__ dst, long long n_mats) {
    TileGeom g = tile_geom(type, rows, cols, rpt);
    const int bb = qk_block_bytes(type), nch = qk_chunks(type);
    const long long row_bytes = (long long)g.nsb * bb;
    const long long per_mat_units = g.n_tiles * g.S * (nch + 1);
    const long long total = per_mat_units * n_mats;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long mat = i / per_mat_units, r = i % per_mat_units;
        long long tile = r / ((long long)g.S * (nch + 1));
        int rem = (int)(r % ((long long)g.S * (nch + 1)));
        int c = rem / g.S, s = rem % g.S;
        long long row = tile * rpt + s / g.nsb;
        int b = s % g.nsb;
        const uint8_t *blk = src + mat * rows * row_bytes + row * row_bytes + (long long)b * bb;
        uint8_t *tb = dst + (mat * g.n_tiles + tile) * (long long)g.tile_bytes;
        bool ok = row < rows;
        if (c < nch) {
            uint8_t *d = tb + (long long)c * g.S * 16 + s * 16;
            if (type == T_Q4_K) {
                uint4 v = ok ? *reinterpret_cast<const uint4 *>(blk + c * 16) : make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4 *>(d) = v;
            } else {
                for (int k = 0; k < 16; k++) d[k] = ok ? blk[c * 16 + k] : 0;
            }
        } else if (type == T_Q6_K) {
            uint8_t *d = tb + 13 * g.S * 16 + s * 2;
            d[0] = ok ? blk[208] : 0;
            d[1] = ok ? blk[209] : 0;
        }
    }
}

// Values of the tiled layout back to row-major floats (C2), one thread per superblock.
__global__ void dequant_tiled_kernel(int type, const uint8_t *__restrict__ tiled, long long rows, long long cols,
                                     int rpt, float *__restrict__ out) {
    TileGeom g = tile_geom(type, rows, cols, rpt);
    long long nsbt = rows * g.nsb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nsbt;
         i += (long long)gridDim.x * blockDim.x) {
        long long row = i / g.nsb;
        int b = (int)(i % g.nsb);
        long long tile = row / rpt;
        int s = (int)(row % rpt) * g.nsb + b;
        const uint8_t *tb = tiled + tile * g.tile_bytes;
        uint8_t blk[210];
        for (int c = 0; c < qk_chunks(type); c++)
            for (int k = 0; k < 16; k++) blk[c * 16 + k] = tb[(long long)c * g.S * 16 + s * 16 + k];
        float *y = out + row * cols + (long long)b * 256;
        if (type == T_Q4_K) {
            float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t *sc = blk + 4, *qs = blk + 16;
            for (int j = 0; j < 8; j++) {
                int scj, mj;
                if (j < 4) {
                    scj = sc[j] & 63;
                    mj = sc[j + 4] & 63;
                } else {
                    scj = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                    mj = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
                }
                float d1 = __fmul_rn(d, (float)scj), m1 = __fmul_rn(dmin, (float)mj);
                int gidx = j / 2, hi = j & 1;
                for (int l = 0; l < 32; l++) {
                    int q = hi ? (qs[32 * gidx + l] >> 4) : (qs[32 * gidx + l] & 0xF);
                    y[64 * gidx + 32 * hi + l] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
                }
            }
        } else {
            blk[208] = tb[13 * g.S * 16 + s * 2];
            blk[209] = tb[13 * g.S * 16 + s * 2 + 1];
            float d = f16_bits_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
            const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
            for (int v = 0; v < 256; v++) {
                int n = v / 128, r = v % 128, quad = r / 32, l = r % 32;
                int lo = quad == 0 ? (blk[64 * n + l] & 0xF)
                                   : quad == 1 ? (blk[64 * n + 32 + l] & 0xF)
                                               : quad == 2 ? (blk[64 * n + l] >> 4) : (blk[64 * n + 32 + l] >> 4);
                int hi = (blk[128 + 32 * n + l] >> (2 * quad)) & 3;
                int q = (lo | (hi << 4)) - 32;
                y[v] = __fmul_rn(__fmul_rn(d, (float)sc[v / 16]), (float)q);
            }
        }
    }
}

__global__ void synth_kernel(int type, uint64_t key, long long n_elems, float mean, float scale,
                             uint8_t *__restrict__ out) {
    const int bb = synth_block_bytes(type);
    const int eb = type == T_F32 ? 4 : (type == T_F16 ? 2 : 0);  // bytes per element of float types
    const long long n_blocks = (n_elems + 255) / 256;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_blocks;
         i += (long long)gridDim.x * blockDim.x) {
        uint8_t blk[1024];
        synth_block(type, key, (uint64_t)i * 256u, mean, scale, blk);
        long long left = n_elems - i * 256;
        int nb = (eb && left < 256) ? (int)left * eb : bb;
        uint8_t *dst = out + (eb ? i * 256 * eb : i * bb);
        for (int k = 0; k < nb; k++) dst[k] = blk[k];
    }
}

// ====================================================================== L2 prefetch of upcoming inputs
// Pieces of 64 KB go round-robin over the CTAs first (then over a CTA's threads), so every
// SM's TMA unit carries a share of the traffic.
constexpr unsigned long long PREFETCH_PIECE = 64ull << 10;

__device__ __forceinline__ bool prefetch_owner(unsigned long long k) {
    return (int)(k % gridDim.x) == (int)blockIdx.x && (int)((k / gridDim.x) % blockDim.x) == (int)threadIdx.x;
}

__device__ void prefetch_ranges_spread(const void *const *ptrs, const unsigned long long *bytes, int n,
                                       unsigned long long &k) {
    for (int i = 0; i < n; i++) {
        const char *c = reinterpret_cast<const char *>(ptrs[i]);
        const unsigned long long np = (bytes[i] + PREFETCH_PIECE - 1) / PREFETCH_PIECE;
        for (unsigned long long q = 0; q < np; q++, k++) {
            if (!prefetch_owner(k)) continue;
            const unsigned long long off = q * PREFETCH_PIECE;
            const unsigned long long len = bytes[i] - off < PREFETCH_PIECE ? bytes[i] - off : PREFETCH_PIECE;
            prefetch_l2(c + off, (uint32_t)(len & ~15ull));
        }
    }
}

__device__ void run_prefetch(const PrefetchSpec &pf) {
    unsigned long long k = 0;
    prefetch_ranges_spread(pf.ptr, pf.bytes, pf.n, k);
    if (pf.kv) {
        const unsigned long long page = 2ull * pf.HK * 16 * pf.D * 2;  // K and V of one page, contiguous
        for (int t = 0; t < pf.T; t++) {
            const int np = pf.pos_of[t] / 16 + 1;
            const int seq = pf.seq_of[t];
            for (int pg = 0; pg < np; pg++, k++) {
                if (!prefetch_owner(k)) continue;
                const int blk = pf.block_table[seq * pf.max_blocks + pg];
                const unsigned long long row = (((unsigned long long)pf.layer * pf.n_blocks + blk) * 2) * pf.HK * 16;
                prefetch_l2(pf.kv + row * pf.D, (uint32_t)page);
            }
        }
    }
}

// ====================================================================== GEMV
// Per-warp scratch of the row reductions (RED_STRIDE, RED_WARP_FLOATS in kernels.cuh): 8 tokens
// x 32 lanes, rows padded to 33 floats so that the lanes reading one superblock index of
// different tokens hit different banks.
// Persistent-style: the grid covers the SMs; CTA c owns a contiguous range of tiles; each
// warp streams its tiles through a private ring of `nst` shared-memory slots with 1-D TMA
// bulk copies (weights do not depend on the previous kernel, so the first slots are
// requested before griddepcontrol.wait), and lane s decodes slot s in registers.
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) kq_rows_kernel(const __grid_constant__ GemvArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *normS = reinterpret_cast<float *>(smem + 512);
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsbK = p.K / 256;
    const int stage_cap = p.tgrp ? p.stage_max : p.T;
    const size_t act_bytes = (size_t)stage_cap * nsbK * sizeof(ActBlock);
    uint8_t *ring = smem + 1024 + ((act_bytes + 127) & ~(size_t)127);
    uint8_t *myring = ring + (size_t)warp * p.nst * p.slot_bytes;
    uint64_t *mybar = bars + warp * p.nst;
    float *red = reinterpret_cast<float *>(ring + (size_t)NWARP * p.nst * p.slot_bytes) + warp * RED_WARP_FLOATS;

    // units: tiles, or (token group, tile) group-major
    const int tg = p.tgrp ? p.tgrp : (p.T > 0 ? p.T : 1);
    const long long n_units = (long long)p.total_tiles * ((p.T + tg - 1) / tg);
    const long long u0 = (long long)blockIdx.x * n_units / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * n_units / gridDim.x;
    const int nmine = (u1 - u0 > warp) ? (int)((u1 - u0 - warp + NWARP - 1) / NWARP) : 0;
    // the tokens this CTA stages: [tA, tB), the groups of units u0 .. u1-1
    const int tA = u1 > u0 ? (int)(u0 / p.total_tiles) * tg : 0;
    const int tB = u1 > u0 ? min(p.T, (int)((u1 - 1) / p.total_tiles + 1) * tg) : 0;
    if (tB - tA > stage_cap) {  // the host sized stage_max too small: nothing is computed
        if (threadIdx.x == 0) atomicOr(p.err, ERR_BAD_INDEX);
        return;
    }

    auto seg_of = [&](long long u) -> int {
        int si = 0;
        if (p.nseg > 1 && u >= p.seg[1].tile0) si = 1;
        if (p.nseg > 2 && u >= p.seg[2].tile0) si = 2;
        return si;
    };
    auto issue = [&](int j) {
        const long long u = (u0 + warp + (long long)j * NWARP) % p.total_tiles;
        const GemvSeg &sg = p.seg[seg_of(u)];
        const uint8_t *src = sg.w + (u - sg.tile0) * (long long)sg.tile_bytes;
        int slot = j % p.nst;
        mbar_arrive_expect_tx(&mybar[slot], sg.tile_bytes);
        bulk_g2s(myring + (size_t)slot * p.slot_bytes, src, sg.tile_bytes, &mybar[slot]);
    };

    if (lane == 0) {
        for (int i = 0; i < p.nst; i++) mbar_init(&mybar[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (lane == 0)
        for (int i = 0; i < p.nst && i < nmine; i++) issue(i);

    pdl_wait();
    run_prefetch(p.pf);
    stage_activations<NWARP>(p.x_rows ? p.x : p.x + (long long)tA * p.x_stride, p.x_stride,
                             p.x_rows ? p.x_rows + tA : nullptr, p.norm_w, p.eps, p.K, tB - tA, act, normS);
    __syncthreads();
    pdl_trigger();

    unsigned long long best[MAX_T];
#pragma unroll
    for (int t = 0; t < MAX_T; t++) best[t] = 0ull;
    int j = 0;
    for (; j < nmine; j++) {
        const int slot = j % p.nst;
        if (!__all_sync(FULL, mbar_wait(&mybar[slot], (j / p.nst) & 1, p.err))) break;
        const long long ug = u0 + warp + (long long)j * NWARP;
        const long long u = ug % p.total_tiles;
        // the unit's tokens [ta, te), staged from token tA on
        const int ta = (int)(ug / p.total_tiles) * tg, te = min(p.T, ta + tg);
        const GemvSeg &sg = p.seg[seg_of(u)];
        const uint8_t *tile = myring + (size_t)slot * p.slot_bytes;
        const long long tl = u - sg.tile0;
        const bool active = lane < sg.S;
        const int b = active ? lane % sg.nsb : 0;
        // lane's superblock decoded into registers once; its dots with the tokens' activation
        // blocks two at a time (independent chains)
        const uint32_t tile_s = smem_u32(tile), act_b = smem_u32(&act[b]);
        const uint32_t tok_stride = (uint32_t)(nsbK * sizeof(ActBlock));
        const int ls = active ? lane : 0;
        // 8 tokens at a time: every lane's superblock partial to shared memory, then one lane
        // per (row, token) adds the row's nsb partials in superblock order (C4)
        auto run_tokens = [&](auto &&dot) {
        for (int t0 = ta; t0 < te; t0 += 8) {
            const int tn = te - t0 < 8 ? te - t0 : 8;
            for (int i = 0; i < tn; i += 2) {
                const int i1 = i + 1 < tn ? i + 1 : i;
                const float v0 = dot(act_b + (uint32_t)(t0 - tA + i) * tok_stride);
                const float v1 = dot(act_b + (uint32_t)(t0 - tA + i1) * tok_stride);
                red[i * RED_STRIDE + lane] = active ? v0 : 0.0f;
                if (i + 1 < tn) red[(i + 1) * RED_STRIDE + lane] = active ? v1 : 0.0f;
            }
            __syncwarp();
            for (int q = lane; q < sg.rpt * 8; q += 32) {
                const int rr = q >> 3, i = q & 7;
                const long long rrow = tl * sg.rpt + rr;
                if (i < tn && rrow < sg.rows) {
                    const float *rv = red + i * RED_STRIDE + rr * sg.nsb;
                    float acc = 0.0f;
                    for (int b2 = 0; b2 < sg.nsb; b2++) acc = __fadd_rn(acc, rv[b2]);
                    const int t = t0 + i;
                    float r = acc;
                    if (p.res) r = __fadd_rn(p.res[t * p.res_stride + sg.out_off + rrow], acc);
                    p.y[t * p.y_stride + sg.out_off + rrow] = r;
                    if (p.amax) {
                        unsigned long long key = ((unsigned long long)((unsigned)total_key(r) ^ 0x80000000u) << 32) |
                                                 (unsigned)(sg.out_off + rrow);
#pragma unroll
                        for (int tt = 0; tt < MAX_T; tt++)
                            if (tt == t && key > best[tt]) best[tt] = key;
                    }
                }
            }
            __syncwarp();
        }
        };
        if (sg.type == T_Q4_K) {
            Q4Reg w;
            q4k_load_r(w, tile_s, sg.S, ls);
            run_tokens([&](uint32_t a) { return q4k_dot_r(w, a); });
        } else {
            Q6Reg w;
            q6k_load_r(w, tile_s, sg.S, ls);
            run_tokens([&](uint32_t a) { return q6k_dot_r(w, a); });
        }
        __syncwarp();
        if (lane == 0 && j + p.nst < nmine) {
            fence_proxy_async();
            issue(j + p.nst);
        }
    }
    if (j < nmine) {  // a wait ran out: let any copy still in flight land (bounded) before exiting
        for (int k = j; k < nmine && k < j + p.nst; k++) mbar_wait(&mybar[k % p.nst], (k / p.nst) & 1, nullptr);
    }
    if (p.amax) {  // argmax of the rows this CTA wrote: one 64-bit atomicMax per token
        __shared__ unsigned long long s_best[MAX_T][NWARP];
        for (int t = 0; t < p.T; t++) {
            unsigned long long b = best[0];
#pragma unroll
            for (int tt = 1; tt < MAX_T; tt++)
                if (tt == t) b = best[tt];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                unsigned long long ob = __shfl_xor_sync(FULL, b, o);
                b = ob > b ? ob : b;
            }
            if (lane == 0) s_best[t][warp] = b;
        }
        __syncthreads();
        if (threadIdx.x < p.T) {
            unsigned long long b = 0;
            for (int w = 0; w < NWARP; w++) b = s_best[threadIdx.x][w] > b ? s_best[threadIdx.x][w] : b;
            atomicMax(p.amax + threadIdx.x, b);
        }
    }
}

size_t gemv_smem_bytes(const GemvArgs &a) {
    size_t act = (size_t)(a.tgrp ? a.stage_max : a.T) * (a.K / 256) * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes +
           (size_t)GEMV_WARPS * RED_WARP_FLOATS * 4;
}

template <typename Kern, typename Arg>
static cudaError_t launch_ex(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, const Arg &a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, a);
}

cudaError_t launch_gemv(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    size_t smem = gemv_smem_bytes(a);
    return launch_ex(kq_rows_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), smem, st, pdl, a);
}

// ====================================================================== experts
// gate/up: unit = (token t, expert slot k, tile) -> the tile of gate_e and of up_e for the
// same rows, two bulk copies into one ring slot; output act = silu(gate) * up (C7).
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) gateup_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsb = p.g_nsb;
    const size_t act_bytes = (size_t)p.T * nsb * sizeof(ActBlock);
    uint8_t *ring = smem + 1024 + ((act_bytes + 127) & ~(size_t)127);
    uint8_t *myring = ring + (size_t)warp * p.nst * p.slot_bytes;
    uint64_t *mybar = bars + warp * p.nst;

    const long long total = (long long)p.T * p.K * p.g_n_tiles;
    const long long u0 = (long long)blockIdx.x * total / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * total / gridDim.x;
    const int nmine = (u1 - u0 > warp) ? (int)((u1 - u0 - warp + NWARP - 1) / NWARP) : 0;

    if (lane == 0) {
        for (int i = 0; i < p.nst; i++) mbar_init(&mybar[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_wait();  // expert ids come from the router
    run_prefetch(p.pf);
    if (p.prefetch_down) {  // the down weights of the selected experts, for the next kernel
        unsigned long long k = 1ull << 40;  // a fresh round-robin start
        for (int q = 0; q < p.T * p.K; q++) {
            const void *ptr = expert_down(p, p.sel_ids[q]);
            const unsigned long long nb = (unsigned long long)p.d_expert_bytes;
            prefetch_ranges_spread(&ptr, &nb, 1, k);
        }
    }

    auto issue = [&](int j) {
        long long u = u0 + warp + (long long)j * NWARP;
        int tile = (int)(u % p.g_n_tiles);
        long long tk = u / p.g_n_tiles;
        int e = p.sel_ids[tk];
        int slot = j % p.nst;
        uint8_t *dst = myring + (size_t)slot * p.slot_bytes;
        mbar_arrive_expect_tx(&mybar[slot], p.g_tile_bytes + p.u_tile_bytes);
        bulk_g2s(dst, expert_gate(p, e) + (long long)tile * p.g_tile_bytes, p.g_tile_bytes, &mybar[slot]);
        bulk_g2s(dst + p.g_tile_bytes, expert_up(p, e) + (long long)tile * p.u_tile_bytes, p.u_tile_bytes,
                 &mybar[slot]);
    };
    if (lane == 0)
        for (int i = 0; i < p.nst && i < nmine; i++) issue(i);

    stage_activations<NWARP>(p.fn, p.E, nullptr, nullptr, 0.0f, p.E, p.T, act, nullptr);
    __syncthreads();
    pdl_trigger();

    int j = 0;
    for (; j < nmine; j++) {
        const int slot = j % p.nst;
        if (!__all_sync(FULL, mbar_wait(&mybar[slot], (j / p.nst) & 1, p.err))) break;
        const long long u = u0 + warp + (long long)j * NWARP;
        const int tile = (int)(u % p.g_n_tiles);
        const long long tk = u / p.g_n_tiles;
        const int t = (int)(tk / p.K);
        const uint8_t *gt = myring + (size_t)slot * p.slot_bytes;
        const uint8_t *ut = gt + p.g_tile_bytes;
        const bool active = lane < p.g_S;
        const int rit = active ? lane / nsb : 0, b = active ? lane % nsb : 0;
        const int row = tile * p.g_rpt + rit;
        float rowv[2];
#pragma unroll 1
        for (int which = 0; which < 2; which++) {  // gate, then up: one copy of the dot code
            const uint8_t *tl = which ? ut : gt;
            const int ty = which ? p.utype : p.gtype;
            float v = 0.0f;
            if (active) {
                const ActBlock &ab = act[t * nsb + b];
                v = ty == T_Q4_K ? q4k_slot_dot(tl, p.g_S, lane, ab) : q6k_slot_dot(tl, p.g_S, lane, ab);
            }
            float r = 0.0f;
            for (int b2 = 0; b2 < nsb; b2++) {
                int srcl = rit * nsb + b2;
                r = __fadd_rn(r, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
            }
            rowv[which] = r;
        }
        const float ag = rowv[0], au = rowv[1];
        if (active && b == 0 && row < p.F) p.act[tk * p.F + row] = __fmul_rn(bt_silu(ag), au);
        __syncwarp();
        if (lane == 0 && j + p.nst < nmine) {
            fence_proxy_async();
            issue(j + p.nst);
        }
    }
    if (j < nmine)
        for (int k = j; k < nmine && k < j + p.nst; k++) mbar_wait(&mybar[k % p.nst], (k / p.nst) & 1, nullptr);
}

// down: unit = (token t, output row) over all K selected experts (one row tile of each);
// the K row values are scaled and summed in the reference's order, then the residual.
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) down_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *wvals = reinterpret_cast<float *>(smem + 512);  // [NWARP][MAX_K]
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsb = p.d_nsb;
    const size_t act_bytes = (size_t)p.T * p.K * nsb * sizeof(ActBlock);
    uint8_t *ring = smem + 1024 + ((act_bytes + 127) & ~(size_t)127);
    uint8_t *myring = ring + (size_t)warp * p.nst * p.slot_bytes;
    uint64_t *mybar = bars + warp * p.nst;

    const long long total = (long long)p.T * p.E;
    const long long u0 = (long long)blockIdx.x * total / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * total / gridDim.x;
    const int nmine = (u1 - u0 > warp) ? (int)((u1 - u0 - warp + NWARP - 1) / NWARP) : 0;

    if (lane == 0) {
        for (int i = 0; i < p.nst; i++) mbar_init(&mybar[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_wait();
    run_prefetch(p.pf);

    auto issue = [&](int j) {
        long long u = u0 + warp + (long long)j * NWARP;
        int row = (int)(u % p.E), t = (int)(u / p.E);
        int slot = j % p.nst;
        uint8_t *dst = myring + (size_t)slot * p.slot_bytes;
        mbar_arrive_expect_tx(&mybar[slot], p.K * p.d_tile_bytes);
        for (int k = 0; k < p.K; k++) {
            int e = p.sel_ids[t * p.K + k];
            bulk_g2s(dst + k * p.d_tile_bytes, expert_down(p, e) + (long long)row * p.d_tile_bytes,
                     p.d_tile_bytes, &mybar[slot]);
        }
    };
    if (lane == 0)
        for (int i = 0; i < p.nst && i < nmine; i++) issue(i);

    stage_activations<NWARP>(p.act, p.F, nullptr, nullptr, 0.0f, p.F, p.T * p.K, act, nullptr);
    __syncthreads();
    pdl_trigger();

    const int epp = 32 / nsb;  // experts per pass
    int j = 0;
    for (; j < nmine; j++) {
        const int slot = j % p.nst;
        if (!__all_sync(FULL, mbar_wait(&mybar[slot], (j / p.nst) & 1, p.err))) break;
        const long long u = u0 + warp + (long long)j * NWARP;
        const int row = (int)(u % p.E), t = (int)(u / p.E);
        const uint8_t *base = myring + (size_t)slot * p.slot_bytes;
        const int kk = lane / nsb, b = lane % nsb;
        for (int k0 = 0; k0 < p.K; k0 += epp) {
            const int k = k0 + kk;
            const bool valid = kk < epp && k < p.K;
            float v = 0.0f;
            if (valid) {
                const ActBlock &ab = act[(t * p.K + k) * nsb + b];
                const uint8_t *tile = base + k * p.d_tile_bytes;
                v = p.dtype == T_Q4_K ? q4k_slot_dot(tile, nsb, b, ab) : q6k_slot_dot(tile, nsb, b, ab);
            }
            float acc = 0.0f;
            for (int b2 = 0; b2 < nsb; b2++) {
                int srcl = kk * nsb + b2;
                acc = __fadd_rn(acc, __shfl_sync(FULL, v, srcl < 32 ? srcl : 31));
            }
            if (valid && b == 0) wvals[warp * MAX_K + k] = acc;
        }
        __syncwarp();
        if (lane == 0) {
            const float *o = wvals + warp * MAX_K;
            const float *w = p.sel_w + t * p.K;
            float sum = 0.0f;
            if (p.single[t]) {
                int workers = p.workers < p.K ? p.workers : p.K;
                if (workers < 1) workers = 1;
                int chunk = (p.K + workers - 1) / workers;
                for (int s0 = 0; s0 < p.K; s0 += chunk) {
                    float tot = __fmul_rn(o[s0], w[s0]);
                    for (int i = s0 + 1; i < p.K && i < s0 + chunk; i++) tot = __fadd_rn(tot, __fmul_rn(o[i], w[i]));
                    sum = workers <= 1 ? tot : __fadd_rn(sum, tot);
                }
            } else {
                for (int i = 0; i < p.K; i++) sum = __fadd_rn(sum, __fmul_rn(o[i], w[i]));
            }
            const long long xi = (long long)t * p.E + row;
            p.x_out[xi] = p.shexp ? __fadd_rn(__fadd_rn(sum, p.shexp[xi]), p.ffn_in[xi]) : __fadd_rn(p.ffn_in[xi], sum);
        }
        __syncwarp();
        if (lane == 0 && j + p.nst < nmine) {
            fence_proxy_async();
            issue(j + p.nst);
        }
    }
    if (j < nmine)
        for (int k = j; k < nmine && k < j + p.nst; k++) mbar_wait(&mybar[k % p.nst], (k / p.nst) & 1, nullptr);
}

size_t gateup_smem_bytes(const ExpertArgs &a) {
    size_t act = (size_t)a.T * a.g_nsb * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes;
}
size_t down_smem_bytes(const ExpertArgs &a) {
    size_t act = (size_t)a.T * a.K * a.d_nsb * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes;
}

cudaError_t launch_gateup(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    return launch_ex(gateup_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), gateup_smem_bytes(a), st, pdl, a);
}

cudaError_t launch_down(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    return launch_ex(down_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), down_smem_bytes(a), st, pdl, a);
}

// ====================================================================== grouped experts (batched steps)
// With many tokens in a step, the per-(token, expert) units above read an expert's weights once
// for every token that selected it. The grouped kernels split each selected expert's rows into
// chunks of at most GROUP_MAXM and make units (chunk, tile): every unit has about the same
// work however skewed the routing, an expert's tile is read from DRAM about once and re-read
// from L2 by its other chunks, and a CTA (a contiguous unit range) stages each chunk's
// activations once. The arithmetic per (token, expert, row) is unchanged.

// One CTA: per expert, the (token, slot) indices tk = t*K + k that selected it, ascending.
__global__ void __launch_bounds__(256) group_kernel(const __grid_constant__ GroupArgs p) {
    extern __shared__ int gsm[];
    const int n = p.T * p.K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int *sel = gsm, *cnt = sel + n, *fill = cnt + p.NE;
    for (int e = tid; e < p.NE; e += blockDim.x) cnt[e] = 0;
    pdl_wait();  // the selections come from the router
    for (int i = tid; i < n; i += blockDim.x) sel[i] = p.sel_ids[i];
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {  // counts (order-free); ids outside [0, NE) are empty slots
        const int e = sel[i];
        if (e >= 0 && e < p.NE) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
        // experts in ascending order: list offsets, the active list and the chunks of at most
        // GROUP_MAXM rows, by warp-wide exclusive scans
        int run = 0, crun = 0, arun = 0;
        for (int e0 = 0; e0 < p.NE; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < p.NE ? cnt[e] : 0;
            const int ch = (c + GROUP_MAXM - 1) / GROUP_MAXM, a = c > 0 ? 1 : 0;
            int ic = c, ich = ch, ia = a;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FULL, ic, o), w = __shfl_up_sync(FULL, ich, o),
                          x = __shfl_up_sync(FULL, ia, o);
                if (lane >= o) {
                    ic += v;
                    ich += w;
                    ia += x;
                }
            }
            if (e < p.NE) {
                const int off = run + ic - c;
                fill[e] = off;
                p.g_count[e] = c;
                p.g_off[e] = off;
                if (a) p.g_active[arun + ia - 1] = e;
                for (int k = 0; k < ch; k++) {
                    p.g_chunk_e[crun + ich - ch + k] = e;
                    p.g_chunk_r0[crun + ich - ch + k] = k * GROUP_MAXM;
                }
            }
            run += __shfl_sync(FULL, ic, 31);
            crun += __shfl_sync(FULL, ich, 31);
            arun += __shfl_sync(FULL, ia, 31);
        }
        if (lane == 0) {
            *p.g_nactive = arun;
            *p.g_nchunks = crun;
        }
        __syncwarp();
        // each expert's list in ascending selection order: 32 selections at a time, a lane's
        // place = the lanes before it with the same expert
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            const int e = i < n ? sel[i] : -1;
            const bool valid = e >= 0 && e < p.NE;
            const unsigned m = __match_any_sync(FULL, valid ? e : -1);
            const int rank = __popc(m & ((1u << lane) - 1u));
            const int base = valid ? fill[e] : 0;
            if (valid) p.g_list[base + rank] = i;
            __syncwarp();
            if (valid && lane == __ffs(m) - 1) fill[e] = base + __popc(m);
            __syncwarp();
        }
    }
    pdl_trigger();
}

// A warp's ring across the chunks of a grouped kernel: copy g goes to slot g % nst and its
// wait uses parity (g / nst) & 1; `issued` and `done` count copies over the whole launch.
struct GroupRing {
    uint8_t *base;
    uint64_t *bars;
    int nst, slot_bytes, issued, done;
};

// gate/up, grouped: unit = (selected expert a, tile); the CTA's units are a contiguous range in
// (a, tile) order, so it walks at most a few experts and stages each one's tokens once.
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) gateup_grouped_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int *rows_s = reinterpret_cast<int *>(smem + 512);  // [GROUP_MAXM] token of each staged row
    int *tk_s = rows_s + GROUP_MAXM;                     // [GROUP_MAXM] its (token, slot) index
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsb = p.g_nsb, nt = p.g_n_tiles;
    const size_t act_bytes = (size_t)GROUP_MAXM * nsb * sizeof(ActBlock);
    GroupRing r;
    r.nst = p.nst;
    r.slot_bytes = p.slot_bytes;
    r.base = smem + 1024 + ((act_bytes + 127) & ~(size_t)127) + (size_t)warp * p.nst * p.slot_bytes;
    r.bars = reinterpret_cast<uint64_t *>(smem) + warp * p.nst;
    r.issued = r.done = 0;
    float *red = reinterpret_cast<float *>(smem + 1024 + ((act_bytes + 127) & ~(size_t)127) +
                                           (size_t)NWARP * p.nst * p.slot_bytes) + warp * 2 * GROUP_RED_FLOATS;
    if (lane == 0) {
        for (int i = 0; i < p.nst; i++) mbar_init(&r.bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_wait();  // the groups come from group_kernel, the activations from the router
    const int total = *p.g_nchunks * nt;
    const int u0 = (int)((unsigned)blockIdx.x * (unsigned)total / gridDim.x);
    const int u1 = (int)((unsigned)(blockIdx.x + 1) * (unsigned)total / gridDim.x);
    pdl_trigger();
    bool ok = true;
    for (int ci = nt ? u0 / nt : 0; ok && ci * nt < u1; ci++) {
        const int e = p.g_chunk_e[ci], c0 = p.g_chunk_r0[ci], m = p.g_count[e], off = p.g_off[e];
        const int lo = (u0 > ci * nt ? u0 : ci * nt) - ci * nt;
        const int hi = (u1 < (ci + 1) * nt ? u1 : (ci + 1) * nt) - ci * nt;
        const int ntw = hi - lo > warp ? (hi - lo - warp + NWARP - 1) / NWARP : 0;
        {
            const int mc = m - c0 < GROUP_MAXM ? m - c0 : GROUP_MAXM;
            __syncthreads();  // the previous chunk's activations are no longer read
            if (tid < mc) {
                const int tk = p.g_list[off + c0 + tid];
                tk_s[tid] = tk;
                rows_s[tid] = tk / p.row_div;
            }
            const int base = r.done;  // this warp's j-th tile of the chunk is copy base + j
            auto issue = [&](int j) {
                const int tile = lo + warp + j * NWARP, slot = (base + j) % r.nst;
                uint8_t *dst = r.base + (size_t)slot * r.slot_bytes;
                mbar_arrive_expect_tx(&r.bars[slot], p.g_tile_bytes + p.u_tile_bytes);
                bulk_g2s(dst, expert_gate(p, e) + (long long)tile * p.g_tile_bytes, p.g_tile_bytes,
                         &r.bars[slot]);
                bulk_g2s(dst + p.g_tile_bytes, expert_up(p, e) + (long long)tile * p.u_tile_bytes,
                         p.u_tile_bytes, &r.bars[slot]);
            };
            if (lane == 0) {
                fence_proxy_async();
                while (r.issued - base < ntw && r.issued - r.done < r.nst) {
                    issue(r.issued - base);
                    r.issued++;
                }
            }
            r.issued = __shfl_sync(FULL, r.issued, 0);
            __syncthreads();  // rows_s, tk_s
            stage_activations<NWARP>(p.fn, p.E, rows_s, nullptr, 0.0f, p.E, mc, act, nullptr);
            __syncthreads();
            for (int j = 0; j < ntw; j++) {
                const int g = base + j, slot = g % r.nst;
                if (!__all_sync(FULL, mbar_wait(&r.bars[slot], (g / r.nst) & 1, p.err))) {
                    ok = false;
                    break;
                }
                r.done = g + 1;
                const int tile = lo + warp + j * NWARP;
                const uint8_t *gt = r.base + (size_t)slot * r.slot_bytes, *ut = gt + p.g_tile_bytes;
                const bool active = lane < p.g_S;
                const int b = active ? lane % nsb : 0;
                const int ls = active ? lane : 0;
                const uint32_t act_b = smem_u32(&act[b]), tok_stride = (uint32_t)(nsb * sizeof(ActBlock));
                // gate then up: the lane's superblock decoded into registers once, its dots with
                // the chunk's tokens two at a time, every partial to shared memory
                auto dots = [&](auto &&dot, float *dst) {
                    for (int i = 0; i < mc; i += 2) {
                        const int i1 = i + 1 < mc ? i + 1 : i;
                        const float v0 = dot(act_b + (uint32_t)i * tok_stride);
                        const float v1 = dot(act_b + (uint32_t)i1 * tok_stride);
                        dst[i * RED_STRIDE + lane] = active ? v0 : 0.0f;
                        if (i + 1 < mc) dst[(i + 1) * RED_STRIDE + lane] = active ? v1 : 0.0f;
                    }
                };
#pragma unroll 1
                for (int which = 0; which < 2; which++) {
                    const uint32_t tl = smem_u32(which ? ut : gt);
                    float *dst = red + which * GROUP_RED_FLOATS;
                    if ((which ? p.utype : p.gtype) == T_Q4_K) {
                        Q4Reg w;
                        q4k_load_r(w, tl, p.g_S, ls);
                        dots([&](uint32_t a) { return q4k_dot_r(w, a); }, dst);
                    } else {
                        Q6Reg w;
                        q6k_load_r(w, tl, p.g_S, ls);
                        dots([&](uint32_t a) { return q6k_dot_r(w, a); }, dst);
                    }
                }
                __syncwarp();
                // one lane per (row, token): the row's nsb partials in superblock order (C4)
                for (int q = lane; q < p.g_rpt * GROUP_MAXM; q += 32) {
                    const int rr = q / GROUP_MAXM, i = q % GROUP_MAXM, rrow = tile * p.g_rpt + rr;
                    if (i < mc && rrow < p.F) {
                        const float *gv = red + i * RED_STRIDE + rr * nsb;
                        const float *uv = gv + GROUP_RED_FLOATS;
                        float ag = 0.0f, au = 0.0f;
                        for (int b2 = 0; b2 < nsb; b2++) {
                            ag = __fadd_rn(ag, gv[b2]);
                            au = __fadd_rn(au, uv[b2]);
                        }
                        p.act[(long long)tk_s[i] * p.F + rrow] = __fmul_rn(bt_silu(ag), au);
                    }
                }
                __syncwarp();
                if (lane == 0 && r.issued - base < ntw) {
                    fence_proxy_async();
                    issue(r.issued - base);
                    r.issued++;
                }
                r.issued = __shfl_sync(FULL, r.issued, 0);
            }
            if (__syncthreads_or(!ok)) ok = false;
        }
    }
    if (!ok && lane == 0)  // a wait ran out: let this warp's copies in flight land (bounded) before exiting
        for (int g = r.done; g < r.issued; g++) mbar_wait(&r.bars[g % r.nst], (g / r.nst) & 1, nullptr);
}

// down, grouped: unit = (selected expert a, group of RG = 32 / nsb output rows): one copy of RG
// consecutive row tiles; lane l decodes slot l % nsb of row l / nsb. Each (token, slot)'s row
// values go to dpart; down_combine_kernel adds them in the reference's order.
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) down_grouped_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int *tk_s = reinterpret_cast<int *>(smem + 512);  // [GROUP_MAXM] (token, slot) index = act row
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsb = p.d_nsb, RG = 32 / nsb, ng = (p.E + RG - 1) / RG;
    const size_t act_bytes = (size_t)GROUP_MAXM * nsb * sizeof(ActBlock);
    GroupRing r;
    r.nst = p.nst;
    r.slot_bytes = p.slot_bytes;
    r.base = smem + 1024 + ((act_bytes + 127) & ~(size_t)127) + (size_t)warp * p.nst * p.slot_bytes;
    r.bars = reinterpret_cast<uint64_t *>(smem) + warp * p.nst;
    r.issued = r.done = 0;
    if (lane == 0) {
        for (int i = 0; i < p.nst; i++) mbar_init(&r.bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_wait();
    const int total = *p.g_nchunks * ng;
    const int u0 = (int)((unsigned)blockIdx.x * (unsigned)total / gridDim.x);
    const int u1 = (int)((unsigned)(blockIdx.x + 1) * (unsigned)total / gridDim.x);
    pdl_trigger();
    bool ok = true;
    for (int ci = ng ? u0 / ng : 0; ok && ci * ng < u1; ci++) {
        const int e = p.g_chunk_e[ci], c0 = p.g_chunk_r0[ci], m = p.g_count[e], off = p.g_off[e];
        const int lo = (u0 > ci * ng ? u0 : ci * ng) - ci * ng;
        const int hi = (u1 < (ci + 1) * ng ? u1 : (ci + 1) * ng) - ci * ng;
        const int nuw = hi - lo > warp ? (hi - lo - warp + NWARP - 1) / NWARP : 0;
        {
            const int mc = m - c0 < GROUP_MAXM ? m - c0 : GROUP_MAXM;
            __syncthreads();
            if (tid < mc) tk_s[tid] = p.g_list[off + c0 + tid];
            const int base = r.done;
            auto issue = [&](int j) {
                const int gr = lo + warp + j * NWARP, slot = (base + j) % r.nst;
                const int r0 = gr * RG, nr = p.E - r0 < RG ? p.E - r0 : RG;
                mbar_arrive_expect_tx(&r.bars[slot], nr * p.d_tile_bytes);
                bulk_g2s(r.base + (size_t)slot * r.slot_bytes, expert_down(p, e) + (long long)r0 * p.d_tile_bytes,
                         nr * p.d_tile_bytes, &r.bars[slot]);
            };
            if (lane == 0) {
                fence_proxy_async();
                while (r.issued - base < nuw && r.issued - r.done < r.nst) {
                    issue(r.issued - base);
                    r.issued++;
                }
            }
            r.issued = __shfl_sync(FULL, r.issued, 0);
            __syncthreads();  // tk_s
            stage_activations<NWARP>(p.act, p.F, tk_s, nullptr, 0.0f, p.F, mc, act, nullptr);
            __syncthreads();
            for (int j = 0; j < nuw; j++) {
                const int g = base + j, slot = g % r.nst;
                if (!__all_sync(FULL, mbar_wait(&r.bars[slot], (g / r.nst) & 1, p.err))) {
                    ok = false;
                    break;
                }
                r.done = g + 1;
                const int gr = lo + warp + j * NWARP, r0 = gr * RG;
                const int nr = p.E - r0 < RG ? p.E - r0 : RG;
                const bool active = lane < nr * nsb;
                const int rr = active ? lane / nsb : 0, b = active ? lane - rr * nsb : 0;
                const uint32_t tile = smem_u32(r.base + (size_t)slot * r.slot_bytes + (size_t)rr * p.d_tile_bytes);
                const uint32_t act_b = smem_u32(&act[b]), tok_stride = (uint32_t)(nsb * sizeof(ActBlock));
                // the lane's superblock in registers once; two tokens at a time, each row's nsb
                // partials added in superblock order across its lanes (C4)
                auto dots = [&](auto &&dot) {
                    for (int i = 0; i < mc; i += 2) {
                        const int i1 = i + 1 < mc ? i + 1 : i;
                        const float v0 = dot(act_b + (uint32_t)i * tok_stride);
                        const float v1 = dot(act_b + (uint32_t)i1 * tok_stride);
                        float acc0 = 0.0f, acc1 = 0.0f;
                        for (int b2 = 0; b2 < nsb; b2++) {
                            const int srcl = rr * nsb + b2;
                            acc0 = __fadd_rn(acc0, __shfl_sync(FULL, v0, srcl < 32 ? srcl : 31));
                            acc1 = __fadd_rn(acc1, __shfl_sync(FULL, v1, srcl < 32 ? srcl : 31));
                        }
                        if (active && b == 0) {
                            p.dpart[(long long)tk_s[i] * p.E + r0 + rr] = acc0;
                            if (i + 1 < mc) p.dpart[(long long)tk_s[i + 1] * p.E + r0 + rr] = acc1;
                        }
                    }
                };
                if (p.dtype == T_Q4_K) {
                    Q4Reg w;
                    q4k_load_r(w, tile, nsb, b);
                    dots([&](uint32_t a) { return q4k_dot_r(w, a); });
                } else {
                    Q6Reg w;
                    q6k_load_r(w, tile, nsb, b);
                    dots([&](uint32_t a) { return q6k_dot_r(w, a); });
                }
                __syncwarp();
                if (lane == 0 && r.issued - base < nuw) {
                    fence_proxy_async();
                    issue(r.issued - base);
                    r.issued++;
                }
                r.issued = __shfl_sync(FULL, r.issued, 0);
            }
            if (__syncthreads_or(!ok)) ok = false;
        }
    }
    if (!ok && lane == 0)
        for (int g = r.done; g < r.issued; g++) mbar_wait(&r.bars[g % r.nst], (g / r.nst) & 1, nullptr);
}

// grid (T, E / 256): x = ffn_in + the K expert rows scaled by their weights and summed in the reference's
// order (the single-token pairs of expert_ffn_single, or the block path's sequential sum).
__global__ void __launch_bounds__(256) down_combine_kernel(const __grid_constant__ ExpertArgs p) {
    const int t = blockIdx.x;
    pdl_wait();
    const float *w = p.sel_w + t * p.K;
    for (int row = blockIdx.y * blockDim.x + threadIdx.x; row < p.E; row += gridDim.y * blockDim.x) {
        float o[MAX_K];
        for (int k = 0; k < p.K; k++) {
            const long long slot = (long long)t * p.K + k;
            const long long src = p.ep_ranks ? (long long)(p.sel_ids[slot] / p.ep_per) * p.ep_slots + slot : slot;
            o[k] = p.dpart[src * p.E + row];
        }
        float sum = 0.0f;
        if (p.single[t]) {
            int workers = p.workers < p.K ? p.workers : p.K;
            if (workers < 1) workers = 1;
            const int chunk = (p.K + workers - 1) / workers;
            for (int s0 = 0; s0 < p.K; s0 += chunk) {
                float tot = __fmul_rn(o[s0], w[s0]);
                for (int i = s0 + 1; i < p.K && i < s0 + chunk; i++) tot = __fadd_rn(tot, __fmul_rn(o[i], w[i]));
                sum = workers <= 1 ? tot : __fadd_rn(sum, tot);
            }
        } else {
            for (int i = 0; i < p.K; i++) sum = __fadd_rn(sum, __fmul_rn(o[i], w[i]));
        }
        const long long xi = (long long)t * p.E + row;
        p.x_out[xi] = p.shexp ? __fadd_rn(__fadd_rn(sum, p.shexp[xi]), p.ffn_in[xi]) : __fadd_rn(p.ffn_in[xi], sum);
    }
    pdl_trigger();
}

// grid slots (the fixed capacity per rank), 256 threads: slot tk = blockIdx.x goes to the rank
// owning its expert with the token's row; every other rank's copy of the slot is marked empty.
__global__ void __launch_bounds__(256) ep_pack_kernel(const __grid_constant__ EpPackArgs p) {
    const int tk = blockIdx.x;
    pdl_wait();
    const int e = tk < p.T * p.K ? p.sel_ids[tk] : -1;
    const int owner = e >= 0 ? e / p.per : -1;
    for (int r = threadIdx.x; r < p.ranks; r += blockDim.x) p.send_meta[r * p.slots + tk] = r == owner ? e : -1;
    if (owner >= 0 && p.send_qs) {  // the token's Q8_K row: values, block scales, 32-value sums
        const long long t = tk / p.K, slot = (long long)owner * p.slots + tk;
        const int nsb = p.E / 256;
        const uint4 *qs = reinterpret_cast<const uint4 *>(p.q8_qs + t * p.E);
        uint4 *dq = reinterpret_cast<uint4 *>(p.send_qs + slot * p.E);
        for (int i = threadIdx.x; i < p.E / 16; i += blockDim.x) dq[i] = qs[i];
        for (int i = threadIdx.x; i < nsb; i += blockDim.x) p.send_d[slot * nsb + i] = p.q8_d[t * nsb + i];
        for (int i = threadIdx.x; i < nsb * 8; i += blockDim.x) p.send_bs[slot * nsb * 8 + i] = p.q8_bs[t * nsb * 8 + i];
    } else if (owner >= 0) {
        const float *src = p.fn + (long long)(tk / p.K) * p.E;
        float *dst = p.send_rows + ((long long)owner * p.slots + tk) * p.E;
        for (int i = threadIdx.x; i < p.E; i += blockDim.x) dst[i] = src[i];
    }
    pdl_trigger();
}

__global__ void __launch_bounds__(256) shexp_act_kernel(const float *__restrict__ gu, float *__restrict__ act, int T,
                                                        int F) {
    pdl_wait();
    const long long n = (long long)T * F;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
        const long long t = i / F, j = i - t * F;
        act[i] = __fmul_rn(bt_silu(gu[t * 2 * F + j]), gu[t * 2 * F + F + j]);
    }
    pdl_trigger();
}

cudaError_t launch_shexp_act(const float *gu, float *act, int T, int F, cudaStream_t st, bool pdl) {
    const long long n = (long long)T * F;
    const int grid = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, shexp_act_kernel, gu, act, T, F);
}

cudaError_t launch_ep_pack(const EpPackArgs &a, cudaStream_t st, bool pdl) {
    return launch_ex(ep_pack_kernel, dim3(a.slots), dim3(256), 0, st, pdl, a);
}

size_t gateup_grouped_smem_bytes(const ExpertArgs &a) {
    size_t act = (size_t)GROUP_MAXM * a.g_nsb * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes +
           (size_t)GEMV_WARPS * 2 * GROUP_RED_FLOATS * 4;
}
size_t down_grouped_smem_bytes(const ExpertArgs &a) {
    size_t act = (size_t)GROUP_MAXM * a.d_nsb * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes;
}
int down_group_rows(const ExpertArgs &a) { return 32 / a.d_nsb; }

cudaError_t launch_group(const GroupArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = ((size_t)a.T * a.K + 2 * (size_t)a.NE + 1) * 4;  // selections, counts, fill
    return launch_ex(group_kernel, dim3(1), dim3(256), smem, st, pdl, a);
}
cudaError_t launch_gateup_grouped(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    return launch_ex(gateup_grouped_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), gateup_grouped_smem_bytes(a),
                     st, pdl, a);
}
cudaError_t launch_down_grouped(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    return launch_ex(down_grouped_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), down_grouped_smem_bytes(a), st,
                     pdl, a);
}
cudaError_t launch_down_combine(const ExpertArgs &a, cudaStream_t st, bool pdl) {
    return launch_ex(down_combine_kernel, dim3(a.T, (a.E + 255) / 256), dim3(256), 0, st, pdl, a);
}

// ====================================================================== router
// grid (ceil(NE/ROUTER_ROWS), T), 32 * ROUTER_ROWS threads: each CTA normalises the token (C6)
// into shared memory and warp w computes router row blockIdx.x*ROUTER_ROWS+w (C5). The
// token's last CTA (atomic ticket) runs soft_max_ext and route(): stable descending order by
// total_cmp, top-K, renormalised over the selection. 16 rows per CTA normalise each token 8
// times at NE = 128 instead of 32: 22.4 against 27.2 µs per batch-64 layer, the same bits.
constexpr int ROUTER_ROWS = 16;  // router rows (warps) per CTA

__global__ void __launch_bounds__(ROUTER_ROWS * 32) router_kernel(const __grid_constant__ RouterArgs p) {
    extern __shared__ float s_y[];  // [E] normalised activations
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.y;
    __shared__ float s_norm;
    __shared__ int s_last;
    __shared__ float s_prob[512];
    __shared__ int s_rank_id[MAX_K];
    __shared__ float s_rank_p[MAX_K];
    pdl_wait();
    const float *x = p.x + (long long)t * p.E;
    if (warp == 0) {
        float acc = warp_sumsq_p2(x, p.E, lane);
        if (lane == 0) s_norm = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)p.E), p.eps)));
    }
    __syncthreads();
    pdl_trigger();
    const float s = s_norm;
    for (int i = threadIdx.x; i < p.E; i += blockDim.x) s_y[i] = __fmul_rn(__fmul_rn(x[i], s), p.norm_w[i]);
    __syncthreads();
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < p.E; i += blockDim.x) p.fn_out[(long long)t * p.E + i] = s_y[i];
    const int r = blockIdx.x * ROUTER_ROWS + warp;
    if (r < p.NE) {
        float acc = warp_dot_p2(p.Wr + (long long)r * p.E, s_y, p.E, lane);
        if (p.bias) acc = __fadd_rn(acc, p.bias[r]);
        if (lane == 0) p.logits[(long long)t * p.NE + r] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&p.cnt[t], 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    __shared__ int s_key[512];
    if (warp == 0) {  // soft_max_ext: max, exp and the P2 sum, then the scaling (C5, C6)
        const float *lg = p.logits + (long long)t * p.NE;
        float m = -__int_as_float(0x7f800000);
        for (int i = lane; i < p.NE; i += 32) {
            float v = __ldcg(lg + i);
            s_prob[i] = v;
            m = fmaxf(m, v);
        }
        m = warp_max(m);
        float acc = 0.0f;
        for (int i = lane; i < p.NE; i += 32) {
            float e = bt_exp(__fsub_rn(s_prob[i], m));
            s_prob[i] = e;
            acc = __fadd_rn(acc, e);
        }
        acc = butterfly_sum(acc);
        const float inv = __fdiv_rn(1.0f, acc);
        for (int i = lane; i < p.NE; i += 32) {
            s_prob[i] = __fmul_rn(s_prob[i], inv);
            s_key[i] = total_key(s_prob[i]);
        }
    }
    __syncthreads();
    // route(): the rank of each probability in the stable descending order, all threads
    for (int i = threadIdx.x; i < p.NE; i += blockDim.x) {
        const int ki = s_key[i];
        int rank = 0;
        for (int jj = 0; jj < p.NE; jj++) {
            const int kj = s_key[jj];
            rank += (kj > ki) || (kj == ki && jj < i);
        }
        if (rank < p.K) {
            s_rank_id[rank] = i;
            s_rank_p[rank] = s_prob[i];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (int q = 0; q < p.K; q++) total = __fadd_rn(total, s_rank_p[q]);
        int ids[MAX_K];
        float ws[MAX_K];
        for (int q = 0; q < p.K; q++) {
            float w = total > 0.0f ? __fdiv_rn(s_rank_p[q], total) : s_rank_p[q];
            ids[q] = s_rank_id[q];
            ws[q] = w;
            p.topk_ids[t * p.K + q] = ids[q];
            p.topk_w[t * p.K + q] = w;
        }
        for (int a = 1; a < p.K; a++)
            for (int b = a; b > 0 && ids[b - 1] > ids[b]; b--) {
                int ti = ids[b]; ids[b] = ids[b - 1]; ids[b - 1] = ti;
                float tw = ws[b]; ws[b] = ws[b - 1]; ws[b - 1] = tw;
            }
        for (int q = 0; q < p.K; q++) {
            p.sel_ids[t * p.K + q] = ids[q];
            p.sel_w[t * p.K + q] = ws[q];
        }
        p.cnt[t] = 0;
    }
}

cudaError_t launch_router(const RouterArgs &a, cudaStream_t st, bool pdl) {
    dim3 grid((a.NE + ROUTER_ROWS - 1) / ROUTER_ROWS, a.T);
    return launch_ex(router_kernel, grid, dim3(ROUTER_ROWS * 32), (size_t)a.E * 4, st, pdl, a);
}

// ====================================================================== q/k norm, RoPE, KV append
// grid (T, ceil((H+2*HK)/8)), warp per head; lane l holds elements l, l+32, ... (C5/C6, C9).
__global__ void __launch_bounds__(256) qkv_post_kernel(const __grid_constant__ QkvPostArgs p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x;
    const int hh = blockIdx.y * 8 + warp;
    pdl_wait();
    pdl_trigger();
    if (hh >= p.H + 2 * p.HK) return;
    const int D = p.D, npl = D / 32;
    const int QW = p.H * D, KW = p.HK * D;
    const float *src = p.qkv + (long long)t * p.qkv_stride;
    float v[8];
    int kind, head;
    if (hh < p.H) {
        kind = 0; head = hh; src += head * D;
    } else if (hh < p.H + p.HK) {
        kind = 1; head = hh - p.H; src += QW + head * D;
    } else {
        kind = 2; head = hh - p.H - p.HK; src += QW + KW + head * D;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = i < npl ? src[lane + 32 * i] : 0.0f;
    const int pos = p.pos_of[t];
    if (kind < 2) {
        const float *w = kind == 0 ? p.q_norm : p.k_norm;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i < npl) acc = fmaf(v[i], v[i], acc);
        acc = butterfly_sum(acc);
        float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), p.eps)));
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i < npl) v[i] = __fmul_rn(__fmul_rn(v[i], s), w[lane + 32 * i]);
        const float *cs = p.rope + (long long)pos * p.n_rot;
        const int half = npl / 2;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (i < half) {
                int d = lane + 32 * i;
                float c = cs[2 * d], sn = cs[2 * d + 1];
                float x0 = v[i], x1 = v[i + half];
                float a = __fmul_rn(x0, c), b = __fmul_rn(x1, sn), e = __fmul_rn(x0, sn), f = __fmul_rn(x1, c);
                v[i] = __fsub_rn(a, b);
                v[i + half] = __fadd_rn(e, f);
            }
        }
    }
    if (kind == 0) {
        float *dst = p.q_out + (long long)t * QW + head * D;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i < npl) dst[lane + 32 * i] = v[i];
    } else {
        const int seq = p.seq_of[t];
        const int blk = p.block_table[seq * p.max_blocks + pos / 16];
        const long long row = ((((long long)p.layer * p.n_blocks + blk) * 2 + (kind - 1)) * p.HK + head) * 16 + pos % 16;
        __half *dst = p.kv + row * D;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i < npl) dst[lane + 32 * i] = __float2half_rn(v[i]);
    }
}

cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t st, bool pdl) {
    dim3 grid(a.T, (a.H + 2 * a.HK + 7) / 8);
    return launch_ex(qkv_post_kernel, grid, dim3(256), 0, st, pdl, a);
}

// ====================================================================== attention
// Persistent: about three 128-thread CTAs per SM (73 KB of shared memory each) walk the step's
// items, an item being (token, kv head, chunk of 128 keys) in that order; CTA b takes the
// contiguous range [b*N/grid, (b+1)*N/grid). K and V pages arrive by 2-D TMA (128-byte swizzle,
// box 64 x 16) into one K and one V buffer: the next item's K is requested as soon as this
// item's scores are done and its V once P*V is done, so the copies overlap the arithmetic.
// Scores: thread = key, all G heads, a sequential fmaf dot over d. P*V: thread = two columns,
// G/2 heads, a sequential fmaf over the chunk's keys. A chunk that is the whole context
// finalises its heads; otherwise it writes (acc, m, l) to scratch and attn_combine_kernel
// merges the chunks in order (C8).
constexpr int ATTN_THREADS = 128;
constexpr int ATTN_PART_ROW = 132;  // floats per (chunk, head) partial: acc[128], m, l, 2 pad

size_t attn_smem_bytes(int G, int T) {
    return 65536 + (size_t)128 * G * 4 + (size_t)ATTN_CHUNK * G * 4 + (32 + 32 + 8 + 8) * 4 + 16 +
           (size_t)(3 * T + 1) * 4 + 1024;
}

template <int N>
__device__ __forceinline__ void lds_vec(float (&dst)[N], const float *src) {
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

// The item loop of the attention kernel. Per item (t, g, c): q rounded to f16 in shared memory
// (when (t, g) changes), then
//   scores: thread = key, all G heads, dims in order (C8: q.k as f16 x f16 + f32 fmas);
//   chunk max, exp and the P3 sum (32-key butterflies, the 4 warp sums in order);
//   P*V: thread = dims 2dp, 2dp+1 and heads hq*G/2 .. +G/2, keys in order;
// and the chunk's partial (acc, m, l), or the output when the context is one chunk.
template <int G>
__global__ void __launch_bounds__(ATTN_THREADS, 3)
    attn_kernel(const __grid_constant__ AttnArgs p, const __grid_constant__ CUtensorMap tmap) {
    constexpr int D = 128, HPT = G / 2, CH = ATTN_CHUNK;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // offset from the shared array itself (not through an integer), so loads stay ld.shared
    uint8_t *smem = smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023u)) & 1023u);
    uint8_t *const K0 = smem, *const K1 = smem + 16384, *const V0 = smem + 32768, *const V1 = smem + 49152;
    float *qs = reinterpret_cast<float *>(smem + 65536);              // [D][G] q rounded to f16, as f32
    float *ps = reinterpret_cast<float *>(smem + 65536 + D * G * 4);  // [CH][G]
    float *red = ps + CH * G;                                         // [4][8]
    float *red2 = red + 32;                                           // [4][8]
    float *s_m = red2 + 32, *s_l = s_m + 8;
    uint64_t *bars = reinterpret_cast<uint64_t *>(s_l + 8);  // [0] K copies, [1] V copies
    int *pre = reinterpret_cast<int *>(bars + 2);            // [T + 1] first item of each token
    int *pos_s = pre + p.T + 1, *seq_s = pos_s + p.T;        // [T] each

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    pdl_wait();
    if (warp == 0) {  // items per token: HK * its chunk count; exclusive prefix over the tokens
        int run = 0;
        for (int t0 = 0; t0 < p.T; t0 += 32) {
            const int t = t0 + lane;
            const int pos = t < p.T ? p.pos_of[t] : 0;
            const int n = t < p.T ? p.HK * ((pos + CH) / CH) : 0;
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += v;
            }
            if (t < p.T) {
                pre[t] = run + incl - n;
                pos_s[t] = pos;
                seq_s[t] = p.seq_of[t];
            }
            run += __shfl_sync(FULL, incl, 31);
        }
        if (lane == 0) pre[p.T] = run;
    }
    __syncthreads();
    pdl_trigger();
    const int N = pre[p.T];
    const int u0 = (int)((long long)blockIdx.x * N / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * N / gridDim.x);
    if (u0 >= u1) return;

    // item i -> token t (the last with pre[t] <= i), kv head g, chunk c
    auto decode = [&](int i, int &t, int &g, int &c) {
        int lo = 0, hi = p.T - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= i) lo = mid;
            else hi = mid - 1;
        }
        t = lo;
        const int nc = (pos_s[t] + CH) / CH, r = i - pre[t];
        g = r / nc;
        c = r - g * nc;
    };
    // warp 0: the page rows of item i (lane = page), kept until its K and V copies are issued
    int nx_pages = 0, nx_row = 0;
    auto locate = [&](int i) {
        int t, g, c;
        decode(i, t, g, c);
        const int nk = pos_s[t] + 1, base = c * CH;
        const int cnt = nk - base < CH ? nk - base : CH;
        nx_pages = (cnt + 15) / 16;
        nx_row = 0;
        if (lane < nx_pages) {
            const int blk = p.block_table[seq_s[t] * p.max_blocks + (base >> 4) + lane];
            nx_row = (int)(((((long long)p.layer * p.n_blocks + blk) * 2 + 0) * p.HK + g) * 16);
        }
    };
    auto issue = [&](int which) {  // which 0: K pages, 1: V pages (row + HK*16)
        if (lane == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(&bars[which], nx_pages * 4096);
        }
        __syncwarp();
        if (lane < nx_pages) {
            const int row = which ? nx_row + p.HK * 16 : nx_row;
            uint8_t *d0 = which ? V0 : K0, *d1 = which ? V1 : K1;
            tma_load_2d(d0 + lane * 2048, &tmap, 0, row, &bars[which]);
            tma_load_2d(d1 + lane * 2048, &tmap, 64, row, &bars[which]);
        }
    };
    int k_issued = 0, v_issued = 0;  // copies requested per buffer (item j's copy is the j-th)
    if (warp == 0) {
        if (lane == 0) prefetch_tmap(&tmap);
        locate(u0);
        issue(0);
        issue(1);
    }
    k_issued = v_issued = 1;
    const int QW = p.H * D, dp = tid & 63, hq = tid >> 6;
    const float NEG_INF = -__int_as_float(0x7f800000);
    int cur_tg = -1;
    bool ok = true;
    for (int i = u0, j = 0; i < u1; i++, j++) {
        int t, g, c;
        decode(i, t, g, c);
        const int nk = pos_s[t] + 1, nc = (nk + CH - 1) / CH, base = c * CH;
        const int cnt = nk - base < CH ? nk - base : CH;
        if (warp == 0 && i + 1 < u1) locate(i + 1);  // the page ids load under this item's arithmetic
        if (t * p.HK + g != cur_tg) {  // every thread passed the last item's scores: qs is free
            cur_tg = t * p.HK + g;
            for (int x = tid; x < D * G; x += ATTN_THREADS) {
                const int h = x / D, d = x % D;
                qs[d * G + h] = __half2float(__float2half_rn(p.q[(long long)t * QW + (g * G + h) * D + d]));
            }
        }
        __syncthreads();
        if (__syncthreads_or(!mbar_wait(&bars[0], j & 1, p.err))) {
            ok = false;
            break;
        }

        // ---- scores
        const int k = tid;
        const bool valid = k < cnt;
        float sc[G];
        {
            // heads in pairs: (sc[2j], sc[2j+1]) += (q[d][2j], q[d][2j+1]) * (k[d], k[d]), one
            // paired fma per pair and dimension, d in order (C8: each an fmaf of two f16 values)
            f32x2 acc[G / 2];
#pragma unroll
            for (int j = 0; j < G / 2; j++) acc[j] = 0ull;
            const uint8_t *krow = K0 + k * 128;
            const int ksw = k & 7;
#pragma unroll 2
            for (int c16 = 0; c16 < 16; c16++) {
                const uint4 w =
                    *reinterpret_cast<const uint4 *>((c16 < 8 ? krow : krow + 16384) + (((c16 & 7) ^ ksw) << 4));
                const uint32_t kw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e2 = 0; e2 < 4; e2++) {
                    const float2 kf = h2f2_fma(kw[e2]);
#pragma unroll
                    for (int hl = 0; hl < 2; hl++) {
                        const int d = c16 * 8 + 2 * e2 + hl;
                        const f32x2 kk = hl ? pk2(kf.y, kf.y) : pk2(kf.x, kf.x);
                        const f32x2 *qd = reinterpret_cast<const f32x2 *>(qs + d * G);
#pragma unroll
                        for (int j = 0; j < G / 2; j++) acc[j] = ffma2(qd[j], kk, acc[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < G / 2; j++) {
                const float2 v = upk2(acc[j]);
                sc[2 * j] = v.x;
                sc[2 * j + 1] = v.y;
            }
        }
#pragma unroll
        for (int h = 0; h < G; h++) {
            sc[h] = valid ? __fmul_rn(sc[h], p.scale) : NEG_INF;
            const float m = warp_max(sc[h]);
            if (lane == 0) red[warp * 8 + h] = m;
        }
        __syncthreads();  // K is no longer read: the next item's K pages may land
        if (warp == 0 && i + 1 < u1) issue(0);
        k_issued += i + 1 < u1;
        if (tid < G) {
            float m = red[tid];
            for (int w = 1; w < 4; w++) m = fmaxf(m, red[w * 8 + tid]);
            s_m[tid] = m;
        }
        __syncthreads();
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
            for (int h4 = 0; h4 < G / 4; h4++)
                prow[h4] = make_float4(sc[4 * h4], sc[4 * h4 + 1], sc[4 * h4 + 2], sc[4 * h4 + 3]);
        } else {
#pragma unroll
            for (int h = 0; h < G; h++) ps[k * G + h] = sc[h];
        }
        __syncthreads();
        if (tid < G) {
            float l = 0.0f;
            for (int w = 0; w < CH / 32; w++) l = __fadd_rn(l, red2[w * 8 + tid]);
            s_l[tid] = l;
        }
        if (__syncthreads_or(!mbar_wait(&bars[1], j & 1, p.err))) {
            ok = false;
            break;
        }
        // ---- P*V
        float acc0[HPT], acc1[HPT];
        {
            // heads in pairs: (acc[d][h], acc[d][h+1]) += (p[h], p[h+1]) * (v[d], v[d]), keys in
            // order (C8)
            constexpr bool PAIRS = HPT % 2 == 0;  // else one head at a time (G = 2, 6)
            constexpr int NP = PAIRS ? HPT / 2 : 1;
            f32x2 a0[NP], a1[NP];
            float s0[HPT], s1[HPT];
#pragma unroll
            for (int j = 0; j < NP; j++) a0[j] = a1[j] = 0ull;
#pragma unroll
            for (int h = 0; h < HPT; h++) s0[h] = s1[h] = 0.0f;
            const int d = 2 * dp, cc = (d & 63) >> 3;
            const uint8_t *vcol = ((d < 64) ? V0 : V1) + (d & 7) * 2;
            int off[8];
#pragma unroll
            for (int kk = 0; kk < 8; kk++) off[kk] = kk * 128 + ((cc ^ kk) << 4);
            const float *pb0 = ps + hq * HPT;
            for (int j0 = 0; j0 < cnt; j0 += 8) {
                const uint8_t *vb = vcol + j0 * 128;
                const float *pb = pb0 + j0 * G;
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    if (j0 + kk < cnt) {
                        const float2 vf = h2f2_fma(*reinterpret_cast<const uint32_t *>(vb + off[kk]));
                        if constexpr (PAIRS) {
                            const f32x2 *pp = reinterpret_cast<const f32x2 *>(pb + kk * G);
                            const f32x2 vx = pk2(vf.x, vf.x), vy = pk2(vf.y, vf.y);
#pragma unroll
                            for (int j = 0; j < NP; j++) {
                                const f32x2 pj = pp[j];
                                a0[j] = ffma2(pj, vx, a0[j]);
                                a1[j] = ffma2(pj, vy, a1[j]);
                            }
                        } else {
#pragma unroll
                            for (int h = 0; h < HPT; h++) {
                                const float pj = pb[kk * G + h];
                                s0[h] = fmaf(pj, vf.x, s0[h]);
                                s1[h] = fmaf(pj, vf.y, s1[h]);
                            }
                        }
                    }
                }
            }
            if constexpr (PAIRS) {
#pragma unroll
                for (int j = 0; j < NP; j++) {
                    const float2 x = upk2(a0[j]), y = upk2(a1[j]);
                    acc0[2 * j] = x.x;
                    acc0[2 * j + 1] = x.y;
                    acc1[2 * j] = y.x;
                    acc1[2 * j + 1] = y.y;
                }
            } else {
#pragma unroll
                for (int h = 0; h < HPT; h++) {
                    acc0[h] = s0[h];
                    acc1[h] = s1[h];
                }
            }
        }
        __syncthreads();  // V is no longer read: the next item's V pages may land
        if (warp == 0 && i + 1 < u1) issue(1);
        v_issued += i + 1 < u1;
        const int d = 2 * dp;
        if (nc == 1) {
#pragma unroll
            for (int h = 0; h < HPT; h++) {
                const int head = hq * HPT + h;
                const float f = bt_exp(__fsub_rn(s_m[head], s_m[head]));
                const float L = fmaf(s_l[head], f, 0.0f);
                float *o = p.out + (long long)t * QW + (g * G + head) * D + d;
                o[0] = __fdiv_rn(fmaf(acc0[h], f, 0.0f), L);
                o[1] = __fdiv_rn(fmaf(acc1[h], f, 0.0f), L);
            }
        } else {
            const long long pbase = (((long long)t * p.HK + g) * p.max_chunks) * G * ATTN_PART_ROW;
#pragma unroll
            for (int h = 0; h < HPT; h++) {
                const int head = hq * HPT + h;
                float *pp = p.part + pbase + ((long long)c * G + head) * ATTN_PART_ROW;
                *reinterpret_cast<float2 *>(pp + d) = make_float2(acc0[h], acc1[h]);
                if (dp == 0) {
                    pp[D] = s_m[head];
                    pp[D + 1] = s_l[head];
                }
            }
        }
        if (!ok) break;
    }
    if (!ok && tid == 0) {
        // a wait ran out: give every copy requested (at most one per buffer beyond those
        // consumed) one more bounded wait before the CTA leaves
        for (int q = 0; q < 2; q++) {
            const int n = q ? v_issued : k_issued;
            mbar_wait(&bars[q], (n - 1) & 1, nullptr);
        }
    }
}

// ====================================================================== attention, one warp pair per chunk
// Batched steps. CTAs of two warp pairs, four CTAs per SM, walk groups (token t, kv head g, two
// consecutive 128-key chunks), CTA b a contiguous range of them; pair pi takes chunk 2 cg + pi of
// group (t, g, cg), and warp hp of the pair takes heads hp*G/2 .. (hp+1)*G/2 - 1. The CTA shares
// the group's q (f16). A pair streams its chunk's K, then V, in pieces of 32 keys (8 KB: two
// 16-row pages in two 128-byte-swizzled column halves) through its own two-slot TMA ring; per
// piece both warps wait for it, meet at a pair barrier (so the slot of the piece before is free)
// and warp 0 requests the next piece -- also the first piece of the pair's next chunk. Lane l
// owns keys l, l + 32, l + 64, l + 96 for the scores (per head a sequential fmaf dot over d;
// heads in f32x2 pairs against each k value converted twice into both halves of a pair) and
// dims 4l .. 4l + 3 for P*V (the warp's heads; dims in f32x2 pairs against probabilities
// stored twice, so a pair operand is one load; full 32-key pieces run without per-key tests). The arithmetic is attn_kernel's (C8): piece j's keys sit on the lanes as
// warp j's keys do there, so the 32-key butterfly sums are the same, and every score and P*V
// sum runs in the same order.
constexpr int AW_PAIRS = 2, AW_WARPS = 2 * AW_PAIRS;
constexpr int AW_PIECE_BYTES = 32 * 256;  // 32 keys of one kv head, f16

size_t attn_warp_smem_bytes(int G, int T) {
    return 1024 + (size_t)AW_PAIRS * 2 * AW_PIECE_BYTES + (size_t)AW_WARPS * ATTN_CHUNK * (G / 2) * 8 +
           (size_t)128 * G * 4 + AW_PAIRS * 2 * 8 + (size_t)(3 * T + 1) * 4 + 64;
}

// both halves of w as one f32x2 of exact f32 values (FMA pipe)
__device__ __forceinline__ f32x2 h2_f32x2(uint32_t w) {
    f32x2 r;
    asm("{\n\t.reg .b16 l, h;\n\t.reg .f32 a, b;\n\tmov.b32 {l, h}, %1;\n\tadd.rn.f32.f16 a, l, %2;\n\t"
        "add.rn.f32.f16 b, h, %2;\n\tmov.b64 %0, {a, b};\n\t}"
        : "=l"(r)
        : "r"(w), "f"(-0.0f));
    return r;
}
// barrier of one warp pair (64 threads, named barrier 1 + pair) that also ANDs v over it
__device__ __forceinline__ bool pair_sync_and(int pair, bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, %2, 64, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((int)v), "r"(1 + pair)
        : "memory");
    return r != 0;
}

template <int G>
__global__ void __launch_bounds__(AW_WARPS * 32, 4)
    attn_warp_kernel(const __grid_constant__ AttnArgs p, const __grid_constant__ CUtensorMap tmap) {
    constexpr int D = 128, CH = ATTN_CHUNK, HH = G / 2;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, pair = warp >> 1, hp = warp & 1;
    uint8_t *ring = smem + pair * 2 * AW_PIECE_BYTES;                                  // [2 slots][piece]
    float *fbase = reinterpret_cast<float *>(smem + AW_PAIRS * 2 * AW_PIECE_BYTES);
    float *pb = fbase + warp * CH * HH * 2;                                            // [CH][HH][2] P twice
    float *qf = fbase + AW_WARPS * CH * HH * 2;                                        // [D][G] q's f16 rounding, as f32
    uint64_t *bars = reinterpret_cast<uint64_t *>(qf + D * G);                         // [pairs][2]
    int *pre = reinterpret_cast<int *>(bars + AW_PAIRS * 2);                           // [T + 1] first group of t
    int *pos_s = pre + p.T + 1, *seq_s = pos_s + p.T;                                  // [T] each
    uint64_t *wb = bars + pair * 2;
    if (hp == 0 && lane == 0) {
        mbar_init(&wb[0], 1);
        mbar_init(&wb[1], 1);
        fence_mbar_init();
    }
    pdl_wait();
    if (warp == 0) {  // groups per token: HK * ceil(chunks / 2); exclusive prefix over the tokens
        int run = 0;
        for (int t0 = 0; t0 < p.T; t0 += 32) {
            const int t = t0 + lane;
            const int pos = t < p.T ? p.pos_of[t] : 0;
            const int n = t < p.T ? p.HK * (((pos + CH) / CH + AW_PAIRS - 1) / AW_PAIRS) : 0;
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += v;
            }
            if (t < p.T) {
                pre[t] = run + incl - n;
                pos_s[t] = pos;
                seq_s[t] = p.seq_of[t];
            }
            run += __shfl_sync(FULL, incl, 31);
        }
        if (lane == 0) pre[p.T] = run;
    }
    __syncthreads();
    pdl_trigger();
    const int NG = pre[p.T];
    const int g0 = (int)((long long)blockIdx.x * NG / gridDim.x);
    const int g1 = (int)((long long)(blockIdx.x + 1) * NG / gridDim.x);
    if (g0 >= g1) return;
    if (warp == 0 && lane == 0) prefetch_tmap(&tmap);

    // group i -> token t (the last with pre[t] <= i), kv head g, chunk group cg
    auto decode = [&](int i, int &t, int &g, int &cg) {
        int lo = 0, hi = p.T - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= i) lo = mid;
            else hi = mid - 1;
        }
        t = lo;
        const int ngc = ((pos_s[t] + CH) / CH + AW_PAIRS - 1) / AW_PAIRS, r = i - pre[t];
        g = r / ngc;
        cg = r - g * ngc;
    };
    // this pair's chunk in group i: chunk c of (t, g) with nk keys, or none
    struct Item {
        int grp, t, g, c, nk, cnt, np;
    };
    auto item_at = [&](int i, Item &it) -> bool {
        int t, g, cg;
        decode(i, t, g, cg);
        const int nk = pos_s[t] + 1, c = cg * AW_PAIRS + pair;
        if (c * CH >= nk) return false;
        it.grp = i;
        it.t = t;
        it.g = g;
        it.c = c;
        it.nk = nk;
        it.cnt = nk - c * CH < CH ? nk - c * CH : CH;
        it.np = (it.cnt + 31) >> 5;
        return true;
    };
    auto next_item = [&](int from, Item &it) -> bool {
        for (int i = from; i < g1; i++)
            if (item_at(i, it)) return true;
        return false;
    };
    // lane < 8: block id of page `lane` of the item's chunk (pages past the keys are not read)
    auto load_pages = [&](const Item &it) -> int {
        const int pg = it.c * (CH / 16) + lane;
        return hp == 0 && lane < 8 && pg * 16 < it.nk ? p.block_table[seq_s[it.t] * p.max_blocks + pg] : 0;
    };
    // (warp 0 of the pair) piece q of item it (K pieces 0 .. np-1, then V pieces) into slot `slot`
    auto issue = [&](int slot, const Item &it, int q, int pages) {
        const int kv = q >= it.np ? 1 : 0, j = kv ? q - it.np : q;
        const int keys = it.cnt - 32 * j < 32 ? it.cnt - 32 * j : 32;
        const int npg = (keys + 15) >> 4;
        const int blk = __shfl_sync(FULL, pages, (2 * j + (lane >> 1)) & 7);
        if (lane == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(&wb[slot], npg * 4096);
        }
        __syncwarp();
        if (lane < 2 * npg) {
            const int row = (int)(((((long long)p.layer * p.n_blocks + blk) * 2 + kv) * p.HK + it.g) * 16);
            tma_load_2d(ring + slot * AW_PIECE_BYTES + (lane & 1) * 4096 + (lane >> 1) * 2048, &tmap, (lane & 1) * 64,
                        row, &wb[slot]);
        }
    };

    const int QW = p.H * D;
    const float NEG_INF = -__int_as_float(0x7f800000);
    Item cur, nxt;
    bool have = next_item(g0, cur);
    int pg_cur = have ? load_pages(cur) : 0;
    bool have_n = have && next_item(cur.grp + 1, nxt);
    int pg_nxt = have_n ? load_pages(nxt) : 0;
    int issued = 0, pc = 0;  // pieces requested and taken by this pair (piece k: slot k & 1)
    if (have && hp == 0) issue(0, cur, 0, pg_cur);
    issued = have ? 1 : 0;
    bool ok = true;
    int cur_tg = -1;
    // piece q of the current item: wait for it; at the pair barrier both warps are past the
    // piece before, so warp 0 may refill that slot with the piece after this one
    auto take = [&](int q) -> bool {
        const bool landed = mbar_wait(&wb[pc & 1], (pc >> 1) & 1, p.err);
        if (!pair_sync_and(pair, landed)) return false;
        if (q + 1 < 2 * cur.np) {
            if (hp == 0) issue(issued & 1, cur, q + 1, pg_cur);
            issued++;
        } else if (have_n) {
            if (hp == 0) issue(issued & 1, nxt, 0, pg_nxt);
            issued++;
        }
        return true;
    };
    for (int i = g0; i < g1; i++) {
        int t, g, cg;
        decode(i, t, g, cg);
        if (t * p.HK + g != cur_tg) {  // every warp is past its scores of the previous (t, g)
            __syncthreads();
            cur_tg = t * p.HK + g;
            for (int x = tid; x < D * G; x += AW_WARPS * 32) {
                const int h = x / D, d = x % D;
                qf[d * G + h] = __half2float(__float2half_rn(p.q[(long long)t * QW + (g * G + h) * D + d]));
            }
            __syncthreads();
        }
        if (!ok || !have || cur.grp != i) continue;
        // ---- scores, piece by piece: lane = key 32 j + lane, this warp's HH heads
        float sc[4][HH];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (j < cur.np) {
                if (!take(j)) {
                    ok = false;
                    break;
                }
                // heads in f32x2 pairs: (s_h, s_h+1) += (q_h, q_h+1) * (k_d, k_d), d in order (C8:
                // each an fmaf of two f16 values); k_d converted twice into both halves of its pair
                constexpr int NP = (HH + 1) / 2;
                f32x2 acc[NP];
#pragma unroll
                for (int jp = 0; jp < NP; jp++) acc[jp] = 0ull;
                const uint8_t *krow = ring + (pc & 1) * AW_PIECE_BYTES + lane * 128;
                const int ksw = lane & 7;
                const float *qb = qf + hp * HH;
#pragma unroll 2
                for (int c16 = 0; c16 < 16; c16++) {
                    const uint4 w =
                        *reinterpret_cast<const uint4 *>((c16 < 8 ? krow : krow + 4096) + (((c16 & 7) ^ ksw) << 4));
                    const uint32_t kw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e2 = 0; e2 < 4; e2++) {
                        f32x2 kb[2];
                        h2_bcast2(kw[e2], kb[0], kb[1]);
#pragma unroll
                        for (int hl = 0; hl < 2; hl++) {
                            const int d = c16 * 8 + 2 * e2 + hl;
                            if constexpr (HH % 2 == 0) {
                                const f32x2 *qd = reinterpret_cast<const f32x2 *>(qb + d * G);
#pragma unroll
                                for (int jp = 0; jp < NP; jp++) acc[jp] = ffma2(qd[jp], kb[hl], acc[jp]);
                            } else {  // odd head count: the last pair's upper half is unused
#pragma unroll
                                for (int jp = 0; jp < NP; jp++) {
                                    const float q0 = qb[d * G + 2 * jp], q1 = 2 * jp + 1 < HH ? qb[d * G + 2 * jp + 1] : 0.0f;
                                    acc[jp] = ffma2(pk2(q0, q1), kb[hl], acc[jp]);
                                }
                            }
                        }
                    }
                }
                float accs[2 * NP];
#pragma unroll
                for (int jp = 0; jp < NP; jp++) {
                    const float2 v = upk2(acc[jp]);
                    accs[2 * jp] = v.x;
                    accs[2 * jp + 1] = v.y;
                }
                const bool valid = 32 * j + lane < cur.cnt;
#pragma unroll
                for (int h = 0; h < HH; h++) sc[j][h] = valid ? __fmul_rn(accs[h], p.scale) : NEG_INF;
                pc++;
            } else {
#pragma unroll
                for (int h = 0; h < HH; h++) sc[j][h] = NEG_INF;
            }
        }
        if (!ok) continue;
        // ---- softmax over the chunk: max, p = exp(s - m), l = the four 32-key butterfly sums in order
        float m[HH], l[HH];
#pragma unroll
        for (int h = 0; h < HH; h++) {
            const float x = fmaxf(fmaxf(sc[0][h], sc[1][h]), fmaxf(sc[2][h], sc[3][h]));
            m[h] = warp_max(x);
            l[h] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const bool valid = 32 * j + lane < cur.cnt;
            float pr[HH];
#pragma unroll
            for (int h = 0; h < HH; h++) {
                pr[h] = valid ? bt_exp(__fsub_rn(sc[j][h], m[h])) : 0.0f;
                l[h] = __fadd_rn(l[h], butterfly_sum(pr[h]));
            }
            if (j < cur.np) {
                f32x2 *prow = reinterpret_cast<f32x2 *>(pb + (32 * j + lane) * HH * 2);
#pragma unroll
                for (int h = 0; h < HH; h++) prow[h] = pk2(pr[h], pr[h]);
            }
        }
        __syncwarp();
        // ---- P*V, piece by piece: lane = dims 4 lane .. 4 lane + 3, keys in order
        f32x2 o01[HH], o23[HH];
#pragma unroll
        for (int h = 0; h < HH; h++) o01[h] = o23[h] = 0ull;
        const int vhalf = lane < 16 ? 0 : 4096, vcc = (lane & 15) >> 1, vsub = (lane & 1) * 8;
#pragma unroll 1
        for (int j = 0; j < cur.np; j++) {
            if (!take(cur.np + j)) {
                ok = false;
                break;
            }
            const uint8_t *vb = ring + (pc & 1) * AW_PIECE_BYTES + vhalf + vsub;
            const int kmax = cur.cnt - 32 * j < 32 ? cur.cnt - 32 * j : 32;
            const float *pj = pb + 32 * j * HH * 2;
            auto pv_key = [&](int kk) {
                const uint2 v = *reinterpret_cast<const uint2 *>(vb + kk * 128 + ((vcc ^ (kk & 7)) << 4));
                const f32x2 v01 = h2_f32x2(v.x), v23 = h2_f32x2(v.y);
                const f32x2 *pr = reinterpret_cast<const f32x2 *>(pj + kk * HH * 2);  // (p_h, p_h)
#pragma unroll
                for (int h = 0; h < HH; h++) {
                    const f32x2 ph = pr[h];
                    o01[h] = ffma2(ph, v01, o01[h]);
                    o23[h] = ffma2(ph, v23, o23[h]);
                }
            };
            if (kmax == 32) {
#pragma unroll 8
                for (int kk = 0; kk < 32; kk++) pv_key(kk);
            } else {
#pragma unroll 1
                for (int kk = 0; kk < kmax; kk++) pv_key(kk);
            }
            pc++;
        }
        if (!ok) continue;
        // ---- the chunk's partial (acc, m, l), or the output when the context is one chunk
        const int nc = (cur.nk + CH - 1) / CH;
#pragma unroll
        for (int hh = 0; hh < HH; hh++) {
            const int h = hp * HH + hh;
            const float2 a01 = upk2(o01[hh]), a23 = upk2(o23[hh]);
            if (nc == 1) {
                const float f = bt_exp(__fsub_rn(m[hh], m[hh]));
                const float L = fmaf(l[hh], f, 0.0f);
                float4 o;
                o.x = __fdiv_rn(fmaf(a01.x, f, 0.0f), L);
                o.y = __fdiv_rn(fmaf(a01.y, f, 0.0f), L);
                o.z = __fdiv_rn(fmaf(a23.x, f, 0.0f), L);
                o.w = __fdiv_rn(fmaf(a23.y, f, 0.0f), L);
                *reinterpret_cast<float4 *>(p.out + (long long)cur.t * QW + (cur.g * G + h) * D + 4 * lane) = o;
            } else {
                float *pp = p.part + ((((long long)cur.t * p.HK + cur.g) * p.max_chunks + cur.c) * G + h) * ATTN_PART_ROW;
                *reinterpret_cast<float4 *>(pp + 4 * lane) = make_float4(a01.x, a01.y, a23.x, a23.y);
                if (lane == 0) {
                    pp[D] = m[hh];
                    pp[D + 1] = l[hh];
                }
            }
        }
        // ---- the next item: its first piece is already requested
        cur = nxt;
        pg_cur = pg_nxt;
        have = have_n;
        have_n = have && next_item(cur.grp + 1, nxt);
        pg_nxt = have_n ? load_pages(nxt) : 0;
    }
    if (!ok && hp == 0 && lane == 0) {
        // a wait ran out: give the copies still requested one more bounded wait before leaving
        for (int s2 = 0; s2 < 2; s2++) {
            long long last = -1;
            for (long long k = issued - 1; k >= 0 && k >= issued - 2; k--)
                if ((k & 1) == s2) last = k;
            if (last >= pc) mbar_wait(&wb[s2], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
}

template <int G>
static cudaError_t launch_attn_warp_g(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl) {
    // a.n_cta = 4 CTAs per SM; fewer when the token tables make the CTA too large for four
    const size_t smem = attn_warp_smem_bytes(G, a.T);
    int per = 0;
    cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, attn_warp_kernel<G>, AW_WARPS * 32, smem);
    if (oe != cudaSuccess) return oe;
    if (per < 1) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(per < 4 ? a.n_cta / 4 * per : a.n_cta);
    cfg.blockDim = dim3(AW_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_warp_kernel<G>, a, tmap);
}

// grid (H, T), 128 threads: merges the chunk partials of one query head in chunk order
// (C8): M = max m_c, f_c = exp(m_c - M), L = fmaf(l_c, f_c, L), O = fmaf(acc_c, f_c, O).
__global__ void __launch_bounds__(128) attn_combine_kernel(const __grid_constant__ AttnArgs p) {
    extern __shared__ float cbuf[];  // m[nc], l[nc], f[nc]
    __shared__ float s_M, s_L;
    const int hd = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    const int pos = p.pos_of[t];
    const int nc = (pos + 1 + ATTN_CHUNK - 1) / ATTN_CHUNK;
    if (nc == 1) return;  // the attention kernel finalised this token
    const int G = p.G, g = hd / G, h = hd % G, D = 128;
    const float *part = p.part + (((long long)t * p.HK + g) * p.max_chunks) * G * ATTN_PART_ROW + (long long)h * ATTN_PART_ROW;
    const long long cstride = (long long)G * ATTN_PART_ROW;
    float *cm = cbuf, *cl = cbuf + nc, *cf = cbuf + 2 * nc;
    for (int c = d; c < nc; c += blockDim.x) {
        cm[c] = part[c * cstride + D];
        cl[c] = part[c * cstride + D + 1];
    }
    __syncthreads();
    if (d < 32) {  // M (order-free)
        float m = -__int_as_float(0x7f800000);
        for (int c = d; c < nc; c += 32) m = fmaxf(m, cm[c]);
        m = warp_max(m);
        if (d == 0) s_M = m;
    }
    __syncthreads();
    for (int c = d; c < nc; c += blockDim.x) cf[c] = bt_exp(__fsub_rn(cm[c], s_M));
    __syncthreads();
    if (d == 0) {
        float L = 0.0f;
        for (int c = 0; c < nc; c++) L = fmaf(cl[c], cf[c], L);
        s_L = L;
    }
    float O = 0.0f;
    const float *pa = part + d;
    int c = 0;
    for (; c + 16 <= nc; c += 16) {
        float a[16];
#pragma unroll
        for (int k = 0; k < 16; k++) a[k] = pa[(long long)(c + k) * cstride];
#pragma unroll
        for (int k = 0; k < 16; k++) O = fmaf(a[k], cf[c + k], O);
    }
    for (; c < nc; c++) O = fmaf(pa[(long long)c * cstride], cf[c], O);
    __syncthreads();
    p.out[(long long)t * p.H * D + hd * D + d] = __fdiv_rn(O, s_L);
}

template <int G>
static cudaError_t launch_attn_g(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_cta);
    cfg.blockDim = dim3(ATTN_THREADS);
    cfg.dynamicSmemBytes = attn_smem_bytes(G, a.T);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_kernel<G>, a, tmap);
}

cudaError_t launch_attn_warp(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl) {
    cudaError_t e;
    switch (a.G) {
    case 2: e = launch_attn_warp_g<2>(a, tmap, st, pdl); break;
    case 4: e = launch_attn_warp_g<4>(a, tmap, st, pdl); break;
    case 6: e = launch_attn_warp_g<6>(a, tmap, st, pdl); break;
    case 8: e = launch_attn_warp_g<8>(a, tmap, st, pdl); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return launch_ex(attn_combine_kernel, dim3(a.H, a.T), dim3(128), (size_t)3 * a.max_chunks * 4, st, pdl, a);
}

cudaError_t launch_attn(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl) {
    cudaError_t e;
    switch (a.G) {
    case 2: e = launch_attn_g<2>(a, tmap, st, pdl); break;
    case 4: e = launch_attn_g<4>(a, tmap, st, pdl); break;
    case 6: e = launch_attn_g<6>(a, tmap, st, pdl); break;
    case 8: e = launch_attn_g<8>(a, tmap, st, pdl); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return launch_ex(attn_combine_kernel, dim3(a.H, a.T), dim3(128), (size_t)3 * a.max_chunks * 4, st, pdl, a);
}

// ====================================================================== embedding and step end
__global__ void __launch_bounds__(256) embed_kernel(const __grid_constant__ EmbedArgs p) {
    const int t = blockIdx.x;
    pdl_wait();
    const int tok = p.tokens[t];
    if (threadIdx.x == 0) p.pos_of[t] = p.dev_len[p.seq_of[t]] + p.local_idx[t];
    pdl_trigger();
    const bool ok = tok >= 0 && tok < p.V;
    if (!ok && threadIdx.x == 0) atomicOr(p.err, ERR_BAD_INDEX);
    const int nsb = p.E / 256;
    const int bb = qk_block_bytes(p.type);
    const uint8_t *row = p.table + (long long)(ok ? tok : 0) * nsb * bb;
    float *x = p.x + (long long)t * p.E;
    for (int i = threadIdx.x; i < p.E; i += blockDim.x) {
        const uint8_t *blk = row + (i / 256) * bb;
        const int v = i % 256;
        float y;
        if (p.type == T_Q4_K) {
            float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t *sc = blk + 4, *qs = blk + 16;
            int j = v / 32, gidx = v / 64, hi = (v / 32) & 1, l = v % 32;
            int scj, mj;
            if (j < 4) {
                scj = sc[j] & 63;
                mj = sc[j + 4] & 63;
            } else {
                scj = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                mj = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
            }
            int q = hi ? (qs[32 * gidx + l] >> 4) : (qs[32 * gidx + l] & 0xF);
            y = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)scj), (float)q), __fmul_rn(dmin, (float)mj));
        } else {
            float d = f16_bits_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
            const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
            int n = v / 128, r = v % 128, quad = r / 32, l = r % 32;
            int lo = quad == 0 ? (blk[64 * n + l] & 0xF)
                               : quad == 1 ? (blk[64 * n + 32 + l] & 0xF)
                                           : quad == 2 ? (blk[64 * n + l] >> 4) : (blk[64 * n + 32 + l] >> 4);
            int hi2 = (blk[128 + 32 * n + l] >> (2 * quad)) & 3;
            y = __fmul_rn(__fmul_rn(d, (float)sc[v / 16]), (float)((lo | (hi2 << 4)) - 32));
        }
        x[i] = ok ? y : 0.0f;
    }
}

cudaError_t launch_embed(const EmbedArgs &a, cudaStream_t st, bool pdl) {
    return launch_ex(embed_kernel, dim3(a.T), dim3(256), 0, st, pdl, a);
}

// grid (n_seqs), 32 threads: the argmax of each sequence's logits was folded by the output
// GEMV into a 64-bit (total_cmp key, row) maximum -- the last maximum wins, as max_by does
// (sample.rs:928-935). Read it, reset the slot for the next step, advance the sequence's
// device length (advance_by) and, for the greedy loop, feed the token back.
__global__ void __launch_bounds__(32) step_end_kernel(const __grid_constant__ StepEndArgs p) {
    const int s = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    const int lrow = p.logit_row ? p.logit_row[s] : -1;
    p.dev_len[p.seq_ids[s]] += p.n_tok[s];
    if (lrow >= 0) {
        const unsigned long long packed = p.amax[lrow];
        p.amax[lrow] = 0ull;
        const int bi = (int)(packed & 0xffffffffull);
        p.next_token[lrow] = bi;
        if (p.tokens_buf) p.tokens_buf[lrow] = bi;
        if (p.gen_out) {
            int k = p.gen_count[lrow]++;
            p.gen_out[(long long)k * p.n_out + lrow] = bi;
        }
    }
}

cudaError_t launch_step_end(const StepEndArgs &a, cudaStream_t st, bool pdl) {
    return launch_ex(step_end_kernel, dim3(a.n_seqs), dim3(32), 0, st, pdl, a);
}

// Large dynamic shared memory must be enabled per kernel and per device before the first
// launch (and outside any stream capture): the engine calls this when it binds a device.
cudaError_t init_kernel_attributes() {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev))) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
    const void *kerns[] = {(const void *)kq_rows_kernel<GEMV_WARPS>, (const void *)gateup_kernel<GEMV_WARPS>,
                           (const void *)down_kernel<GEMV_WARPS>, (const void *)gateup_grouped_kernel<GEMV_WARPS>,
                           (const void *)down_grouped_kernel<GEMV_WARPS>, (const void *)group_kernel,
                           (const void *)attn_kernel<2>,
                           (const void *)attn_kernel<4>,          (const void *)attn_kernel<6>,
                           (const void *)attn_kernel<8>,          (const void *)attn_warp_kernel<2>,
                           (const void *)attn_warp_kernel<4>,     (const void *)attn_warp_kernel<6>,
                           (const void *)attn_warp_kernel<8>};
    for (const void *k : kerns) {
        cudaFuncAttributes fa;
        if ((e = cudaFuncGetAttributes(&fa, k))) return e;
        int dyn = optin - (int)fa.sharedSizeBytes;
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn))) return e;
    }
    return init_mma_attributes();
}

int max_dynamic_smem() {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return optin - 2048;  // headroom for the kernels' static shared memory
}

// ====================================================================== one-off launchers
cudaError_t launch_repack(int type, const uint8_t *src, long long rows, long long cols, int rpt, uint8_t *dst,
                          long long n_mats, cudaStream_t st) {
    TileGeom g = tile_geom(type, rows, cols, rpt);
    long long total = g.n_tiles * g.S * (qk_chunks(type) + 1) * n_mats;
    long long blocks = (total + 255) / 256;
    if (blocks > 65535LL * 8) blocks = 65535LL * 8;
    repack_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, src, rows, cols, rpt, dst, n_mats);
    return cudaGetLastError();
}

cudaError_t launch_dequant_tiled(int type, const uint8_t *tiled, long long rows, long long cols, int rpt, float *out,
                                 cudaStream_t st) {
    long long n = rows * (cols / 256);
    long long blocks = (n + 127) / 128;
    if (blocks > 65535) blocks = 65535;
    dequant_tiled_kernel<<<(unsigned)blocks, 128, 0, st>>>(type, tiled, rows, cols, rpt, out);
    return cudaGetLastError();
}

cudaError_t launch_synth(int type, uint64_t key, long long n_elems, float mean, float scale, uint8_t *out,
                         cudaStream_t st) {
    long long nb = (n_elems + 255) / 256;
    long long blocks = (nb + 127) / 128;
    if (blocks > 65535LL * 4) blocks = 65535LL * 4;
    if (blocks < 1) blocks = 1;
    synth_kernel<<<(unsigned)blocks, 128, 0, st>>>(type, key, n_elems, mean, scale, out);
    return cudaGetLastError();
}


// ====================================================================== KV gather / scatter, untile
// Copies positions [p0, p0+n) of one sequence and layer between the paged pool and dense
// kv.rs-layout buffers ([pos][HK*D] f16 for k and for v). to_pool selects the direction.
__global__ void kv_copy_kernel(__half *pool, const int *__restrict__ table_row, int layer, int n_blocks, int HK, int D,
                               int p0, int n, __half *kbuf, __half *vbuf, int to_pool) {
    const long long per = 2LL * HK * D;
    const long long total = (long long)n * per;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int pi = (int)(i / per);
        int r = (int)(i % per);
        int kvsel = r / (HK * D), e = r % (HK * D), head = e / D, d = e % D;
        int pos = p0 + pi;
        int blk = table_row[pos / 16];
        long long row = ((((long long)layer * n_blocks + blk) * 2 + kvsel) * HK + head) * 16 + pos % 16;
        __half *pp = pool + row * D + d;
        __half *bb = (kvsel ? vbuf : kbuf) + (long long)pi * HK * D + e;
        if (to_pool) *pp = *bb;
        else *bb = *pp;
    }
}

cudaError_t launch_kv_copy(__half *pool, const int *table_row, int layer, int n_blocks, int HK, int D, int p0, int n,
                           __half *kbuf, __half *vbuf, int to_pool, cudaStream_t st) {
    long long total = (long long)n * 2 * HK * D;
    if (total <= 0) return cudaSuccess;
    long long blocks = (total + 255) / 256;
    if (blocks > 65535LL * 4) blocks = 65535LL * 4;
    kv_copy_kernel<<<(unsigned)blocks, 256, 0, st>>>(pool, table_row, layer, n_blocks, HK, D, p0, n, kbuf, vbuf, to_pool);
    return cudaGetLastError();
}

// Inverse of repack_kernel: tiled layout back to GGUF row-major bytes.
__global__ void untile_kernel(int type, const uint8_t *__restrict__ tiled, long long rows, long long cols, int rpt,
                              uint8_t *__restrict__ dst, long long n_mats) {
    TileGeom g = tile_geom(type, rows, cols, rpt);
    const int bb = qk_block_bytes(type);
    const long long nsb_all = n_mats * rows * g.nsb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nsb_all;
         i += (long long)gridDim.x * blockDim.x) {
        long long mat = i / (rows * g.nsb), r = i % (rows * g.nsb);
        long long row = r / g.nsb;
        int b = (int)(r % g.nsb);
        long long tile = row / rpt;
        int s = (int)(row % rpt) * g.nsb + b;
        const uint8_t *tb = tiled + (mat * g.n_tiles + tile) * (long long)g.tile_bytes;
        uint8_t *out = dst + i * bb;
        for (int c = 0; c < qk_chunks(type); c++)
            for (int k = 0; k < 16; k++) out[c * 16 + k] = tb[(long long)c * g.S * 16 + s * 16 + k];
        if (type == T_Q6_K) {
            out[208] = tb[13 * g.S * 16 + s * 2];
            out[209] = tb[13 * g.S * 16 + s * 2 + 1];
        }
    }
}

cudaError_t launch_untile(int type, const uint8_t *tiled, long long rows, long long cols, int rpt, uint8_t *dst,
                          long long n_mats, cudaStream_t st) {
    long long n = n_mats * rows * (cols / 256);
    long long blocks = (n + 127) / 128;
    if (blocks > 65535LL * 4) blocks = 65535LL * 4;
    untile_kernel<<<(unsigned)blocks, 128, 0, st>>>(type, tiled, rows, cols, rpt, dst, n_mats);
    return cudaGetLastError();
}

}  // namespace bt
