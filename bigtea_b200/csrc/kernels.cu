// kernels.cu -- the sm_100a kernels of the decode-step layer.
//
// Reference call sites each kernel replaces (Chaos tree, core/arch/src/stream.rs unless noted):
//   embed_kernel      get_rows on token_embd                           2192-2231
//   gemv_kernel       rms_norm+mul then mul_mat (q/k/v, attn_output, output head)
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

// ====================================================================== activation staging
// C3 over one 256-value block held 8 values per lane (lane l: elements 8l..8l+7).
__device__ __forceinline__ void quantize_block_warp(const float v[8], ActBlock *dst, int lane) {
    float am = 0.0f;
    int ai = 1 << 30;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float av = fabsf(v[i]);
        if (av > am) {
            am = av;
            ai = lane * 8 + i;
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        float om = __shfl_xor_sync(FULL, am, o);
        int oi = __shfl_xor_sync(FULL, ai, o);
        if (om > am || (om == am && oi < ai)) {
            am = om;
            ai = oi;
        }
    }
    int sel = ai & 7;
    float mine = v[0];
#pragma unroll
    for (int i = 1; i < 8; i++)
        if (sel == i) mine = v[i];
    float mx = __shfl_sync(FULL, mine, (ai >> 3) & 31);
    uint32_t w0 = 0, w1 = 0;
    int s8 = 0;
    float d = 0.0f;
    if (am != 0.0f) {
        float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int q = (int)rintf(__fmul_rn(iscale, v[i]));
            q = q > 127 ? 127 : q;
            s8 += q;
            uint32_t b = (uint32_t)(q & 0xff);
            if (i < 4) w0 |= b << (8 * i);
            else w1 |= b << (8 * (i - 4));
        }
        d = __fdiv_rn(1.0f, iscale);
    }
    *reinterpret_cast<uint2 *>(dst->qs + lane * 8) = make_uint2(w0, w1);
    int s16 = s8 + __shfl_xor_sync(FULL, s8, 1);
    int s32 = s16 + __shfl_xor_sync(FULL, s16, 2);
    if ((lane & 3) == 0) dst->bs32[lane >> 2] = s32;
    if (lane == 0) dst->d = d;
}

// Stage T activation rows (optionally RMS-normalised, C6) as Q8_K blocks. All threads.
template <int NWARP>
__device__ void stage_activations(const float *x, long long x_stride, const int *x_rows, const float *norm_w,
                                  float eps, int K, int T, ActBlock *act, float *normS) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (norm_w) {
        for (int t = warp; t < T; t += NWARP) {
            const float *xt = x + (long long)(x_rows ? x_rows[t] : t) * x_stride;
            float acc = 0.0f;
            for (int i = lane; i < K; i += 32) acc = fmaf(xt[i], xt[i], acc);
            acc = butterfly_sum(acc);
            if (lane == 0) normS[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)K), eps)));
        }
        __syncthreads();
    }
    const int nsb = K / 256;
    for (int blk = warp; blk < T * nsb; blk += NWARP) {
        int t = blk / nsb, b = blk % nsb;
        const float *xt = x + (long long)(x_rows ? x_rows[t] : t) * x_stride + b * 256 + lane * 8;
        float v[8];
        float4 a0 = *reinterpret_cast<const float4 *>(xt), a1 = *reinterpret_cast<const float4 *>(xt + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        if (norm_w) {
            float s = normS[t];
            const float *w = norm_w + b * 256 + lane * 8;
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], s), w[i]);
        }
        quantize_block_warp(v, act + blk, lane);
    }
}

// ====================================================================== GEMV
// Persistent-style: the grid covers the SMs; CTA c owns a contiguous range of tiles; each
// warp streams its tiles through a private ring of `nst` shared-memory slots with 1-D TMA
// bulk copies (weights do not depend on the previous kernel, so the first slots are
// requested before griddepcontrol.wait), and lane s decodes slot s in registers.
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) gemv_kernel(const __grid_constant__ GemvArgs p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *normS = reinterpret_cast<float *>(smem + 512);
    ActBlock *act = reinterpret_cast<ActBlock *>(smem + 1024);
    const int nsbK = p.K / 256;
    const size_t act_bytes = (size_t)p.T * nsbK * sizeof(ActBlock);
    uint8_t *ring = smem + 1024 + ((act_bytes + 127) & ~(size_t)127);
    uint8_t *myring = ring + (size_t)warp * p.nst * p.slot_bytes;
    uint64_t *mybar = bars + warp * p.nst;

    const long long u0 = (long long)blockIdx.x * p.total_tiles / gridDim.x;
    const long long u1 = (long long)(blockIdx.x + 1) * p.total_tiles / gridDim.x;
    const int nmine = (u1 - u0 > warp) ? (int)((u1 - u0 - warp + NWARP - 1) / NWARP) : 0;

    auto seg_of = [&](long long u) -> int {
        int si = 0;
        if (p.nseg > 1 && u >= p.seg[1].tile0) si = 1;
        if (p.nseg > 2 && u >= p.seg[2].tile0) si = 2;
        return si;
    };
    auto issue = [&](int j) {
        long long u = u0 + warp + (long long)j * NWARP;
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
    stage_activations<NWARP>(p.x, p.x_stride, p.x_rows, p.norm_w, p.eps, p.K, p.T, act, normS);
    __syncthreads();
    pdl_trigger();

    int j = 0;
    for (; j < nmine; j++) {
        const int slot = j % p.nst;
        if (!__all_sync(FULL, mbar_wait(&mybar[slot], (j / p.nst) & 1, p.err))) break;
        const long long u = u0 + warp + (long long)j * NWARP;
        const GemvSeg &sg = p.seg[seg_of(u)];
        const uint8_t *tile = myring + (size_t)slot * p.slot_bytes;
        const long long tl = u - sg.tile0;
        const bool active = lane < sg.S;
        const int rit = active ? lane / sg.nsb : 0, b = active ? lane % sg.nsb : 0;
        const long long row = tl * sg.rpt + rit;
        const bool writer = active && b == 0 && row < sg.rows;
        for (int t = 0; t < p.T; t++) {
            float v = 0.0f;
            if (active) {
                const ActBlock &ab = act[t * nsbK + b];
                v = (sg.type == T_Q4_K) ? q4k_slot_dot(tile, sg.S, lane, ab) : q6k_slot_dot(tile, sg.S, lane, ab);
            }
            float acc = 0.0f;
            for (int b2 = 0; b2 < sg.nsb; b2++) {
                int srcl = rit * sg.nsb + b2;
                float o = __shfl_sync(FULL, v, srcl < 32 ? srcl : 31);
                acc = __fadd_rn(acc, o);
            }
            if (writer) {
                float r = acc;
                if (p.res) r = __fadd_rn(p.res[t * p.res_stride + sg.out_off + row], acc);
                p.y[t * p.y_stride + sg.out_off + row] = r;
            }
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
}

size_t gemv_smem_bytes(const GemvArgs &a) {
    size_t act = (size_t)a.T * (a.K / 256) * sizeof(ActBlock);
    return 1024 + ((act + 127) & ~(size_t)127) + (size_t)GEMV_WARPS * a.nst * a.slot_bytes;
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
    return launch_ex(gemv_kernel<GEMV_WARPS>, dim3(grid), dim3(GEMV_WARPS * 32), smem, st, pdl, a);
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

    auto issue = [&](int j) {
        long long u = u0 + warp + (long long)j * NWARP;
        int tile = (int)(u % p.g_n_tiles);
        long long tk = u / p.g_n_tiles;
        int e = p.sel_ids[tk];
        int slot = j % p.nst;
        uint8_t *dst = myring + (size_t)slot * p.slot_bytes;
        mbar_arrive_expect_tx(&mybar[slot], p.g_tile_bytes + p.u_tile_bytes);
        bulk_g2s(dst, p.gate + e * p.g_expert_bytes + (long long)tile * p.g_tile_bytes, p.g_tile_bytes, &mybar[slot]);
        bulk_g2s(dst + p.g_tile_bytes, p.up + e * p.u_expert_bytes + (long long)tile * p.u_tile_bytes, p.u_tile_bytes,
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
        float vg = 0.0f, vu = 0.0f;
        if (active) {
            const ActBlock &ab = act[t * nsb + b];
            vg = p.gtype == T_Q4_K ? q4k_slot_dot(gt, p.g_S, lane, ab) : q6k_slot_dot(gt, p.g_S, lane, ab);
            vu = p.utype == T_Q4_K ? q4k_slot_dot(ut, p.g_S, lane, ab) : q6k_slot_dot(ut, p.g_S, lane, ab);
        }
        float ag = 0.0f, au = 0.0f;
        for (int b2 = 0; b2 < nsb; b2++) {
            int srcl = rit * nsb + b2;
            srcl = srcl < 32 ? srcl : 31;
            ag = __fadd_rn(ag, __shfl_sync(FULL, vg, srcl));
            au = __fadd_rn(au, __shfl_sync(FULL, vu, srcl));
        }
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

    auto issue = [&](int j) {
        long long u = u0 + warp + (long long)j * NWARP;
        int row = (int)(u % p.E), t = (int)(u / p.E);
        int slot = j % p.nst;
        uint8_t *dst = myring + (size_t)slot * p.slot_bytes;
        mbar_arrive_expect_tx(&mybar[slot], p.K * p.d_tile_bytes);
        for (int k = 0; k < p.K; k++) {
            int e = p.sel_ids[t * p.K + k];
            bulk_g2s(dst + k * p.d_tile_bytes, p.down + e * p.d_expert_bytes + (long long)row * p.d_tile_bytes,
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
            p.x_out[(long long)t * p.E + row] = __fadd_rn(p.ffn_in[(long long)t * p.E + row], sum);
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

// ====================================================================== router
// grid (ceil(NE/rows_per_cta), T), 128 threads. Each CTA normalises the token (C6), computes
// its rows of the F32 router (C5); the last CTA of a token (atomic ticket) runs soft_max_ext
// and route(): stable descending order by total_cmp, top-K, renormalised over the selection.
__global__ void __launch_bounds__(128) router_kernel(const __grid_constant__ RouterArgs p) {
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
        float acc = 0.0f;
        for (int i = lane; i < p.E; i += 32) acc = fmaf(x[i], x[i], acc);
        acc = butterfly_sum(acc);
        if (lane == 0) s_norm = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)p.E), p.eps)));
    }
    __syncthreads();
    pdl_trigger();
    const float s = s_norm;
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < p.E; i += blockDim.x)
            p.fn_out[(long long)t * p.E + i] = __fmul_rn(__fmul_rn(x[i], s), p.norm_w[i]);
    const int r0 = blockIdx.x * p.rows_per_cta;
    for (int r = r0 + warp; r < r0 + p.rows_per_cta && r < p.NE; r += 4) {
        const float *wr = p.Wr + (long long)r * p.E;
        float acc = 0.0f;
        for (int i = lane; i < p.E; i += 32) acc = fmaf(wr[i], __fmul_rn(__fmul_rn(x[i], s), p.norm_w[i]), acc);
        acc = butterfly_sum(acc);
        if (lane == 0) p.logits[(long long)t * p.NE + r] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&p.cnt[t], 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (warp != 0) return;
    const float *lg = p.logits + (long long)t * p.NE;
    float m = -__int_as_float(0x7f800000);
    for (int i = lane; i < p.NE; i += 32) m = fmaxf(m, __ldcg(lg + i));
    m = warp_max(m);
    float acc = 0.0f;
    for (int i = lane; i < p.NE; i += 32) {
        float e = bt_exp(__fsub_rn(__ldcg(lg + i), m));
        s_prob[i] = e;
        acc = __fadd_rn(acc, e);
    }
    acc = butterfly_sum(acc);
    const float inv = __fdiv_rn(1.0f, acc);
    for (int i = lane; i < p.NE; i += 32) s_prob[i] = __fmul_rn(s_prob[i], inv);
    __syncwarp();
    for (int i = lane; i < p.NE; i += 32) {
        int ki = total_key(s_prob[i]);
        int rank = 0;
        for (int jj = 0; jj < p.NE; jj++) {
            int kj = total_key(s_prob[jj]);
            rank += (kj > ki) || (kj == ki && jj < i);
        }
        if (rank < p.K) {
            s_rank_id[rank] = i;
            s_rank_p[rank] = s_prob[i];
        }
    }
    __syncwarp();
    if (lane == 0) {
        float total = 0.0f;
        for (int r = 0; r < p.K; r++) total = __fadd_rn(total, s_rank_p[r]);
        int ids[MAX_K];
        float ws[MAX_K];
        for (int r = 0; r < p.K; r++) {
            float w = total > 0.0f ? __fdiv_rn(s_rank_p[r], total) : s_rank_p[r];
            ids[r] = s_rank_id[r];
            ws[r] = w;
            p.topk_ids[t * p.K + r] = ids[r];
            p.topk_w[t * p.K + r] = w;
        }
        for (int a = 1; a < p.K; a++)
            for (int b = a; b > 0 && ids[b - 1] > ids[b]; b--) {
                int ti = ids[b]; ids[b] = ids[b - 1]; ids[b - 1] = ti;
                float tw = ws[b]; ws[b] = ws[b - 1]; ws[b - 1] = tw;
            }
        for (int r = 0; r < p.K; r++) {
            p.sel_ids[t * p.K + r] = ids[r];
            p.sel_w[t * p.K + r] = ws[r];
        }
        p.cnt[t] = 0;
    }
}

cudaError_t launch_router(const RouterArgs &a, cudaStream_t st, bool pdl) {
    dim3 grid((a.NE + a.rows_per_cta - 1) / a.rows_per_cta, a.T);
    return launch_ex(router_kernel, grid, dim3(128), 0, st, pdl, a);
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
// grid (max_chunks, HK, T), 256 threads, one CTA per (token, kv head, chunk of 256 keys).
// K and V pages are fetched with 2-D TMA (128-byte swizzle, box 64 x 16) into shared memory;
// thread j owns key j for the scores, thread (d, head group) owns an output column for P*V.
// A chunk writes (m, l, acc) to scratch; the last chunk of a (token, head) combines (C8).
constexpr int ATTN_THREADS = 256;

size_t attn_smem_bytes(int G) {
    return 4 * 32768 + (size_t)128 * G * 4 + (size_t)ATTN_CHUNK * G * 4 + 8 * 8 * 4 * 2 + 64 + 1024;
}

__global__ void __launch_bounds__(ATTN_THREADS, 1)
    attn_kernel(const __grid_constant__ AttnArgs p, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *Kr[2] = {smem, smem + 32768};
    uint8_t *Vr[2] = {smem + 65536, smem + 98304};
    const int G = p.G, D = 128;
    float *qs = reinterpret_cast<float *>(smem + 131072);          // [D][G]
    float *ps = qs + D * G;                                        // [256][G]
    float *red = ps + ATTN_CHUNK * G;                              // [8][8]
    float *red2 = red + 64;                                        // [8][8]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red2 + 64);
    __shared__ int s_last;
    __shared__ float s_m[8], s_l[8];

    const int c = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    const int seq = p.seq_of[t], pos = p.pos_of[t];
    const int nk = pos + 1, nc = (nk + ATTN_CHUNK - 1) / ATTN_CHUNK;
    if (c >= nc) {
        pdl_trigger();
        return;
    }
    const int base = c * ATTN_CHUNK;
    const int cnt = nk - base < ATTN_CHUNK ? nk - base : ATTN_CHUNK;
    const int npages = (cnt + 15) / 16;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        prefetch_tmap(&tmap);
        mbar_arrive_expect_tx(bar, npages * 8192);
        for (int pg = 0; pg < npages; pg++) {
            int blk = p.block_table[seq * p.max_blocks + (base >> 4) + pg];
            int rowK = (int)(((((long long)p.layer * p.n_blocks + blk) * 2 + 0) * p.HK + g) * 16);
            int rowV = rowK + p.HK * 16;
            tma_load_2d(Kr[0] + pg * 2048, &tmap, 0, rowK, bar);
            tma_load_2d(Kr[1] + pg * 2048, &tmap, 64, rowK, bar);
            tma_load_2d(Vr[0] + pg * 2048, &tmap, 0, rowV, bar);
            tma_load_2d(Vr[1] + pg * 2048, &tmap, 64, rowV, bar);
        }
    }
    pdl_trigger();
    for (int i = tid; i < D * G; i += ATTN_THREADS) {
        int h = i / D, d = i % D;
        qs[d * G + h] = f16_round(p.q[(long long)t * p.H * D + (g * G + h) * D + d]);
    }
    __syncthreads();
    const bool landed = mbar_wait(bar, 0, p.err);
    if (__syncthreads_or(!landed)) {  // a wait ran out: give the copies one more bounded wait, then leave
        if (tid == 0) mbar_wait(bar, 0, nullptr);
        return;
    }
    // scores: thread j owns key j (sequential fmaf over d, C8)
    const int j = tid;
    const bool valid = j < cnt;
    float s[8];
#pragma unroll
    for (int h = 0; h < 8; h++) s[h] = 0.0f;
    if (valid) {
#pragma unroll 1
        for (int c16 = 0; c16 < 16; c16++) {
            const uint8_t *kr = Kr[c16 >> 3] + j * 128 + ((((c16 & 7) ^ (j & 7))) << 4);
            uint4 kv = *reinterpret_cast<const uint4 *>(kr);
            const __half *hk = reinterpret_cast<const __half *>(&kv);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                float kf = __half2float(hk[e]);
                const float *qd = qs + (c16 * 8 + e) * G;
#pragma unroll
                for (int h = 0; h < 8; h++)
                    if (h < G) s[h] = fmaf(qd[h], kf, s[h]);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < 8; h++) s[h] = valid ? __fmul_rn(s[h], p.scale) : -__int_as_float(0x7f800000);
    // per-head chunk max
#pragma unroll
    for (int h = 0; h < 8; h++) {
        float m = warp_max(s[h]);
        if (lane == 0) red[warp * 8 + h] = m;
    }
    __syncthreads();
    if (tid < G) {
        float m = red[tid];
        for (int w = 1; w < 8; w++) m = fmaxf(m, red[w * 8 + tid]);
        s_m[tid] = m;
    }
    __syncthreads();
    // probabilities and the P3 sum
#pragma unroll
    for (int h = 0; h < 8; h++) {
        if (h < G) {
            float pr = valid ? bt_exp(__fsub_rn(s[h], s_m[h])) : 0.0f;
            ps[j * G + h] = pr;
            float ws = butterfly_sum(pr);
            if (lane == 0) red2[warp * 8 + h] = ws;
        }
    }
    __syncthreads();
    if (tid < G) {
        float l = 0.0f;
        for (int w = 0; w < 8; w++) l = __fadd_rn(l, red2[w * 8 + tid]);
        s_l[tid] = l;
    }
    // P*V: thread owns column d for heads [hq*G/2, hq*G/2 + G/2)
    const int d = tid & 127, hq = tid >> 7, hpt = G / 2;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    {
        const uint8_t *vreg = Vr[d >> 6];
        const int cc = (d & 63) >> 3, within = (d & 7) * 2;
        for (int jj = 0; jj < cnt; jj++) {
            const __half hv = *reinterpret_cast<const __half *>(vreg + jj * 128 + (((cc ^ (jj & 7))) << 4) + within);
            const float vf = __half2float(hv);
            const float *pj = ps + jj * G + hq * hpt;
#pragma unroll
            for (int h = 0; h < 4; h++)
                if (h < hpt) acc[h] = fmaf(pj[h], vf, acc[h]);
        }
    }
    __syncthreads();
    const int QW = p.H * D;
    if (nc == 1) {
        for (int h = 0; h < hpt; h++) {
            int hh = hq * hpt + h;
            float M = s_m[hh];
            float f = bt_exp(__fsub_rn(s_m[hh], M));
            float L = fmaf(s_l[hh], f, 0.0f);
            float O = fmaf(acc[h], f, 0.0f);
            p.out[(long long)t * QW + (g * G + hh) * D + d] = __fdiv_rn(O, L);
        }
        return;
    }
    const long long pbase = (((long long)t * p.HK + g) * p.max_chunks) * G * (D + 2);
    for (int h = 0; h < hpt; h++) {
        int hh = hq * hpt + h;
        float *pp = p.part + pbase + ((long long)c * G + hh) * (D + 2);
        pp[d] = acc[h];
        if (d == 0) {
            pp[D] = s_m[hh];
            pp[D + 1] = s_l[hh];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.cnt[t * p.HK + g], 1) == nc - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int h = 0; h < hpt; h++) {
        int hh = hq * hpt + h;
        float M = -__int_as_float(0x7f800000);
        for (int cc = 0; cc < nc; cc++) M = fmaxf(M, __ldcg(p.part + pbase + ((long long)cc * G + hh) * (D + 2) + D));
        float L = 0.0f, O = 0.0f;
        for (int cc = 0; cc < nc; cc++) {
            const float *pp = p.part + pbase + ((long long)cc * G + hh) * (D + 2);
            float f = bt_exp(__fsub_rn(__ldcg(pp + D), M));
            L = fmaf(__ldcg(pp + D + 1), f, L);
            O = fmaf(__ldcg(pp + d), f, O);
        }
        p.out[(long long)t * QW + (g * G + hh) * D + d] = __fdiv_rn(O, L);
    }
    if (tid == 0) p.cnt[t * p.HK + g] = 0;
}

cudaError_t launch_attn(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl) {
    size_t smem = attn_smem_bytes(a.G);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.max_chunks, a.HK, a.T);
    cfg.blockDim = dim3(ATTN_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_kernel, a, tmap);
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

// grid (n_seqs), 1024 threads: argmax with total_cmp, last maximum wins (sample.rs:928-935);
// then advance the sequence's device length (advance_by) and, for the greedy loop, feed the
// token back. CTA s handles sequence s of the step; logit_row[s] < 0 means no logits.
__global__ void __launch_bounds__(1024) step_end_kernel(const __grid_constant__ StepEndArgs p) {
    const int s = blockIdx.x;
    __shared__ int s_key[32], s_idx[32];
    pdl_wait();
    pdl_trigger();
    const int lrow = p.logit_row ? p.logit_row[s] : -1;
    int bk = -2147483647 - 1, bi = -1;
    if (lrow >= 0) {
        const float *lg = p.logits + (long long)lrow * p.V;
        for (int i = threadIdx.x; i < p.V; i += blockDim.x) {
            int k = total_key(lg[i]);
            if (k >= bk) {
                bk = k;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            int ok = __shfl_xor_sync(FULL, bk, o), oi = __shfl_xor_sync(FULL, bi, o);
            if (ok > bk || (ok == bk && oi > bi)) {
                bk = ok;
                bi = oi;
            }
        }
        if ((threadIdx.x & 31) == 0) {
            s_key[threadIdx.x >> 5] = bk;
            s_idx[threadIdx.x >> 5] = bi;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            int nw = blockDim.x >> 5;
            bk = threadIdx.x < nw ? s_key[threadIdx.x] : (-2147483647 - 1);
            bi = threadIdx.x < nw ? s_idx[threadIdx.x] : -1;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                int ok = __shfl_xor_sync(FULL, bk, o), oi = __shfl_xor_sync(FULL, bi, o);
                if (ok > bk || (ok == bk && oi > bi)) {
                    bk = ok;
                    bi = oi;
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        p.dev_len[p.seq_ids[s]] += p.n_tok[s];
        if (lrow >= 0) {
            p.next_token[lrow] = bi;
            if (p.tokens_buf) p.tokens_buf[lrow] = bi;
            if (p.gen_out) {
                int k = p.gen_count[lrow]++;
                p.gen_out[(long long)k * p.n_out + lrow] = bi;
            }
        }
    }
}

cudaError_t launch_step_end(const StepEndArgs &a, cudaStream_t st, bool pdl) {
    return launch_ex(step_end_kernel, dim3(a.n_seqs), dim3(1024), 0, st, pdl, a);
}

// Large dynamic shared memory must be enabled per kernel and per device before the first
// launch (and outside any stream capture): the engine calls this when it binds a device.
cudaError_t init_kernel_attributes() {
    const int cap = 227 * 1024;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<GEMV_WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap))) return e;
    if ((e = cudaFuncSetAttribute(gateup_kernel<GEMV_WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap))) return e;
    if ((e = cudaFuncSetAttribute(down_kernel<GEMV_WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap))) return e;
    return cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
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
