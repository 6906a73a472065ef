// Tensor-core (tcgen05, kind::i8) kernels of the K-quant contractions.
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "kernels.cuh"
#include "kquant.cuh"
#include "stage.cuh"
#include "umma.cuh"

namespace bt {

// One CTA of 128 threads: D[128][N] = A[128][K] (unsigned 8-bit) . B[N][K]^T (signed 8-bit) in
// int32, K / 32 MMAs accumulating in TMEM; the parity hook of the operand layouts and
// descriptors the grouped expert kernel uses.
__global__ void __launch_bounds__(128) i8_mma_probe_kernel(const uint8_t *__restrict__ A, const int8_t *__restrict__ B,
                                                           int32_t *__restrict__ D, int N, int K, int *err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sa = smem;            // [K/32][128 rows][32]
    uint8_t *sb = smem + 128 * K;  // [K/32][N rows][32]
    uint64_t *bar = reinterpret_cast<uint64_t *>(sb + N * K);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 128 * K; i += 128) sa[umma_off(i / K, i % K, 128)] = A[i];
    for (int i = tid; i < N * K; i += 128) sb[umma_off(i / K, i % K, N)] = (uint8_t)B[i];
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), 32);
    fence_proxy_async();  // the operands were written by the generic proxy; the MMA reads them
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tid == 0) {
        const uint32_t idesc = umma_idesc_u8s8(128, N);
        for (int s = 0; s < K / 32; s++)
            umma_i8(tmem, umma_desc(smem_u32(sa) + (uint32_t)s * 128 * 32, 128, 256),
                    umma_desc(smem_u32(sb) + (uint32_t)(s * N * 32), 128, 256), idesc, s > 0);
        umma_commit(smem_u32(bar));
    }
    const bool ok = mbar_wait(bar, 0, err);
    tc_fence_after();
    if (__syncthreads_and(ok)) {
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (c0 + j < N) D[(warp * 32 + lane) * N + c0 + j] = (int32_t)v[j];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 32);
}

size_t i8_mma_probe_smem(int N, int K) { return (size_t)(128 + N) * K + 16; }

// ====================================================================== grouped gate/up on tcgen05
// Q4_K gate and up of the grouped batched path. Unit = (chunk of at most 16 rows of one
// expert, block of 128 output rows); CTA b takes units [b*U/grid, (b+1)*U/grid), chunk-major,
// so consecutive units share the chunk's staged activations. Per unit, 16 steps (gate then
// up, superblock 0..7):
//   - thread r (= output row r of the block, = TMEM lane r) loads its row's 144-byte
//     superblock (header + 128 bytes of nibbles) straight from the tiled weights, one step
//     ahead, and unpacks the nibbles into the 8-bit A operand (8 sub-blocks x 128 rows x 32);
//   - one thread issues 8 MMAs (M = 128, N = 16, K = 32: one per 32-value sub-block, each into
//     its own 16 TMEM columns) against the chunk's Q8_K activations (the B operand) and
//     commits them to the step's mbarrier;
//   - the previous step's epilogue reads its 8 x 16 integer sub-block dots from TMEM and
//     finishes C4 per (row, token): sumi = sum sc_j dot_j, summ = sum m_j bs32_j, then
//     (float)sumi * (d * d_a) - (float)summ * (dmin * d_a), added to the row's running sum in
//     superblock order -- the integers are exact, so the result equals the dp4a kernels' bits.
// A and TMEM are double-buffered by step parity. Every wait is bounded; on a timeout the CTA
// waits (bounded) for its MMAs in flight, frees its TMEM and leaves.
constexpr int MMA_N = 16;                     // tokens per MMA (the chunk, zero-padded)
constexpr int MMA_A_BYTES = 8 * 128 * 32;     // one superblock of 128 rows, 8 K steps
constexpr int MMA_TMEM_COLS = 256;            // 2 buffers x 8 sub-blocks x 16 tokens

size_t gateup_mma_smem_bytes(int E) {
    const size_t nsb = (size_t)E / 256;
    return 1024 + (size_t)MMA_N * E + 2 * MMA_A_BYTES + (size_t)MMA_N * nsb * sizeof(ActBlock) + 256;
}

__global__ void __launch_bounds__(256, 1) gateup_mma_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int E = p.E, nsb = E / 256, S = p.g_S;
    uint8_t *sB = smem;                                                  // [E/32 K steps][16 rows][32]
    uint8_t *sA = sB + MMA_N * E;                                        // [2][8 K steps][128 rows][32]
    ActBlock *act = reinterpret_cast<ActBlock *>(sA + 2 * MMA_A_BYTES);  // [16][nsb]
    int *tk_s = reinterpret_cast<int *>(act + MMA_N * nsb);             // [16]
    int *rows_s = tk_s + MMA_N;                                          // [16]
    uint64_t *bars = reinterpret_cast<uint64_t *>(rows_s + MMA_N);      // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    // thread (row r of the block, half h): h loads and unpacks nibble groups 2h, 2h+1 of the
    // row and finishes the epilogue of tokens 8h .. 8h+7
    const int r = tid & 127, h = tid >> 7;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), MMA_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lanes
    pdl_wait();  // the groups come from group_kernel, the activations from the router
    const int nrb = p.F / 128;
    const int total = *p.g_nchunks * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    pdl_trigger();
    const uint32_t idesc = umma_idesc_u8s8(128, MMA_N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    int cur_chunk = -1, mc = 0;
    uint32_t gstep = 0;  // steps issued by this CTA: buffer gstep & 1, its barrier phase (gstep >> 1) & 1
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int ci = u / nrb, rb = u - ci * nrb;
        const int e = p.g_chunk_e[ci];
        if (ci != cur_chunk) {  // stage the chunk: Q8_K blocks, then the B operand (zero rows past mc)
            cur_chunk = ci;
            const int c0 = p.g_chunk_r0[ci], m = p.g_count[e], off = p.g_off[e];
            mc = m - c0 < MMA_N ? m - c0 : MMA_N;
            __syncthreads();  // the previous chunk's operands are no longer read
            if (tid < mc) {
                const int tk = p.g_list[off + c0 + tid];
                tk_s[tid] = tk;
                rows_s[tid] = tk / p.row_div;
            }
            __syncthreads();
            stage_activations<8>(p.fn, p.E, rows_s, nullptr, 0.0f, p.E, mc, act, nullptr);
            __syncthreads();
            for (int i = tid; i < MMA_N * E / 16; i += 256) {  // 16-byte pieces of the B operand
                const int t = i / (E / 16), k = (i - t * (E / 16)) * 16;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (t < mc) v = *reinterpret_cast<const uint4 *>(act[t * nsb + k / 256].qs + (k & 255));
                *reinterpret_cast<uint4 *>(sB + umma_off(t, k, MMA_N)) = v;
            }
        }
        // this thread's row of the block: tile (row / rpt), slot (row % rpt) * nsb + superblock
        const int row = rb * 128 + r;
        const int rpt = p.g_rpt;
        const uint8_t *gbase = expert_gate(p, e) + (long long)(row / rpt) * p.g_tile_bytes;
        const uint8_t *ubase = expert_up(p, e) + (long long)(row / rpt) * p.u_tile_bytes;
        const int slot0 = (row % rpt) * nsb;
        // chunk 0 (header) and this half's four nibble chunks 1 + 4h .. 4 + 4h
        auto load_raw = [&](int st, uint4 (&w)[5]) {
            const uint8_t *b = (st < nsb ? gbase : ubase) + (size_t)(slot0 + (st < nsb ? st : st - nsb)) * 16;
            w[0] = __ldg(reinterpret_cast<const uint4 *>(b));
#pragma unroll
            for (int c = 0; c < 4; c++)
                w[1 + c] = __ldg(reinterpret_cast<const uint4 *>(b + (size_t)(1 + 4 * h + c) * S * 16));
        };
        float acc_g[8], acc_u[8];
#pragma unroll
        for (int t = 0; t < 8; t++) acc_g[t] = acc_u[t] = 0.0f;
        uint4 raw[5], nxt[5];
        load_raw(0, raw);
        int sc[8], mn[8];
        float dw = 0.0f, dminw = 0.0f;
        int psc[8], pmn[8];
        float pdw = 0.0f, pdminw = 0.0f;
        const int nsteps = 2 * nsb;
        auto epilogue = [&](int st, uint32_t gs) -> bool {  // the integer dots of step st -> the row sums
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            const int sb = st < nsb ? st : st - nsb;
            int sumi[8];
#pragma unroll
            for (int t = 0; t < 8; t++) sumi[t] = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint32_t v[8];
                tmem_ld8(tmem + tlane + (gs & 1) * 128 + j * 16 + h * 8, v);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 8; t++) sumi[t] += psc[j] * (int)v[t];
            }
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int tt = 8 * h + t;
                const ActBlock &ab = act[(tt < mc ? tt : 0) * nsb + sb];
                const int4 b0 = *reinterpret_cast<const int4 *>(ab.bs32);
                const int4 b1 = *reinterpret_cast<const int4 *>(ab.bs32 + 4);
                const int summ = pmn[0] * b0.x + pmn[1] * b0.y + pmn[2] * b0.z + pmn[3] * b0.w + pmn[4] * b1.x +
                                 pmn[5] * b1.y + pmn[6] * b1.z + pmn[7] * b1.w;
                const float da = ab.d;
                const float t1 = __fmul_rn(pdw, da);
                const float t2 = __fmul_rn(__int2float_rn(sumi[t]), t1);
                const float t3 = __fmul_rn(pdminw, da);
                const float t4 = __fmul_rn(__int2float_rn(summ), t3);
                const float v = __fsub_rn(t2, t4);
                if (st < nsb) acc_g[t] = __fadd_rn(acc_g[t], v);
                else acc_u[t] = __fadd_rn(acc_u[t], v);
            }
            return true;
        };
        for (int st = 0; st < nsteps; st++) {
            const uint32_t gs = gstep++;
            // header: d, dmin and the 6-bit scales/mins of this row's superblock (get_scale_min_k4)
            {
                const uint4 hd = raw[0];
                dw = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffff)));
                dminw = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
                const uint32_t s03 = hd.y, s47 = hd.z, s811 = hd.w;
                const uint32_t sc_lo = s03 & 0x3F3F3F3Fu, m_lo = s47 & 0x3F3F3F3Fu;
                const uint32_t sc_hi = (s811 & 0x0F0F0F0Fu) | ((s03 >> 2) & 0x30303030u);
                const uint32_t m_hi = ((s811 >> 4) & 0x0F0F0F0Fu) | ((s47 >> 2) & 0x30303030u);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    sc[j] = byte_u(sc_lo, j);
                    sc[j + 4] = byte_u(sc_hi, j);
                    mn[j] = byte_u(m_lo, j);
                    mn[j + 4] = byte_u(m_hi, j);
                }
            }
            // the A operand: nibble group g = 2h + gg; sub-block 2g = low nibbles, 2g + 1 = high
            uint8_t *a = sA + (gs & 1) * MMA_A_BYTES;
#pragma unroll
            for (int gg = 0; gg < 2; gg++) {
                const int g = 2 * h + gg;
                const uint4 w0 = raw[1 + 2 * gg], w1 = raw[2 + 2 * gg];
                const uint4 lo0 = make_uint4(w0.x & 0x0F0F0F0Fu, w0.y & 0x0F0F0F0Fu, w0.z & 0x0F0F0F0Fu, w0.w & 0x0F0F0F0Fu);
                const uint4 lo1 = make_uint4(w1.x & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu, w1.z & 0x0F0F0F0Fu, w1.w & 0x0F0F0F0Fu);
                const uint4 hi0 = make_uint4((w0.x >> 4) & 0x0F0F0F0Fu, (w0.y >> 4) & 0x0F0F0F0Fu, (w0.z >> 4) & 0x0F0F0F0Fu,
                                             (w0.w >> 4) & 0x0F0F0F0Fu);
                const uint4 hi1 = make_uint4((w1.x >> 4) & 0x0F0F0F0Fu, (w1.y >> 4) & 0x0F0F0F0Fu, (w1.z >> 4) & 0x0F0F0F0Fu,
                                             (w1.w >> 4) & 0x0F0F0F0Fu);
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g) * 32, 128)) = lo0;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g) * 32 + 16, 128)) = lo1;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g + 1) * 32, 128)) = hi0;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g + 1) * 32 + 16, 128)) = hi1;
            }
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const int sb = st < nsb ? st : st - nsb;
#pragma unroll 1
                for (int j = 0; j < 8; j++)
                    umma_i8(tmem + (gs & 1) * 128 + j * 16,
                            umma_desc(aBase + (gs & 1) * MMA_A_BYTES + j * 4096, 128, 256),
                            umma_desc(bBase + (uint32_t)(sb * 8 + j) * MMA_N * 32, 128, 256), idesc, false);
                umma_commit(smem_u32(&bars[gs & 1]));
            }
            if (st + 1 < nsteps) load_raw(st + 1, nxt);
            if (st > 0 && !__syncthreads_and(epilogue(st - 1, gs - 1))) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                psc[j] = sc[j];
                pmn[j] = mn[j];
            }
            pdw = dw;
            pdminw = dminw;
#pragma unroll
            for (int c = 0; c < 5; c++) raw[c] = nxt[c];
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsteps - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
        if (row < p.F)
            for (int t = 0; t < 8; t++)
                if (8 * h + t < mc)
                    p.act[(long long)tk_s[8 * h + t] * p.F + row] = __fmul_rn(bt_silu(acc_g[t]), acc_u[t]);
    }
    if (!ok && tid == 0) {  // let this CTA's MMAs in flight finish (bounded) before the TMEM goes
        for (uint32_t b = 0; b < 2; b++) {
            // the last step issued on buffer b
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, MMA_TMEM_COLS);
}

cudaError_t launch_gateup_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    const size_t smem = gateup_mma_smem_bytes(a.E);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gateup_mma_kernel, a);
}

// ====================================================================== batched GEMV on tcgen05
// y[t][out_off + r] = W[r,:] . x[t,:] (+ res) for Q4_K segments of whole 128-row blocks and T > 8
// tokens (q/k/v and attn_output of batched steps). Unit = (chunk of 32 tokens, block of 128
// rows of one segment), token-chunk-major. The activations of a chunk are RMS-normed (q/k/v)
// and quantised exactly as the dp4a kernel stages them, into the 8-bit B operand plus each
// block's d and 32-value sums. Per superblock step, thread r unpacks its row's nibbles into A
// (double-buffered), one thread issues 8 MMAs (M = 128, N = 32, one per sub-block, each into
// its own 32 TMEM columns; TMEM double-buffered), and the previous step's epilogue turns the
// integer sub-block dots into the superblock's C4 value per (row, token) and adds it to the
// row's running sum in superblock order.
constexpr int GM_N = 32;

size_t gemv_mma_smem_bytes(int K) {
    const size_t nsb = (size_t)K / 256;
    return 1024 + (size_t)GM_N * K + (size_t)GM_N * nsb * (4 + 32) + 8 * sizeof(ActBlock) + 2 * MMA_A_BYTES +
           GM_N * 4 + 256;
}

__global__ void __launch_bounds__(256, 1) gemv_mma_kernel(const __grid_constant__ GemvArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int K = p.K, nsb = K / 256;
    uint8_t *sA = smem;                                                  // [2][8 K steps][128 rows][32]
    uint8_t *sB = sA + 2 * MMA_A_BYTES;                                  // [K/32 steps][32 rows][32]
    float *dA = reinterpret_cast<float *>(sB + (size_t)GM_N * K);        // [32][nsb]
    int *bsA = reinterpret_cast<int *>(dA + GM_N * nsb);                 // [32][nsb][8]
    ActBlock *tmp = reinterpret_cast<ActBlock *>(bsA + GM_N * nsb * 8);  // [8] one per warp
    float *normS = reinterpret_cast<float *>(tmp + 8);                   // [32]
    uint64_t *bars = reinterpret_cast<uint64_t *>(normS + GM_N);         // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // thread (row r of the block, half h): h unpacks nibble groups 2h, 2h+1 of the row and
    // finishes the epilogue of tokens 16h .. 16h+15
    const int r = tid & 127, h = tid >> 7;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait();
    int nrb = 0;  // 128-row blocks over the segments
    for (int i = 0; i < p.nseg; i++) nrb += p.seg[i].rows / 128;
    const int ntc = (p.T + GM_N - 1) / GM_N;
    const int total = ntc * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    pdl_trigger();
    const uint32_t idesc = umma_idesc_u8s8(128, GM_N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    int cur_tc = -1, tn = 0;
    uint32_t gstep = 0;
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int tc = u / nrb;
        int rb = u - tc * nrb, si = 0;
        while (rb >= p.seg[si].rows / 128) {
            rb -= p.seg[si].rows / 128;
            si++;
        }
        const GemvSeg &sg = p.seg[si];
        if (tc != cur_tc) {  // stage the chunk's 32 token rows (zeros past the last token)
            cur_tc = tc;
            const int t0 = tc * GM_N;
            tn = p.T - t0 < GM_N ? p.T - t0 : GM_N;
            __syncthreads();  // the previous chunk's operands are no longer read
            if (p.norm_w) {
                for (int t = warp; t < tn; t += 8) {
                    const float *xt = p.x + (long long)(p.x_rows ? p.x_rows[t0 + t] : t0 + t) * p.x_stride;
                    const float acc = warp_sumsq_p2(xt, K, lane);
                    if (lane == 0) normS[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)K), p.eps)));
                }
                __syncthreads();
            }
            for (int blk = warp; blk < GM_N * nsb; blk += 8) {
                const int t = blk / nsb, b = blk - t * nsb;
                uint2 q8 = make_uint2(0, 0);
                float dv = 0.0f;
                int bsv = 0;
                if (t < tn) {
                    const float *xt = p.x + (long long)(p.x_rows ? p.x_rows[t0 + t] : t0 + t) * p.x_stride + b * 256 +
                                      lane * 8;
                    float v[8];
                    const float4 a0 = *reinterpret_cast<const float4 *>(xt), a1 = *reinterpret_cast<const float4 *>(xt + 4);
                    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
                    v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
                    if (p.norm_w) {
                        const float sN = normS[t];
                        const float *w = p.norm_w + b * 256 + lane * 8;
#pragma unroll
                        for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], sN), w[i]);
                    }
                    quantize_block_warp(v, tmp + warp, lane);
                    __syncwarp();
                    q8 = *reinterpret_cast<const uint2 *>(tmp[warp].qs + lane * 8);
                    dv = tmp[warp].d;
                    bsv = lane < 8 ? tmp[warp].bs32[lane] : 0;
                    __syncwarp();  // tmp is read before the warp's next block overwrites it
                }
                const int k = b * 256 + lane * 8;
                *reinterpret_cast<uint2 *>(sB + umma_off(t, k, GM_N)) = q8;
                if (lane == 0) dA[t * nsb + b] = dv;
                if (lane < 8) bsA[(t * nsb + b) * 8 + lane] = bsv;
            }
        }
        // this thread's row: tile row / rpt of the segment, slot (row % rpt) * nsb + superblock
        const int row = rb * 128 + r;
        const uint8_t *wbase = sg.w + (long long)(row / sg.rpt) * sg.tile_bytes;
        const int slot0 = (row % sg.rpt) * nsb, S = sg.S;
        auto load_raw = [&](int st, uint4 (&w)[5]) {  // header and this half's four nibble chunks
            const uint8_t *b = wbase + (size_t)(slot0 + st) * 16;
            w[0] = __ldg(reinterpret_cast<const uint4 *>(b));
#pragma unroll
            for (int c = 0; c < 4; c++)
                w[1 + c] = __ldg(reinterpret_cast<const uint4 *>(b + (size_t)(1 + 4 * h + c) * S * 16));
        };
        constexpr int HT = GM_N / 2;  // tokens per half
        float acc[HT];
#pragma unroll
        for (int t = 0; t < HT; t++) acc[t] = 0.0f;
        uint4 raw[5], nxt[5];
        load_raw(0, raw);
        int sc[8], mn[8], psc[8], pmn[8];
        float dw = 0.0f, dminw = 0.0f, pdw = 0.0f, pdminw = 0.0f;
        auto epilogue = [&](int sb, uint32_t gs) -> bool {
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            int sumi[HT];
#pragma unroll
            for (int t = 0; t < HT; t++) sumi[t] = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint32_t v[16];
                tmem_ld16(tmem + tlane + (gs & 1) * 256 + j * GM_N + h * HT, v);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < HT; t++) sumi[t] += psc[j] * (int)v[t];
            }
#pragma unroll
            for (int tt = 0; tt < HT; tt++) {
                const int t = HT * h + tt;
                const int4 b0 = *reinterpret_cast<const int4 *>(bsA + (t * nsb + sb) * 8);
                const int4 b1 = *reinterpret_cast<const int4 *>(bsA + (t * nsb + sb) * 8 + 4);
                const int summ = pmn[0] * b0.x + pmn[1] * b0.y + pmn[2] * b0.z + pmn[3] * b0.w + pmn[4] * b1.x +
                                 pmn[5] * b1.y + pmn[6] * b1.z + pmn[7] * b1.w;
                const float da = dA[t * nsb + sb];
                const float t1 = __fmul_rn(pdw, da);
                const float t2 = __fmul_rn(__int2float_rn(sumi[tt]), t1);
                const float t3 = __fmul_rn(pdminw, da);
                const float t4 = __fmul_rn(__int2float_rn(summ), t3);
                acc[tt] = __fadd_rn(acc[tt], __fsub_rn(t2, t4));
            }
            return true;
        };
        for (int st = 0; st < nsb; st++) {
            const uint32_t gs = gstep++;
            {
                const uint4 h = raw[0];
                dw = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffff)));
                dminw = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
                const uint32_t s03 = h.y, s47 = h.z, s811 = h.w;
                const uint32_t sc_lo = s03 & 0x3F3F3F3Fu, m_lo = s47 & 0x3F3F3F3Fu;
                const uint32_t sc_hi = (s811 & 0x0F0F0F0Fu) | ((s03 >> 2) & 0x30303030u);
                const uint32_t m_hi = ((s811 >> 4) & 0x0F0F0F0Fu) | ((s47 >> 2) & 0x30303030u);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    sc[j] = byte_u(sc_lo, j);
                    sc[j + 4] = byte_u(sc_hi, j);
                    mn[j] = byte_u(m_lo, j);
                    mn[j + 4] = byte_u(m_hi, j);
                }
            }
            uint8_t *a = sA + (gs & 1) * MMA_A_BYTES;
#pragma unroll
            for (int gg = 0; gg < 2; gg++) {
                const int g = 2 * h + gg;
                const uint4 w0 = raw[1 + 2 * gg], w1 = raw[2 + 2 * gg];
                const uint4 lo0 = make_uint4(w0.x & 0x0F0F0F0Fu, w0.y & 0x0F0F0F0Fu, w0.z & 0x0F0F0F0Fu, w0.w & 0x0F0F0F0Fu);
                const uint4 lo1 = make_uint4(w1.x & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu, w1.z & 0x0F0F0F0Fu, w1.w & 0x0F0F0F0Fu);
                const uint4 hi0 = make_uint4((w0.x >> 4) & 0x0F0F0F0Fu, (w0.y >> 4) & 0x0F0F0F0Fu, (w0.z >> 4) & 0x0F0F0F0Fu,
                                             (w0.w >> 4) & 0x0F0F0F0Fu);
                const uint4 hi1 = make_uint4((w1.x >> 4) & 0x0F0F0F0Fu, (w1.y >> 4) & 0x0F0F0F0Fu, (w1.z >> 4) & 0x0F0F0F0Fu,
                                             (w1.w >> 4) & 0x0F0F0F0Fu);
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g) * 32, 128)) = lo0;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g) * 32 + 16, 128)) = lo1;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g + 1) * 32, 128)) = hi0;
                *reinterpret_cast<uint4 *>(a + umma_off(r, (2 * g + 1) * 32 + 16, 128)) = hi1;
            }
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll 1
                for (int j = 0; j < 8; j++)
                    umma_i8(tmem + (gs & 1) * 256 + j * GM_N,
                            umma_desc(aBase + (gs & 1) * MMA_A_BYTES + j * 4096, 128, 256),
                            umma_desc(bBase + (uint32_t)(st * 8 + j) * GM_N * 32, 128, 256), idesc, false);
                umma_commit(smem_u32(&bars[gs & 1]));
            }
            if (st + 1 < nsb) load_raw(st + 1, nxt);
            if (st > 0 && !__syncthreads_and(epilogue(st - 1, gs - 1))) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                psc[j] = sc[j];
                pmn[j] = mn[j];
            }
            pdw = dw;
            pdminw = dminw;
#pragma unroll
            for (int c = 0; c < 5; c++) raw[c] = nxt[c];
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsb - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
        const int t0 = tc * GM_N + HT * h;
        for (int t = 0; t < HT && HT * h + t < tn; t++) {
            const long long yi = (long long)(t0 + t) * p.y_stride + sg.out_off + row;
            float y = acc[t];
            if (p.res) y = __fadd_rn(p.res[(long long)(t0 + t) * p.res_stride + sg.out_off + row], acc[t]);
            p.y[yi] = y;
        }
    }
    if (!ok && tid == 0) {
        for (uint32_t b = 0; b < 2; b++) {
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

cudaError_t launch_gemv_mma(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = gemv_mma_smem_bytes(a.K);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_mma_kernel, a);
}

cudaError_t init_mma_attributes() {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev))) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
    const void *kerns[] = {(const void *)gateup_mma_kernel, (const void *)gemv_mma_kernel};
    for (const void *k : kerns) {
        cudaFuncAttributes fa;
        if ((e = cudaFuncGetAttributes(&fa, k))) return e;
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes)))
            return e;
    }
    return cudaSuccess;
}

cudaError_t launch_i8_mma_probe(const uint8_t *A, const int8_t *B, int32_t *D, int N, int K, int *err,
                                cudaStream_t st) {
    const size_t smem = i8_mma_probe_smem(N, K);
    cudaError_t e = cudaFuncSetAttribute(i8_mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    i8_mma_probe_kernel<<<1, 128, smem, st>>>(A, B, D, N, K, err);
    return cudaGetLastError();
}

}  // namespace bt
