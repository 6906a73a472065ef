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
//   - thread r (= output row r of the block, = TMEM lane r) takes its row's 144-byte
//     superblock (header + 128 bytes of nibbles) from the raw-weight ring and unpacks the
//     nibbles into the 8-bit A operand (8 sub-blocks x 128 rows x 32);
//   - one thread issues 8 MMAs (M = 128, N = 16, K = 32: one per 32-value sub-block, each into
//     its own 16 TMEM columns) against the chunk's Q8_K activations (the B operand) and
//     commits them to the step's mbarrier;
//   - the previous step's epilogue reads its 8 x 16 integer sub-block dots from TMEM and
//     finishes C4 per (row, token): sumi = sum sc_j dot_j, summ = sum m_j bs32_j, then
//     (float)sumi * (d * d_a) - (float)summ * (dmin * d_a), added to the row's running sum in
//     superblock order -- the integers are exact, so the result equals the dp4a kernels' bits.
// The raw-weight ring: each thread copies its own 5 x 16 bytes of a step (the header and the
// four nibble chunks of its half) with cp.async RAW_D steps ahead, across unit boundaries, so
// the weight stream does not wait for a DRAM round trip per step. The chunk's activations come
// as Q8_K rows quantised once per step by q8_stage_kernel and are copied in with cp.async. A and
// TMEM are double-buffered by step parity. Every wait is bounded; on a timeout the CTA waits
// (bounded) for its MMAs in flight, frees its TMEM and leaves.
constexpr int MMA_N = 16;                     // tokens per MMA (the chunk, zero-padded)
constexpr int MMA_A_BYTES = 8 * 128 * 32;     // one superblock of 128 rows, 8 K steps
constexpr int MMA_TMEM_COLS = 256;            // 2 buffers x 8 sub-blocks x 16 tokens
constexpr int RAW_D = 3, RAW_R = RAW_D + 1;   // ring: steps in flight ahead, stages
constexpr int RAW_CHUNK = 256 * 16;           // one 16-byte piece per thread
constexpr int RAW_STAGE = 5 * RAW_CHUNK;      // header + four nibble chunks per thread
constexpr size_t MMA_SMEM_LIMIT = 230400;     // sm_100 opt-in per block less the engine's 2 KB headroom

size_t gateup_mma_smem_bytes(int E) {
    const size_t nsb = (size_t)E / 256;
    return 1024 + (size_t)MMA_N * E + 2 * MMA_A_BYTES + (size_t)RAW_R * RAW_STAGE + (size_t)MMA_N * nsb * (4 + 32) +
           2 * MMA_N * 4 + 256;
}

// 8 or 16 consecutive TMEM columns of this warp's lanes
template <int HT>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[HT]) {
    if constexpr (HT == 16) tmem_ld16(taddr, v);
    else tmem_ld8(taddr, v);
}

// The C4 epilogue of one step for HT tokens of this thread's row: the 8 sub-block integer
// dots of token t at TMEM column col0 + j * jstride + t, loaded JB sub-blocks per wait.
template <int HT>
__device__ __forceinline__ void tmem_sumi(uint32_t col0, int jstride, const int (&psc)[8], int (&sumi)[HT]) {
    constexpr int JB = HT == 16 ? 2 : 4;
#pragma unroll
    for (int t = 0; t < HT; t++) sumi[t] = 0;
#pragma unroll
    for (int j0 = 0; j0 < 8; j0 += JB) {
        uint32_t v[JB][HT];
#pragma unroll
        for (int jj = 0; jj < JB; jj++) tmem_ld_cols<HT>(col0 + (uint32_t)((j0 + jj) * jstride), v[jj]);
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < JB; jj++) tmem_pin(v[jj]);
#pragma unroll
        for (int jj = 0; jj < JB; jj++)
#pragma unroll
            for (int t = 0; t < HT; t++) sumi[t] += psc[j0 + jj] * (int)v[jj][t];
    }
}

// Header of a Q4_K superblock (get_scale_min_k4): d, dmin and the 6-bit scales and mins.
__device__ __forceinline__ void q4k_header(const uint4 hd, float &dw, float &dminw, int (&sc)[8], int (&mn)[8]) {
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

// The A operand of one step: nibble groups 2h, 2h+1 of row r (sub-block 2g = low nibbles,
// 2g + 1 = high) from the four 16-byte chunks raw[1..4].
__device__ __forceinline__ void q4k_unpack_a(uint8_t *a, const uint4 (&raw)[5], int r, int h) {
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
}

// Step q's 5 x 16 bytes of this thread: from the ring (after waiting for its copies), then the
// copies of step q + RAW_D go out into the stage step q - 1 used.
template <typename IssueFn>
__device__ __forceinline__ void ring_take(const uint8_t *ring_t, int q, uint4 (&raw)[5], IssueFn &&issue) {
    cp_async_wait<RAW_D - 1>();
    const uint8_t *src = ring_t + (size_t)(q % RAW_R) * RAW_STAGE;
#pragma unroll
    for (int c = 0; c < 5; c++) raw[c] = *reinterpret_cast<const uint4 *>(src + c * RAW_CHUNK);
    issue(q + RAW_D);
}

__global__ void __launch_bounds__(256, 1) gateup_mma_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int E = p.E, nsb = E / 256, S = p.g_S;
    uint8_t *sB = smem;                                                  // [E/32 K steps][16 rows][32]
    uint8_t *sA = sB + MMA_N * E;                                        // [2][8 K steps][128 rows][32]
    uint8_t *ring = sA + 2 * MMA_A_BYTES;                                // [RAW_R][5][256 threads][16]
    float *dA = reinterpret_cast<float *>(ring + RAW_R * RAW_STAGE);     // [16][nsb] activation scales
    int *bsA = reinterpret_cast<int *>(dA + MMA_N * nsb);                // [16][nsb][8] 32-value sums
    int *tk_s = bsA + MMA_N * nsb * 8;                                   // [16]
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
    const int rpt = p.g_rpt, nsteps = 2 * nsb;
    // this thread's row of unit u: tile (row / rpt), slot (row % rpt) * nsb + superblock
    auto unit_src = [&](int u, const uint8_t *&gb, const uint8_t *&ub, int &s0) {
        const int ci = u / nrb, rb = u - ci * nrb;
        const int e = p.g_chunk_e[ci];
        const int row = rb * 128 + r;
        gb = expert_gate(p, e) + (long long)(row / rpt) * p.g_tile_bytes;
        ub = expert_up(p, e) + (long long)(row / rpt) * p.u_tile_bytes;
        s0 = (row % rpt) * nsb;
    };
    // ring: step q of this CTA is (unit u0 + q / nsteps, step q % nsteps)
    const int Q = u1 > u0 ? (u1 - u0) * nsteps : 0;
    const uint8_t *ring_t = ring + tid * 16;
    const uint32_t ring_s = smem_u32(ring) + (uint32_t)tid * 16;
    int pf_u = -1, pf_s0 = 0;
    const uint8_t *pf_g = nullptr, *pf_up = nullptr;
    auto issue = [&](int q) {
        if (q < Q) {
            const int qu = q / nsteps, sq = q - qu * nsteps;
            if (u0 + qu != pf_u) {
                pf_u = u0 + qu;
                unit_src(pf_u, pf_g, pf_up, pf_s0);
            }
            const bool g = sq < nsb;
            const uint8_t *b = (g ? pf_g : pf_up) + (size_t)(pf_s0 + (g ? sq : sq - nsb)) * 16;
            const uint32_t dst = ring_s + (uint32_t)(q % RAW_R) * RAW_STAGE;
            cp_async16(dst, b);
#pragma unroll
            for (int c = 0; c < 4; c++)
                cp_async16(dst + (uint32_t)(1 + c) * RAW_CHUNK, b + (size_t)(1 + 4 * h + c) * S * 16);
        }
        cp_async_commit();
    };
    for (int q = 0; q < RAW_D; q++) issue(q);
    int cur_chunk = -1, mc = 0, q = 0;
    uint32_t gstep = 0;  // steps issued by this CTA: buffer gstep & 1, its barrier phase (gstep >> 1) & 1
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int ci = u / nrb, rb = u - ci * nrb;
        const int e = p.g_chunk_e[ci];
        if (ci != cur_chunk) {  // the chunk's Q8_K rows: B operand (zero rows past mc), scales, sums
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
            const uint32_t sB_s = smem_u32(sB);
            for (int i = tid; i < MMA_N * E / 16; i += 256) {  // 16-byte pieces of the B operand
                const int t = i / (E / 16), k = (i - t * (E / 16)) * 16;
                if (t < mc) cp_async16(sB_s + umma_off(t, k, MMA_N), p.q8_qs + (long long)rows_s[t] * E + k);
                else *reinterpret_cast<uint4 *>(sB + umma_off(t, k, MMA_N)) = make_uint4(0, 0, 0, 0);
            }
            for (int i = tid; i < MMA_N * nsb * 2; i += 256) {  // 32-value sums, two 16-byte halves per block
                const int t = i / (nsb * 2), j = i - t * nsb * 2;
                if (t < mc) cp_async16(smem_u32(bsA + t * nsb * 8 + j * 4), p.q8_bs + (long long)rows_s[t] * nsb * 8 + j * 4);
                else *reinterpret_cast<int4 *>(bsA + t * nsb * 8 + j * 4) = make_int4(0, 0, 0, 0);
            }
            for (int i = tid; i < MMA_N * nsb; i += 256) {
                const int t = i / nsb, b = i - t * nsb;
                dA[i] = t < mc ? p.q8_d[(long long)rows_s[t] * nsb + b] : 0.0f;
            }
            cp_async_commit();
            cp_async_wait<0>();  // (the ring's copies in flight complete here too)
            __syncthreads();
        }
        const int row = rb * 128 + r;
        float acc_g[8], acc_u[8];
#pragma unroll
        for (int t = 0; t < 8; t++) acc_g[t] = acc_u[t] = 0.0f;
        uint4 raw[5];
        int sc[8], mn[8];
        float dw = 0.0f, dminw = 0.0f;
        int psc[8], pmn[8];
        float pdw = 0.0f, pdminw = 0.0f;
        auto epilogue = [&](int st, uint32_t gs) -> bool {  // the integer dots of step st -> the row sums
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            const int sb = st < nsb ? st : st - nsb;
            int sumi[8];
            tmem_sumi<8>(tmem + tlane + (gs & 1) * 128 + h * 8, 16, psc, sumi);
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int tt = 8 * h + t;
                const int4 b0 = *reinterpret_cast<const int4 *>(bsA + (tt * nsb + sb) * 8);
                const int4 b1 = *reinterpret_cast<const int4 *>(bsA + (tt * nsb + sb) * 8 + 4);
                const int summ = pmn[0] * b0.x + pmn[1] * b0.y + pmn[2] * b0.z + pmn[3] * b0.w + pmn[4] * b1.x +
                                 pmn[5] * b1.y + pmn[6] * b1.z + pmn[7] * b1.w;
                const float da = dA[tt * nsb + sb];
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
        for (int st = 0; st < nsteps; st++, q++) {
            const uint32_t gs = gstep++;
            ring_take(ring_t, q, raw, issue);
            q4k_header(raw[0], dw, dminw, sc, mn);
            q4k_unpack_a(sA + (gs & 1) * MMA_A_BYTES, raw, r, h);
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
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives it
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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = gateup_mma_smem_bytes(a.E);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gateup_mma_kernel, a);
}

// ====================================================================== grouped down on tcgen05
// Q4_K down of the grouped batched path: the gate/up kernel's scheme with one matrix. Unit =
// (chunk of at most 16 (token, slot) rows of one expert, block of 128 output rows); K = F, one
// superblock per step. The B operand is the chunk's SiLU-product rows as Q8_K (staged per
// (token, slot) row by q8_stage_kernel, as the dp4a kernel stages them); the epilogue writes each
// (token, slot)'s row sums to dpart for the combine. Thread r reads row r of the block from its
// tile (d_rpt rows of nsb superblocks each); Q4_K tiles start on 16 bytes.
size_t down_mma_smem_bytes(int F) {
    const size_t nsb = (size_t)F / 256;
    return 1024 + (size_t)MMA_N * F + 2 * MMA_A_BYTES + (size_t)RAW_R * RAW_STAGE + (size_t)MMA_N * nsb * (4 + 32) +
           2 * MMA_N * 4 + 256;
}

__global__ void __launch_bounds__(256, 1) down_mma_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int F = p.F, nsb = F / 256, rpt = p.d_rpt, S = rpt * nsb;
    uint8_t *sB = smem;                                                  // [F/32 K steps][16 rows][32]
    uint8_t *sA = sB + MMA_N * F;                                        // [2][8 K steps][128 rows][32]
    uint8_t *ring = sA + 2 * MMA_A_BYTES;                                // [RAW_R][5][256 threads][16]
    float *dA = reinterpret_cast<float *>(ring + RAW_R * RAW_STAGE);     // [16][nsb] activation scales
    int *bsA = reinterpret_cast<int *>(dA + MMA_N * nsb);                // [16][nsb][8] 32-value sums
    int *tk_s = bsA + MMA_N * nsb * 8;                                   // [16]
    uint64_t *bars = reinterpret_cast<uint64_t *>(tk_s + 2 * MMA_N);    // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    // thread (row r of the block, half h): h loads and unpacks nibble groups 2h, 2h+1 of the
    // row and finishes the epilogue of rows 8h .. 8h+7 of the chunk
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
    pdl_wait();  // the groups and the staged products come from the kernels before
    const int nrb = p.E / 128;
    const int total = *p.g_nchunks * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    pdl_trigger();
    const uint32_t idesc = umma_idesc_u8s8(128, MMA_N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    // this thread's row of unit u: tile (row / rpt), slot (row % rpt) * nsb + superblock
    auto unit_src = [&](int u, const uint8_t *&db, int &s0) {
        const int ci = u / nrb, rb = u - ci * nrb;
        const int row = rb * 128 + r;
        db = expert_down(p, p.g_chunk_e[ci]) + (long long)(row / rpt) * p.d_tile_bytes;
        s0 = (row % rpt) * nsb;
    };
    const int Q = u1 > u0 ? (u1 - u0) * nsb : 0;
    const uint8_t *ring_t = ring + tid * 16;
    const uint32_t ring_s = smem_u32(ring) + (uint32_t)tid * 16;
    int pf_u = -1, pf_s0 = 0;
    const uint8_t *pf_d = nullptr;
    auto issue = [&](int q) {
        if (q < Q) {
            const int qu = q / nsb, sq = q - qu * nsb;
            if (u0 + qu != pf_u) {
                pf_u = u0 + qu;
                unit_src(pf_u, pf_d, pf_s0);
            }
            const uint8_t *b = pf_d + (size_t)(pf_s0 + sq) * 16;
            const uint32_t dst = ring_s + (uint32_t)(q % RAW_R) * RAW_STAGE;
            cp_async16(dst, b);
#pragma unroll
            for (int c = 0; c < 4; c++)
                cp_async16(dst + (uint32_t)(1 + c) * RAW_CHUNK, b + (size_t)(1 + 4 * h + c) * S * 16);
        }
        cp_async_commit();
    };
    for (int q = 0; q < RAW_D; q++) issue(q);
    int cur_chunk = -1, mc = 0, q = 0;
    uint32_t gstep = 0;  // steps issued by this CTA: buffer gstep & 1, its barrier phase (gstep >> 1) & 1
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int ci = u / nrb, rb = u - ci * nrb;
        if (ci != cur_chunk) {  // the chunk's Q8_K rows: B operand (zero rows past mc), scales, sums
            cur_chunk = ci;
            const int e = p.g_chunk_e[ci];
            const int c0 = p.g_chunk_r0[ci], m = p.g_count[e], off = p.g_off[e];
            mc = m - c0 < MMA_N ? m - c0 : MMA_N;
            __syncthreads();  // the previous chunk's operands are no longer read
            if (tid < mc) tk_s[tid] = p.g_list[off + c0 + tid];
            __syncthreads();
            const uint32_t sB_s = smem_u32(sB);
            for (int i = tid; i < MMA_N * F / 16; i += 256) {  // 16-byte pieces of the B operand
                const int t = i / (F / 16), k = (i - t * (F / 16)) * 16;
                if (t < mc) cp_async16(sB_s + umma_off(t, k, MMA_N), p.q8_qs + (long long)tk_s[t] * F + k);
                else *reinterpret_cast<uint4 *>(sB + umma_off(t, k, MMA_N)) = make_uint4(0, 0, 0, 0);
            }
            for (int i = tid; i < MMA_N * nsb * 2; i += 256) {  // 32-value sums, two 16-byte halves per block
                const int t = i / (nsb * 2), j = i - t * nsb * 2;
                if (t < mc) cp_async16(smem_u32(bsA + t * nsb * 8 + j * 4), p.q8_bs + (long long)tk_s[t] * nsb * 8 + j * 4);
                else *reinterpret_cast<int4 *>(bsA + t * nsb * 8 + j * 4) = make_int4(0, 0, 0, 0);
            }
            for (int i = tid; i < MMA_N * nsb; i += 256) {
                const int t = i / nsb, b = i - t * nsb;
                dA[i] = t < mc ? p.q8_d[(long long)tk_s[t] * nsb + b] : 0.0f;
            }
            cp_async_commit();
            cp_async_wait<0>();  // (the ring's copies in flight complete here too)
            __syncthreads();
        }
        const int row = rb * 128 + r;
        float acc[8];
#pragma unroll
        for (int t = 0; t < 8; t++) acc[t] = 0.0f;
        uint4 raw[5];
        int sc[8], mn[8];
        float dw = 0.0f, dminw = 0.0f;
        int psc[8], pmn[8];
        float pdw = 0.0f, pdminw = 0.0f;
        auto epilogue = [&](int sb, uint32_t gs) -> bool {  // the integer dots of superblock sb -> the row sums
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            int sumi[8];
            tmem_sumi<8>(tmem + tlane + (gs & 1) * 128 + h * 8, 16, psc, sumi);
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int tt = 8 * h + t;
                const int4 b0 = *reinterpret_cast<const int4 *>(bsA + (tt * nsb + sb) * 8);
                const int4 b1 = *reinterpret_cast<const int4 *>(bsA + (tt * nsb + sb) * 8 + 4);
                const int summ = pmn[0] * b0.x + pmn[1] * b0.y + pmn[2] * b0.z + pmn[3] * b0.w + pmn[4] * b1.x +
                                 pmn[5] * b1.y + pmn[6] * b1.z + pmn[7] * b1.w;
                const float da = dA[tt * nsb + sb];
                const float t1 = __fmul_rn(pdw, da);
                const float t2 = __fmul_rn(__int2float_rn(sumi[t]), t1);
                const float t3 = __fmul_rn(pdminw, da);
                const float t4 = __fmul_rn(__int2float_rn(summ), t3);
                acc[t] = __fadd_rn(acc[t], __fsub_rn(t2, t4));
            }
            return true;
        };
        for (int st = 0; st < nsb; st++, q++) {
            const uint32_t gs = gstep++;
            ring_take(ring_t, q, raw, issue);
            q4k_header(raw[0], dw, dminw, sc, mn);
            q4k_unpack_a(sA + (gs & 1) * MMA_A_BYTES, raw, r, h);
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll 1
                for (int j = 0; j < 8; j++)
                    umma_i8(tmem + (gs & 1) * 128 + j * 16,
                            umma_desc(aBase + (gs & 1) * MMA_A_BYTES + j * 4096, 128, 256),
                            umma_desc(bBase + (uint32_t)(st * 8 + j) * MMA_N * 32, 128, 256), idesc, false);
                umma_commit(smem_u32(&bars[gs & 1]));
            }
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
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsb - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
        for (int t = 0; t < 8; t++)
            if (8 * h + t < mc) p.dpart[(long long)tk_s[8 * h + t] * p.E + row] = acc[t];
    }
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives it
    if (!ok && tid == 0) {  // let this CTA's MMAs in flight finish (bounded) before the TMEM goes
        for (uint32_t b = 0; b < 2; b++) {
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, MMA_TMEM_COLS);
}

cudaError_t launch_down_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    if (a.F % 256 || a.d_rpt < 1 || a.d_rpt * (a.F / 256) > 32 || a.E % 128 || a.dtype != T_Q4_K || a.d_nsb != a.F / 256 ||
        a.d_tile_bytes != 9 * 16 * a.d_rpt * (a.F / 256))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = down_mma_smem_bytes(a.F);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, down_mma_kernel, a);
}

// ====================================================================== Q8_K activation rows
// One CTA per row: the row's RMSNorm factor (warp 0, C5/C6) when norm_w, then the 256-value
// blocks quantised (C3) by the warps in turn, written as the tensor-core kernels read them: the
// 8-bit values in row order, each block's scale and its eight 32-value sums. The arithmetic is
// the dp4a kernels' staging, so both paths see the same bits.
__global__ void __launch_bounds__(256) q8_stage_kernel(const float *x, long long xs, const int *x_rows,
                                                       const float *norm_w, float eps, int K, int8_t *qs, float *dq,
                                                       int *bs) {
    __shared__ ActBlock tmp[8];
    __shared__ float s_norm;
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nsb = K / 256;
    pdl_wait();
    const float *xt = x + (long long)(x_rows ? x_rows[t] : t) * xs;
    if (norm_w) {
        if (warp == 0) {
            const float acc = warp_sumsq_p2(xt, K, lane);
            if (lane == 0) s_norm = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)K), eps)));
        }
        __syncthreads();
    }
    pdl_trigger();
    for (int b = warp; b < nsb; b += 8) {
        const float *src = xt + b * 256 + lane * 8;
        float v[8];
        const float4 a0 = *reinterpret_cast<const float4 *>(src), a1 = *reinterpret_cast<const float4 *>(src + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        if (norm_w) {
            const float sN = s_norm;
            const float *w = norm_w + b * 256 + lane * 8;
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], sN), w[i]);
        }
        quantize_block_warp(v, tmp + warp, lane);
        __syncwarp();
        *reinterpret_cast<uint2 *>(qs + (long long)t * K + b * 256 + lane * 8) =
            *reinterpret_cast<const uint2 *>(tmp[warp].qs + lane * 8);
        if (lane == 0) dq[(long long)t * nsb + b] = tmp[warp].d;
        if (lane < 8) bs[((long long)t * nsb + b) * 8 + lane] = tmp[warp].bs32[lane];
        __syncwarp();  // tmp is read before the warp's next block overwrites it
    }
}

cudaError_t launch_q8_stage(const float *x, long long x_stride, const int *x_rows, const float *norm_w, float eps, int K,
                            int T, int8_t *qs, float *d, int *bs, cudaStream_t st, bool pdl) {
    if (T <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q8_stage_kernel, x, x_stride, x_rows, norm_w, eps, K, qs, d, bs);
}

// ====================================================================== batched GEMV on tcgen05
// y[t][out_off + r] = W[r,:] . x[t,:] (+ res) for Q4_K segments of whole 128-row blocks and T > 8
// tokens (q/k/v and attn_output of batched steps). Unit = (chunk of N tokens, block of 128
// rows of one segment), token-chunk-major; N = 32 where the operands fit beside the raw-weight
// ring, else 16 (K of 4096). The activations come as Q8_K rows, RMS-normed (q/k/v) and quantised
// once per step by q8_stage_kernel exactly as the dp4a kernel stages them; a chunk copies its
// rows into the 8-bit B operand plus each block's d and 32-value sums. Per superblock step, thread r takes its row's superblock from the ring
// (cp.async, RAW_D steps ahead across units) and unpacks its nibbles into A (double-buffered),
// one thread issues 8 MMAs (M = 128, one per sub-block, each into its own N TMEM columns; TMEM
// double-buffered), and the previous step's epilogue turns the integer sub-block dots into the
// superblock's C4 value per (row, token) and adds it to the row's running sum in superblock
// order.
template <int N>
static size_t gemv_mma_bytes(int K) {
    const size_t nsb = (size_t)K / 256;
    return 1024 + (size_t)N * K + (size_t)N * nsb * (4 + 32) + 2 * MMA_A_BYTES + (size_t)RAW_R * RAW_STAGE + 256;
}

int gemv_mma_tokens(int K) {
    if (K % 256) return 0;
    if (gemv_mma_bytes<32>(K) <= MMA_SMEM_LIMIT) return 32;
    if (gemv_mma_bytes<16>(K) <= MMA_SMEM_LIMIT) return 16;
    return 0;
}

size_t gemv_mma_smem_bytes(int K) {
    const int n = gemv_mma_tokens(K);
    return n == 32 ? gemv_mma_bytes<32>(K) : n == 16 ? gemv_mma_bytes<16>(K) : (size_t)-1;
}

template <int N>
__global__ void __launch_bounds__(256, 1) kq_rows_mma_kernel(const __grid_constant__ GemvArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int K = p.K, nsb = K / 256;
    uint8_t *sA = smem;                                                  // [2][8 K steps][128 rows][32]
    uint8_t *ring = sA + 2 * MMA_A_BYTES;                                // [RAW_R][5][256 threads][16]
    uint8_t *sB = ring + RAW_R * RAW_STAGE;                              // [K/32 steps][N rows][32]
    float *dA = reinterpret_cast<float *>(sB + (size_t)N * K);           // [N][nsb]
    int *bsA = reinterpret_cast<int *>(dA + N * nsb);                    // [N][nsb][8]
    uint64_t *bars = reinterpret_cast<uint64_t *>(bsA + N * nsb * 8);    // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    constexpr int HT = N / 2;                // tokens per half
    constexpr uint32_t TCOLS = 2 * 8 * N;    // 2 buffers x 8 sub-blocks x N tokens
    const int tid = threadIdx.x, warp = tid >> 5;
    // thread (row r of the block, half h): h unpacks nibble groups 2h, 2h+1 of the row and
    // finishes the epilogue of tokens HT*h .. HT*h + HT-1
    const int r = tid & 127, h = tid >> 7;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    int nrb = 0;  // 128-row blocks over the segments
    for (int i = 0; i < p.nseg; i++) nrb += p.seg[i].rows / 128;
    const int ntc = (p.T + N - 1) / N;
    const int total = ntc * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    // this thread's row of unit u: the segment, tile (row / rpt), slot (row % rpt) * nsb
    auto unit_src = [&](int u, const uint8_t *&wb, int &s0, int &S, int &si, int &row) {
        int rb = u - (u / nrb) * nrb;
        si = 0;
        while (rb >= p.seg[si].rows / 128) {
            rb -= p.seg[si].rows / 128;
            si++;
        }
        row = rb * 128 + r;
        wb = p.seg[si].w + (long long)(row / p.seg[si].rpt) * p.seg[si].tile_bytes;
        s0 = (row % p.seg[si].rpt) * nsb;
        S = p.seg[si].S;
    };
    const int Q = u1 > u0 ? (u1 - u0) * nsb : 0;
    const uint8_t *ring_t = ring + tid * 16;
    const uint32_t ring_s = smem_u32(ring) + (uint32_t)tid * 16;
    int pf_u = -1, pf_s0 = 0, pf_S = 0;
    const uint8_t *pf_w = nullptr;
    auto issue = [&](int q) {
        if (q < Q) {
            const int qu = q / nsb, sq = q - qu * nsb;
            if (u0 + qu != pf_u) {
                int si_, row_;
                pf_u = u0 + qu;
                unit_src(pf_u, pf_w, pf_s0, pf_S, si_, row_);
            }
            const uint8_t *b = pf_w + (size_t)(pf_s0 + sq) * 16;
            const uint32_t dst = ring_s + (uint32_t)(q % RAW_R) * RAW_STAGE;
            cp_async16(dst, b);
#pragma unroll
            for (int c = 0; c < 4; c++)
                cp_async16(dst + (uint32_t)(1 + c) * RAW_CHUNK, b + (size_t)(1 + 4 * h + c) * pf_S * 16);
        }
        cp_async_commit();
    };
    // the weights do not depend on the previous kernel: their first copies go out before the wait
    for (int q = 0; q < RAW_D; q++) issue(q);
    pdl_wait();
    pdl_trigger();
    const uint32_t idesc = umma_idesc_u8s8(128, N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    int cur_tc = -1, tn = 0, q = 0;
    uint32_t gstep = 0;
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int tc = u / nrb;
        const uint8_t *wb_;
        int s0_, S_, si, row;
        unit_src(u, wb_, s0_, S_, si, row);
        const GemvSeg &sg = p.seg[si];
        if (tc != cur_tc) {  // the chunk's N token rows as Q8_K: B operand (zeros past the last token), scales, sums
            cur_tc = tc;
            const int t0 = tc * N;
            tn = p.T - t0 < N ? p.T - t0 : N;
            __syncthreads();  // the previous chunk's operands are no longer read
            const uint32_t sB_s = smem_u32(sB);
            for (int i = tid; i < N * K / 16; i += 256) {  // 16-byte pieces of the B operand
                const int t = i / (K / 16), k = (i - t * (K / 16)) * 16;
                if (t < tn) cp_async16(sB_s + umma_off(t, k, N), p.q8_qs + (long long)(t0 + t) * K + k);
                else *reinterpret_cast<uint4 *>(sB + umma_off(t, k, N)) = make_uint4(0, 0, 0, 0);
            }
            for (int i = tid; i < N * nsb * 2; i += 256) {  // 32-value sums, two 16-byte halves per block
                const int t = i / (nsb * 2), j = i - t * nsb * 2;
                if (t < tn) cp_async16(smem_u32(bsA + t * nsb * 8 + j * 4), p.q8_bs + (long long)(t0 + t) * nsb * 8 + j * 4);
                else *reinterpret_cast<int4 *>(bsA + t * nsb * 8 + j * 4) = make_int4(0, 0, 0, 0);
            }
            for (int i = tid; i < N * nsb; i += 256) {
                const int t = i / nsb, b = i - t * nsb;
                dA[i] = t < tn ? p.q8_d[(long long)(t0 + t) * nsb + b] : 0.0f;
            }
            cp_async_commit();
            cp_async_wait<0>();  // (the ring's copies in flight complete here too)
            __syncthreads();
        }
        float acc[HT];
#pragma unroll
        for (int t = 0; t < HT; t++) acc[t] = 0.0f;
        uint4 raw[5];
        int sc[8], mn[8], psc[8], pmn[8];
        float dw = 0.0f, dminw = 0.0f, pdw = 0.0f, pdminw = 0.0f;
        auto epilogue = [&](int sb, uint32_t gs) -> bool {
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            int sumi[HT];
            tmem_sumi<HT>(tmem + tlane + (gs & 1) * 8 * N + h * HT, N, psc, sumi);
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
        for (int st = 0; st < nsb; st++, q++) {
            const uint32_t gs = gstep++;
            ring_take(ring_t, q, raw, issue);
            q4k_header(raw[0], dw, dminw, sc, mn);
            q4k_unpack_a(sA + (gs & 1) * MMA_A_BYTES, raw, r, h);
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll 1
                for (int j = 0; j < 8; j++)
                    umma_i8(tmem + (gs & 1) * 8 * N + j * N,
                            umma_desc(aBase + (gs & 1) * MMA_A_BYTES + j * 4096, 128, 256),
                            umma_desc(bBase + (uint32_t)(st * 8 + j) * N * 32, 128, 256), idesc, false);
                umma_commit(smem_u32(&bars[gs & 1]));
            }
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
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsb - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
        const int t0 = tc * N + HT * h;
        for (int t = 0; t < HT && HT * h + t < tn; t++) {
            const long long yi = (long long)(t0 + t) * p.y_stride + sg.out_off + row;
            float y = acc[t];
            if (p.res) y = __fadd_rn(p.res[(long long)(t0 + t) * p.res_stride + sg.out_off + row], acc[t]);
            p.y[yi] = y;
        }
    }
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives it
    if (!ok && tid == 0) {
        for (uint32_t b = 0; b < 2; b++) {
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, TCOLS);
}

// ====================================================================== Q6_K rows on tcgen05
// The same GEMV for Q6_K segments of whole 128-row blocks, optionally with the output head's
// per-token argmax keys. Q6_K scales each 16-value sub-block on its own while one MMA of kind::i8
// covers K = 32, so each K step runs two MMAs against the same A (the row's 6-bit values as
// unsigned bytes, 0..63): one whose B holds the step's first 16 activation values and zeros for
// the other 16, one the other way round. Neither B is stored: per K step the chunk's
// activations lie in shared memory as [first halves][zeros][second halves], 16 token rows x 16
// bytes each, and the two descriptors start at the first and at the zero block with the K halves
// one block apart (LBO 256 B, SBO 128 B). 16 MMAs per superblock step write the 16 sub-block
// dots of 128 rows x 16 tokens into their own TMEM columns (2 x 256 columns, double-buffered); the
// epilogue finishes C4's Q6_K form per (row, token) -- sumi = sum_j sc_j (dot_j - 32 bs16_j),
// then (float)sumi * (d * d_a) added to the row's sum in superblock order -- the dp4a kernel's
// bits. Thread (row r, half h) copies its row's ql and qh of half h (4 + 2 pieces of 16 bytes)
// and either the 16 scales (h = 0) or the 16 bytes holding the superblock's d (h = 1) with
// cp.async Q6_RAW_D steps ahead; after the step's barrier each thread reads the other half's
// piece from the ring, and only then are the next copies requested, so no stage is rewritten
// while a thread still reads it.
constexpr int Q6_N = 16, Q6_HT = 8;
constexpr int Q6_RAW_D = 2, Q6_RAW_R = Q6_RAW_D + 1;
constexpr int Q6_RAW_STAGE = 7 * RAW_CHUNK;
constexpr int Q6_B_STEP = 3 * Q6_N * 16;      // one K step of B: first halves, zeros, second halves
constexpr uint32_t Q6_TCOLS = 2 * 16 * Q6_N;  // 2 buffers x 16 sub-blocks x 16 tokens

size_t gemv_mma6_smem_bytes(int K) {
    if (K <= 0 || K % 256) return (size_t)-1;
    const size_t nsb = (size_t)K / 256;
    const size_t b = 1024 + 2 * MMA_A_BYTES + (size_t)Q6_RAW_R * Q6_RAW_STAGE + (size_t)(K / 32) * Q6_B_STEP +
                     (size_t)Q6_N * nsb * 4 + (size_t)Q6_N * (K / 16) * 4 + 256;
    return b <= MMA_SMEM_LIMIT ? b : (size_t)-1;
}

// The A operand of one step: values 128h .. 128h+127 of row r (low 4 bits from ql, high 2 from
// qh) as unsigned bytes in natural order, value 128h + 32q + l at K step 4h + q, position l.
// raw[0..1] = ql[64h .. 64h+31], raw[2..3] = ql[64h+32 .. 64h+63], raw[4..5] = qh[32h .. 32h+31].
__device__ __forceinline__ void q6k_unpack_a(uint8_t *a, const uint4 (&raw)[6], int r, int h) {
    const uint32_t lo[8] = {raw[0].x, raw[0].y, raw[0].z, raw[0].w, raw[1].x, raw[1].y, raw[1].z, raw[1].w};
    const uint32_t hi[8] = {raw[2].x, raw[2].y, raw[2].z, raw[2].w, raw[3].x, raw[3].y, raw[3].z, raw[3].w};
    const uint32_t qh[8] = {raw[4].x, raw[4].y, raw[4].z, raw[4].w, raw[5].x, raw[5].y, raw[5].z, raw[5].w};
    uint32_t u[4][8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        u[0][i] = (lo[i] & 0x0F0F0F0Fu) | ((qh[i] << 4) & 0x30303030u);
        u[1][i] = (hi[i] & 0x0F0F0F0Fu) | ((qh[i] << 2) & 0x30303030u);
        u[2][i] = ((lo[i] >> 4) & 0x0F0F0F0Fu) | (qh[i] & 0x30303030u);
        u[3][i] = ((hi[i] >> 4) & 0x0F0F0F0Fu) | ((qh[i] >> 2) & 0x30303030u);
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
        *reinterpret_cast<uint4 *>(a + umma_off(r, (4 * h + q) * 32, 128)) = make_uint4(u[q][0], u[q][1], u[q][2], u[q][3]);
        *reinterpret_cast<uint4 *>(a + umma_off(r, (4 * h + q) * 32 + 16, 128)) =
            make_uint4(u[q][4], u[q][5], u[q][6], u[q][7]);
    }
}

// byte offset of the 16-byte piece k16 (values 16 k16 .. 16 k16 + 15) of token row t in B
__device__ __forceinline__ uint32_t q6_b_off(int t, int k16) {
    return (uint32_t)(k16 >> 1) * Q6_B_STEP + (uint32_t)(k16 & 1) * (2 * Q6_N * 16) + (uint32_t)(t >> 3) * 128 +
           (uint32_t)(t & 7) * 16;
}

__global__ void __launch_bounds__(256, 1) kq6_rows_mma_kernel(const __grid_constant__ GemvArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int K = p.K, nsb = K / 256, n16 = K / 16;
    uint8_t *sA = smem;                                                       // [2][8 K steps][128 rows][32]
    uint8_t *ring = sA + 2 * MMA_A_BYTES;                                     // [Q6_RAW_R][7][256 threads][16]
    uint8_t *sB = ring + Q6_RAW_R * Q6_RAW_STAGE;                             // [K/32][3][16 rows][16]
    float *dA = reinterpret_cast<float *>(sB + (size_t)(K / 32) * Q6_B_STEP);  // [16][nsb]
    int *bs16 = reinterpret_cast<int *>(dA + Q6_N * nsb);                     // [16][K/16]
    uint64_t *bars = reinterpret_cast<uint64_t *>(bs16 + Q6_N * n16);         // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // thread (row r of the block, half h): h unpacks values 128h .. 128h+127 of the row and
    // finishes the epilogue of tokens 8h .. 8h+7
    const int r = tid & 127, h = tid >> 7;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), Q6_TCOLS);
    for (int i = tid; i < (K / 32) * Q6_N; i += 256)  // the zero blocks of B, once
        *reinterpret_cast<uint4 *>(sB + (size_t)(i / Q6_N) * Q6_B_STEP + Q6_N * 16 + (i % Q6_N) * 16) =
            make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    int nrb = 0;  // 128-row blocks over the segments
    for (int i = 0; i < p.nseg; i++) nrb += p.seg[i].rows / 128;
    const int ntc = (p.T + Q6_N - 1) / Q6_N;
    const int total = ntc * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    // this thread's row of unit u: the segment, its tile, the row's first slot
    auto unit_src = [&](int u, const uint8_t *&wb, int &s0, int &S, int &si, int &row) {
        int rb = u - (u / nrb) * nrb;
        si = 0;
        while (rb >= p.seg[si].rows / 128) {
            rb -= p.seg[si].rows / 128;
            si++;
        }
        row = rb * 128 + r;
        wb = p.seg[si].w + (long long)(row / p.seg[si].rpt) * p.seg[si].tile_bytes;
        s0 = (row % p.seg[si].rpt) * nsb;
        S = p.seg[si].S;
    };
    const int Q = u1 > u0 ? (u1 - u0) * nsb : 0;
    const uint8_t *ring_t = ring + tid * 16;
    const uint32_t ring_s = smem_u32(ring) + (uint32_t)tid * 16;
    int pf_u = -1, pf_s0 = 0, pf_S = 0;
    const uint8_t *pf_w = nullptr;
    auto issue = [&](int q) {
        if (q < Q) {
            const int qu = q / nsb, sq = q - qu * nsb;
            if (u0 + qu != pf_u) {
                int si_, row_;
                pf_u = u0 + qu;
                unit_src(pf_u, pf_w, pf_s0, pf_S, si_, row_);
            }
            const int s = pf_s0 + sq;
            const size_t cs = (size_t)pf_S * 16;
            const uint8_t *b = pf_w + (size_t)s * 16;
            const uint32_t dst = ring_s + (uint32_t)(q % Q6_RAW_R) * Q6_RAW_STAGE;
#pragma unroll
            for (int c = 0; c < 4; c++) cp_async16(dst + (uint32_t)c * RAW_CHUNK, b + (size_t)(4 * h + c) * cs);
#pragma unroll
            for (int c = 0; c < 2; c++) cp_async16(dst + (uint32_t)(4 + c) * RAW_CHUNK, b + (size_t)(8 + 2 * h + c) * cs);
            if (h == 0) cp_async16(dst + 6u * RAW_CHUNK, b + 12 * cs);                          // the 16 scales
            else cp_async16(dst + 6u * RAW_CHUNK, pf_w + 13 * cs + (size_t)((2 * s) & ~15));  // d's 16 bytes
        }
        cp_async_commit();
    };
    // the weights do not depend on the previous kernel: their first copies go out before the wait
    for (int q = 0; q < Q6_RAW_D; q++) issue(q);
    pdl_wait();
    pdl_trigger();
    const uint32_t idesc = umma_idesc_u8s8(128, Q6_N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    int cur_tc = -1, tn = 0, q = 0;
    uint32_t gstep = 0;
    bool ok = true;
    unsigned long long best[Q6_HT];
#pragma unroll
    for (int t = 0; t < Q6_HT; t++) best[t] = 0ull;
    // the current chunk's argmax keys: per token, the max over this CTA's rows, one atomic per warp
    auto flush_best = [&]() {
        if (!p.amax || cur_tc < 0) return;
#pragma unroll
        for (int tt = 0; tt < Q6_HT; tt++) {
            unsigned long long b = best[tt];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const unsigned long long ob = __shfl_xor_sync(FULL, b, o);
                b = ob > b ? ob : b;
            }
            if (lane == 0 && Q6_HT * h + tt < tn) atomicMax(p.amax + cur_tc * Q6_N + Q6_HT * h + tt, b);
            best[tt] = 0ull;
        }
    };
    for (int u = u0; ok && u < u1; u++) {
        const int tc = u / nrb;
        const uint8_t *wb_;
        int s0, S_, si, row;
        unit_src(u, wb_, s0, S_, si, row);
        const GemvSeg &sg = p.seg[si];
        if (tc != cur_tc) {  // the chunk's 16 token rows as Q8_K: B (zeros past the last token), scales, 16-value sums
            flush_best();
            cur_tc = tc;
            const int t0 = tc * Q6_N;
            tn = p.T - t0 < Q6_N ? p.T - t0 : Q6_N;
            __syncthreads();  // the previous chunk's operands are no longer read
            const uint32_t sB_s = smem_u32(sB);
            for (int i = tid; i < Q6_N * n16; i += 256) {
                const int t = i / n16, k16 = i - t * n16;
                if (t < tn) cp_async16(sB_s + q6_b_off(t, k16), p.q8_qs + (long long)(t0 + t) * K + k16 * 16);
                else *reinterpret_cast<uint4 *>(sB + q6_b_off(t, k16)) = make_uint4(0, 0, 0, 0);
            }
            for (int i = tid; i < Q6_N * nsb; i += 256) {
                const int t = i / nsb, b = i - t * nsb;
                dA[i] = t < tn ? p.q8_d[(long long)(t0 + t) * nsb + b] : 0.0f;
            }
            cp_async_commit();
            cp_async_wait<0>();  // (the ring's copies in flight complete here too)
            __syncthreads();
            for (int i = tid; i < Q6_N * n16; i += 256) {  // bs16[t][k16]: the sum of those 16 values
                const uint4 v = *reinterpret_cast<const uint4 *>(sB + q6_b_off(i / n16, i % n16));
                int s = __dp4a((int)v.x, 0x01010101, 0);
                s = __dp4a((int)v.y, 0x01010101, s);
                s = __dp4a((int)v.z, 0x01010101, s);
                bs16[i] = __dp4a((int)v.w, 0x01010101, s);
            }
            __syncthreads();
        }
        float acc[Q6_HT];
#pragma unroll
        for (int t = 0; t < Q6_HT; t++) acc[t] = 0.0f;
        uint4 raw[6];
        int sc[16], psc[16];
        float dw = 0.0f, pdw = 0.0f;
        auto epilogue = [&](int sb, uint32_t gs) -> bool {
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            int sumi[Q6_HT];
#pragma unroll
            for (int t = 0; t < Q6_HT; t++) sumi[t] = 0;
            const uint32_t col0 = tmem + tlane + (gs & 1) * 16 * Q6_N + h * Q6_HT;
#pragma unroll
            for (int j0 = 0; j0 < 16; j0 += 4) {
                uint32_t v[4][8];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) tmem_ld8(col0 + (uint32_t)((j0 + jj) * Q6_N), v[jj]);
                tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 4; jj++) tmem_pin(v[jj]);
#pragma unroll
                for (int jj = 0; jj < 4; jj++)
#pragma unroll
                    for (int t = 0; t < Q6_HT; t++) sumi[t] += psc[j0 + jj] * (int)v[jj][t];
            }
#pragma unroll
            for (int tt = 0; tt < Q6_HT; tt++) {
                const int t = Q6_HT * h + tt;
                const int4 *bq = reinterpret_cast<const int4 *>(bs16 + t * n16 + sb * 16);
                int corr = 0;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int4 b = bq[c];
                    corr += psc[4 * c] * b.x + psc[4 * c + 1] * b.y + psc[4 * c + 2] * b.z + psc[4 * c + 3] * b.w;
                }
                const int si_ = sumi[tt] - 32 * corr;
                acc[tt] = __fadd_rn(acc[tt], __fmul_rn(__int2float_rn(si_), __fmul_rn(pdw, dA[t * nsb + sb])));
            }
            return true;
        };
        for (int st = 0; st < nsb; st++, q++) {
            const uint32_t gs = gstep++;
            cp_async_wait<Q6_RAW_D - 1>();  // this thread's pieces of step q have landed
            const uint8_t *stage = ring + (size_t)(q % Q6_RAW_R) * Q6_RAW_STAGE;
#pragma unroll
            for (int c = 0; c < 6; c++) raw[c] = *reinterpret_cast<const uint4 *>(stage + c * RAW_CHUNK + tid * 16);
            q6k_unpack_a(sA + (gs & 1) * MMA_A_BYTES, raw, r, h);
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint32_t a0 = aBase + (gs & 1) * MMA_A_BYTES;
#pragma unroll 1
                for (int j = 0; j < 8; j++) {
                    const uint64_t ad = umma_desc(a0 + j * 4096, 128, 256);
                    const uint32_t bj = bBase + (uint32_t)(st * 8 + j) * Q6_B_STEP;
                    const uint32_t d0 = tmem + (gs & 1) * 16 * Q6_N + (uint32_t)(2 * j) * Q6_N;
                    umma_i8(d0, ad, umma_desc(bj, 256, 128), idesc, false);
                    umma_i8(d0 + Q6_N, ad, umma_desc(bj + 2 * 128, 256, 128), idesc, false);
                }
                umma_commit(smem_u32(&bars[gs & 1]));
            }
            {  // the step's scales and d from both halves' pieces (visible after the barrier)
                const uint4 scv = *reinterpret_cast<const uint4 *>(stage + 6 * RAW_CHUNK + r * 16);
                const uint4 dv = *reinterpret_cast<const uint4 *>(stage + 6 * RAW_CHUNK + (128 + r) * 16);
                const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
                for (int j = 0; j < 16; j++) sc[j] = byte_s(scw[j >> 2], j & 3);
                const int o = (2 * (s0 + st)) & 15;  // d's byte offset in the piece (even)
                const unsigned long long dword = o < 8 ? ((unsigned long long)dv.y << 32) | dv.x
                                                       : ((unsigned long long)dv.w << 32) | dv.z;
                dw = __half2float(__ushort_as_half((unsigned short)((dword >> (8 * (o & 7))) & 0xffffu)));
            }
            issue(q + Q6_RAW_D);  // into the stage of step q - 1, which every thread has finished reading
            if (st > 0 && !__syncthreads_and(epilogue(st - 1, gs - 1))) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 16; j++) psc[j] = sc[j];
            pdw = dw;
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsb - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
        const int t0 = tc * Q6_N + Q6_HT * h;
#pragma unroll
        for (int tt = 0; tt < Q6_HT; tt++) {
            if (Q6_HT * h + tt < tn) {
                float y = acc[tt];
                if (p.res) y = __fadd_rn(p.res[(long long)(t0 + tt) * p.res_stride + sg.out_off + row], acc[tt]);
                p.y[(long long)(t0 + tt) * p.y_stride + sg.out_off + row] = y;
                const unsigned long long key =
                    ((unsigned long long)((unsigned)total_key(y) ^ 0x80000000u) << 32) | (unsigned)(sg.out_off + row);
                best[tt] = key > best[tt] ? key : best[tt];
            }
        }
    }
    if (ok) flush_best();
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives it
    if (!ok && tid == 0) {
        for (uint32_t b = 0; b < 2; b++) {
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, Q6_TCOLS);
}

// Q6_K down of the grouped batched path: kq6_rows_mma_kernel's arithmetic (two MMAs per K step
// against the halves of the activations, the Q6_K epilogue) over down_mma_kernel's units (chunk of
// at most 16 (token, slot) rows of one expert, block of 128 output rows), K = F, the rows' sums to
// dpart for the combine.
size_t down6_mma_smem_bytes(int F) {
    if (F <= 0 || F % 256) return (size_t)-1;
    const size_t nsb = (size_t)F / 256;
    const size_t b = 1024 + 2 * MMA_A_BYTES + (size_t)Q6_RAW_R * Q6_RAW_STAGE + (size_t)(F / 32) * Q6_B_STEP +
                     (size_t)Q6_N * nsb * 4 + (size_t)Q6_N * (F / 16) * 4 + 2 * Q6_N * 4 + 256;
    return b <= MMA_SMEM_LIMIT ? b : (size_t)-1;
}

__global__ void __launch_bounds__(256, 1) down6_mma_kernel(const __grid_constant__ ExpertArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int F = p.F, nsb = F / 256, n16 = F / 16, rpt = p.d_rpt, S = rpt * nsb;
    uint8_t *sA = smem;                                                       // [2][8 K steps][128 rows][32]
    uint8_t *ring = sA + 2 * MMA_A_BYTES;                                     // [Q6_RAW_R][7][256 threads][16]
    uint8_t *sB = ring + Q6_RAW_R * Q6_RAW_STAGE;                             // [F/32][3][16 rows][16]
    float *dA = reinterpret_cast<float *>(sB + (size_t)(F / 32) * Q6_B_STEP);  // [16][nsb]
    int *bs16 = reinterpret_cast<int *>(dA + Q6_N * nsb);                     // [16][F/16]
    int *tk_s = bs16 + Q6_N * n16;                                            // [16]
    uint64_t *bars = reinterpret_cast<uint64_t *>(tk_s + 2 * Q6_N);          // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & 127, h = tid >> 7;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), Q6_TCOLS);
    for (int i = tid; i < (F / 32) * Q6_N; i += 256)  // the zero blocks of B, once
        *reinterpret_cast<uint4 *>(sB + (size_t)(i / Q6_N) * Q6_B_STEP + Q6_N * 16 + (i % Q6_N) * 16) =
            make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_wait();  // the groups and the staged products come from the kernels before
    const int nrb = p.E / 128;
    const int total = *p.g_nchunks * nrb;
    const int u0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    pdl_trigger();
    // this thread's row of unit u: its tile and first slot
    auto unit_src = [&](int u, const uint8_t *&db, int &s0) {
        const int ci = u / nrb, rb = u - ci * nrb;
        const int row = rb * 128 + r;
        db = expert_down(p, p.g_chunk_e[ci]) + (long long)(row / rpt) * p.d_tile_bytes;
        s0 = (row % rpt) * nsb;
    };
    const int Q = u1 > u0 ? (u1 - u0) * nsb : 0;
    const uint32_t ring_s = smem_u32(ring) + (uint32_t)tid * 16;
    int pf_u = -1, pf_s0 = 0;
    const uint8_t *pf_w = nullptr;
    auto issue = [&](int q) {
        if (q < Q) {
            const int qu = q / nsb, sq = q - qu * nsb;
            if (u0 + qu != pf_u) {
                pf_u = u0 + qu;
                unit_src(pf_u, pf_w, pf_s0);
            }
            const int s = pf_s0 + sq;
            const size_t cs = (size_t)S * 16;
            const uint8_t *b = pf_w + (size_t)s * 16;
            const uint32_t dst = ring_s + (uint32_t)(q % Q6_RAW_R) * Q6_RAW_STAGE;
#pragma unroll
            for (int c = 0; c < 4; c++) cp_async16(dst + (uint32_t)c * RAW_CHUNK, b + (size_t)(4 * h + c) * cs);
#pragma unroll
            for (int c = 0; c < 2; c++) cp_async16(dst + (uint32_t)(4 + c) * RAW_CHUNK, b + (size_t)(8 + 2 * h + c) * cs);
            if (h == 0) cp_async16(dst + 6u * RAW_CHUNK, b + 12 * cs);                          // the 16 scales
            else cp_async16(dst + 6u * RAW_CHUNK, pf_w + 13 * cs + (size_t)((2 * s) & ~15));  // d's 16 bytes
        }
        cp_async_commit();
    };
    for (int q = 0; q < Q6_RAW_D; q++) issue(q);
    const uint32_t idesc = umma_idesc_u8s8(128, Q6_N);
    const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
    int cur_chunk = -1, mc = 0, q = 0;
    uint32_t gstep = 0;
    bool ok = true;
    for (int u = u0; ok && u < u1; u++) {
        const int ci = u / nrb, rb = u - ci * nrb;
        int s0;
        {
            const uint8_t *db_;
            unit_src(u, db_, s0);
        }
        if (ci != cur_chunk) {  // the chunk's rows as Q8_K: B (zeros past mc), scales, 16-value sums
            cur_chunk = ci;
            const int e = p.g_chunk_e[ci];
            const int c0 = p.g_chunk_r0[ci], m = p.g_count[e], off = p.g_off[e];
            mc = m - c0 < Q6_N ? m - c0 : Q6_N;
            __syncthreads();  // the previous chunk's operands are no longer read
            if (tid < mc) tk_s[tid] = p.g_list[off + c0 + tid];
            __syncthreads();
            const uint32_t sB_s = smem_u32(sB);
            for (int i = tid; i < Q6_N * n16; i += 256) {
                const int t = i / n16, k16 = i - t * n16;
                if (t < mc) cp_async16(sB_s + q6_b_off(t, k16), p.q8_qs + (long long)tk_s[t] * F + k16 * 16);
                else *reinterpret_cast<uint4 *>(sB + q6_b_off(t, k16)) = make_uint4(0, 0, 0, 0);
            }
            for (int i = tid; i < Q6_N * nsb; i += 256) {
                const int t = i / nsb, b = i - t * nsb;
                dA[i] = t < mc ? p.q8_d[(long long)tk_s[t] * nsb + b] : 0.0f;
            }
            cp_async_commit();
            cp_async_wait<0>();  // (the ring's copies in flight complete here too)
            __syncthreads();
            for (int i = tid; i < Q6_N * n16; i += 256) {  // bs16[t][k16]: the sum of those 16 values
                const uint4 v = *reinterpret_cast<const uint4 *>(sB + q6_b_off(i / n16, i % n16));
                int s = __dp4a((int)v.x, 0x01010101, 0);
                s = __dp4a((int)v.y, 0x01010101, s);
                s = __dp4a((int)v.z, 0x01010101, s);
                bs16[i] = __dp4a((int)v.w, 0x01010101, s);
            }
            __syncthreads();
        }
        const int row = rb * 128 + r;
        float acc[Q6_HT];
#pragma unroll
        for (int t = 0; t < Q6_HT; t++) acc[t] = 0.0f;
        uint4 raw[6];
        int sc[16], psc[16];
        float dw = 0.0f, pdw = 0.0f;
        auto epilogue = [&](int sb, uint32_t gs) -> bool {
            if (!mbar_wait(&bars[gs & 1], (gs >> 1) & 1, p.err)) return false;
            tc_fence_after();
            int sumi[Q6_HT];
#pragma unroll
            for (int t = 0; t < Q6_HT; t++) sumi[t] = 0;
            const uint32_t col0 = tmem + tlane + (gs & 1) * 16 * Q6_N + h * Q6_HT;
#pragma unroll
            for (int j0 = 0; j0 < 16; j0 += 4) {
                uint32_t v[4][8];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) tmem_ld8(col0 + (uint32_t)((j0 + jj) * Q6_N), v[jj]);
                tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 4; jj++) tmem_pin(v[jj]);
#pragma unroll
                for (int jj = 0; jj < 4; jj++)
#pragma unroll
                    for (int t = 0; t < Q6_HT; t++) sumi[t] += psc[j0 + jj] * (int)v[jj][t];
            }
#pragma unroll
            for (int tt = 0; tt < Q6_HT; tt++) {
                const int t = Q6_HT * h + tt;
                const int4 *bq = reinterpret_cast<const int4 *>(bs16 + t * n16 + sb * 16);
                int corr = 0;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int4 b = bq[c];
                    corr += psc[4 * c] * b.x + psc[4 * c + 1] * b.y + psc[4 * c + 2] * b.z + psc[4 * c + 3] * b.w;
                }
                const int si_ = sumi[tt] - 32 * corr;
                acc[tt] = __fadd_rn(acc[tt], __fmul_rn(__int2float_rn(si_), __fmul_rn(pdw, dA[t * nsb + sb])));
            }
            return true;
        };
        for (int st = 0; st < nsb; st++, q++) {
            const uint32_t gs = gstep++;
            cp_async_wait<Q6_RAW_D - 1>();  // this thread's pieces of step q have landed
            const uint8_t *stage = ring + (size_t)(q % Q6_RAW_R) * Q6_RAW_STAGE;
#pragma unroll
            for (int c = 0; c < 6; c++) raw[c] = *reinterpret_cast<const uint4 *>(stage + c * RAW_CHUNK + tid * 16);
            q6k_unpack_a(sA + (gs & 1) * MMA_A_BYTES, raw, r, h);
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint32_t a0 = aBase + (gs & 1) * MMA_A_BYTES;
#pragma unroll 1
                for (int j = 0; j < 8; j++) {
                    const uint64_t ad = umma_desc(a0 + j * 4096, 128, 256);
                    const uint32_t bj = bBase + (uint32_t)(st * 8 + j) * Q6_B_STEP;
                    const uint32_t d0 = tmem + (gs & 1) * 16 * Q6_N + (uint32_t)(2 * j) * Q6_N;
                    umma_i8(d0, ad, umma_desc(bj, 256, 128), idesc, false);
                    umma_i8(d0 + Q6_N, ad, umma_desc(bj + 2 * 128, 256, 128), idesc, false);
                }
                umma_commit(smem_u32(&bars[gs & 1]));
            }
            {  // the step's scales and d from both halves' pieces (visible after the barrier)
                const uint4 scv = *reinterpret_cast<const uint4 *>(stage + 6 * RAW_CHUNK + r * 16);
                const uint4 dv = *reinterpret_cast<const uint4 *>(stage + 6 * RAW_CHUNK + (128 + r) * 16);
                const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
                for (int j = 0; j < 16; j++) sc[j] = byte_s(scw[j >> 2], j & 3);
                const int o = (2 * (s0 + st)) & 15;  // d's byte offset in the piece (even)
                const unsigned long long dword = o < 8 ? ((unsigned long long)dv.y << 32) | dv.x
                                                       : ((unsigned long long)dv.w << 32) | dv.z;
                dw = __half2float(__ushort_as_half((unsigned short)((dword >> (8 * (o & 7))) & 0xffffu)));
            }
            issue(q + Q6_RAW_D);  // into the stage of step q - 1, which every thread has finished reading
            if (st > 0 && !__syncthreads_and(epilogue(st - 1, gs - 1))) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 16; j++) psc[j] = sc[j];
            pdw = dw;
            tc_fence_before();
        }
        if (!ok) break;
        if (!__syncthreads_and(epilogue(nsb - 1, gstep - 1))) {
            ok = false;
            break;
        }
        tc_fence_before();
#pragma unroll
        for (int tt = 0; tt < Q6_HT; tt++)
            if (Q6_HT * h + tt < mc) p.dpart[(long long)tk_s[Q6_HT * h + tt] * p.E + row] = acc[tt];
    }
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives it
    if (!ok && tid == 0) {
        for (uint32_t b = 0; b < 2; b++) {
            const long long last = gstep == 0 ? -1 : ((long long)((gstep - 1) & 1) == b ? gstep - 1 : (long long)gstep - 2);
            if (last >= 0) mbar_wait(&bars[b], (uint32_t)(last >> 1) & 1, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, Q6_TCOLS);
}

cudaError_t launch_down6_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    const size_t smem = down6_mma_smem_bytes(a.F);
    if (smem == (size_t)-1 || a.d_rpt < 1 || a.d_rpt * (a.F / 256) > 32 || a.E % 128 || a.dtype != T_Q6_K ||
        a.d_nsb != a.F / 256 || a.d_tile_bytes % 16 ||
        a.d_tile_bytes != 13 * 16 * a.d_rpt * (a.F / 256) + (2 * a.d_rpt * (a.F / 256) + 15) / 16 * 16)
        return cudaErrorInvalidValue;
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
    return cudaLaunchKernelEx(&cfg, down6_mma_kernel, a);
}

cudaError_t launch_gemv_mma6(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    const size_t smem = gemv_mma6_smem_bytes(a.K);
    if (smem == (size_t)-1) return cudaErrorInvalidValue;
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
    return cudaLaunchKernelEx(&cfg, kq6_rows_mma_kernel, a);
}

cudaError_t launch_gemv_mma(const GemvArgs &a, int grid, cudaStream_t st, bool pdl) {
    const int n = gemv_mma_tokens(a.K);
    if (!n) return cudaErrorInvalidValue;
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
    return n == 32 ? cudaLaunchKernelEx(&cfg, kq_rows_mma_kernel<32>, a) : cudaLaunchKernelEx(&cfg, kq_rows_mma_kernel<16>, a);
}

cudaError_t init_mma_attributes() {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev))) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))) return e;
    const void *kerns[] = {(const void *)gateup_mma_kernel, (const void *)kq_rows_mma_kernel<32>,
                           (const void *)kq_rows_mma_kernel<16>, (const void *)kq6_rows_mma_kernel,
                           (const void *)down_mma_kernel, (const void *)down6_mma_kernel};
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
