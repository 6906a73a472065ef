// stage.cuh -- staging of activations as Q8_K blocks in shared memory (contracts C3, C5, C6),
// shared by the per-phase kernels and the persistent decode-step kernel.
#pragma once
#include "bt_common.cuh"
#include "kquant.cuh"

namespace bt {

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
    if ((lane & 1) == 0) dst->bs16[lane >> 1] = (int16_t)s16;
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
            float acc = warp_sumsq_p2(xt, K, lane);
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

}  // namespace bt
