// kquant.cuh -- Q4_K / Q6_K block formats, the HBM tile layout, the seeded synthetic
// quantiser and the per-slot integer dot products of the GEMV kernels.
//
// Block formats (ggml block_q4_K / block_q6_K; Chaos reads them at core/model/src/validate.rs:60-75
// and sizes them at core/gguf/src/tensor.rs:30-32):
//   Q4_K, 144 B / 256 values: f16 d, f16 dmin, 12 bytes of packed 6-bit scales and mins,
//         128 bytes of 4-bit quants; value = (d*sc)*q - (dmin*m).
//   Q6_K, 210 B / 256 values: 128 B low nibbles, 64 B high 2-bit pairs, 16 int8 scales,
//         f16 d; value = (d*sc)*(q-32).
//
// HBM tile layout ("tiled-S"): a matrix of R rows x nsb superblocks is cut into tiles of
// `rpt` rows; tile t holds the S = rpt*nsb superblocks of rows [t*rpt, t*rpt+rpt) as slots
// s = (row - t*rpt)*nsb + b. A superblock's 16-byte chunk c lives at c*S*16 + s*16 inside
// the tile, so one warp whose lane s reads chunk c touches S*16 contiguous bytes: every
// 16-byte load of a superblock is coalesced across the warp. Q6_K's trailing f16 d (the
// bytes after its 13 whole chunks) goes to a plane at 13*S*16 + s*2, padded to 16 bytes.
// The permutation is lossless: a tile carries exactly the GGUF bytes of its rows.
#pragma once
#include <cuda_fp16.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

namespace bt {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_K = 12, T_Q6_K = 14 };

__host__ __device__ inline int qk_block_bytes(int type) { return type == T_Q4_K ? 144 : (type == T_Q6_K ? 210 : 0); }
__host__ __device__ inline int qk_chunks(int type) { return type == T_Q4_K ? 9 : 13; }

struct TileGeom {
    int type, nsb, rpt, S, tile_bytes;
    long long n_tiles;
    long long rows;
};

__host__ __device__ inline TileGeom tile_geom(int type, long long rows, long long cols, int rpt) {
    TileGeom g;
    g.type = type;
    g.nsb = (int)(cols / 256);
    g.rpt = rpt;
    g.S = rpt * g.nsb;
    g.rows = rows;
    if (type == T_Q4_K) g.tile_bytes = 9 * g.S * 16;
    else g.tile_bytes = 13 * g.S * 16 + ((g.S * 2 + 15) / 16) * 16;
    g.n_tiles = (rows + rpt - 1) / rpt;
    return g;
}

// the row count per tile a warp-wide GEMV uses: as many whole rows as fit in 32 slots
__host__ __device__ inline int default_rpt(long long cols) {
    int nsb = (int)(cols / 256);
    return nsb > 0 && nsb <= 32 ? 32 / nsb : 0;
}

// ------------------------------------------------------------------ f16 on host and device
__host__ __device__ inline uint16_t f32_to_f16_bits(float f) {
#ifdef __CUDA_ARCH__
    return __half_as_ushort(__float2half_rn(f));
#else
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, e8 = (x >> 23) & 0xffu, mant = x & 0x7fffffu;
    if (e8 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    int e = (int)e8 - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1u), mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13), rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
#endif
}

__host__ __device__ inline float f16_bits_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
    return __half2float(__ushort_as_half(h));
#else
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16, e = ((uint32_t)h >> 10) & 0x1fu, m = (uint32_t)h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
#endif
}

// ------------------------------------------------------------------ seeded synthetic values
__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Irwin-Hall(4) approximation of N(mean, sigma): four 16-bit uniforms from one 64-bit hash.
// Integer sum, one int->float conversion and two rounded float ops: the same bits on the
// host and the device.
__host__ __device__ inline float synth_value(uint64_t key, uint64_t idx, float mean, float scale) {
    uint64_t h = splitmix64(key + idx * 0xD1B54A32D192ED03ull);
    int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) + (int)(h >> 48);
    float z = (float)(s - 131070) * scale;
    return mean + z;
}

__host__ __device__ inline uint64_t synth_key(uint64_t seed, uint64_t tensor_id) {
    return splitmix64(seed ^ splitmix64(tensor_id));
}

// sigma * sqrt(3) / 65536: unit variance for the centred sum of four 16-bit uniforms
__host__ __device__ inline float synth_scale(float sigma) { return sigma * 2.64296052e-05f; }

__host__ __device__ inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// A simple K-quant quantiser: per 32-value sub-block min/max, 6-bit scales and mins.
__host__ __device__ inline void quant_q4k_block(const float *x, uint8_t *out) {
    float scl[8], mns[8];
    for (int j = 0; j < 8; j++) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; l++) {
            float v = x[32 * j + l];
            mn = v < mn ? v : mn;
            mx = v > mx ? v : mx;
        }
        if (mn > 0.0f) mn = 0.0f;
        scl[j] = (mx - mn) / 15.0f;
        mns[j] = -mn;
    }
    float ms = 0.0f, mm = 0.0f;
    for (int j = 0; j < 8; j++) {
        ms = scl[j] > ms ? scl[j] : ms;
        mm = mns[j] > mm ? mns[j] : mm;
    }
    uint16_t dh = f32_to_f16_bits(ms / 63.0f), dmh = f32_to_f16_bits(mm / 63.0f);
    float df = f16_bits_to_f32(dh), dmf = f16_bits_to_f32(dmh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = df > 0.0f ? clampi((int)rintf(scl[j] / df), 0, 63) : 0;
        m[j] = dmf > 0.0f ? clampi((int)rintf(mns[j] / dmf), 0, 63) : 0;
    }
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(dmh & 0xff);
    out[3] = (uint8_t)(dmh >> 8);
    uint8_t *s = out + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t *qs = out + 16;
    for (int g = 0; g < 4; g++) {
        float d0 = df * (float)sc[2 * g], m0 = dmf * (float)m[2 * g];
        float d1 = df * (float)sc[2 * g + 1], m1 = dmf * (float)m[2 * g + 1];
        for (int l = 0; l < 32; l++) {
            int q0 = d0 > 0.0f ? clampi((int)rintf((x[64 * g + l] + m0) / d0), 0, 15) : 0;
            int q1 = d1 > 0.0f ? clampi((int)rintf((x[64 * g + 32 + l] + m1) / d1), 0, 15) : 0;
            qs[32 * g + l] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

__host__ __device__ inline void quant_q6k_block(const float *x, uint8_t *out) {
    float ds[16];
    for (int s = 0; s < 16; s++) {
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 16; i++) {
            float v = x[16 * s + i], av = fabsf(v);
            if (av > amax) {
                amax = av;
                mx = v;
            }
        }
        ds[s] = amax == 0.0f ? 0.0f : mx / -32.0f;
    }
    float amax = 0.0f, smax = 0.0f;
    for (int s = 0; s < 16; s++) {
        float av = fabsf(ds[s]);
        if (av > amax) {
            amax = av;
            smax = ds[s];
        }
    }
    int L[256];
    int8_t sc[16];
    uint16_t dh = 0;
    if (amax == 0.0f) {
        for (int i = 0; i < 256; i++) L[i] = 32;
        for (int s = 0; s < 16; s++) sc[s] = 0;
    } else {
        float iscale = -128.0f / smax;
        dh = f32_to_f16_bits(1.0f / iscale);
        float df = f16_bits_to_f32(dh);
        for (int s = 0; s < 16; s++) {
            sc[s] = (int8_t)clampi((int)rintf(iscale * ds[s]), -128, 127);
            float den = df * (float)sc[s];
            for (int i = 0; i < 16; i++) {
                int q = den != 0.0f ? clampi((int)rintf(x[16 * s + i] / den), -32, 31) : 0;
                L[16 * s + i] = q + 32;
            }
        }
    }
    uint8_t *ql = out, *qh = out + 128;
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            int L1 = L[128 * n + l], L2 = L[128 * n + 32 + l], L3 = L[128 * n + 64 + l], L4 = L[128 * n + 96 + l];
            ql[64 * n + l] = (uint8_t)((L1 & 0xF) | ((L3 & 0xF) << 4));
            ql[64 * n + 32 + l] = (uint8_t)((L2 & 0xF) | ((L4 & 0xF) << 4));
            qh[32 * n + l] = (uint8_t)((L1 >> 4) | ((L2 >> 4) << 2) | ((L3 >> 4) << 4) | ((L4 >> 4) << 6));
        }
    for (int s = 0; s < 16; s++) out[192 + s] = (uint8_t)sc[s];
    out[208] = (uint8_t)(dh & 0xff);
    out[209] = (uint8_t)(dh >> 8);
}

// One superblock (or, for F32/F16, 256 elements) of a synthetic tensor, element index base
// `e0` in row-major order.
__host__ __device__ inline void synth_block(int type, uint64_t key, uint64_t e0, float mean, float scale,
                                            uint8_t *out) {
    float x[256];
    for (int i = 0; i < 256; i++) x[i] = synth_value(key, e0 + (uint64_t)i, mean, scale);
    if (type == T_Q4_K) quant_q4k_block(x, out);
    else if (type == T_Q6_K) quant_q6k_block(x, out);
    else if (type == T_F32) memcpy(out, x, sizeof x);
    else if (type == T_F16) {
        for (int i = 0; i < 256; i++) {
            uint16_t h = f32_to_f16_bits(x[i]);
            out[2 * i] = (uint8_t)(h & 0xff);
            out[2 * i + 1] = (uint8_t)(h >> 8);
        }
    }
}

__host__ __device__ inline int synth_block_bytes(int type) {
    return type == T_Q4_K ? 144 : type == T_Q6_K ? 210 : type == T_F32 ? 1024 : 512;
}

// FNV-1a of a tensor name: the tensor id of the synthetic generator
inline uint64_t name_id(const char *s) {
    uint64_t h = 1469598103934665603ull;
    while (*s) {
        h ^= (uint8_t)*s++;
        h *= 1099511628211ull;
    }
    return h;
}

// ------------------------------------------------------------------ device-side decode
#ifdef __CUDACC__

// Q8_K activation block as staged in shared memory: 256 quants, scale, the sums of the 8
// sub-blocks of 32 (the Q4_K min term) and of the 16 sub-blocks of 16 (the Q6_K offset term).
// 336 bytes = 21 x 16, so 8 consecutive blocks start in 8 different 16-byte bank groups.
struct __align__(16) ActBlock {
    int8_t qs[256];
    float d;
    int pad[3];
    int bs32[8];
    int16_t bs16[16];
};
static_assert(sizeof(ActBlock) == 336, "ActBlock layout");
static_assert(offsetof(ActBlock, d) == 256 && offsetof(ActBlock, bs32) == 272 && offsetof(ActBlock, bs16) == 304,
              "ActBlock field offsets");

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }
// unsigned bytes of a times signed bytes of b, accumulated into c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int byte_u(uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xffu); }
__device__ __forceinline__ int byte_s(uint32_t w, int k) { return (int)(int8_t)((w >> (8 * k)) & 0xffu); }

// Shared-memory loads at 32-bit shared-window addresses. The dots below take such addresses,
// so a non-inlined copy of them still reads shared memory with shared loads. The "memory"
// clobber keeps them after the waits that make the data valid.
__device__ __forceinline__ uint4 lds_u4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint16_t lds_u16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
    return v;
}
// ActBlock field offsets, for the address-based dots
constexpr uint32_t ACT_D = 256, ACT_BS32 = 272, ACT_BS16 = 304;

// C4 for one Q4_K superblock (slot s of a tile at shared address tile_s, S slots) against the
// activation block at act_s: sumi = sum_j sc_j * (q . a over sub-block j), summ = sum_j m_j *
// bs32_j (integers, so the grouping below gives the same values as any other order), then
// (float)sumi * (d * d_a) - (float)summ * (dmin * d_a). High nibbles enter the dot unshifted
// (unsigned x signed dp4a) and the exact multiple of 16 is shifted out afterwards.
__device__ __forceinline__ float q4k_dot_s(uint32_t tile_s, int S, int s, uint32_t act_s) {
    const uint32_t base = tile_s + (uint32_t)s * 16u, cstride = (uint32_t)S * 16u;
    const uint4 h = lds_u4(base);
    const float dw = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffff)));
    const float dminw = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t s03 = h.y, s47 = h.z, s811 = h.w;  // the 12 packed scale bytes (get_scale_min_k4)
    const uint32_t sc_lo = s03 & 0x3F3F3F3Fu, m_lo = s47 & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (s811 & 0x0F0F0F0Fu) | ((s03 >> 2) & 0x30303030u);
    const uint32_t m_hi = ((s811 >> 4) & 0x0F0F0F0Fu) | ((s47 >> 2) & 0x30303030u);
    int dot[8];
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const uint4 w0 = lds_u4(base + (1 + 2 * g) * cstride), w1 = lds_u4(base + (2 + 2 * g) * cstride);
        const uint4 al0 = lds_u4(act_s + 64 * g), al1 = lds_u4(act_s + 64 * g + 16);
        const uint4 ah0 = lds_u4(act_s + 64 * g + 32), ah1 = lds_u4(act_s + 64 * g + 48);
        int dlo = 0, dhi = 0;
        dlo = dp4a(w0.x & 0x0F0F0F0F, al0.x, dlo);
        dlo = dp4a(w0.y & 0x0F0F0F0F, al0.y, dlo);
        dlo = dp4a(w0.z & 0x0F0F0F0F, al0.z, dlo);
        dlo = dp4a(w0.w & 0x0F0F0F0F, al0.w, dlo);
        dlo = dp4a(w1.x & 0x0F0F0F0F, al1.x, dlo);
        dlo = dp4a(w1.y & 0x0F0F0F0F, al1.y, dlo);
        dlo = dp4a(w1.z & 0x0F0F0F0F, al1.z, dlo);
        dlo = dp4a(w1.w & 0x0F0F0F0F, al1.w, dlo);
        dhi = dp4a_us(w0.x & 0xF0F0F0F0u, ah0.x, dhi);
        dhi = dp4a_us(w0.y & 0xF0F0F0F0u, ah0.y, dhi);
        dhi = dp4a_us(w0.z & 0xF0F0F0F0u, ah0.z, dhi);
        dhi = dp4a_us(w0.w & 0xF0F0F0F0u, ah0.w, dhi);
        dhi = dp4a_us(w1.x & 0xF0F0F0F0u, ah1.x, dhi);
        dhi = dp4a_us(w1.y & 0xF0F0F0F0u, ah1.y, dhi);
        dhi = dp4a_us(w1.z & 0xF0F0F0F0u, ah1.z, dhi);
        dhi = dp4a_us(w1.w & 0xF0F0F0F0u, ah1.w, dhi);
        dot[2 * g] = dlo;
        dot[2 * g + 1] = dhi >> 4;
    }
    const uint4 b0 = lds_u4(act_s + ACT_BS32), b1 = lds_u4(act_s + ACT_BS32 + 16);
    const int bs[8] = {(int)b0.x, (int)b0.y, (int)b0.z, (int)b0.w, (int)b1.x, (int)b1.y, (int)b1.z, (int)b1.w};
    int sumi = 0, summ = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int sc = j < 4 ? byte_u(sc_lo, j) : byte_u(sc_hi, j - 4);
        const int m = j < 4 ? byte_u(m_lo, j) : byte_u(m_hi, j - 4);
        sumi += sc * dot[j];
        summ += m * bs[j];
    }
    const float da = lds_f32(act_s + ACT_D);
    const float t1 = __fmul_rn(dw, da);
    const float t2 = __fmul_rn(__int2float_rn(sumi), t1);
    const float t3 = __fmul_rn(dminw, da);
    const float t4 = __fmul_rn(__int2float_rn(summ), t3);
    return __fsub_rn(t2, t4);
}

// C4 for one Q6_K superblock: sumi = sum over the 16 sub-blocks of sc * (q - 32) . a, computed
// as sc * (u . a - 32 * bs16) with u = q + 32 in [0, 63] (unsigned x signed dp4a; integers, so
// equal to the per-value form), then (float)sumi * (d * d_a). Value v of the superblock:
// n = v / 128, quad = (v % 128) / 32, l = v % 32; low nibble from ql[64n + 32 * (quad & 1) + l]
// (high nibble when quad >= 2), two high bits from qh[32n + l] >> 2 * quad; sub-block v / 16.
// In the tile: chunks 0-7 ql, 8-11 qh, 12 the scales, and d in a plane after chunk row 12.
__device__ __forceinline__ float q6k_dot_s(uint32_t tile_s, int S, int s, uint32_t act_s) {
    const uint32_t base = tile_s + (uint32_t)s * 16u, cstride = (uint32_t)S * 16u;
    const uint16_t dbits = lds_u16(tile_s + 13u * cstride + 2u * (uint32_t)s);
    const float dw = __half2float(__ushort_as_half(dbits));
    const uint4 scv = lds_u4(base + 12u * cstride);  // the 16 int8 sub-block scales
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
    const uint4 bq0 = lds_u4(act_s + ACT_BS16), bq1 = lds_u4(act_s + ACT_BS16 + 16);
    const uint32_t bsw[8] = {bq0.x, bq0.y, bq0.z, bq0.w, bq1.x, bq1.y, bq1.z, bq1.w};
    int sumi = 0;
#pragma unroll
    for (int n = 0; n < 2; n++) {
        const uint4 qa0 = lds_u4(base + (4 * n + 0) * cstride), qa1 = lds_u4(base + (4 * n + 1) * cstride);
        const uint4 qb0 = lds_u4(base + (4 * n + 2) * cstride), qb1 = lds_u4(base + (4 * n + 3) * cstride);
        const uint4 hh0 = lds_u4(base + (8 + 2 * n) * cstride), hh1 = lds_u4(base + (9 + 2 * n) * cstride);
        const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
        const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
        const uint32_t wh[8] = {hh0.x, hh0.y, hh0.z, hh0.w, hh1.x, hh1.y, hh1.z, hh1.w};
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {  // l = 16 hf .. 16 hf + 15: sub-blocks 8n + 2 quad + hf
            const uint4 A0 = lds_u4(act_s + 16 * (8 * n + 0 + hf)), A1 = lds_u4(act_s + 16 * (8 * n + 2 + hf));
            const uint4 A2 = lds_u4(act_s + 16 * (8 * n + 4 + hf)), A3 = lds_u4(act_s + 16 * (8 * n + 6 + hf));
            const uint32_t a0[4] = {A0.x, A0.y, A0.z, A0.w}, a1[4] = {A1.x, A1.y, A1.z, A1.w};
            const uint32_t a2[4] = {A2.x, A2.y, A2.z, A2.w}, a3[4] = {A3.x, A3.y, A3.z, A3.w};
            int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int l4 = 4 * hf + i;
                const uint32_t hq = wh[l4];
                const uint32_t u1 = (wa[l4] & 0x0F0F0F0Fu) | ((hq << 4) & 0x30303030u);
                const uint32_t u2 = (wb[l4] & 0x0F0F0F0Fu) | ((hq << 2) & 0x30303030u);
                const uint32_t u3 = ((wa[l4] >> 4) & 0x0F0F0F0Fu) | (hq & 0x30303030u);
                const uint32_t u4 = ((wb[l4] >> 4) & 0x0F0F0F0Fu) | ((hq >> 2) & 0x30303030u);
                acc0 = dp4a_us(u1, (int)a0[i], acc0);
                acc1 = dp4a_us(u2, (int)a1[i], acc1);
                acc2 = dp4a_us(u3, (int)a2[i], acc2);
                acc3 = dp4a_us(u4, (int)a3[i], acc3);
            }
            const int accs[4] = {acc0, acc1, acc2, acc3};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int sub = 8 * n + 2 * q + hf;
                const int sc = byte_s(scw[sub >> 2], sub & 3);
                const int bs = (int)(int16_t)((bsw[sub >> 1] >> (16 * (sub & 1))) & 0xffffu);
                sumi += sc * (accs[q] - 32 * bs);
            }
        }
    }
    return __fmul_rn(__int2float_rn(sumi), __fmul_rn(dw, lds_f32(act_s + ACT_D)));
}

// Register-resident forms for several tokens against one weight superblock: *_load_r decodes
// lane s's superblock of the tile once (nibbles masked, 6-bit values assembled, scales
// unpacked), *_dot_r then computes one token's dot from its activation block. Each is the same
// integer and float arithmetic, in the same order, as q4k_dot_s / q6k_dot_s.
struct Q4Reg {
    uint32_t lo[32], hi[32];  // per 32-value group g: words 8g..8g+7, low and high nibbles in place
    int sc[8], mn[8];
    float dw, dminw;
};
__device__ __forceinline__ void q4k_load_r(Q4Reg &r, uint32_t tile_s, int S, int s) {
    const uint32_t base = tile_s + (uint32_t)s * 16u, cstride = (uint32_t)S * 16u;
    const uint4 h = lds_u4(base);
    r.dw = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffff)));
    r.dminw = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t s03 = h.y, s47 = h.z, s811 = h.w;
    const uint32_t sc_lo = s03 & 0x3F3F3F3Fu, m_lo = s47 & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (s811 & 0x0F0F0F0Fu) | ((s03 >> 2) & 0x30303030u);
    const uint32_t m_hi = ((s811 >> 4) & 0x0F0F0F0Fu) | ((s47 >> 2) & 0x30303030u);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        r.sc[j] = byte_u(sc_lo, j);
        r.sc[j + 4] = byte_u(sc_hi, j);
        r.mn[j] = byte_u(m_lo, j);
        r.mn[j + 4] = byte_u(m_hi, j);
    }
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const uint4 w0 = lds_u4(base + (1 + 2 * g) * cstride), w1 = lds_u4(base + (2 + 2 * g) * cstride);
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            r.lo[8 * g + i] = w[i] & 0x0F0F0F0Fu;
            r.hi[8 * g + i] = w[i] & 0xF0F0F0F0u;
        }
    }
}
__device__ __forceinline__ float q4k_dot_r(const Q4Reg &r, uint32_t act_s) {
    int dot[8];
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const uint4 al0 = lds_u4(act_s + 64 * g), al1 = lds_u4(act_s + 64 * g + 16);
        const uint4 ah0 = lds_u4(act_s + 64 * g + 32), ah1 = lds_u4(act_s + 64 * g + 48);
        const uint32_t al[8] = {al0.x, al0.y, al0.z, al0.w, al1.x, al1.y, al1.z, al1.w};
        const uint32_t ah[8] = {ah0.x, ah0.y, ah0.z, ah0.w, ah1.x, ah1.y, ah1.z, ah1.w};
        int dlo = 0, dhi = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            dlo = dp4a((int)r.lo[8 * g + i], (int)al[i], dlo);
            dhi = dp4a_us(r.hi[8 * g + i], (int)ah[i], dhi);
        }
        dot[2 * g] = dlo;
        dot[2 * g + 1] = dhi >> 4;
    }
    const uint4 b0 = lds_u4(act_s + ACT_BS32), b1 = lds_u4(act_s + ACT_BS32 + 16);
    const int bs[8] = {(int)b0.x, (int)b0.y, (int)b0.z, (int)b0.w, (int)b1.x, (int)b1.y, (int)b1.z, (int)b1.w};
    int sumi = 0, summ = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        sumi += r.sc[j] * dot[j];
        summ += r.mn[j] * bs[j];
    }
    const float da = lds_f32(act_s + ACT_D);
    const float t1 = __fmul_rn(r.dw, da);
    const float t2 = __fmul_rn(__int2float_rn(sumi), t1);
    const float t3 = __fmul_rn(r.dminw, da);
    const float t4 = __fmul_rn(__int2float_rn(summ), t3);
    return __fsub_rn(t2, t4);
}

struct Q6Reg {
    uint32_t u[64];  // [n][hf][i][q]: the 6-bit values q + 32 of sub-blocks 8n + 2q + hf, bytes 4i..4i+3
    int sc[16];
    float dw;
};
__device__ __forceinline__ void q6k_load_r(Q6Reg &r, uint32_t tile_s, int S, int s) {
    const uint32_t base = tile_s + (uint32_t)s * 16u, cstride = (uint32_t)S * 16u;
    r.dw = __half2float(__ushort_as_half(lds_u16(tile_s + 13u * cstride + 2u * (uint32_t)s)));
    const uint4 scv = lds_u4(base + 12u * cstride);
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
    for (int j = 0; j < 16; j++) r.sc[j] = byte_s(scw[j >> 2], j & 3);
#pragma unroll
    for (int n = 0; n < 2; n++) {
        const uint4 qa0 = lds_u4(base + (4 * n + 0) * cstride), qa1 = lds_u4(base + (4 * n + 1) * cstride);
        const uint4 qb0 = lds_u4(base + (4 * n + 2) * cstride), qb1 = lds_u4(base + (4 * n + 3) * cstride);
        const uint4 hh0 = lds_u4(base + (8 + 2 * n) * cstride), hh1 = lds_u4(base + (9 + 2 * n) * cstride);
        const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
        const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
        const uint32_t wh[8] = {hh0.x, hh0.y, hh0.z, hh0.w, hh1.x, hh1.y, hh1.z, hh1.w};
#pragma unroll
        for (int hf = 0; hf < 2; hf++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int l4 = 4 * hf + i;
                const uint32_t hq = wh[l4];
                uint32_t *u = r.u + ((n * 2 + hf) * 4 + i) * 4;
                u[0] = (wa[l4] & 0x0F0F0F0Fu) | ((hq << 4) & 0x30303030u);
                u[1] = (wb[l4] & 0x0F0F0F0Fu) | ((hq << 2) & 0x30303030u);
                u[2] = ((wa[l4] >> 4) & 0x0F0F0F0Fu) | (hq & 0x30303030u);
                u[3] = ((wb[l4] >> 4) & 0x0F0F0F0Fu) | ((hq >> 2) & 0x30303030u);
            }
    }
}
__device__ __forceinline__ float q6k_dot_r(const Q6Reg &r, uint32_t act_s) {
    const uint4 bq0 = lds_u4(act_s + ACT_BS16), bq1 = lds_u4(act_s + ACT_BS16 + 16);
    const uint32_t bsw[8] = {bq0.x, bq0.y, bq0.z, bq0.w, bq1.x, bq1.y, bq1.z, bq1.w};
    int sumi = 0;
#pragma unroll
    for (int n = 0; n < 2; n++)
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            const uint4 A0 = lds_u4(act_s + 16 * (8 * n + 0 + hf)), A1 = lds_u4(act_s + 16 * (8 * n + 2 + hf));
            const uint4 A2 = lds_u4(act_s + 16 * (8 * n + 4 + hf)), A3 = lds_u4(act_s + 16 * (8 * n + 6 + hf));
            const uint32_t a[4][4] = {{A0.x, A0.y, A0.z, A0.w}, {A1.x, A1.y, A1.z, A1.w}, {A2.x, A2.y, A2.z, A2.w},
                                      {A3.x, A3.y, A3.z, A3.w}};
            int acc[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[q] = dp4a_us(r.u[((n * 2 + hf) * 4 + i) * 4 + q], (int)a[q][i], acc[q]);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int sub = 8 * n + 2 * q + hf;
                const int bs = (int)(int16_t)((bsw[sub >> 1] >> (16 * (sub & 1))) & 0xffffu);
                sumi += r.sc[sub] * (acc[q] - 32 * bs);
            }
        }
    return __fmul_rn(__int2float_rn(sumi), __fmul_rn(r.dw, lds_f32(act_s + ACT_D)));
}

// The same dots on generic pointers into shared memory.
__device__ __forceinline__ float q4k_slot_dot(const uint8_t *tile, int S, int s, const ActBlock &a) {
    return q4k_dot_s((uint32_t)__cvta_generic_to_shared(tile), S, s, (uint32_t)__cvta_generic_to_shared(&a));
}
__device__ __forceinline__ float q6k_slot_dot(const uint8_t *tile, int S, int s, const ActBlock &a) {
    return q6k_dot_s((uint32_t)__cvta_generic_to_shared(tile), S, s, (uint32_t)__cvta_generic_to_shared(&a));
}

#endif  // __CUDACC__

}  // namespace bt
