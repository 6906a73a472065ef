// Tensor-core (tcgen05, kind::i8) kernels of the K-quant contractions.
#include <cuda_runtime.h>

#include "bt_common.cuh"
#include "kernels.cuh"
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

cudaError_t launch_i8_mma_probe(const uint8_t *A, const int8_t *B, int32_t *D, int N, int K, int *err,
                                cudaStream_t st) {
    const size_t smem = i8_mma_probe_smem(N, K);
    cudaError_t e = cudaFuncSetAttribute(i8_mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    i8_mma_probe_kernel<<<1, 128, smem, st>>>(A, B, D, N, K, err);
    return cudaGetLastError();
}

}  // namespace bt
