// expert_stream.cuh -- parameters of the multi-layer expert-FFN stream kernel (expert_stream.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "step_kernel.cuh"

namespace bt {

struct ExpertStreamArgs {
    const LayerDev *layers;  // [n_layer]: gate, up and down are read
    int n_layer, T, K, E, F, workers;
    const int *sel;     // [n_layer][T][K] expert ids, distinct per token, ascending
    const float *wts;   // [n_layer][T][K] route weights
    const float *xin;   // gate/up input of layer s at xin + s * xin_stride: [T][E], already normalised
    long long xin_stride;
    float *act;         // [n_layer][T * K][F] SiLU(gate) * up
    float *out;         // [n_layer][T][E] the expert sum (plus a zero residual)
    unsigned *bar;      // arrival counter, zeroed before the launch
    int *err;
    long long wait_limit;  // SM cycles of every bounded wait
    int nslot, slot_bytes;  // the CTA's ring: nslot slots, each holding the largest unit
    int consumers;          // consumer warps per CTA: 4 (two CTAs per SM) or 8 (one)
};

size_t expert_stream_fixed_smem(int T, int E, int K, int F);
int expert_stream_max_slots();
int expert_stream_max_rows();  // down rows a CTA may own per layer (T * E / grid, rounded up)
// sets the kernel's shared-memory limit for a's ring and reports how many CTAs an SM then holds;
// call once before launching (or capturing) it
cudaError_t prepare_expert_stream(const ExpertStreamArgs &a, int *blocks_per_sm);
int expert_stream_regs();  // registers per thread of the kernel (-1 if unknown)
cudaError_t launch_expert_stream(const ExpertStreamArgs &a, int grid, cudaStream_t st);

}  // namespace bt
