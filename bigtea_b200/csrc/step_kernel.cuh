// step_kernel.cuh -- parameters of the persistent decode-step kernel (step_kernel.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "xcache_dev.cuh"

namespace bt {

constexpr int STEP_MAX_T = 4;                    // sequences one persistent step carries
constexpr int STEP_REGION_BYTES = 150 * 1024;    // rings / attention tiles
constexpr int STEP_ACT_BYTES = 32 * 1024;        // Q8_K activation blocks
constexpr int STEP_CBUF_BYTES = 16 * 1024;       // norm vector, router probabilities, combine scratch
constexpr int STEP_ROUTER_ROWS = 4;              // router rows one CTA computes
constexpr int STEP_RES = 256;                    // residual values one CTA prefetches for a phase
constexpr int STEP_DOWN_ROWS = 128;              // down rows one CTA owns per layer: T * E / grid, rounded up
constexpr int STEP_MAX_NSB_F = 8;                // expert width F / 256 the down phase stages per warp

// A quantised matrix in the tiled layout, as the device reads it.
struct QMatDev {
    const uint8_t *w;
    int type, nsb, rpt, S, tile_bytes, rows, n_tiles;
    long long mat_bytes;  // one expert's matrix
};

// One layer's tensors as the device reads them; the persistent kernel copies it into shared
// memory word by word.
struct LayerDev {
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm, *gate_inp;
    const float *gate_bias;  // [NE] added to the router logits, or null
    QMatDev q, k, v, o, gate, up, down;
    // the shared expert (C10), when the model has one (sgate.w != null): gate and up in the
    // GEMV layout, down with one row per tile like the routed experts' down matrices
    QMatDev sgate, sup, sdown;
};

struct StepArgs {
    const LayerDev *layers;
    int n_layer;
    QMatDev out;
    const float *out_norm;
    const uint8_t *embd;
    int embd_type;
    int E, H, HK, D, G, NE, K, F, V, workers, n_rot;
    float eps, scale;
    const float *rope;
    int T;
    const int *tokens, *seq_of;
    int *pos_of, *dev_len;
    __half *kv;
    const int *block_table;
    int max_blocks, n_blocks, max_chunks;
    float *x, *ffn_in, *qkv, *att, *part, *rlog, *act;
    int FS;         // shared expert width (0: none)
    float *shact;   // [T][FS] SiLU(gate) * up of the shared expert
    // the expert cache with its policy on the device (xc_on): after each layer's routing, CTA 0
    // looks the selected experts up, every CTA fills missed slots from the pinned host blocks,
    // and the expert tiles come from the slot pool (slot: gate | up | down of one expert)
    int xc_on;
    XcDev xd;
    const uint8_t *const *xc_host;  // [n_layer] device addresses of the experts' host blocks
    uint8_t *xc_pool;
    long long xc_stride;
    int xc_bounce;
    XcCopy *xc_copies;
    int *xc_ncopies;
    int *xc_rows;  // [n_layer][NE] each expert's slot (rows written by the lookups)
    int *dbg_ids;
    float *dbg_w;
    int TB;
    float *logits;
    unsigned long long *amax;
    int *next_token, *tokens_buf, *gen_out, *gen_count;
    int n_out;
    unsigned *bar;  // grid barrier arrival counter, zeroed before each launch
    int *err;
    // every bounded wait of the step gives up after this many SM cycles (about 1 s by default)
    long long wait_limit;
    // failure drill, off when fault_barrier is 0: CTA fault_cta leaves at its grid barrier number
    // fault_barrier (1-based, counted from the start of the launch) without arriving, as a CTA
    // that died would; the others' bounded waits then run out
    int fault_cta, fault_barrier;
    // second drill, off at 0: in layer fault_copy - 1, CTA fault_cta requests none of its expert
    // gate/up tiles, so its own bounded ring waits run out (the failure exit with copies missing)
    int fault_copy;
    // optional timeline: per barrier, every CTA's arrival time and CTA 0's departure time
    // (%globaltimer ns), rows of gridDim.x + 1 at trace[(layer * STEP_PHASES + phase) * (grid + 1)]
    unsigned long long *trace;
};

constexpr int STEP_PHASES = 32;  // timeline slots per layer: 8 barriers, then 24 points inside phases

size_t step_smem_bytes(int max_chunks);
cudaError_t init_step_kernel_attributes();
cudaError_t launch_decode_step(const StepArgs &a, const CUtensorMap &tmap, int grid, cudaStream_t st);

}  // namespace bt
