// kernels.cuh -- parameter blocks and launchers of the decode-layer kernels (sm_100a).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kquant.cuh"

namespace bt {

constexpr int MAX_T = 8;        // tokens one GEMV / expert launch carries in shared memory
constexpr int MAX_K = 16;       // experts used per token
constexpr int ATTN_CHUNK = 128; // attention keys per chunk (contract C8)
constexpr int GEMV_WARPS = 8;
// per-warp scratch of the row reductions: 8 tokens x 32 lanes, rows padded to 33 floats
constexpr int RED_STRIDE = 33, RED_WARP_FLOATS = 8 * RED_STRIDE;

// Ranges to start pulling into L2 while a kernel runs (the next kernels' inputs), and
// optionally one layer's KV pages of the step's sequences.
struct PrefetchSpec {
    const void *ptr[4];
    unsigned long long bytes[4];
    int n;
    // KV pages of `layer` for every token's sequence (positions 0..pos_of[t])
    const __half *kv;
    const int *block_table, *seq_of, *pos_of;
    int max_blocks, layer, n_blocks, HK, D, T;
};

struct GemvSeg {
    const uint8_t *w;  // tiled weights
    int type, nsb, rpt, S, tile_bytes;
    int rows;
    int n_tiles;
    int tile0;    // first global unit of this segment
    int out_off;  // column offset in y
};

struct GemvArgs {
    GemvSeg seg[3];
    int nseg, total_tiles;
    const float *x;
    long long x_stride;
    const int *x_rows;     // optional row indirection for the activations
    const float *norm_w;   // optional RMSNorm weight (C6) applied before quantising
    float eps;
    int K, T;
    float *y;
    long long y_stride;
    const float *res;      // optional residual added to the output
    long long res_stride;
    int *err;
    int slot_bytes, nst;
    unsigned long long *amax;  // optional: per token, max of (total_cmp key, row) over the output
    PrefetchSpec pf;
    // the activations as Q8_K rows (q8_stage_kernel): [T][K] values, [T][K/256] scales,
    // [T][K/256][8] 32-value sums; read by the tensor-core GEMV
    const int8_t *q8_qs;
    const float *q8_d;
    const int *q8_bs;
    // token groups (dp4a kernel, no amax): 0 = every unit carries all T tokens; else the units
    // are (group of tgrp tokens, tile), group-major, and a CTA stages only the tokens of the
    // groups its units cover, at most stage_max of them
    int tgrp, stage_max;
};

struct ExpertArgs {
    const uint8_t *gate, *up, *down;
    int gtype, utype, dtype;
    int g_nsb, g_rpt, g_S, g_tile_bytes, g_n_tiles;
    int u_tile_bytes;
    long long g_expert_bytes, u_expert_bytes, d_expert_bytes;
    int d_nsb, d_tile_bytes, d_rpt;  // down: superblocks per row, tile bytes, rows per tile
    int E, F, K, T, workers;
    const int *sel_ids;        // [T][K] ascending expert ids
    const float *sel_w;        // [T][K] their renormalised weights
    const float *fn;           // [T][E] post-norm activations (gate/up input)
    float *act;                // [T][K][F] silu(gate)*up
    const float *ffn_in;       // [T][E] residual
    float *x_out;              // [T][E]
    const unsigned char *single;  // [T] 1 = the token was a single-token step (paired order)
    int *err;
    int slot_bytes, nst;
    PrefetchSpec pf;
    int prefetch_down;  // gate/up: pull the selected experts' down weights into L2
    // grouped form (batched steps): the tokens of each selected expert, from group_kernel
    const int *g_count, *g_off, *g_list, *g_active, *g_nactive;
    const int *g_chunk_e, *g_chunk_r0, *g_nchunks;  // the chunks of at most GROUP_MAXM rows
    float *dpart;  // [T][K][E] each (token, expert slot)'s down rows before the expert sum
    int row_div;   // grouped gate/up: the activation row of list entry i is i / row_div
    const int8_t *q8_qs;  // fn as Q8_K rows (q8_stage_kernel), read by the tensor-core gate/up
    const float *q8_d;
    const int *q8_bs;
    // expert parallelism: the combine reads slot (t, k) of the rank owning expert sel_ids[t*K+k]
    // from dpart[(owner * ep_slots + t*K + k) * E]; ep_ranks = 0 outside expert parallelism
    int ep_ranks, ep_per, ep_slots;
    // expert cache: expert e's gate | up | down matrices sit in slot slot_of[e] of the pool
    // (slot_stride bytes each); slot_of = null when every expert is resident
    const int *slot_of;
    const uint8_t *pool;
    // expert parallelism with sharded expert memory: the resident matrices are those of the
    // experts [expert_base, expert_base + per), expert e at position e - expert_base
    int expert_base;
    long long slot_stride;
    // the shared expert's output rows [T][E], added to the routed sum before the residual; or null
    const float *shexp;
};

// the weights of expert e: its resident matrices, or its slot of the expert cache
__device__ __forceinline__ const uint8_t *expert_gate(const ExpertArgs &p, int e) {
    return p.slot_of ? p.pool + (long long)p.slot_of[e] * p.slot_stride : p.gate + (e - p.expert_base) * p.g_expert_bytes;
}
__device__ __forceinline__ const uint8_t *expert_up(const ExpertArgs &p, int e) {
    return p.slot_of ? p.pool + (long long)p.slot_of[e] * p.slot_stride + p.g_expert_bytes
                     : p.up + (e - p.expert_base) * p.u_expert_bytes;
}
__device__ __forceinline__ const uint8_t *expert_down(const ExpertArgs &p, int e) {
    return p.slot_of ? p.pool + (long long)p.slot_of[e] * p.slot_stride + p.g_expert_bytes + p.u_expert_bytes
                     : p.down + (e - p.expert_base) * p.d_expert_bytes;
}

// Expert-parallel dispatch: the rows of every (token, slot) pair, packed for the rank that owns
// the pair's expert (ranks own ep_per consecutive experts each).
struct EpPackArgs {
    const int *sel_ids;  // [T][K] global expert ids
    const float *fn;     // [T][E] the experts' input rows
    int T, K, E, ranks, per, slots;
    int *send_meta;      // [ranks][slots] expert id, or -1 where the slot is not for that rank
    float *send_rows;    // [ranks][slots][E]
    // Q8_K dispatch (when send_qs is set): the T token rows already quantised by q8_stage_kernel
    // go to the owner's slot in place of the f32 rows, a quarter of the bytes
    const int8_t *q8_qs;
    const float *q8_d;
    const int *q8_bs;
    int8_t *send_qs;     // [ranks][slots][E]
    float *send_d;       // [ranks][slots][E/256]
    int *send_bs;        // [ranks][slots][E/256][8]
};

// Tokens grouped by expert for the batched expert kernels: for every expert e, the (token,
// slot) indices tk = t*K + k that selected it, in ascending tk; the experts with at least one
// token in ascending id order.
struct GroupArgs {
    const int *sel_ids;  // [T][K]
    int T, K, NE;
    int *g_count, *g_off, *g_list, *g_active, *g_nactive;
    int *g_chunk_e, *g_chunk_r0, *g_nchunks;  // chunk i: expert g_chunk_e[i], its rows from g_chunk_r0[i]
};
constexpr int GROUP_MAXM = 16;  // tokens of one expert whose activations a CTA stages at a time
constexpr int GROUP_RED_FLOATS = GROUP_MAXM * RED_STRIDE;  // a warp's partials of one chunk (gate or up)
// chunks of a grouped step: at most one partial chunk per expert
inline int group_max_chunks(int rows, int NE) { return rows / GROUP_MAXM + NE + 1; }

struct RouterArgs {
    const float *x, *norm_w;
    float eps;
    int E;
    const float *Wr;
    const float *bias;  // [NE] added to the logits, or null
    int NE, K, T, rows_per_cta;
    float *fn_out, *logits;
    int *cnt;
    int *topk_ids;
    float *topk_w;
    int *sel_ids;
    float *sel_w;
};

struct QkvPostArgs {
    const float *qkv;
    int qkv_stride;
    const float *q_norm, *k_norm;
    float eps;
    const float *rope;
    int n_rot, H, HK, D, T;
    const int *seq_of, *pos_of, *block_table;
    int max_blocks, layer, n_blocks;
    __half *kv;
    float *q_out;
};

struct AttnArgs {
    const float *q;
    int H, HK, D, G, T;
    const int *seq_of, *pos_of, *block_table;
    int max_blocks, layer, n_blocks, max_chunks;
    int n_cta;  // persistent grid of the attention kernel
    float scale;
    float *part;
    int *cnt;
    float *out;
    int *err;
};

struct EmbedArgs {
    const uint8_t *table;  // raw GGUF rows
    int type, E, V, T;
    const int *tokens, *seq_of, *local_idx;
    const int *dev_len;
    int *pos_of;
    float *x;
    int *err;
};

struct StepEndArgs {
    const float *logits;  // [n_out][V]
    int V, n_seqs, n_out;
    const int *seq_ids, *n_tok;
    const int *logit_row; // [n_seqs]: row of `logits` holding the sequence's last token, or -1
    unsigned long long *amax;  // [n_out] argmax packed by the output GEMV; read and reset here
    int *dev_len;
    int *next_token;      // [n_out]
    int *tokens_buf;      // if non-null: tokens_buf[row] = argmax (greedy feed-back)
    int *gen_out;         // if non-null: gen_out[gen_count[row]*n_out + row] = argmax
    int *gen_count;
};

cudaError_t init_kernel_attributes();
int max_dynamic_smem();  // per-block dynamic shared memory the ring sizing may use

// ---- launchers (all asynchronous on `st`; `pdl` enables programmatic dependent launch)
size_t gemv_smem_bytes(const GemvArgs &a);
cudaError_t launch_gemv(const GemvArgs &a, int grid, cudaStream_t st, bool pdl);
size_t gateup_smem_bytes(const ExpertArgs &a);
size_t down_smem_bytes(const ExpertArgs &a);
cudaError_t launch_gateup(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_down(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_router(const RouterArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_group(const GroupArgs &a, cudaStream_t st, bool pdl);
size_t gateup_grouped_smem_bytes(const ExpertArgs &a);
size_t down_grouped_smem_bytes(const ExpertArgs &a);
int down_group_rows(const ExpertArgs &a);  // output rows of one grouped down unit
cudaError_t launch_gateup_grouped(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_down_grouped(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_down_combine(const ExpertArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_ep_pack(const EpPackArgs &a, cudaStream_t st, bool pdl);
// tcgen05 kind::i8 probe: D[128][N] = A[128][K] . B[N][K]^T (u8 x s8 -> s32)
cudaError_t launch_i8_mma_probe(const uint8_t *A, const int8_t *B, int32_t *D, int N, int K, int *err,
                                cudaStream_t st);
// grouped gate/up on tcgen05 (Q4_K gate and up, F a multiple of 128); one CTA per SM
size_t gateup_mma_smem_bytes(int E);
cudaError_t launch_gateup_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
// grouped down on tcgen05 (Q4_K down, tiles of 32 / nsb rows, E a multiple of 128); its B operand
// is the SiLU products as Q8_K rows, one per (token, slot); one CTA per SM
size_t down_mma_smem_bytes(int F);
cudaError_t launch_down_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
// the same for a Q6_K down ((size_t)-1: F does not fit)
size_t down6_mma_smem_bytes(int F);
cudaError_t launch_down6_mma(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl);
cudaError_t init_mma_attributes();
// batched GEMV on tcgen05 (Q4_K segments of whole 128-row blocks, no argmax); one CTA per SM
size_t gemv_mma_smem_bytes(int K);
// tokens per unit of the batched tensor-core GEMV (32 or 16; 0: does not fit)
int gemv_mma_tokens(int K);
// T rows of K activations (row t = x_rows[t] or t; RMSNorm first when norm_w) as Q8_K rows:
// qs [T][K], d [T][K/256], bs [T][K/256][8] (C3/C6, the dp4a kernels' staging bit for bit)
cudaError_t launch_q8_stage(const float *x, long long x_stride, const int *x_rows, const float *norm_w, float eps, int K,
                            int T, int8_t *qs, float *d, int *bs, cudaStream_t st, bool pdl);
cudaError_t launch_gemv_mma(const GemvArgs &a, int grid, cudaStream_t st, bool pdl);
// Q6_K segments of whole 128-row blocks on tcgen05 (16-token chunks), with optional argmax keys;
// (size_t)-1 = K does not fit
size_t gemv_mma6_smem_bytes(int K);
cudaError_t launch_gemv_mma6(const GemvArgs &a, int grid, cudaStream_t st, bool pdl);
// act[t][j] = silu(gu[t][j]) * gu[t][F + j] for the shared expert (C7)
cudaError_t launch_shexp_act(const float *gu, float *act, int T, int F, cudaStream_t st, bool pdl);
cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t st, bool pdl);
size_t attn_smem_bytes(int G, int T);
cudaError_t launch_attn(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl);
// the batched steps' attention with one warp per 128-key chunk (attn_warp_kernel), then the combine
cudaError_t launch_attn_warp(const AttnArgs &a, const CUtensorMap &tmap, cudaStream_t st, bool pdl);
size_t attn_warp_smem_bytes(int G, int T);
cudaError_t launch_embed(const EmbedArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_step_end(const StepEndArgs &a, cudaStream_t st, bool pdl);

cudaError_t launch_repack(int type, const uint8_t *src, long long rows, long long cols, int rpt, uint8_t *dst,
                          long long n_mats, cudaStream_t st);
cudaError_t launch_dequant_tiled(int type, const uint8_t *tiled, long long rows, long long cols, int rpt,
                                 float *out, cudaStream_t st);
cudaError_t launch_kv_copy(__half *pool, const int *table_row, int layer, int n_blocks, int HK, int D, int p0, int n,
                           __half *kbuf, __half *vbuf, int to_pool, cudaStream_t st);
cudaError_t launch_untile(int type, const uint8_t *tiled, long long rows, long long cols, int rpt, uint8_t *dst,
                          long long n_mats, cudaStream_t st);
cudaError_t launch_synth(int type, uint64_t key, long long n_elems, float mean, float scale, uint8_t *out,
                         cudaStream_t st);

}  // namespace bt
