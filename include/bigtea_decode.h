/*
 * bigtea_decode.h -- C ABI of the B200 decode-step layer.
 *
 * Drop-in for the qwen3moe decode path of Chaos (aturzone/Bigtea). Every entry point
 * names the reference interface it replaces (paths relative to the Chaos tree).
 * Conventions: every call returns BT_OK (0) or a bt_status; on failure
 * bt_last_error() holds a message for the calling thread. Nothing aborts. Handles are
 * opaque; one engine is driven from one thread at a time (the reference's
 * StreamingRunner is `&mut self`, core/arch/src/stream.rs:1933). Output buffers are
 * caller-owned host memory unless a name says otherwise.
 */
#ifndef BIGTEA_DECODE_H
#define BIGTEA_DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BT_ABI_VERSION 2

typedef enum {
    BT_OK = 0,
    BT_ERR_INVALID = 1,        /* bad argument, shape or state */
    BT_ERR_CUDA = 2,           /* a CUDA runtime call failed */
    BT_ERR_OOM = 3,            /* device or pinned-host allocation failed */
    BT_ERR_MISSING_TENSOR = 4, /* ArchError::MissingTensor, core/arch/src/lib.rs */
    BT_ERR_KV = 5,             /* KvError::WrongSize and capacity, core/arch/src/kv.rs:171-178 */
    BT_ERR_TIMEOUT = 6,        /* a bounded device wait ran out; the context stays usable */
    BT_ERR_UNSUPPORTED = 7     /* a tensor type or shape this build has no kernel for */
} bt_status;

/* ggml type ids (core/gguf/src/tensor.rs:18-57) accepted by this build */
enum { BT_TYPE_F32 = 0, BT_TYPE_F16 = 1, BT_TYPE_Q4_K = 12, BT_TYPE_Q6_K = 14 };
/* KvType (core/arch/src/kv.rs:44-55); only F16 is on the device path */
enum { BT_KV_F16 = 1 };

/* Qwen3Config fields the decode layer reads (core/arch/src/qwen3.rs:565-844). */
typedef struct {
    uint32_t n_layer, n_embd, n_head, n_head_kv, head_dim;
    uint32_t n_expert, n_expert_used, n_ff_exp, n_vocab, n_rot;
    float rms_eps, rope_freq_base;
    /* CHAOS_EXPERT_WORKERS (stream.rs:1305-1312, default 4): fixes the order in which
     * one position's expert outputs are summed. */
    uint32_t expert_workers;
    /* longest sequence the RoPE table covers (positions 0..max_positions-1) */
    uint32_t max_positions;
    /* width of a shared expert (blk.N.ffn_{gate,up,down}_shexp), 0 = none. Not in the
     * reference's qwen3moe tensor set: the DeepSeek-style workload has one, added unweighted
     * to the routed sum before the residual, as llama.cpp's deepseek2 graph does:
     * x = (moe + shexp(x_n)) + ffn_inp. */
    uint32_t n_ff_shexp;
} bt_model_desc;

/* One GGUF tensor as Model::read_tensor returns it (core/model/src/lib.rs:390-470):
 * ggml dims (ne[0] innermost) and host bytes. The engine copies the bytes to HBM
 * during bt_engine_create; the caller may free them afterwards. */
typedef struct {
    const char *name;
    uint32_t type;
    uint32_t n_dims;
    uint64_t ne[4];
    const void *data;
    uint64_t nbytes;
} bt_tensor_view;

typedef struct bt_engine bt_engine;
typedef struct bt_kv bt_kv;

/* Phase timers, the device analogue of StreamStats (stream.rs:134-194). */
typedef struct {
    uint64_t forward_calls;
    uint64_t tokens;
    double forward_seconds;     /* host wall time inside bt_forward / bt_generate_greedy */
    uint64_t weight_bytes;      /* bytes of weights resident in HBM */
    uint64_t graph_replays;     /* decode steps served from a captured CUDA graph */
} bt_stats;

const char *bt_last_error(void);
int bt_abi_version(void);

/* StreamingRunner::new + load_resident (stream.rs:586, 1793-1876): upload every tensor
 * (experts included: the model is HBM-resident) and build the kernels' layouts.
 * `device` is a CUDA ordinal. */
int bt_engine_create(const bt_model_desc *desc, const bt_tensor_view *tensors, size_t n_tensors,
                     int device, bt_engine **out);
/* Same engine with seeded synthetic weights generated on the device (N(0, sigma)
 * quantised to each tensor's type; norms 1 + N(0, sigma)). `types` gives, per layer,
 * the ggml types of attn_q, attn_k, attn_v, attn_output, ffn_gate_exps, ffn_up_exps,
 * ffn_down_exps (7 entries per layer); token_embd and output use `embd_type`/`out_type`.
 * The bytes are identical to bt_synth_tensor's for the same seed and tensor id. */
int bt_engine_create_synthetic(const bt_model_desc *desc, const uint32_t *types, uint32_t embd_type,
                               uint32_t out_type, uint64_t seed, float sigma, int device,
                               bt_engine **out);
/* Destroy every bt_kv of the engine before the engine itself. */
void bt_engine_destroy(bt_engine *e);
int bt_engine_stats(const bt_engine *e, bt_stats *out);
/* copy a resident tensor's GGUF bytes back to the host (for a CPU check of synthetic weights) */
int bt_engine_tensor_bytes(const bt_engine *e, const char *name, void *host_out, uint64_t nbytes);

/* KvCache::with_type (kv.rs:114-160) as a paged device pool: `max_seqs` sequences of up to
 * `max_positions` positions each, `block_tokens` (16) positions per page. */
int bt_kv_create(bt_engine *e, uint32_t kind, uint32_t max_seqs, uint32_t max_positions,
                 uint32_t block_tokens, bt_kv **out);
void bt_kv_destroy(bt_kv *kv);
int bt_kv_len(const bt_kv *kv, uint32_t seq, uint32_t *len);                 /* kv.rs:151-153 */
int bt_kv_clear(bt_kv *kv, uint32_t seq);                                    /* kv.rs:232-238 */
int bt_kv_truncate(bt_kv *kv, uint32_t seq, uint32_t n);                     /* kv.rs:280-292 */
int bt_kv_shift_out(bt_kv *kv, uint32_t seq, uint32_t keep, uint32_t drop);  /* kv.rs:314-328 */
int bt_kv_set_positions(bt_kv *kv, uint32_t seq, uint32_t n);                /* kv.rs:270-272 */
int bt_kv_bytes(const bt_kv *kv, uint64_t *bytes);                          /* kv.rs:162-166 */
int bt_kv_is_consistent(const bt_kv *kv, uint32_t seq, int *consistent);     /* kv.rs:330-338 */
/* keys()/values() of one layer in the kv.rs byte layout ([pos][n_head_kv*head_dim] f16)
 * (kv.rs:222-228): the first bytes / (n_head_kv*head_dim*2) positions, into k_out and v_out
 * of `bytes` each; `bytes` must be whole positions and at most what the layer holds. */
int bt_kv_export_layer(const bt_kv *kv, uint32_t seq, uint32_t layer, void *k_out, void *v_out,
                       uint64_t bytes);
/* restore_layer (kv.rs:252-264): replaces the layer's positions with `bytes` of k and v. */
int bt_kv_import_layer(bt_kv *kv, uint32_t seq, uint32_t layer, const void *k, const void *v,
                       uint64_t bytes);

/* ---- isolated expert-FFN timing (no counterpart in the reference) ----
 * The routed experts' arithmetic alone, over every layer of the model, with T tokens a layer:
 * a seeded selection of K distinct experts per token, seeded weights and activation rows.
 * kernel 0: the kernels a decode step of T single tokens runs, layer after layer (the
 *   per-token ones up to 8 tokens, the grouped ones above; T = 1..the step capacity);
 * kernel 1: one persistent kernel that is given every layer's selections up front and streams
 *   the experts' tiles through a CTA-wide TMA ring, layer s's gate/up and layer s-1's down in
 *   one stage (T = 1..4); the same arithmetic as kernel 0, bit for bit.
 * Captured as one CUDA graph, replayed once to warm up and then n_iters times between CUDA
 * events: *ms_per_pass is the mean device time of one pass over the layers, *bytes_per_pass the
 * weight bytes one pass reads (every layer's distinct selected experts' gate, up and down
 * matrices), so bytes / time is the kernels' HBM bandwidth with the routing and the rest of the
 * step taken away. out_last (optional, host, [T][n_embd] f32) receives the last layer's expert
 * sum. Overwrites the engine's step scratch; not for an expert-parallel engine or one with the
 * expert cache. */
int bt_bench_experts(bt_engine *e, uint32_t T, uint32_t n_iters, uint64_t seed, uint32_t kernel,
                     double *ms_per_pass, uint64_t *bytes_per_pass, float *out_last);

/* StreamingRunner::forward_cached (stream.rs:1933-1975), batched over sequences.
 * Sequence i appends n_tokens[i] tokens (tokens are concatenated in `tokens`) at
 * pos_start[i], which must equal that sequence's cache length. Writes the logits of
 * each sequence's last token to logits_out[i * n_vocab ...] (host). */
int bt_forward(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *tokens,
               const uint32_t *n_tokens, const uint32_t *pos_start, uint32_t n_seqs,
               float *logits_out);
/* The chaos-run greedy decode loop (cli/run/src/main.rs:3914-4070, temp 0, argmax of
 * core/arch/src/sample.rs:928-935) run on the device: starting from `first_tokens`
 * (one per sequence, not yet in the cache), runs n_steps single-token steps and writes
 * the n_steps tokens each step produced to tokens_out[step * n_seqs + i]. The last
 * step's logits go to last_logits (n_seqs * n_vocab, may be NULL). */
int bt_generate_greedy(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *first_tokens,
                       uint32_t n_seqs, uint32_t n_steps, uint32_t *tokens_out, float *last_logits);

/* ---- token sampling on the device: Sampler (core/arch/src/sample.rs:306-680) ---- */
/* SamplerStage (sample.rs:43-50) */
enum { BT_STAGE_TOP_K = 0, BT_STAGE_TYPICAL_P = 1, BT_STAGE_TOP_P = 2, BT_STAGE_MIN_P = 3, BT_STAGE_XTC = 4,
       BT_STAGE_TEMPERATURE = 5 };
/* SamplerConfig (sample.rs:84-180), field for field; the list fields are host arrays. eos < 0 is
 * None; chain == NULL is the default chain (top_k, typical_p, top_p, min_p, xtc, temperature),
 * at most 32 stages otherwise. bt_sampler_config_default fills SamplerConfig::default() (greedy)
 * and bt_sampler_config_llamacpp llamacpp_defaults(). */
typedef struct bt_sampler_config {
    float temperature;
    uint32_t top_k;
    float top_p, min_p, typical_p, top_n_sigma;
    float xtc_probability, xtc_threshold;
    float dynatemp_range, dynatemp_exponent;
    float repeat_penalty, frequency_penalty, presence_penalty;
    uint32_t repeat_last_n;
    float dry_multiplier, dry_base;
    uint32_t dry_allowed_length, dry_penalty_last_n;
    uint32_t mirostat;
    float mirostat_tau, mirostat_eta;
    float adaptive_p, adaptive_decay;
    int32_t ignore_eos, eos;
    const int32_t *chain;
    uint32_t n_chain;
    const uint32_t *bias_ids;
    const float *bias_values;
    uint32_t n_bias;
    const uint32_t *suppress_ids; /* infill_suppress */
    uint32_t n_suppress;
    const uint32_t *dry_breakers; /* dry_sequence_breakers */
    uint32_t n_dry_breakers;
    uint64_t seed;
} bt_sampler_config;
/* The state a Sampler carries from token to token (sample.rs:306-321): the SplitMix64 word,
 * mirostat's mu and adaptive-p's two accumulators. Caller-owned, one per sequence. */
typedef struct bt_sampler_state {
    uint64_t rng;
    float mu, ap_weighted, ap_total;
} bt_sampler_state;
void bt_sampler_config_default(bt_sampler_config *c);
void bt_sampler_config_llamacpp(bt_sampler_config *c);
/* Sampler::new (sample.rs:324-344): the state of a fresh sampler for `c` (host only). */
int bt_sampler_init(const bt_sampler_config *c, bt_sampler_state *state);
/* Sampler::sample (sample.rs:474-680) for n_seqs sequences at once, on the device. `logits` is
 * NULL for the engine's own logits of the last bt_forward or bt_generate_greedy call (row i is
 * that call's sequence i; no logits cross to the host), else a host array [n_seqs][n_vocab].
 * Sequence i's history (the tokens so far, for the penalties and DRY) is
 * history[sum(history_len[0..i)) ...] of history_len[i] tokens; history_len may be NULL (no
 * history). states[i] is read and advanced as the reference's Sampler advances. The results
 * equal the reference's algorithm with this library's exp/ln/pow and tie rules (the smaller id
 * first among equal logits). typical_p runs on at most 4096 candidates: BT_ERR_UNSUPPORTED
 * beyond that (set top_k, or put top_p or min_p before it in the chain). */
int bt_sample(bt_engine *e, const bt_sampler_config *cfg, bt_sampler_state *states, uint32_t n_seqs,
              const float *logits, const uint32_t *history, const uint32_t *history_len, uint32_t *tokens_out);

/* Device time (CUDA events on the engine stream) of the last bt_generate_greedy replay loop. */
int bt_last_device_ms(const bt_engine *e, double *ms);
/* Page-locked host memory (no counterpart in the reference). bt_forward copies logits straight
 * into an output buffer from here, without the staging copy a pageable buffer takes; the
 * latency-bound single-token loop is where that shows. bt_host_free releases a block. */
int bt_host_alloc(uint64_t bytes, void **out);
int bt_host_free(void *p);

/* StreamStats-style per-kernel timing (stream.rs:134-194): runs n_steps greedy steps with
 * serialised launches, each bracketed by CUDA events; fills one entry per kernel kind. */
typedef struct {
    char name[32];
    uint64_t launches;
    double total_ms;
} bt_kernel_time;
int bt_profile_decode(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *first_tokens,
                      uint32_t n_seqs, uint32_t n_steps, bt_kernel_time *out, uint32_t max_out, uint32_t *n_out);
/* Engine switches: "pdl" (programmatic dependent launch between the step's kernels, default 1),
 * "prefetch" (L2 bulk prefetch of the next kernels' weights and KV pages, default 0),
 * "persistent" (run single-token steps of up to 4 sequences as one cooperative kernel that
 * holds every SM for the whole step, default 1; 0 = one kernel per phase), "mma" (Q4_K
 * contractions of batched steps on the tensor cores, default 1), "mma_min_units" (the batched
 * GEMV goes to the tensor cores from this many 128-row x token-chunk units, default 32),
 * "mma_grid" (CTAs of the tensor-core kernels, default 0 = one per SM), "token_groups" (a
 * batched dp4a GEMV with fewer tiles than half the grid's warps, such as a 512-row Q6_K attn_v,
 * runs as one launch over units of (token group, tile), default 1; 0 = token chunks whose units
 * carry every token of the chunk; the results are the same bits), "wait_limit_us" (every
 * bounded wait of the persistent step gives up after this long, default 0 = about 1 s), and the
 * failure drill "fault_cta" / "fault_barrier" (off at 0): in each persistent step, CTA fault_cta
 * leaves at its grid barrier number fault_barrier (1-based) without arriving, as a CTA that died
 * would; the other CTAs' waits run out, the first one poisons the barrier, every CTA leaves at its
 * next barrier, and the call returns BT_ERR_TIMEOUT after about one wait limit; "fault_copy" (off
 * at 0): in layer fault_copy - 1, CTA fault_cta requests none of its expert tiles, so its own
 * waits run out and it takes the failure exit (barrier poisoned, its copies drained);
 * "stream_slots" (ring slots of bt_bench_experts' stream kernel, default 0 = as many as fit in
 * 160 KB of shared memory); "stream_warps" (its consumer warps per CTA: 8, one CTA per SM, the
 * default; or 4, two CTAs per SM); "xcache_device" (the expert cache's policy runs on the device after
 * each layer's router and fills missed slots from the pinned host copies with a kernel, so a
 * step needs no host round trip per layer; default 1; 0 = the host decides each layer; a
 * change starts a new, empty cache). */
int bt_set_option(bt_engine *e, const char *name, int value);

/* Router bias of one layer: n == n_expert F32 values added to the router logits before the
 * softmax (a ggml_add after the ffn_gate_inp mul_mat), or bias == NULL to remove it. Not part
 * of the reference's qwen3moe tensor set (stream.rs:2784-2831 has no bias): the skewed-routing
 * workloads use it. bt_engine_create also takes it as the optional tensor
 * blk.N.ffn_gate_inp.bias. */
int bt_engine_set_router_bias(bt_engine *e, uint32_t layer, const float *bias, uint32_t n);

/* ---- expert cache (models whose experts do not fit in HBM) ----
 * The experts move to pinned host memory; each step copies the experts a layer selects into
 * slots of an HBM pool of `cache_bytes` (cudaMemcpyAsync on the engine's stream, ordered
 * before that layer's expert kernels). The reference streams expert slices from disk into a
 * host cache instead (core/arch/src/stream.rs:1400-1475, admission stream.rs:1314-1379,
 * core/arch/src/expert_cache.rs); here the slow tier is host memory and the cache is HBM.
 * Policies: BT_XCACHE_LRU evicts the least recently used expert; BT_XCACHE_FREQ is the
 * reference's frequency-gated admission (a newcomer replaces the least-used of 8 sampled
 * entries only when selected strictly more often; else it is used once from a bounce slot).
 * Steps run as per-phase kernels with one host round trip per layer; results are the same
 * bits as with every expert resident. Not combinable with expert parallelism. */
enum { BT_XCACHE_LRU = 0, BT_XCACHE_FREQ = 1 };
typedef struct bt_xcache_stats {
    uint64_t hits, misses, evictions, admissions, bypasses, bytes_copied;
    uint64_t capacity_slots, slot_bytes;
} bt_xcache_stats;
/* a second call starts a new, empty cache of the given size and policy */
int bt_engine_enable_expert_cache(bt_engine *e, uint64_t cache_bytes, int policy);
int bt_expert_cache_stats(const bt_engine *e, bt_xcache_stats *out);
/* the policy alone, on the host: a trace of n_steps x n_layer groups of n_sel expert ids
 * (layer-major within a step), looked up in order; no device is touched */
int bt_expert_cache_simulate(int policy, uint32_t capacity, uint32_t n_layer, uint32_t n_expert, uint32_t n_sel,
                             const int32_t *trace, uint32_t n_steps, bt_xcache_stats *out);
/* the same trace through the device policy (the lookup kernel an engine with the option
 * "xcache_device" runs after each layer's router) on the current device: the same counts as
 * bt_expert_cache_simulate; n_expert <= 1024, n_sel <= 1024 */
int bt_expert_cache_simulate_device(int policy, uint32_t capacity, uint32_t n_layer, uint32_t n_expert,
                                    uint32_t n_sel, const int32_t *trace, uint32_t n_steps, bt_xcache_stats *out);

/* ---- expert parallelism (batched decode over the GPUs of one node) ----
 * No counterpart in the reference, which has no distributed code. One engine per GPU, one
 * process each. With n ranks, rank r computes the experts [r*NE/n, (r+1)*NE/n). Each layer of
 * a step then runs as follows:
 *   - every (token, slot) row goes to the rank that owns the slot's expert;
 *   - that rank runs the expert FFN on the rows it received;
 *   - the expert outputs come back (NCCL send/recv over NVLink);
 *   - the token's own rank adds them in the reference's order (stream.rs:1232-1284), so the
 *     results equal a single-GPU run bit for bit.
 * Attention, the router and the head stay on each sequence's rank (data parallel). Every
 * rank must run the same sequence of steps: the exchange has fixed sizes (64 tokens x
 * n_expert_used slots per rank pair; a call's tokens run in steps of at most 64 here) and all
 * ranks take part in every layer. */
/* an NCCL unique id for bt_engine_enable_ep (nbytes >= 128); rank 0 makes it and shares it */
int bt_ep_unique_id(void *out, size_t nbytes);
/* collective over the n_ranks engines; disables the persistent single-kernel step */
int bt_engine_enable_ep(bt_engine *e, const void *unique_id, size_t nbytes, int rank, int n_ranks);

/* ---- parity hooks: each runs one device kernel on host buffers ---- */
/* dequantize() (core/ggml/src/lib.rs:233-290): n values of `type` through the device layout */
int bt_debug_dequant(uint32_t type, const void *bytes, uint64_t n, float *out);
/* route() result for one layer and token (stream.rs:869-888): ids in descending probability,
 * renormalised weights. `token` indexes the token list of the last bt_forward; only its last
 * step (its last 128 tokens at most: a call's tokens run in steps of up to 128) is kept. After bt_generate_greedy, token i is sequence i's last step. */
int bt_debug_topk(const bt_engine *e, uint32_t layer, uint32_t token, int32_t *ids, float *weights);
/* residual stream after the last layer for `token`, indexed as for bt_debug_topk (n_embd floats) */
int bt_debug_hidden(const bt_engine *e, uint32_t token, float *out);
/* one quantised mul_mat (graph.rs:690): y[t][r] = W[r,:] . x[t,:] for T tokens */
int bt_op_gemv(uint32_t type, const void *w_bytes, uint32_t rows, uint32_t cols, const float *x,
               uint32_t T, float *y);

/* parity hook of the tensor-core path (tcgen05.mma kind::i8, the operand layouts and
 * descriptors of the grouped expert kernel): d[128][n] = a[128][k] . b[n][k]^T in int32, a
 * unsigned 8-bit, b signed 8-bit, host buffers; n in {8, 16, 32}, k a multiple of 32 up to 512 */
int bt_op_i8_mma(const uint8_t *a, const int8_t *b, uint32_t n, uint32_t k, int32_t *d);

/* ---- allocation-free GEMV (no counterpart in the reference) ----
 * bt_op_gemv on caller-owned DEVICE buffers that allocates nothing: no cudaMalloc, cudaFree,
 * stream or event creation, and no allocating library call. It is for callers that cannot
 * allocate inside a step: cudaMalloc and cudaFree synchronise the whole device, and they fail
 * once the engine's weights and KV pool have reserved HBM, so a serving loop that owns the
 * device's memory and overlaps work on several streams needs a call that only uses memory
 * reserved up front. Its scratch is one file-scope device array of BT_NOALLOC_SCRATCH_BYTES
 * per device, reserved when the library loads: a 256-byte header holding the error word (the
 * call zeroes it on `stream` before its kernels; nothing else must start at zero) and the
 * tiled copy of W. A matrix whose tiled copy does not fit (rows * cols/256 * block bytes >
 * BT_NOALLOC_SCRATCH_BYTES - 256; e.g. the 151936 x 2048 Q6_K output head) is rejected with
 * BT_ERR_INVALID before anything runs. Calls on one device share the scratch, so overlapping
 * calls (other threads, or other streams without ordering) race: serialise them. The first
 * call on a device does that device's set-up (the scratch's address, the kernels' shared-memory
 * limits) with the device current; make it before any stream capture. The call waits for
 * `stream` (a cudaStream_t, NULL for the legacy default stream) before it returns.
 * w_dev: rows x cols GGUF bytes (Q4_K or Q6_K, row-major); x_dev: T x cols f32; y_dev: T x rows
 * f32, y[t][r] = W[r,:] . x[t,:] with the same arithmetic as bt_op_gemv. */
#define BT_NOALLOC_SCRATCH_BYTES (16u << 20)
int bt_op_gemv_noalloc(uint32_t type, const void *w_dev, uint32_t rows, uint32_t cols, const float *x_dev, uint32_t T,
                       float *y_dev, void *stream);

/* ---- synthetic weights (seeded; same bytes on host and device) ---- */
/* fill `out` (rows * row_bytes) with N(mean, sigma) values quantised to `type` */
int bt_synth_tensor(uint32_t type, uint64_t rows, uint64_t cols, uint64_t seed, uint64_t tensor_id,
                    float mean, float sigma, void *out);
/* the tensor id bt_engine_create_synthetic uses for a tensor name (64-bit FNV-1a) */
uint64_t bt_tensor_id(const char *name);

#ifdef __cplusplus
}
#endif
#endif
