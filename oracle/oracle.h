/*
 * oracle.h -- CPU restatement of the Chaos decode-step layer (TEST INFRASTRUCTURE).
 *
 * This library is the parity checker for the sm_100a kernels in bigtea_b200/csrc.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
 * `--impl reference` arm) may load it. The product never links, calls or falls
 * back to it.
 *
 * What it restates (reference paths relative to the Chaos source tree):
 *   - StreamingRunner::forward_cached_inner, qwen3moe branch
 *       core/arch/src/stream.rs:2106-2915 (op order, residual adds, output head)
 *   - route(): stable descending sort, top-k, renormalise   stream.rs:869-888
 *   - expert_ffn_single / expert_chunk reduction order      stream.rs:1084-1289
 *   - expert_ffn_block (n_tokens > 1) accumulation order     stream.rs:1051-1058
 *   - KvCache::push f16 layout                               core/arch/src/kv.rs:171-205
 *   - argmax tie rule (last max wins, total_cmp)             core/arch/src/sample.rs:928-935
 *   - Q4_K / Q6_K block layouts                              core/model/src/validate.rs:60-75,
 *                                                            core/gguf/src/tensor.rs:30-32
 * The arithmetic below those calls lives in ggml (llama.cpp, unpinned HEAD, absent
 * from the tree). It is restated from ggml's published algorithm where ggml fixes
 * the result (K-quant dequant, Q8_K activation quantisation, integer K-quant dot
 * products, NeoX RoPE cache recurrence, soft_max scale-by-reciprocal) and follows a
 * documented ARITHMETIC CONTRACT where ggml's result depends on SIMD width or
 * thread count (float reduction orders, exp). The CUDA kernels implement the same
 * contract, which is what makes KV bytes, top-k ids and logits bit-exact between
 * the two. Agreement with ggml itself is unverified here (ggml is not available).
 * Dequantisation is pinned bit-exactly against gguf-py 0.19.0 (llama.cpp's own
 * numpy restatement) by tests/golden.
 */
#ifndef BIGTEA_ORACLE_H
#define BIGTEA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_K = 12, OR_Q6_K = 14 };

/* ggml's block_q8_K: one f32 scale, 256 int8 quants, 16 sums of 16 quants. */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} or_block_q8k;

/* ---- scalar contract helpers ---- */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);
float or_exp(float x);
float or_silu(float x);

/* ---- formats ---- */
int64_t or_row_bytes(int type, int64_t n);
int or_dequant(int type, const void *src, int64_t n, float *dst);
void or_quantize_q8k(const float *x, int64_t n, or_block_q8k *y);

/* ---- ops (each restates one ggml call site of the reference) ---- */
/* y[r] = W[r,:] . x for rows [0, rows); W in GGUF row-major bytes of `type`. */
int or_gemv(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y);
/* the same with the plain C dots, single-threaded (the check of the AVX2 dots) */
int or_gemv_scalar_dots(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y);
void or_rmsnorm(const float *x, const float *w, int n, float eps, float *y);
float or_sumsq_p2(const float *x, int n);
float or_dot_p2(const float *a, const float *b, int n);
void or_rope_table(int n_pos, int n_rot, float base, float *cs /* [n_pos][n_rot/2][2] */);
void or_rope_neox(float *x, int n_rot, const float *cs_pos /* [n_rot/2][2] */);
/* router: softmax over n logits, then route() of stream.rs:869-888 */
void or_softmax(const float *logits, int n, float *probs);
void or_route(const float *probs, int n, int k, int32_t *ids, float *weights);
/* one query head over nk visible keys (f16, row stride ld halves), chunked per contract */
void or_attn_head(const float *q, const uint16_t *k, const uint16_t *v, int64_t ld, int nk,
                  int head_dim, float scale, int chunk, float *out);
uint32_t or_argmax(const float *logits, int64_t n);

/* ---- whole model ---- */
typedef struct {
    int n_layer, n_embd, n_head, n_head_kv, head_dim;
    int n_expert, n_expert_used, n_ff_exp, n_vocab;
    int n_rot;
    float rms_eps, rope_base;
    int expert_workers; /* reference default 4 (stream.rs:1305-1312) */
    int attn_chunk;     /* attention contract chunk, 128 */
    int max_positions;  /* RoPE table / KV capacity */
    /* 0 (OR_NUM_CONTRACT): the arithmetic contract the device implements -- the parity oracle.
     * Otherwise a set of OR_NUM_* bits: each op whose bit is set computes with ggml-cpu's
     * generic algorithm instead (OR_NUM_GGML: all of them), to measure the distance. */
    int numerics;
} or_config;

enum {
    OR_NUM_CONTRACT = 0,
    OR_NUM_NORM = 1,       /* rms_norm: squares summed in double */
    OR_NUM_QDOT = 2,       /* K-quant x Q8_K dots: the generic eight-lane sums */
    OR_NUM_FDOT = 4,       /* F32 dots (the router): products summed in double */
    OR_NUM_SOFTMAX = 8,    /* soft_max: libm expf, double sum */
    OR_NUM_SILU = 16,      /* silu: libm expf */
    OR_NUM_ATTN = 32,      /* flash_attn_ext: serial online softmax, f16 accumulator */
    OR_NUM_ATTN_F32V = 64, /* the same with an f32 accumulator */
    OR_NUM_FMA = 128,      /* the dot lanes and the attention accumulator contracted into fmaf */
    OR_NUM_GGML = 63
};
/* single ops of the ggml mode */
void or_ggml_rmsnorm(const float *x, const float *w, int n, float eps, float *y);
int or_ggml_gemv(int type, const void *W, int64_t rows, int64_t cols, const float *x, float *y);
void or_ggml_softmax(const float *x, int n, float *y);
void or_ggml_attn_head(const float *q, const uint16_t *k, const uint16_t *v, int64_t ld, int nk, int head_dim,
                       float scale, int f32_acc, float *out);

typedef struct {
    const char *name;
    int type;
    int64_t ne[4];
    const void *data;
} or_tensor;

typedef struct or_model or_model;
typedef struct or_kv or_kv;

or_model *or_model_new(const or_config *cfg, const or_tensor *tensors, int n_tensors);
void or_model_free(or_model *m);
const char *or_last_error(void);

or_kv *or_kv_new(const or_model *m);
void or_kv_free(or_kv *kv);
int or_kv_len(const or_kv *kv);
void or_kv_set_len(or_kv *kv, int n);
/* f16 bytes of one layer in kv.rs layout: [pos][n_head_kv*head_dim] */
void or_kv_read(const or_kv *kv, int layer, int n_pos, uint16_t *k, uint16_t *v);
void or_kv_write(or_kv *kv, int layer, int n_pos, const uint16_t *k, const uint16_t *v);

/* forward_cached(tokens, pos_start): logits of the last position (n_vocab floats). */
int or_forward(or_model *m, or_kv *kv, const int32_t *tokens, int n_tokens, int pos_start,
               float *logits);
/* the (ids, weights) route() chose for token t of the last forward, per layer */
int or_debug_topk(const or_model *m, int layer, int t, int32_t *ids, float *weights);
/* the residual stream after the last layer for token t of the last forward */
int or_debug_hidden(const or_model *m, int t, float *out);
int or_set_threads(int n);
/* route() replaced by src's choice for the same layer and token of src's last forward (NULL: off) */
void or_model_route_from(or_model *m, const or_model *src);
/* the K-th largest router probability minus the (K+1)-th, for token t of the last forward */
int or_debug_route_gap(const or_model *m, int layer, int t, float *gap);

/* ---- seeded synthetic weights (the tests' and the CPU arm's model bytes) ---- */
/* FNV-1a of a tensor name: the tensor id of the generator */
uint64_t or_tensor_id(const char *name);
/* rows x cols values of N(mean, sigma) (Irwin-Hall(4)) quantised to `type`, GGUF row-major */
int or_synth_tensor(int type, int64_t rows, int64_t cols, uint64_t seed, uint64_t tensor_id, float mean,
                    float sigma, void *out);

/* STREAM-style host copy bandwidth (read + write bytes), best of reps, GB/s */
double or_copy_gbs(int64_t bytes, int threads, int reps);

/* ---- the token sampler (core/arch/src/sample.rs), restated in sample.c ---- */
/* S5 ln and S6 pow: the sampler's own functions (sample.c) */
float or_ln(float x);
float or_pow(float x, float y);

/* SamplerStage (sample.rs:43-50), in the enum's order */
enum { OR_STAGE_TOP_K = 0, OR_STAGE_TYPICAL_P, OR_STAGE_TOP_P, OR_STAGE_MIN_P, OR_STAGE_XTC,
       OR_STAGE_TEMPERATURE };

/* SamplerConfig (sample.rs:84-180); the same layout as bt_sampler_config */
typedef struct {
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
    const int32_t *chain; /* NULL: the default chain */
    uint32_t n_chain;
    const uint32_t *bias_ids;
    const float *bias_values;
    uint32_t n_bias;
    const uint32_t *suppress_ids;
    uint32_t n_suppress;
    const uint32_t *dry_breakers;
    uint32_t n_dry_breakers;
    uint64_t seed;
} or_sampler_config;

/* the state a Sampler keeps between tokens (sample.rs:306-321) */
typedef struct {
    uint64_t rng;
    float mu, ap_weighted, ap_total;
} or_sampler_state;

void or_sampler_config_default(or_sampler_config *c);  /* SamplerConfig::default, sample.rs:183-222 */
void or_sampler_config_llamacpp(or_sampler_config *c); /* llamacpp_defaults, sample.rs:228-268 */
void or_sampler_init(const or_sampler_config *c, or_sampler_state *st); /* Sampler::new, sample.rs:324-344 */
float or_sampler_next_f32(or_sampler_state *st);                         /* sample.rs:462-472 */
/* Sampler::sample (sample.rs:474-680); -1 with or_last_error() on a bad config */
int64_t or_sample(const or_sampler_config *c, or_sampler_state *st, const float *logits, int64_t n_vocab,
                  const uint32_t *history, int64_t n_history);
/* the stage functions on a candidate list (ids, vals; n entries), for the reference's unit tests;
 * each returns the new length */
int64_t or_stage_top_p(uint32_t *ids, float *vals, int64_t n, float top_p);
int64_t or_stage_min_p(uint32_t *ids, float *vals, int64_t n, float min_p);
int64_t or_stage_typical_p(uint32_t *ids, float *vals, int64_t n, float typical_p);
int64_t or_stage_top_n_sigma(uint32_t *ids, float *vals, int64_t n, float n_sigma);
int64_t or_stage_xtc(uint32_t *ids, float *vals, int64_t n, float probability, float threshold, float roll);
void or_stage_temperature(float *vals, int64_t n, float temperature);
float or_dynamic_temperature(const float *vals, int64_t n, float temperature, float range, float exponent);
void or_stage_penalties(const uint32_t *ids, float *vals, int64_t n, const uint32_t *history, int64_t n_history,
                        float repeat, float frequency, float presence, uint32_t last_n);
void or_stage_dry(const uint32_t *ids, float *vals, int64_t n, const uint32_t *history, int64_t n_history,
                  float multiplier, float base, uint32_t allowed_length, uint32_t penalty_last_n,
                  const uint32_t *breakers, uint32_t n_breakers);

#ifdef __cplusplus
}
#endif
#endif
