// The token sampler on the device: Chaos's Sampler::sample (core/arch/src/sample.rs:474-680) over
// the engine's logits rows, one CTA per sequence. The host side (validation, staging, the C ABI)
// is bt_sample in engine.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

constexpr int SAMP_MAX_CHAIN = 32;   // stages in one chain
constexpr int SAMP_TYPICAL_MAX = 4096;  // candidates typical_p can sort in shared memory

// the scalars of bt_sampler_config (sample.rs:84-180), plus is_greedy()
struct SampParams {
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
    int ignore_eos, eos;
    int n_chain;
    int chain[SAMP_MAX_CHAIN];
    int n_bias, n_suppress, n_breakers;
    int greedy;  // SamplerConfig::is_greedy (sample.rs:277-295)
};

// device copies of the list fields and the histories (hist_off[s] .. hist_off[s + 1])
struct SampLists {
    const uint32_t *bias_ids;
    const float *bias_values;
    const uint32_t *suppress_ids;
    const uint32_t *breakers;
    const uint32_t *hist;
    const uint32_t *hist_off;
};

// bt_sampler_state
struct SampState {
    unsigned long long rng;
    float mu, ap_weighted, ap_total;
};

// status words of one sequence
enum { SAMP_OK = 0, SAMP_DONE_ARGMAX = 1, SAMP_ERR_TYPICAL_TOO_MANY = 2 };

// scratch bytes for n_seqs rows of V logits (the sort's temporary storage included)
size_t sampler_scratch_bytes(int n_seqs, int V);

// Sample one token for each of n_seqs rows of `logits` (device, row-major [n_seqs][V]).
// `state`, `tok` and `status` are device arrays of n_seqs entries; `state` is read and advanced.
cudaError_t sampler_launch(cudaStream_t st, const SampParams &P, const SampLists &L, const float *logits, int V,
                           int n_seqs, void *scratch, size_t scratch_bytes, SampState *state, uint32_t *tok,
                           int *status);
