// engine.cu -- host runtime and C ABI of the decode-step layer (include/bigtea_decode.h).
//
// The engine owns the HBM-resident weights (GGUF bytes rearranged into the tiled layout of
// kquant.cuh), the RoPE table, the per-step scratch and the CUDA graphs of the greedy loop.
// bt_kv is the paged f16 KV pool. Reference interfaces: StreamingRunner::new / load_resident /
// forward_cached (core/arch/src/stream.rs:586, 1793, 1933) and KvCache (core/arch/src/kv.rs).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>  // types of the NCCL calls; the library itself is opened at run time
#include <string.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/bigtea_decode.h"
#include "bt_common.cuh"
#include "expert_cache.h"
#include "kernels.cuh"
#include "step_kernel.cuh"
#include "expert_stream.cuh"

// Under expert parallelism every exchange carries a step's full capacity of (token, expert)
// slots to every rank, so the steps are kept at 64 tokens there.
constexpr int EP_STEP_TOKENS = 64;
#ifndef BT_STEP_TOKENS
#define BT_STEP_TOKENS 128  // tokens of one step of the per-phase kernels (longer calls are cut into steps)
#endif
#include "xcache_dev.cuh"
#include "sampler.cuh"

using namespace bt;

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}
#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) return fail(BT_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

extern "C" const char *bt_last_error(void) { return g_err.c_str(); }
extern "C" int bt_abi_version(void) { return BT_ABI_VERSION; }

// ------------------------------------------------------------------ device buffers
struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), n(o.n) {
        o.p = nullptr;
        o.n = 0;
    }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) {
            if (p) cudaFree(p);
            p = o.p;
            n = o.n;
            o.p = nullptr;
            o.n = 0;
        }
        return *this;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    cudaError_t alloc(size_t bytes) {
        if (p) cudaFree(p);
        p = nullptr;
        n = bytes;
        return cudaMalloc(&p, bytes ? bytes : 16);
    }
    template <typename T> T *as() const { return reinterpret_cast<T *>(p); }
};

// A quantised matrix (or stack of per-expert matrices) in the tiled layout.
struct QMat {
    DevBuf buf;
    DevBuf raw;  // GGUF bytes, kept only where a row gather needs them (token_embd)
    int type = -1;
    long long rows = 0, cols = 0, n_mats = 1;
    TileGeom g{};
    long long mat_bytes = 0;  // bytes of one expert's matrix
};

struct Layer {
    DevBuf attn_norm, q_norm, k_norm, ffn_norm, gate_inp;
    DevBuf gate_bias;  // optional ffn_gate_inp.bias [n_expert], added to the router logits
    QMat q, k, v, o, gate, up, down;
    QMat gate_sh, up_sh, down_sh;  // the shared expert, when the model has one (n_ff_shexp)
    // the shared expert's down matrix again with one row per tile, for the persistent step's
    // down units (a layout copy: not counted in the weight bytes)
    QMat down_sh1;
};

struct GraphKey {
    const void *kv;
    std::vector<uint32_t> seqs;
    bool operator<(const GraphKey &o) const { return kv != o.kv ? kv < o.kv : seqs < o.seqs; }
};

struct KernelTimer {
    std::string name;
    uint64_t launches = 0;
    double ms = 0;
};

struct bt_engine {
    bt_model_desc d{};
    int device = 0;
    int n_sm = 148;
    cudaStream_t st = nullptr;
    std::vector<Layer> L;
    QMat embd, out;
    DevBuf out_norm, rope;
    // per-step scratch, sized for TB tokens and max_seqs outputs
    int TB = BT_STEP_TOKENS;
    int max_out = 0;
    DevBuf x, ffn_in, fn, qkv, qbuf, att, rlog, rcnt, sel_ids, sel_w, act, part, acnt;
    DevBuf q8_qs, q8_d, q8_bs;  // activation rows as Q8_K for the tensor-core kernels (q8_rows x q8_k)
    size_t q8_rows = 0, q8_k = 0;
    DevBuf g_count, g_off, g_list, g_active, g_nactive, dpart;  // grouped experts of batched steps
    DevBuf g_chunk_e, g_chunk_r0, g_nchunks;
    DevBuf sh_gu, sh_act, sh_out;  // the shared expert: [TB][2F] gate|up, [TB][F] silu*up, [TB][E] rows
    // expert parallelism (bt_engine_enable_ep): this rank computes experts [rank*NE/n, (rank+1)*NE/n)
    bool ep = false;
    int ep_rank = 0, ep_n = 1;
    // sharded expert memory under expert parallelism: the resident routed experts are
    // [ep_e0, ep_e0 + ep_ne) of every layer (ep_ne = 0: all of them)
    int ep_e0 = 0, ep_ne = 0;
    ncclComm_t ep_comm = nullptr;
    int ep_timeout_ms = 60000;  // a host wait on an expert-parallel step longer than this aborts the exchange
    bool ep_aborted = false;
    bool mma = true;  // grouped Q4_K gate/up on tcgen05 (option "mma")
    int mma_min_units = 32;  // batched GEMVs on tcgen05 from this many (tokens, rows) units on (option)
    int token_groups = 1;    // batched dp4a GEMVs with few tiles split their tokens into groups (option)
    int mma_grid = 0;        // CTAs of the tensor-core kernels (0: one per SM; option, for tests)
    bool attn_warp = true;   // batched attention with one warp per 128-key chunk (option "attn_warp")
    // the persistent step's bounded waits, in microseconds (option "wait_limit_us"; 0 = about 1 s)
    int wait_limit_us = 0;
    // ring slots of the expert stream kernel (option "stream_slots"; 0 = as many as fit in
    // 160 KB of shared memory with the staging buffers, which leaves the SM about 90 KB of L1
    // for the prefetched activation rows)
    int stream_slots = 0;
    int stream_warps = 8;  // consumer warps per CTA of the stream kernel (option "stream_warps": 4 or 8)
    // failure drill of the persistent step (options "fault_cta", "fault_barrier"; off at 0):
    // CTA fault_cta leaves at its grid barrier number fault_barrier without arriving
    int fault_cta = 0, fault_barrier = 0;
    int fault_copy = 0;  // option "fault_copy": in layer fault_copy - 1, CTA fault_cta requests no expert tiles
    // expert cache: experts in pinned host memory, the ones a layer selects copied into slots
    // of a device pool before its expert kernels (bt_engine_enable_expert_cache)
    bool xcache = false;
    ExpertCachePolicy xpol;
    XCacheStats xstats;
    int x_bounce = 0;               // bounce slots, after the cache's own
    long long x_stride = 0;         // bytes of a slot: one expert's gate | up | down
    DevBuf x_pool, x_slot_dev;      // (capacity + bounce) slots; [n_layer][NE] slot of each expert
    std::vector<uint8_t *> x_host;  // per layer, pinned: [NE] experts of x_stride bytes
    int *x_sel_host = nullptr;      // pinned: a step's selections
    int *x_slot_host = nullptr;     // pinned [n_layer][NE]: staging of x_slot_dev
    cudaEvent_t x_ev = nullptr;
    // the policy on the device (option "xcache_device", default 1): no host round trip per layer
    bool xdev = true;
    XcDev xd{};
    DevBuf xd_buf;                            // the device policy's arrays
    DevBuf x_copies, x_ncopies;               // a layer's slot copies
    std::vector<const uint8_t *> x_host_dev;  // device addresses of x_host
    DevBuf x_host_devarr;                     // the same, in device memory
    DevBuf ep_send_meta, ep_send_rows, ep_recv_meta, ep_recv_rows, ep_act, ep_dpart, ep_ret;
    DevBuf ep_send_qs, ep_send_d, ep_send_bs, ep_recv_qs, ep_recv_d, ep_recv_bs;  // Q8_K dispatch
    DevBuf dbg_ids, dbg_w;  // [n_layer][TB][K]
    DevBuf tokens, seq_of, local_idx, pos_of, single, x_rows;
    DevBuf st_seq, st_ntok, st_lrow, next_tok, gen_out, gen_count, logits, amax;
    DevBuf err;
    // pinned host staging of a call's small transfers: the step plan's vectors go up from
    // plan_host without a host wait (plan_ev marks when its last copies have been read), and a
    // call of up to STEP_MAX_T sequences brings its error word and logits back through err_host
    // and logits_host behind one stream wait
    uint8_t *plan_host = nullptr;
    size_t plan_seg = 0;  // bytes of one plan vector's slot in plan_host (8 slots)
    cudaEvent_t plan_ev = nullptr;
    bool plan_ev_live = false;
    int *err_host = nullptr;
    float *logits_host = nullptr;
    int part_chunks = 0;
    size_t gen_cap = 0;
    uint64_t weight_bytes = 0;
    bt_stats stats{};
    std::map<GraphKey, cudaGraphExec_t> graphs;
    cudaGraph_t graph_objs[64] = {};
    int last_T = 0;        // tokens in the last step of the last bt_forward
    int last_rows = 0;     // logits rows the last bt_forward / bt_generate_greedy left in `logits`
    DevBuf samp_scratch, samp_aux, samp_in;  // bt_sample: sort and chain scratch, lists, host logits
    size_t last_first = 0; // index (in that call's token list) of the step's first token
    // profiling
    bool timing = false;
    std::map<std::string, KernelTimer> timers;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
    std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> ev_used;
    double last_device_ms = 0;
    bool pdl = true;
    bool mega = true;      // run single-token steps of up to STEP_MAX_T sequences as one persistent kernel
    DevBuf layer_dev;      // LayerDev[n_layer] for the persistent kernel
    QMatDev out_dev{};
    DevBuf gbar;           // grid barrier words of the persistent kernel
    DevBuf trace;          // persistent-kernel timeline (profiling only)
    bool tracing = false;
    // L2 bulk prefetch of the next kernels' inputs: measured slower (the issuing CTAs wait on
    // their prefetches), so off unless asked for
    bool prefetch = false;
};

struct bt_kv {
    bt_engine *e = nullptr;
    uint32_t max_seqs = 0, max_positions = 0, block_tokens = 16;
    int n_blocks = 0, max_blocks = 0;
    DevBuf pool;                       // [n_layer][n_blocks][2][HK][16][D] f16
    DevBuf bt_dev;                     // [max_seqs][max_blocks] int32
    DevBuf dev_len;                    // [max_seqs] int32
    DevBuf tmp;                        // export/import/shift staging
    std::vector<int> table;            // host mirror of the block table
    std::vector<int> free_blocks;
    std::vector<std::vector<int>> pages;
    std::vector<uint32_t> len;         // host mirror of the lengths
    std::vector<std::vector<uint32_t>> layer_pos;  // positions held per layer (is_consistent)
    CUtensorMap tmap;
    bool table_dirty = true;
};

// ------------------------------------------------------------------ driver entry point for TMA maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// ------------------------------------------------------------------ helpers
// Ring depth per warp: at most 3 slots and about 110 KB per CTA, so that the CTAs of the next
// kernel (programmatic dependent launch) fit beside a running CTA on the same SM.
static int pick_nst(size_t slot_bytes, size_t fixed_bytes) {
    static size_t cap = 0;
    if (!cap) {
        cap = (size_t)max_dynamic_smem();
        if (cap > 110 * 1024) cap = 110 * 1024;
    }
    int nst = 3;
    while (nst > 1 && fixed_bytes + (size_t)GEMV_WARPS * nst * slot_bytes > cap) nst--;
    return nst;
}

// the same choice with an explicit cap on the CTA's shared memory (the batched kernels use all of it)
static int pick_nst_cap(size_t slot_bytes, size_t fixed_bytes, size_t cap) {
    int nst = 3;
    while (nst > 1 && fixed_bytes + (size_t)GEMV_WARPS * nst * slot_bytes > cap) nst--;
    return nst;
}

// Tokens one GEMV launch carries in a step of T > MAX_T tokens: as many as fit beside a two-slot
// ring in the CTA's shared memory, split evenly (the weights are read once per launch).
static int gemv_chunk(int T, int K, int slot_bytes) {
    if (T <= MAX_T) return MAX_T;
    const size_t cap = (size_t)max_dynamic_smem();
    const size_t ring = (size_t)GEMV_WARPS * 2 * slot_bytes + (size_t)GEMV_WARPS * RED_WARP_FLOATS * 4;
    const size_t per = (size_t)(K / 256) * sizeof(ActBlock);
    long long n = cap > 1024 + 128 + ring ? (long long)((cap - 1024 - 128 - ring) / per) : MAX_T;
    if (n < MAX_T) n = MAX_T;
    const int chunks = (int)((T + n - 1) / n);
    return (T + chunks - 1) / chunks;
}

static int grid_for(const bt_engine *e, long long units) {
    long long g = units < e->n_sm ? units : e->n_sm;
    return (int)(g < 1 ? 1 : g);
}

static void rope_table(const bt_model_desc &d, std::vector<float> &cs) {
    // ggml_rope_cache_init's recurrence for NeoX with freq_scale 1, ext_factor 0, attn_factor 1
    // (core/ggml/src/graph.rs:542-562 fixes those parameters for qwen3moe).
    int n_rot = (int)d.n_rot;
    cs.resize((size_t)d.max_positions * n_rot);
    float theta_scale = powf(d.rope_freq_base, -2.0f / (float)n_rot);
    for (uint32_t p = 0; p < d.max_positions; p++) {
        float theta = (float)p;
        float *row = cs.data() + (size_t)p * n_rot;
        for (int i = 0; i < n_rot / 2; i++) {
            row[2 * i] = cosf(theta);
            row[2 * i + 1] = sinf(theta);
            theta *= theta_scale;
        }
    }
}

static bool is_norm_name(const std::string &n) {
    return n.find("_norm.weight") != std::string::npos;
}

// Upload one tensor (host or device source) into its resident form.
static int ingest_qmat(bt_engine *e, QMat &m, int type, long long rows, long long cols, long long n_mats,
                       const void *src, bool src_device, int rpt, bool keep_raw, DevBuf &staging) {
    if (type != T_Q4_K && type != T_Q6_K)
        return fail(BT_ERR_UNSUPPORTED, "quantised matrices must be Q4_K or Q6_K (got type " + std::to_string(type) + ")");
    if (cols % 256) return fail(BT_ERR_UNSUPPORTED, "row length must be a multiple of 256");
    if (cols / 256 > 32) return fail(BT_ERR_UNSUPPORTED, "rows longer than 8192 values are not supported");
    m.type = type;
    m.rows = rows;
    m.cols = cols;
    m.n_mats = n_mats;
    m.g = tile_geom(type, rows, cols, rpt);
    m.mat_bytes = m.g.n_tiles * (long long)m.g.tile_bytes;
    size_t raw_bytes = (size_t)n_mats * rows * (cols / 256) * qk_block_bytes(type);
    const uint8_t *dsrc = reinterpret_cast<const uint8_t *>(src);
    if (!src_device) {
        if (staging.n < raw_bytes) CK(staging.alloc(raw_bytes));
        CK(cudaMemcpyAsync(staging.p, src, raw_bytes, cudaMemcpyHostToDevice, e->st));
        dsrc = staging.as<uint8_t>();
    }
    CK(m.buf.alloc((size_t)m.mat_bytes * n_mats));
    CK(launch_repack(type, dsrc, rows, cols, rpt, m.buf.as<uint8_t>(), n_mats, e->st));
    if (keep_raw) {
        CK(m.raw.alloc(raw_bytes));
        CK(cudaMemcpyAsync(m.raw.p, dsrc, raw_bytes, cudaMemcpyDeviceToDevice, e->st));
    }
    CK(cudaStreamSynchronize(e->st));
    e->weight_bytes += raw_bytes;
    return BT_OK;
}

static int ingest_f32(bt_engine *e, DevBuf &b, const void *src, bool src_device, size_t n) {
    CK(b.alloc(n * 4));
    CK(cudaMemcpyAsync(b.p, src, n * 4, src_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, e->st));
    CK(cudaStreamSynchronize(e->st));
    e->weight_bytes += n * 4;
    return BT_OK;
}

struct SrcTensor {
    int type;
    uint64_t ne[4];
    int n_dims;
    const void *data;
    bool device;
    uint64_t nbytes;
};

static uint64_t expected_bytes(int type, uint64_t n) {
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q4_K: return n / 256 * 144;
    case T_Q6_K: return n / 256 * 210;
    default: return 0;
    }
}

static int validate_desc(const bt_model_desc *d) {
    if (!d) return fail(BT_ERR_INVALID, "null model description");
    if (d->n_layer == 0 || d->n_embd == 0 || d->n_head == 0 || d->n_head_kv == 0 || d->n_expert == 0 ||
        d->n_expert_used == 0 || d->n_ff_exp == 0 || d->n_vocab == 0 || d->max_positions == 0)
        return fail(BT_ERR_INVALID, "model description has a zero dimension");
    if (d->head_dim != 128) return fail(BT_ERR_UNSUPPORTED, "head_dim must be 128");
    if (d->n_rot != d->head_dim) return fail(BT_ERR_UNSUPPORTED, "partial rotary embeddings are not supported");
    if (d->n_head % d->n_head_kv || (d->n_head / d->n_head_kv) > 8 || ((d->n_head / d->n_head_kv) & 1))
        return fail(BT_ERR_UNSUPPORTED, "GQA group must be 2, 4, 6 or 8 query heads per KV head");
    if (d->n_expert_used > (uint32_t)MAX_K || d->n_expert_used > d->n_expert)
        return fail(BT_ERR_UNSUPPORTED, "n_expert_used must be at most 16 and at most n_expert");
    if (d->n_expert > 512) return fail(BT_ERR_UNSUPPORTED, "n_expert must be at most 512");
    if (d->n_embd % 256 || d->n_ff_exp % 256 || (d->n_head * d->head_dim) % 256 || d->n_ff_shexp % 256)
        return fail(BT_ERR_UNSUPPORTED, "n_embd, n_ff_exp, n_ff_shexp and n_head*head_dim must be multiples of 256");
    return BT_OK;
}

// ------------------------------------------------------------------ NCCL, opened at run time
// Only expert parallelism needs NCCL, so the library is opened on first use (in a process that
// already holds torch's NCCL, dlopen returns that one).
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
};

static const NcclApi *nccl_api() {
    static NcclApi api{};
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
        api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(h, "ncclGroupStart"));
        api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
        api.Send = reinterpret_cast<decltype(api.Send)>(dlsym(h, "ncclSend"));
        api.Recv = reinterpret_cast<decltype(api.Recv)>(dlsym(h, "ncclRecv"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort && api.CommGetAsyncError &&
             api.GroupStart && api.GroupEnd && api.Send && api.Recv && api.GetErrorString;
    });
    return ok ? &api : nullptr;
}

#define NK(call)                                                                                     \
    do {                                                                                             \
        ncclResult_t r_ = (call);                                                                    \
        if (r_ != ncclSuccess) return fail(BT_ERR_CUDA, std::string("NCCL: ") + nccl_api()->GetErrorString(r_)); \
    } while (0)

// Waits for the engine's stream. Without expert parallelism this is cudaStreamSynchronize. With
// it, a step can only finish when every rank takes part in the exchange, so the wait is bounded:
// past ep_timeout_ms (or on an NCCL error) the communicator is aborted, which ends its pending
// transfers, and the engine refuses further steps (BT_ERR_TIMEOUT).
static int wait_stream(bt_engine *e) {
    if (!e->ep || !e->ep_comm) {
        CK(cudaStreamSynchronize(e->st));
        return BT_OK;
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaStreamQuery(e->st);
        if (q == cudaSuccess) return BT_OK;
        if (q != cudaErrorNotReady) CK(q);
        ncclResult_t ar = ncclSuccess;
        nccl_api()->CommGetAsyncError(e->ep_comm, &ar);
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if ((ar != ncclSuccess && ar != ncclInProgress) || ms > e->ep_timeout_ms) {
            nccl_api()->CommAbort(e->ep_comm);
            e->ep_comm = nullptr;
            e->ep_aborted = true;
            // the aborted transfers return; the kernels queued after them finish on stale rows
            const auto t1 = std::chrono::steady_clock::now();
            while (cudaStreamQuery(e->st) == cudaErrorNotReady &&
                   std::chrono::steady_clock::now() - t1 < std::chrono::seconds(10))
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            return fail(BT_ERR_TIMEOUT, ar != ncclSuccess && ar != ncclInProgress
                                            ? std::string("expert-parallel exchange failed: ") + nccl_api()->GetErrorString(ar)
                                            : "expert-parallel exchange timed out (a rank did not take part); the "
                                              "communicator was aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(ms < 5 ? 5 : 100));
    }
}

// Q8_K activation rows for the tensor-core kernels: `rows` rows of up to max(hidden, heads x
// head_dim) values.
static cudaError_t alloc_q8(bt_engine *e, size_t rows) {
    const size_t K = std::max<size_t>(e->d.n_embd, (size_t)e->d.n_head * e->d.head_dim), nsb = K / 256;
    if (rows <= e->q8_rows && K <= e->q8_k) return cudaSuccess;
    cudaError_t r;
    if ((r = e->q8_qs.alloc(rows * K))) return r;
    if ((r = e->q8_d.alloc(rows * nsb * 4))) return r;
    if ((r = e->q8_bs.alloc(rows * nsb * 8 * 4))) return r;
    e->q8_rows = rows;
    e->q8_k = K;
    return cudaSuccess;
}

// tokens of one step: the scratch capacity, or less under expert parallelism
static int step_cap(const bt_engine *e) { return e->ep && EP_STEP_TOKENS < e->TB ? EP_STEP_TOKENS : e->TB; }

static int alloc_scratch(bt_engine *e) {
    const bt_model_desc &d = e->d;
    const int TB = e->TB, E = d.n_embd, QW = d.n_head * d.head_dim, KW = d.n_head_kv * d.head_dim;
    const int K = d.n_expert_used, NE = d.n_expert, F = d.n_ff_exp, G = d.n_head / d.n_head_kv;
    e->part_chunks = (int)((d.max_positions + ATTN_CHUNK - 1) / ATTN_CHUNK);
    e->max_out = 256;
    // Q8_K staging: TB rows of the widest GEMV input, or TB * K rows of SiLU products (the grouped
    // down's input), whichever needs more
    {
        const size_t kd = std::max<size_t>(d.n_embd, (size_t)d.n_head * d.head_dim);
        CK(alloc_q8(e, std::max<size_t>((size_t)TB, ((size_t)TB * K * F + kd - 1) / kd)));
    }
    CK(e->x.alloc((size_t)TB * E * 4));
    CK(e->ffn_in.alloc((size_t)TB * E * 4));
    CK(e->fn.alloc((size_t)TB * E * 4));
    CK(e->qkv.alloc((size_t)TB * (QW + 2 * KW) * 4));
    CK(e->qbuf.alloc((size_t)TB * QW * 4));
    CK(e->att.alloc((size_t)TB * QW * 4));
    CK(e->rlog.alloc((size_t)TB * NE * 4));
    CK(e->rcnt.alloc((size_t)TB * 4));
    CK(cudaMemset(e->rcnt.p, 0, (size_t)TB * 4));
    CK(e->sel_ids.alloc((size_t)TB * K * 4));
    CK(e->sel_w.alloc((size_t)TB * K * 4));
    CK(e->act.alloc((size_t)TB * K * F * 4));
    CK(e->part.alloc((size_t)TB * d.n_head_kv * e->part_chunks * G * (d.head_dim + 4) * 4));
    CK(e->acnt.alloc((size_t)TB * d.n_head_kv * 4));
    CK(e->g_count.alloc((size_t)NE * 4));
    CK(e->g_off.alloc((size_t)NE * 4));
    CK(e->g_list.alloc((size_t)TB * K * 4));
    CK(e->g_active.alloc((size_t)NE * 4));
    CK(e->g_nactive.alloc(4));
    CK(e->g_nchunks.alloc(4));
    CK(e->g_chunk_e.alloc((size_t)group_max_chunks(TB * K, NE) * 4));
    CK(e->g_chunk_r0.alloc((size_t)group_max_chunks(TB * K, NE) * 4));
    CK(e->dpart.alloc((size_t)TB * K * E * 4));
    if (d.n_ff_shexp) {
        CK(e->sh_gu.alloc((size_t)TB * 2 * d.n_ff_shexp * 4));
        CK(e->sh_act.alloc((size_t)TB * d.n_ff_shexp * 4));
        CK(e->sh_out.alloc((size_t)TB * E * 4));
    }
    CK(cudaMemset(e->acnt.p, 0, (size_t)TB * d.n_head_kv * 4));
    CK(e->dbg_ids.alloc((size_t)d.n_layer * TB * K * 4));
    CK(e->dbg_w.alloc((size_t)d.n_layer * TB * K * 4));
    CK(e->tokens.alloc((size_t)TB * 4));
    CK(e->seq_of.alloc((size_t)TB * 4));
    CK(e->local_idx.alloc((size_t)TB * 4));
    CK(e->pos_of.alloc((size_t)TB * 4));
    CK(e->single.alloc((size_t)TB));
    CK(e->x_rows.alloc((size_t)e->max_out * 4));
    CK(e->st_seq.alloc((size_t)e->max_out * 4));
    CK(e->st_ntok.alloc((size_t)e->max_out * 4));
    CK(e->st_lrow.alloc((size_t)e->max_out * 4));
    CK(e->next_tok.alloc((size_t)e->max_out * 4));
    CK(e->gen_count.alloc((size_t)e->max_out * 4));
    CK(e->logits.alloc((size_t)e->max_out * d.n_vocab * 4));
    CK(e->amax.alloc((size_t)e->max_out * 8));
    CK(cudaMemset(e->amax.p, 0, (size_t)e->max_out * 8));
    CK(e->err.alloc(4));
    CK(cudaMemset(e->err.p, 0, 4));
    const int plan_rows = TB > e->max_out ? TB : e->max_out;
    e->plan_seg = ((size_t)plan_rows * 4 + 255) & ~(size_t)255;
    if (!e->plan_host) CK(cudaHostAlloc((void **)&e->plan_host, 8 * e->plan_seg, cudaHostAllocDefault));
    if (!e->plan_ev) CK(cudaEventCreateWithFlags(&e->plan_ev, cudaEventDisableTiming));
    if (!e->err_host) CK(cudaHostAlloc((void **)&e->err_host, 4, cudaHostAllocDefault));
    if (!e->logits_host)
        CK(cudaHostAlloc((void **)&e->logits_host, (size_t)STEP_MAX_T * d.n_vocab * 4, cudaHostAllocDefault));
    return BT_OK;
}

static QMatDev qmat_dev(const QMat &m) {
    QMatDev d{};
    d.w = m.buf.as<uint8_t>();
    d.type = m.type;
    d.nsb = m.g.nsb;
    d.rpt = m.g.rpt;
    d.S = m.g.S;
    d.tile_bytes = m.g.tile_bytes;
    d.rows = (int)m.rows;
    d.n_tiles = (int)m.g.n_tiles;
    d.mat_bytes = m.mat_bytes;
    return d;
}

// the per-layer pointer table of the persistent kernel
static int upload_layer_dev(bt_engine *e) {
    std::vector<LayerDev> ld(e->d.n_layer);
    for (uint32_t il = 0; il < e->d.n_layer; il++) {
        Layer &l = e->L[il];
        LayerDev &x = ld[il];
        x.attn_norm = l.attn_norm.as<float>();
        x.q_norm = l.q_norm.as<float>();
        x.k_norm = l.k_norm.as<float>();
        x.ffn_norm = l.ffn_norm.as<float>();
        x.gate_inp = l.gate_inp.as<float>();
        x.gate_bias = l.gate_bias.p ? l.gate_bias.as<float>() : nullptr;
        x.q = qmat_dev(l.q);
        x.k = qmat_dev(l.k);
        x.v = qmat_dev(l.v);
        x.o = qmat_dev(l.o);
        x.gate = qmat_dev(l.gate);
        x.up = qmat_dev(l.up);
        x.down = qmat_dev(l.down);
        if (e->d.n_ff_shexp) {
            x.sgate = qmat_dev(l.gate_sh);
            x.sup = qmat_dev(l.up_sh);
            x.sdown = qmat_dev(l.down_sh1);
        } else {
            x.sgate = x.sup = x.sdown = QMatDev{};
        }
    }
    if (!e->layer_dev.p) CK(e->layer_dev.alloc(ld.size() * sizeof(LayerDev)));
    CK(cudaMemcpy(e->layer_dev.p, ld.data(), ld.size() * sizeof(LayerDev), cudaMemcpyHostToDevice));
    return BT_OK;
}

static int finish_create(bt_engine *e) {
    int ur = upload_layer_dev(e);
    if (ur) return ur;
    e->out_dev = qmat_dev(e->out);
    CK(e->gbar.alloc(64));
    CK(cudaMemset(e->gbar.p, 0, 64));
    std::vector<float> cs;
    rope_table(e->d, cs);
    CK(e->rope.alloc(cs.size() * 4));
    CK(cudaMemcpy(e->rope.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    int r = alloc_scratch(e);
    if (r) return r;
    e->stats.weight_bytes = e->weight_bytes;
    return BT_OK;
}

static int find_src(const std::map<std::string, SrcTensor> &m, const std::string &n, const SrcTensor **out) {
    auto it = m.find(n);
    if (it == m.end()) return fail(BT_ERR_MISSING_TENSOR, "missing tensor " + n);
    *out = &it->second;
    return BT_OK;
}

static int check_shape(const std::string &n, const SrcTensor *t, std::initializer_list<uint64_t> want) {
    uint64_t n_el = 1;
    int i = 0;
    for (uint64_t w : want) {
        if (i >= 4 || t->ne[i] != w)
            return fail(BT_ERR_INVALID, "tensor " + n + " has an unexpected shape (dim " + std::to_string(i) + ")");
        n_el *= w;
        i++;
    }
    for (; i < 4; i++)
        if (t->ne[i] > 1) return fail(BT_ERR_INVALID, "tensor " + n + " has extra dimensions");
    uint64_t eb = expected_bytes(t->type, n_el);
    if (eb == 0) return fail(BT_ERR_UNSUPPORTED, "tensor " + n + " has unsupported type " + std::to_string(t->type));
    if (t->nbytes && t->nbytes != eb) return fail(BT_ERR_INVALID, "tensor " + n + " byte size does not match its shape");
    return BT_OK;
}

// Ingests the tensors in `src`: the embedding and output head when `globals`, layers [l0, l1),
// then (when `finish`) the per-engine tables. The synthetic path calls it one layer at a time.
static int build_engine(bt_engine *e, const std::map<std::string, SrcTensor> &src, uint32_t l0, uint32_t l1,
                        bool globals, bool finish) {
    const bt_model_desc &d = e->d;
    const uint64_t E = d.n_embd, QW = d.n_head * d.head_dim, KW = d.n_head_kv * d.head_dim;
    const uint64_t NE = d.n_expert, F = d.n_ff_exp, V = d.n_vocab, D = d.head_dim;
    DevBuf staging;
    const SrcTensor *t;
    int r;
#define NEED(name, ...)                                  \
    if ((r = find_src(src, name, &t))) return r;         \
    if ((r = check_shape(name, t, {__VA_ARGS__}))) return r;
    if (globals) {
    NEED("token_embd.weight", E, V);
    if ((r = ingest_qmat(e, e->embd, t->type, V, E, 1, t->data, t->device, default_rpt(E), true, staging))) return r;
    NEED("output_norm.weight", E);
    if (t->type != T_F32) return fail(BT_ERR_UNSUPPORTED, "norm weights must be F32");
    if ((r = ingest_f32(e, e->out_norm, t->data, t->device, E))) return r;
    {
        const SrcTensor *o = nullptr;
        auto it = src.find("output.weight");
        o = it == src.end() ? nullptr : &it->second;
        if (!o) {
            NEED("token_embd.weight", E, V);
            o = t;  // tied output head (stream.rs:2892-2896)
        } else if ((r = check_shape("output.weight", o, {E, V}))) {
            return r;
        }
        if ((r = ingest_qmat(e, e->out, o->type, V, E, 1, o->data, o->device, default_rpt(E), false, staging)))
            return r;
    }
    }
    if (e->L.size() != d.n_layer) e->L.resize(d.n_layer);
    for (uint32_t il = l0; il < l1; il++) {
        Layer &l = e->L[il];
        std::string p = "blk." + std::to_string(il) + ".";
        auto f32 = [&](const char *suffix, DevBuf &b, uint64_t n) -> int {
            std::string nm = p + suffix;
            const SrcTensor *tt;
            int rr;
            if ((rr = find_src(src, nm, &tt))) return rr;
            if ((rr = check_shape(nm, tt, {n}))) return rr;
            if (tt->type != T_F32) return fail(BT_ERR_UNSUPPORTED, nm + " must be F32");
            return ingest_f32(e, b, tt->data, tt->device, n);
        };
        auto mat = [&](const char *suffix, QMat &m, uint64_t cols, uint64_t rows, uint64_t nm_, int rpt) -> int {
            std::string nm = p + suffix;
            const SrcTensor *tt;
            int rr;
            if ((rr = find_src(src, nm, &tt))) return rr;
            if (nm_ > 1) {
                if ((rr = check_shape(nm, tt, {cols, rows, nm_}))) return rr;
            } else if ((rr = check_shape(nm, tt, {cols, rows}))) {
                return rr;
            }
            return ingest_qmat(e, m, tt->type, rows, cols, nm_, tt->data, tt->device, rpt, false, staging);
        };
        if ((r = f32("attn_norm.weight", l.attn_norm, E))) return r;
        if ((r = f32("attn_q_norm.weight", l.q_norm, D))) return r;
        if ((r = f32("attn_k_norm.weight", l.k_norm, D))) return r;
        if ((r = f32("ffn_norm.weight", l.ffn_norm, E))) return r;
        {
            std::string nm = p + "ffn_gate_inp.weight";
            const SrcTensor *tt;
            if ((r = find_src(src, nm, &tt))) return r;
            if ((r = check_shape(nm, tt, {E, NE}))) return r;
            if (tt->type != T_F32) return fail(BT_ERR_UNSUPPORTED, nm + " must be F32");
            if ((r = ingest_f32(e, l.gate_inp, tt->data, tt->device, E * NE))) return r;
            // optional: a router bias (not in the reference's qwen3moe tensors; the skewed-routing
            // workloads carry one)
            nm = p + "ffn_gate_inp.bias";
            if (find_src(src, nm, &tt) == BT_OK) {
                if ((r = check_shape(nm, tt, {NE}))) return r;
                if (tt->type != T_F32) return fail(BT_ERR_UNSUPPORTED, nm + " must be F32");
                if ((r = ingest_f32(e, l.gate_bias, tt->data, tt->device, NE))) return r;
            }
            g_err.clear();
        }
        if ((r = mat("attn_q.weight", l.q, E, QW, 1, default_rpt(E)))) return r;
        if ((r = mat("attn_k.weight", l.k, E, KW, 1, default_rpt(E)))) return r;
        if ((r = mat("attn_v.weight", l.v, E, KW, 1, default_rpt(E)))) return r;
        if ((r = mat("attn_output.weight", l.o, QW, E, 1, default_rpt(QW)))) return r;
        if ((r = mat("ffn_gate_exps.weight", l.gate, E, F, NE, default_rpt(E)))) return r;
        if ((r = mat("ffn_up_exps.weight", l.up, E, F, NE, default_rpt(E)))) return r;
        if ((r = mat("ffn_down_exps.weight", l.down, F, E, NE, 1))) return r;
        if (d.n_ff_shexp) {
            const uint64_t FS = d.n_ff_shexp;
            if ((r = mat("ffn_gate_shexp.weight", l.gate_sh, E, FS, 1, default_rpt(E)))) return r;
            if ((r = mat("ffn_up_shexp.weight", l.up_sh, E, FS, 1, default_rpt(E)))) return r;
            if ((r = mat("ffn_down_shexp.weight", l.down_sh, FS, E, 1, default_rpt(FS)))) return r;
            const uint64_t wb = e->weight_bytes;
            if ((r = mat("ffn_down_shexp.weight", l.down_sh1, FS, E, 1, 1))) return r;
            e->weight_bytes = wb;
        }
        if (l.gate.g.tile_bytes != l.up.g.tile_bytes && l.gate.type == l.up.type)
            return fail(BT_ERR_INVALID, "gate and up experts disagree in shape");
    }
#undef NEED
    CK(cudaStreamSynchronize(e->st));  // the sources may be freed after this returns
    return finish ? finish_create(e) : BT_OK;
}

static int engine_init_device(bt_engine *e, int device) {
    e->device = device;
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return fail(BT_ERR_UNSUPPORTED, "this build targets sm_100a (B200)");
    e->n_sm = prop.multiProcessorCount;
    CK(init_kernel_attributes());
    CK(init_step_kernel_attributes());
    CK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    return BT_OK;
}

extern "C" int bt_engine_create(const bt_model_desc *desc, const bt_tensor_view *tensors, size_t n_tensors, int device,
                                bt_engine **out) {
    if (!out) return fail(BT_ERR_INVALID, "null output handle");
    *out = nullptr;
    int r = validate_desc(desc);
    if (r) return r;
    std::unique_ptr<bt_engine> e(new bt_engine());
    e->d = *desc;
    if (e->d.expert_workers == 0) e->d.expert_workers = 4;
    if ((r = engine_init_device(e.get(), device))) return r;
    std::map<std::string, SrcTensor> src;
    for (size_t i = 0; i < n_tensors; i++) {
        const bt_tensor_view &tv = tensors[i];
        if (!tv.name || !tv.data) return fail(BT_ERR_INVALID, "tensor view with a null name or data");
        SrcTensor s{};
        s.type = (int)tv.type;
        for (int k = 0; k < 4; k++) s.ne[k] = k < (int)tv.n_dims ? tv.ne[k] : 1;
        s.n_dims = (int)tv.n_dims;
        s.data = tv.data;
        s.device = false;
        s.nbytes = tv.nbytes;
        src[tv.name] = s;
    }
    if ((r = build_engine(e.get(), src, 0, e->d.n_layer, true, true))) {
        std::string keep = g_err;
        bt_engine_destroy(e.release());
        g_err = keep;
        return r;
    }
    *out = e.release();
    return BT_OK;
}

extern "C" int bt_engine_create_synthetic(const bt_model_desc *desc, const uint32_t *types, uint32_t embd_type,
                                          uint32_t out_type, uint64_t seed, float sigma, int device,
                                          bt_engine **out) {
    if (!out || !types) return fail(BT_ERR_INVALID, "null argument");
    *out = nullptr;
    int r = validate_desc(desc);
    if (r) return r;
    std::unique_ptr<bt_engine> e(new bt_engine());
    e->d = *desc;
    if (e->d.expert_workers == 0) e->d.expert_workers = 4;
    if ((r = engine_init_device(e.get(), device))) return r;
    const bt_model_desc &d = e->d;
    const uint64_t E = d.n_embd, QW = d.n_head * d.head_dim, KW = d.n_head_kv * d.head_dim;
    const uint64_t NE = d.n_expert, F = d.n_ff_exp, V = d.n_vocab, D = d.head_dim;
    // Generate the tensors on the device (synth_kernel), one layer at a time, each layer's raw
    // bytes freed once the engine has ingested them.
    std::vector<std::unique_ptr<DevBuf>> raws;
    std::map<std::string, SrcTensor> src;
    auto gen = [&](const std::string &name, int type, std::vector<uint64_t> ne) -> int {
        uint64_t n = 1;
        for (auto v : ne) n *= v;
        uint64_t bytes = expected_bytes(type, n);
        if (!bytes) return fail(BT_ERR_UNSUPPORTED, "synthetic tensor " + name + " has unsupported type");
        std::unique_ptr<DevBuf> b(new DevBuf());
        CK(b->alloc(bytes));
        float mean = is_norm_name(name) ? 1.0f : 0.0f;
        CK(launch_synth(type, synth_key(seed, name_id(name.c_str())), (long long)n, mean, synth_scale(sigma),
                        b->as<uint8_t>(), e->st));
        SrcTensor s{};
        s.type = type;
        for (int k = 0; k < 4; k++) s.ne[k] = k < (int)ne.size() ? ne[k] : 1;
        s.n_dims = (int)ne.size();
        s.data = b->p;
        s.device = true;
        s.nbytes = bytes;
        src[name] = s;
        raws.push_back(std::move(b));
        return BT_OK;
    };
    auto ingest = [&](uint32_t l0, uint32_t l1, bool globals) -> int {
        CK(cudaStreamSynchronize(e->st));
        int rr = build_engine(e.get(), src, l0, l1, globals, false);
        raws.clear();  // build_engine synchronised: the raw copies go
        src.clear();
        return rr;
    };
    auto bail = [&](int rr) {
        std::string keep = g_err;
        bt_engine_destroy(e.release());
        g_err = keep;
        return rr;
    };
    if ((r = gen("token_embd.weight", (int)embd_type, {E, V}))) return r;
    if ((r = gen("output_norm.weight", T_F32, {E}))) return r;
    if ((r = gen("output.weight", (int)out_type, {E, V}))) return r;
    if ((r = ingest(0, 0, true))) return bail(r);
    for (uint32_t il = 0; il < d.n_layer; il++) {
        std::string p = "blk." + std::to_string(il) + ".";
        const uint32_t *ty = types + 7 * il;
        if ((r = gen(p + "attn_norm.weight", T_F32, {E}))) return r;
        if ((r = gen(p + "attn_q.weight", (int)ty[0], {E, QW}))) return r;
        if ((r = gen(p + "attn_k.weight", (int)ty[1], {E, KW}))) return r;
        if ((r = gen(p + "attn_v.weight", (int)ty[2], {E, KW}))) return r;
        if ((r = gen(p + "attn_q_norm.weight", T_F32, {D}))) return r;
        if ((r = gen(p + "attn_k_norm.weight", T_F32, {D}))) return r;
        if ((r = gen(p + "attn_output.weight", (int)ty[3], {QW, E}))) return r;
        if ((r = gen(p + "ffn_norm.weight", T_F32, {E}))) return r;
        if ((r = gen(p + "ffn_gate_inp.weight", T_F32, {E, NE}))) return r;
        if ((r = gen(p + "ffn_gate_exps.weight", (int)ty[4], {E, F, NE}))) return r;
        if ((r = gen(p + "ffn_up_exps.weight", (int)ty[5], {E, F, NE}))) return r;
        if ((r = gen(p + "ffn_down_exps.weight", (int)ty[6], {F, E, NE}))) return r;
        if (d.n_ff_shexp) {  // the shared expert in the routed experts' types
            const uint64_t FS = d.n_ff_shexp;
            if ((r = gen(p + "ffn_gate_shexp.weight", (int)ty[4], {E, FS}))) return r;
            if ((r = gen(p + "ffn_up_shexp.weight", (int)ty[5], {E, FS}))) return r;
            if ((r = gen(p + "ffn_down_shexp.weight", (int)ty[6], {FS, E}))) return r;
        }
        // ingest this layer right away: peak memory is the engine plus one raw layer
        if ((r = ingest(il, il + 1, false))) return bail(r);
    }
    if ((r = finish_create(e.get()))) return bail(r);
    *out = e.release();
    return BT_OK;
}

extern "C" void bt_engine_destroy(bt_engine *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->st) cudaStreamSynchronize(e->st);
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    if (e->ep_comm && nccl_api()) nccl_api()->CommDestroy(e->ep_comm);
    for (uint8_t *h : e->x_host) cudaFreeHost(h);
    if (e->x_sel_host) cudaFreeHost(e->x_sel_host);
    if (e->x_slot_host) cudaFreeHost(e->x_slot_host);
    if (e->x_ev) cudaEventDestroy(e->x_ev);
    if (e->plan_host) cudaFreeHost(e->plan_host);
    if (e->plan_ev) cudaEventDestroy(e->plan_ev);
    if (e->err_host) cudaFreeHost(e->err_host);
    if (e->logits_host) cudaFreeHost(e->logits_host);
    for (auto &p : e->ev_pool) {
        cudaEventDestroy(p.first);
        cudaEventDestroy(p.second);
    }
    for (auto &p : e->ev_used) {
        cudaEventDestroy(p.second.first);
        cudaEventDestroy(p.second.second);
    }
    e->L.clear();
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

extern "C" int bt_engine_stats(const bt_engine *e, bt_stats *out) {
    if (!e || !out) return fail(BT_ERR_INVALID, "null argument");
    *out = e->stats;
    return BT_OK;
}

// ------------------------------------------------------------------ KV pool
static int kv_build_tmap(bt_kv *kv) {
    const bt_model_desc &d = kv->e->d;
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return fail(BT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t rows = (cuuint64_t)d.n_layer * kv->n_blocks * 2 * d.n_head_kv * 16;
    if (rows >= (1ull << 32)) return fail(BT_ERR_UNSUPPORTED, "KV pool too large for one tensor map");
    cuuint64_t dims[2] = {d.head_dim, rows};
    cuuint64_t strides[1] = {(cuuint64_t)d.head_dim * 2};
    cuuint32_t box[2] = {64, 16};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&kv->tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kv->pool.p, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return BT_OK;
}

extern "C" int bt_kv_create(bt_engine *e, uint32_t kind, uint32_t max_seqs, uint32_t max_positions,
                            uint32_t block_tokens, bt_kv **out) {
    if (!e || !out) return fail(BT_ERR_INVALID, "null argument");
    *out = nullptr;
    if (kind != BT_KV_F16) return fail(BT_ERR_UNSUPPORTED, "only the f16 KV cache is on the device path");
    if (block_tokens != 16) return fail(BT_ERR_UNSUPPORTED, "pages hold 16 positions");
    if (max_seqs == 0 || max_positions == 0) return fail(BT_ERR_INVALID, "empty KV pool");
    if (max_positions > e->d.max_positions)
        return fail(BT_ERR_INVALID, "max_positions exceeds the model's RoPE table");
    if (max_seqs > (uint32_t)e->max_out) return fail(BT_ERR_UNSUPPORTED, "at most 256 sequences per pool");
    CK(cudaSetDevice(e->device));
    std::unique_ptr<bt_kv> kv(new bt_kv());
    kv->e = e;
    kv->max_seqs = max_seqs;
    kv->max_positions = max_positions;
    kv->max_blocks = (int)((max_positions + 15) / 16);
    kv->n_blocks = kv->max_blocks * (int)max_seqs;
    const bt_model_desc &d = e->d;
    size_t pool = (size_t)d.n_layer * kv->n_blocks * 2 * d.n_head_kv * 16 * d.head_dim * 2;
    if (kv->pool.alloc(pool) != cudaSuccess) return fail(BT_ERR_OOM, "KV pool allocation failed");
    CK(cudaMemset(kv->pool.p, 0, pool));
    CK(kv->bt_dev.alloc((size_t)max_seqs * kv->max_blocks * 4));
    CK(kv->dev_len.alloc((size_t)max_seqs * 4));
    CK(cudaMemset(kv->dev_len.p, 0, (size_t)max_seqs * 4));
    kv->table.assign((size_t)max_seqs * kv->max_blocks, 0);
    for (int b = kv->n_blocks - 1; b >= 0; b--) kv->free_blocks.push_back(b);
    kv->len.assign(max_seqs, 0);
    kv->layer_pos.assign(max_seqs, std::vector<uint32_t>(d.n_layer, 0));
    kv->pages.assign(max_seqs, std::vector<int>());
    int r = kv_build_tmap(kv.get());
    if (r) return r;
    *out = kv.release();
    return BT_OK;
}

extern "C" void bt_kv_destroy(bt_kv *kv) {
    if (!kv) return;
    cudaSetDevice(kv->e->device);
    cudaStreamSynchronize(kv->e->st);
    for (auto it = kv->e->graphs.begin(); it != kv->e->graphs.end();) {
        if (it->first.kv == kv) {
            cudaGraphExecDestroy(it->second);
            it = kv->e->graphs.erase(it);
        } else {
            ++it;
        }
    }
    delete kv;
}

// Page bookkeeping: pages[seq] lists the pool blocks holding positions [16*i, 16*i+16).
static int kv_reserve(bt_kv *kv, uint32_t seq, uint32_t n_positions) {
    size_t need = (n_positions + 15) / 16;
    if (need > (size_t)kv->max_blocks) return fail(BT_ERR_KV, "sequence would exceed max_positions");
    auto &pg = kv->pages[seq];
    while (pg.size() < need) {
        if (kv->free_blocks.empty()) return fail(BT_ERR_OOM, "KV pool has no free pages");
        int b = kv->free_blocks.back();
        kv->free_blocks.pop_back();
        kv->table[(size_t)seq * kv->max_blocks + pg.size()] = b;
        pg.push_back(b);
        kv->table_dirty = true;
    }
    return BT_OK;
}

static void kv_release_beyond(bt_kv *kv, uint32_t seq, uint32_t n_positions) {
    size_t keep = (n_positions + 15) / 16;
    auto &pg = kv->pages[seq];
    while (pg.size() > keep) {
        kv->free_blocks.push_back(pg.back());
        kv->table[(size_t)seq * kv->max_blocks + pg.size() - 1] = 0;
        pg.pop_back();
        kv->table_dirty = true;
    }
}

static int kv_sync(bt_kv *kv) {
    if (kv->table_dirty) {
        CK(cudaMemcpyAsync(kv->bt_dev.p, kv->table.data(), kv->table.size() * 4, cudaMemcpyHostToDevice, kv->e->st));
        kv->table_dirty = false;
    }
    return BT_OK;
}

static int kv_set_len(bt_kv *kv, uint32_t seq, uint32_t n) {
    kv->len[seq] = n;
    int v = (int)n;
    CK(cudaMemcpyAsync(kv->dev_len.as<int>() + seq, &v, 4, cudaMemcpyHostToDevice, kv->e->st));
    CK(cudaStreamSynchronize(kv->e->st));
    return BT_OK;
}

static int kv_check_seq(const bt_kv *kv, uint32_t seq) {
    if (!kv) return fail(BT_ERR_INVALID, "null KV handle");
    if (seq >= kv->max_seqs) return fail(BT_ERR_INVALID, "sequence id out of range");
    return BT_OK;
}

extern "C" int bt_kv_len(const bt_kv *kv, uint32_t seq, uint32_t *len) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    if (!len) return fail(BT_ERR_INVALID, "null output");
    *len = kv->len[seq];
    return BT_OK;
}

extern "C" int bt_kv_bytes(const bt_kv *kv, uint64_t *bytes) {
    if (!kv || !bytes) return fail(BT_ERR_INVALID, "null argument");
    // bytes held, as KvCache::bytes counts them: positions * per-position bytes, k and v, all layers
    const bt_model_desc &d = kv->e->d;
    uint64_t total = 0;
    for (uint32_t s = 0; s < kv->max_seqs; s++)
        for (uint32_t l = 0; l < d.n_layer; l++) total += (uint64_t)kv->layer_pos[s][l] * d.n_head_kv * d.head_dim * 2 * 2;
    *bytes = total;
    return BT_OK;
}

extern "C" int bt_kv_is_consistent(const bt_kv *kv, uint32_t seq, int *consistent) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    if (!consistent) return fail(BT_ERR_INVALID, "null output");
    int ok = 1;
    for (uint32_t l = 0; l < kv->e->d.n_layer; l++) ok &= kv->layer_pos[seq][l] == kv->len[seq];
    *consistent = ok;
    return BT_OK;
}

extern "C" int bt_kv_clear(bt_kv *kv, uint32_t seq) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    kv_release_beyond(kv, seq, 0);
    for (auto &c : kv->layer_pos[seq]) c = 0;
    return kv_set_len(kv, seq, 0);
}

extern "C" int bt_kv_truncate(bt_kv *kv, uint32_t seq, uint32_t n) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    if (n >= kv->len[seq]) return BT_OK;  // truncate_to keeps everything when n >= len (kv.rs:280-283)
    kv_release_beyond(kv, seq, n);
    for (auto &c : kv->layer_pos[seq]) c = c < n ? c : n;
    return kv_set_len(kv, seq, n);
}

extern "C" int bt_kv_set_positions(bt_kv *kv, uint32_t seq, uint32_t n) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    if (n > kv->max_positions) return fail(BT_ERR_KV, "positions exceed the pool's max_positions");
    if ((r = kv_reserve(kv, seq, n))) return r;
    if ((r = kv_sync(kv))) return r;
    return kv_set_len(kv, seq, n);
}

static int kv_tmp(bt_kv *kv, size_t bytes) {
    if (kv->tmp.n < bytes) CK(kv->tmp.alloc(bytes));
    return BT_OK;
}

extern "C" int bt_kv_shift_out(bt_kv *kv, uint32_t seq, uint32_t keep, uint32_t drop) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    uint32_t n = kv->len[seq];
    if (drop == 0 || keep >= n) return BT_OK;  // kv.rs:314-317
    if (drop > n - keep) drop = n - keep;
    const bt_model_desc &d = kv->e->d;
    const uint32_t tail = n - keep - drop;
    const size_t per = (size_t)d.n_head_kv * d.head_dim;
    if ((r = kv_sync(kv))) return r;
    if (tail) {
        if ((r = kv_tmp(kv, tail * per * 2 * 2))) return r;
        __half *kb = kv->tmp.as<__half>(), *vb = kb + tail * per;
        const int *row = kv->bt_dev.as<int>() + (size_t)seq * kv->max_blocks;
        for (uint32_t l = 0; l < d.n_layer; l++) {
            CK(launch_kv_copy(kv->pool.as<__half>(), row, (int)l, kv->n_blocks, d.n_head_kv, d.head_dim, keep + drop,
                              tail, kb, vb, 0, kv->e->st));
            CK(launch_kv_copy(kv->pool.as<__half>(), row, (int)l, kv->n_blocks, d.n_head_kv, d.head_dim, keep, tail, kb,
                              vb, 1, kv->e->st));
        }
    }
    CK(cudaStreamSynchronize(kv->e->st));
    kv_release_beyond(kv, seq, n - drop);
    for (auto &c : kv->layer_pos[seq]) c = c > drop ? c - drop : 0;
    return kv_set_len(kv, seq, n - drop);
}

extern "C" int bt_kv_export_layer(const bt_kv *kvc, uint32_t seq, uint32_t layer, void *k_out, void *v_out,
                                  uint64_t bytes) {
    bt_kv *kv = const_cast<bt_kv *>(kvc);
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    const bt_model_desc &d = kv->e->d;
    if (layer >= d.n_layer) return fail(BT_ERR_INVALID, "layer out of range");
    const size_t step = (size_t)d.n_head_kv * d.head_dim * 2;
    const uint32_t held = kv->layer_pos[seq][layer];
    if (bytes % step || bytes > held * step)
        return fail(BT_ERR_KV, "export size must be whole positions, at most the layer's");
    const uint32_t n = (uint32_t)(bytes / step);
    if (!n) return BT_OK;
    if (!k_out || !v_out) return fail(BT_ERR_INVALID, "null output buffer");
    if ((r = kv_sync(kv))) return r;
    if ((r = kv_tmp(kv, 2 * bytes))) return r;
    __half *kb = kv->tmp.as<__half>(), *vb = kb + bytes / 2;
    CK(launch_kv_copy(kv->pool.as<__half>(), kv->bt_dev.as<int>() + (size_t)seq * kv->max_blocks, (int)layer,
                      kv->n_blocks, d.n_head_kv, d.head_dim, 0, (int)n, kb, vb, 0, kv->e->st));
    CK(cudaMemcpyAsync(k_out, kb, bytes, cudaMemcpyDeviceToHost, kv->e->st));
    CK(cudaMemcpyAsync(v_out, vb, bytes, cudaMemcpyDeviceToHost, kv->e->st));
    CK(cudaStreamSynchronize(kv->e->st));
    return BT_OK;
}

extern "C" int bt_kv_import_layer(bt_kv *kv, uint32_t seq, uint32_t layer, const void *k, const void *v,
                                  uint64_t bytes) {
    int r = kv_check_seq(kv, seq);
    if (r) return r;
    const bt_model_desc &d = kv->e->d;
    const size_t step = (size_t)d.n_head_kv * d.head_dim * 2;
    if (layer >= d.n_layer || bytes % step) return fail(BT_ERR_KV, "restore_layer needs whole positions");
    const uint32_t n = (uint32_t)(bytes / step);
    if (n > kv->max_positions) return fail(BT_ERR_KV, "restored layer exceeds max_positions");
    if (n && (!k || !v)) return fail(BT_ERR_INVALID, "null input buffer");
    uint32_t hold = n > kv->len[seq] ? n : kv->len[seq];
    if ((r = kv_reserve(kv, seq, hold))) return r;
    if ((r = kv_sync(kv))) return r;
    if (n) {
        if ((r = kv_tmp(kv, 2 * bytes))) return r;
        __half *kb = kv->tmp.as<__half>(), *vb = kb + bytes / 2;
        CK(cudaMemcpyAsync(kb, k, bytes, cudaMemcpyHostToDevice, kv->e->st));
        CK(cudaMemcpyAsync(vb, v, bytes, cudaMemcpyHostToDevice, kv->e->st));
        CK(launch_kv_copy(kv->pool.as<__half>(), kv->bt_dev.as<int>() + (size_t)seq * kv->max_blocks, (int)layer,
                          kv->n_blocks, d.n_head_kv, d.head_dim, 0, (int)n, kb, vb, 1, kv->e->st));
        CK(cudaStreamSynchronize(kv->e->st));
    }
    kv->layer_pos[seq][layer] = n;
    return BT_OK;
}

// ------------------------------------------------------------------ one forward step
struct StepPlan {
    int T = 0;
    std::vector<int> tokens, seq_of, local_idx;
    std::vector<unsigned char> single;
    std::vector<int> st_seq, st_ntok, st_lrow;
    std::vector<int> x_rows;  // token index of each output row produced in this step
    int out_first = 0;        // first output row
};

static void timer_begin(bt_engine *e, const char *name) {
    if (!e->timing) return;
    std::pair<cudaEvent_t, cudaEvent_t> ev;
    if (!e->ev_pool.empty()) {
        ev = e->ev_pool.back();
        e->ev_pool.pop_back();
    } else {
        cudaEventCreate(&ev.first);
        cudaEventCreate(&ev.second);
    }
    cudaEventRecord(ev.first, e->st);
    e->ev_used.push_back({name, ev});
}

static void timer_end(bt_engine *e) {
    if (!e->timing) return;
    cudaEventRecord(e->ev_used.back().second.second, e->st);
}

static void timer_collect(bt_engine *e) {
    for (auto &u : e->ev_used) {
        float ms = 0;
        cudaEventElapsedTime(&ms, u.second.first, u.second.second);
        KernelTimer &k = e->timers[u.first];
        k.name = u.first;
        k.launches++;
        k.ms += ms;
        e->ev_pool.push_back(u.second);
    }
    e->ev_used.clear();
}

static GemvSeg make_seg(const QMat &m, int tile0, int out_off) {
    GemvSeg s{};
    s.w = m.buf.as<uint8_t>();
    s.type = m.type;
    s.nsb = m.g.nsb;
    s.rpt = m.g.rpt;
    s.S = m.g.S;
    s.tile_bytes = m.g.tile_bytes;
    s.rows = (int)m.rows;
    s.n_tiles = (int)m.g.n_tiles;
    s.tile0 = tile0;
    s.out_off = out_off;
    return s;
}

static cudaError_t run_gemv(bt_engine *e, const QMat *const *mats, const int *out_offs, int nseg, const float *x,
                            long long x_stride, const int *x_rows, const float *norm_w, int K, int T, float *y,
                            long long y_stride, const float *res, long long res_stride, const char *name,
                            unsigned long long *amax = nullptr, const PrefetchSpec *pf = nullptr, int tgrp = 0) {
    GemvArgs a{};
    a.amax = amax;
    if (pf) a.pf = *pf;
    int tile0 = 0, slot = 0;
    for (int i = 0; i < nseg; i++) {
        a.seg[i] = make_seg(*mats[i], tile0, out_offs[i]);
        tile0 += a.seg[i].n_tiles;
        slot = a.seg[i].tile_bytes > slot ? a.seg[i].tile_bytes : slot;
    }
    a.nseg = nseg;
    a.total_tiles = tile0;
    a.x = x;
    a.x_stride = x_stride;
    a.x_rows = x_rows;
    a.norm_w = norm_w;
    a.eps = e->d.rms_eps;
    a.K = K;
    a.T = T;
    a.y = y;
    a.y_stride = y_stride;
    a.res = res;
    a.res_stride = res_stride;
    a.err = e->err.as<int>();
    a.slot_bytes = slot;
    long long n_units = tile0;
    if (tgrp > 0 && !amax) {
        // units (group of tgrp tokens, tile); a CTA's contiguous range of at most upc units
        // covers at most (upc - 1) / tiles + 2 groups, whose tokens it stages
        a.tgrp = tgrp;
        n_units = (long long)tile0 * ((T + tgrp - 1) / tgrp);
        const long long g = grid_for(e, n_units), upc = (n_units + g - 1) / g;
        const long long span = ((upc - 1) / tile0 + 2) * tgrp;
        a.stage_max = (int)(span < T ? span : T);
        if (a.stage_max > 128) return cudaErrorInvalidValue;  // the RMSNorm scales: 128 floats
    }
    a.nst = 1;
    size_t fixed = gemv_smem_bytes(a) - (size_t)GEMV_WARPS * slot;
    a.nst = T > MAX_T ? pick_nst_cap(slot, fixed, (size_t)max_dynamic_smem()) : pick_nst(slot, fixed);
    if (gemv_smem_bytes(a) > (size_t)max_dynamic_smem()) return cudaErrorInvalidValue;
    timer_begin(e, name);
    cudaError_t r = launch_gemv(a, grid_for(e, n_units), e->st, e->pdl);
    timer_end(e);
    return r;
}

// Q6_K matrices the tensor-core kernel takes: whole 128-row blocks (a tile's run of superblock
// scales d is padded to 16 bytes, so every tile starts on 16 bytes and each d's 16-byte piece lies
// inside its tile)
static bool mma6_fits(const QMat &m) {
    return m.type == T_Q6_K && m.rows % 128 == 0 && m.g.tile_bytes % 16 == 0;
}

// The arguments of a tensor-core GEMV over n segments (activations from the Q8_K staging)
static GemvArgs mma_args(bt_engine *e, const QMat *const *m, const int *offs, int n, int K, int T, float *y,
                         long long y_stride, const float *res, long long res_stride, unsigned long long *amax) {
    GemvArgs a{};
    int tile0 = 0;
    for (int i = 0; i < n; i++) {
        a.seg[i] = make_seg(*m[i], tile0, offs[i]);
        tile0 += a.seg[i].n_tiles;
    }
    a.nseg = n;
    a.total_tiles = tile0;
    a.K = K;
    a.T = T;
    a.y = y;
    a.y_stride = y_stride;
    a.res = res;
    a.res_stride = res_stride;
    a.err = e->err.as<int>();
    a.amax = amax;
    a.q8_qs = e->q8_qs.as<int8_t>();
    a.q8_d = e->q8_d.as<float>();
    a.q8_bs = e->q8_bs.as<int>();
    return a;
}

// T activation rows (x_rows[t] or t) as Q8_K rows for the tensor-core GEMVs, RMS-normed first
// when norm_w
static cudaError_t stage_q8(bt_engine *e, const float *x, long long x_stride, const int *x_rows, const float *norm_w,
                            int K, int T) {
    if ((size_t)T > e->q8_rows) return cudaErrorInvalidValue;
    return launch_q8_stage(x, x_stride, x_rows, norm_w, e->d.rms_eps, K, T, e->q8_qs.as<int8_t>(), e->q8_d.as<float>(),
                           e->q8_bs.as<int>(), e->st, e->pdl);
}

// A batched GEMV (T > MAX_T tokens): the Q4_K segments of whole 128-row blocks run on tcgen05 in
// one launch over all tokens, the Q6_K ones in another (both from one Q8_K staging), when they
// cover mma_min_units CTAs; the other segments run through the dp4a kernel.
static int run_gemv_batched(bt_engine *e, const QMat *const *mats, const int *offs, int nseg, const float *x,
                            long long x_stride, const float *norm_w, int K, int T, float *y, long long y_stride,
                            const float *res, long long res_stride, const char *name, const PrefetchSpec *pf) {
    const QMat *mm[3], *m6[3], *dm[3];
    int mo[3], o6[3], dof[3], nm = 0, n6 = 0, nd = 0;
    // the tensor-core kernels' units are (N tokens, 128 rows), one CTA per SM: they pay once
    // they cover mma_min_units CTAs
    const int gn = gemv_mma_tokens(K);
    long long units = 0, units6 = 0;
    for (int i = 0; i < nseg; i++) {
        if (mats[i]->type == T_Q4_K && mats[i]->rows % 128 == 0) units += (long long)(mats[i]->rows / 128);
        if (mma6_fits(*mats[i])) units6 += (long long)(mats[i]->rows / 128);
    }
    units *= gn ? (T + gn - 1) / gn : 0;
    units6 *= (T + 15) / 16;
    const bool mma_ok = e->mma && gn && gemv_mma_smem_bytes(K) <= (size_t)max_dynamic_smem() &&
                        units >= e->mma_min_units && (size_t)T <= e->q8_rows;
    const bool mma6_ok = e->mma && gemv_mma6_smem_bytes(K) <= (size_t)max_dynamic_smem() &&
                         units6 >= e->mma_min_units && (size_t)T <= e->q8_rows;
    for (int i = 0; i < nseg; i++) {
        if (mma_ok && mats[i]->type == T_Q4_K && mats[i]->rows % 128 == 0) {
            mm[nm] = mats[i];
            mo[nm++] = offs[i];
        } else if (mma6_ok && mma6_fits(*mats[i])) {
            m6[n6] = mats[i];
            o6[n6++] = offs[i];
        } else {
            dm[nd] = mats[i];
            dof[nd++] = offs[i];
        }
    }
    if (nm || n6) {
        timer_begin(e, name);
        cudaError_t ce = stage_q8(e, x, x_stride, nullptr, norm_w, K, T);
        if (ce == cudaSuccess && nm) {
            const GemvArgs a = mma_args(e, mm, mo, nm, K, T, y, y_stride, res, res_stride, nullptr);
            ce = launch_gemv_mma(a, e->mma_grid ? e->mma_grid : e->n_sm, e->st, e->pdl);
        }
        if (ce == cudaSuccess && n6) {
            const GemvArgs a = mma_args(e, m6, o6, n6, K, T, y, y_stride, res, res_stride, nullptr);
            ce = launch_gemv_mma6(a, e->mma_grid ? e->mma_grid : e->n_sm, e->st, e->pdl);
        }
        timer_end(e);
        CK(ce);
    }
    if (nd) {
        int slot = 0;
        long long tiles = 0;
        for (int i = 0; i < nd; i++) {
            slot = dm[i]->g.tile_bytes > slot ? dm[i]->g.tile_bytes : slot;
            tiles += dm[i]->g.n_tiles;
        }
        // fewer tiles than half the grid's warps (a 512-row attn_v: 128 tiles): one launch whose
        // units are (group of 8k tokens, tile), enough of them for every warp
        const long long warps = (long long)grid_for(e, 1ll << 30) * GEMV_WARPS;
        if (e->token_groups && tiles * 2 <= warps) {
            const int ng = (int)((warps + tiles - 1) / tiles);
            int tgrp = (T + ng - 1) / ng;
            tgrp = (tgrp + 7) / 8 * 8;
            GemvArgs probe{};
            probe.K = K;
            probe.tgrp = tgrp;
            probe.stage_max = 2 * tgrp < T ? 2 * tgrp : T;
            probe.slot_bytes = slot;
            probe.nst = 1;
            if (probe.stage_max <= 128 && gemv_smem_bytes(probe) <= (size_t)max_dynamic_smem()) {
                CK(run_gemv(e, dm, dof, nd, x, x_stride, nullptr, norm_w, K, T, y, y_stride, res, res_stride, name,
                            nullptr, pf, tgrp));
                return BT_OK;
            }
        }
        const int chunk = gemv_chunk(T, K, slot);
        for (int t0 = 0; t0 < T; t0 += chunk) {
            const int tg = T - t0 < chunk ? T - t0 : chunk;
            CK(run_gemv(e, dm, dof, nd, x + (size_t)t0 * x_stride, x_stride, nullptr, norm_w, K, tg,
                        y + (size_t)t0 * y_stride, y_stride, res ? res + (size_t)t0 * res_stride : nullptr, res_stride,
                        name, nullptr, t0 == 0 ? pf : nullptr));
        }
    }
    return BT_OK;
}

// The plan's vectors are copied into the engine's pinned staging and sent from there, so the
// host does not wait for the device here. The staging is rewritten only once the previous
// plan's copies have run (plan_ev); in stream order those copies also follow every kernel of
// the step before, so no step reads a plan vector that a later plan overwrites.
static int upload_plan(bt_engine *e, const StepPlan &p) {
    cudaStream_t st = e->st;
    if (e->plan_ev_live) {
        CK(cudaEventSynchronize(e->plan_ev));
        e->plan_ev_live = false;
    }
    int slot = 0;
    auto put = [&](DevBuf &dst, const void *src, size_t n) -> cudaError_t {
        if (n == 0) return cudaSuccess;
        if (n > e->plan_seg) return cudaErrorInvalidValue;
        uint8_t *h = e->plan_host + (size_t)slot++ * e->plan_seg;
        memcpy(h, src, n);
        return cudaMemcpyAsync(dst.p, h, n, cudaMemcpyHostToDevice, st);
    };
    CK(put(e->tokens, p.tokens.data(), (size_t)p.T * 4));
    CK(put(e->seq_of, p.seq_of.data(), (size_t)p.T * 4));
    CK(put(e->local_idx, p.local_idx.data(), (size_t)p.T * 4));
    CK(put(e->single, p.single.data(), (size_t)p.T));
    CK(put(e->st_seq, p.st_seq.data(), p.st_seq.size() * 4));
    CK(put(e->st_ntok, p.st_ntok.data(), p.st_ntok.size() * 4));
    CK(put(e->st_lrow, p.st_lrow.data(), p.st_lrow.size() * 4));
    CK(put(e->x_rows, p.x_rows.data(), p.x_rows.size() * 4));
    CK(cudaEventRecord(e->plan_ev, st));
    e->plan_ev_live = true;
    return BT_OK;
}

// Can this step run as one persistent kernel? Single-token steps of up to STEP_MAX_T
// sequences whose activations fit the kernel's shared memory.
static bool step_eligible(const bt_engine *e, const bt_kv *kv, const StepPlan &p) {
    // (the expert cache: only with the device policy, and without a shared expert)
    if (e->xcache && (!e->xdev || e->d.n_ff_shexp || (e->d.n_head != 4 * e->d.n_head_kv &&
                                                     e->d.n_head != 8 * e->d.n_head_kv)))
        return false;
    if (!e->mega || e->ep || p.T > STEP_MAX_T || p.out_first != 0 || (int)p.x_rows.size() != p.T) return false;
    for (int t = 0; t < p.T; t++)
        if (!p.single[t] || p.local_idx[t] != 0 || p.x_rows[t] != t || p.st_lrow[t] != t) return false;
    if ((int)p.st_seq.size() != p.T) return false;
    const bt_model_desc &d = e->d;
    const int nsbE = d.n_embd / 256, nsbQ = d.n_head * d.head_dim / 256, nsbF = d.n_ff_exp / 256;
    int blocks = nsbE > nsbQ ? nsbE : nsbQ;
    blocks = (int)d.n_expert_used * nsbF > blocks ? (int)d.n_expert_used * nsbF : blocks;
    if ((size_t)p.T * blocks * sizeof(ActBlock) > (size_t)STEP_ACT_BYTES) return false;
    // the down phase: each warp stages one expert's products, and a CTA's rows fit its table
    if (nsbF > STEP_MAX_NSB_F || (p.T * (int)d.n_embd + e->n_sm - 1) / e->n_sm > STEP_DOWN_ROWS) return false;
    // the shared expert is expert index K of the down units
    // (a shared expert: only the kernel with 4 query heads per KV head carries it)
    if (d.n_ff_shexp && ((int)d.n_ff_shexp / 256 > STEP_MAX_NSB_F || (int)d.n_expert_used + 1 > MAX_K ||
                         d.n_head != 4 * d.n_head_kv))
        return false;
    if ((long long)e->L[0].gate.g.nsb * 1 > 32 || 32 / nsbF < 1) return false;
    const int max_chunks = (int)((kv->max_positions + ATTN_CHUNK - 1) / ATTN_CHUNK);
    if (3 * max_chunks * 4 > STEP_CBUF_BYTES || d.n_expert > 512) return false;
    if ((long long)d.n_expert_used * e->L[0].down.g.tile_bytes > STEP_REGION_BYTES / 8) return false;
    // router: rows of a CTA plus the normalised rows in the region, probabilities and keys in cbuf
    if (d.n_expert % 4 != 0 || (int)d.n_expert > STEP_ROUTER_ROWS * e->n_sm) return false;
    if ((size_t)(STEP_ROUTER_ROWS + p.T) * d.n_embd * 4 > (size_t)STEP_REGION_BYTES) return false;
    if ((size_t)d.n_embd * 4 > (size_t)STEP_CBUF_BYTES || (size_t)2 * p.T * d.n_expert * 4 > (size_t)STEP_CBUF_BYTES)
        return false;
    // residual rows one CTA prefetches: the down rows and the attn_output tiles' rows
    if ((long long)p.T * d.n_embd / e->n_sm + 1 > STEP_RES) return false;
    const long long o_tiles = e->L[0].o.g.n_tiles;
    if ((long long)p.T * ((o_tiles + e->n_sm - 1) / e->n_sm + 1) * e->L[0].o.g.rpt > STEP_RES) return false;
    return true;
}

static int launch_persistent_step(bt_engine *e, bt_kv *kv, const StepPlan &p, bool greedy) {
    const bt_model_desc &d = e->d;
    StepArgs a{};
    a.layers = e->layer_dev.as<LayerDev>();
    a.n_layer = (int)d.n_layer;
    a.out = e->out_dev;
    a.out_norm = e->out_norm.as<float>();
    a.embd = e->embd.raw.as<uint8_t>();
    a.embd_type = e->embd.type;
    a.E = d.n_embd;
    a.H = d.n_head;
    a.HK = d.n_head_kv;
    a.D = d.head_dim;
    a.G = d.n_head / d.n_head_kv;
    a.NE = d.n_expert;
    a.K = d.n_expert_used;
    a.F = d.n_ff_exp;
    a.V = d.n_vocab;
    a.workers = (int)d.expert_workers;
    a.n_rot = d.n_rot;
    a.eps = d.rms_eps;
    a.scale = 1.0f / sqrtf((float)d.head_dim);
    a.rope = e->rope.as<float>();
    a.T = p.T;
    a.tokens = e->tokens.as<int>();
    a.seq_of = e->seq_of.as<int>();
    a.pos_of = e->pos_of.as<int>();
    a.dev_len = kv->dev_len.as<int>();
    a.kv = kv->pool.as<__half>();
    a.block_table = kv->bt_dev.as<int>();
    a.max_blocks = kv->max_blocks;
    a.n_blocks = kv->n_blocks;
    a.max_chunks = (int)((kv->max_positions + ATTN_CHUNK - 1) / ATTN_CHUNK);
    a.x = e->x.as<float>();
    a.ffn_in = e->ffn_in.as<float>();
    a.qkv = e->qkv.as<float>();
    a.att = e->att.as<float>();
    a.part = e->part.as<float>();
    a.rlog = e->rlog.as<float>();
    a.act = e->act.as<float>();
    a.dbg_ids = e->dbg_ids.as<int>();
    a.dbg_w = e->dbg_w.as<float>();
    a.TB = e->TB;
    a.logits = e->logits.as<float>();
    a.amax = e->amax.as<unsigned long long>();
    a.next_token = e->next_tok.as<int>();
    a.tokens_buf = greedy ? e->tokens.as<int>() : nullptr;
    a.gen_out = greedy ? e->gen_out.as<int>() : nullptr;
    a.gen_count = e->gen_count.as<int>();
    a.n_out = p.T;
    a.FS = (int)e->d.n_ff_shexp;
    a.shact = e->d.n_ff_shexp ? e->sh_act.as<float>() : nullptr;
    a.xc_on = e->xcache ? 1 : 0;
    if (e->xcache) {
        a.xd = e->xd;
        a.xc_host = e->x_host_devarr.as<const uint8_t *>();
        a.xc_pool = e->x_pool.as<uint8_t>();
        a.xc_stride = e->x_stride;
        a.xc_bounce = e->x_bounce;
        a.xc_copies = e->x_copies.as<XcCopy>();
        a.xc_ncopies = e->x_ncopies.as<int>();
        a.xc_rows = e->x_slot_dev.as<int>();
    }
    a.bar = e->gbar.as<unsigned>();
    a.err = e->err.as<int>();
    a.wait_limit = WAIT_LIMIT_CYCLES;
    if (e->wait_limit_us > 0) {
        int clk_khz = 0;
        CK(cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, e->device));
        a.wait_limit = (long long)e->wait_limit_us * (clk_khz > 0 ? clk_khz : 1965000) / 1000;
    }
    a.fault_cta = e->fault_cta;
    a.fault_barrier = e->fault_barrier;
    a.fault_copy = e->fault_copy;
    a.trace = e->tracing ? e->trace.as<unsigned long long>() : nullptr;
    // the barrier's arrival count starts from zero even if an earlier launch stopped early
    CK(cudaMemsetAsync(e->gbar.p, 0, 8, e->st));
    timer_begin(e, "decode_step");
    CK(launch_decode_step(a, kv->tmap, e->n_sm, e->st));
    timer_end(e);
    return BT_OK;
}

// All kernels of one step on e->st. Capturable: no host synchronisation inside.
// Expert cache, one layer: read the layer's selections back, decide hits and misses, copy the
// missing experts from pinned host memory into their slots (ordered before the expert kernels
// on the stream) and upload the layer's slot table. Earlier layers' kernels have finished when
// the selections arrive, so any slot not used by this layer can be overwritten.
static int xcache_layer(bt_engine *e, int il, int T) {
    const int K = (int)e->d.n_expert_used, NE = (int)e->d.n_expert, n = T * K;
    CK(cudaMemcpyAsync(e->x_sel_host, e->sel_ids.p, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaEventRecord(e->x_ev, e->st));
    CK(cudaEventSynchronize(e->x_ev));
    std::vector<int> distinct;
    std::vector<char> seen(NE, 0);
    for (int i = 0; i < n; i++) {
        const int x = e->x_sel_host[i];
        if (x < 0 || x >= NE) return fail(BT_ERR_INVALID, "expert id out of range");
        if (!seen[x]) {
            seen[x] = 1;
            distinct.push_back(x);
        }
    }
    const int nd = (int)distinct.size();
    std::vector<int> slot(nd);
    std::unique_ptr<bool[]> copy(new bool[nd]);
    e->xpol.lookup(il, distinct.data(), nd, slot.data(), copy.get(), e->xstats);
    const Layer &l = e->L[il];
    const size_t bytes = (size_t)(l.gate.mat_bytes + l.up.mat_bytes + l.down.mat_bytes);
    int *row = e->x_slot_host + (size_t)il * NE;
    int bounce = 0;
    for (int i = 0; i < nd; i++) {
        int s = slot[i];
        bool c = copy[i];
        if (s < 0) {
            if (bounce >= e->x_bounce) return fail(BT_ERR_INVALID, "more distinct experts than bounce slots");
            s = e->xpol.capacity() + bounce++;
            c = true;
        }
        row[distinct[i]] = s;
        if (c) {
            CK(cudaMemcpyAsync(e->x_pool.as<uint8_t>() + (size_t)s * e->x_stride,
                               e->x_host[il] + (size_t)distinct[i] * e->x_stride, bytes, cudaMemcpyHostToDevice, e->st));
            e->xstats.bytes_copied += bytes;
        }
    }
    CK(cudaMemcpyAsync(e->x_slot_dev.as<int>() + (size_t)il * NE, row, (size_t)NE * 4, cudaMemcpyHostToDevice, e->st));
    return BT_OK;
}

// The device policy's state for a new, empty cache: the same initial state as
// ExpertCachePolicy (every slot free, popped in ascending order; the xorshift seed).
static int xdev_init(DevBuf &buf, XcDev &x, int policy, int capacity, int n_layer, int n_expert, cudaStream_t st) {
    const size_t LN = (size_t)n_layer * n_expert, C = (size_t)capacity;
    x = XcDev{};
    x.policy = policy;
    x.cap = capacity;
    x.NE = n_expert;
    x.keycap = (int)(4 * LN);
    const size_t bytes = LN * 4 + LN * 4 + C * 4 + C * 8 + C * 8 + C * 4 + (size_t)x.keycap * 4 + XC_NCTR * 4 +
                         XC_N * 8 + 64;
    CK(buf.alloc(bytes));
    uint8_t *p = buf.as<uint8_t>();
    auto take = [&p](size_t n) {
        uint8_t *q = p;
        p += (n + 7) & ~(size_t)7;
        return q;
    };
    x.st = reinterpret_cast<unsigned long long *>(take(XC_N * 8));
    x.last = reinterpret_cast<unsigned long long *>(take(C * 8));
    x.inuse = reinterpret_cast<unsigned long long *>(take(C * 8));
    x.slot_of = reinterpret_cast<int *>(take(LN * 4));
    x.freq = reinterpret_cast<unsigned *>(take(LN * 4));
    x.key_of = reinterpret_cast<int *>(take(C * 4));
    x.free_list = reinterpret_cast<int *>(take(C * 4));
    x.keys = reinterpret_cast<int *>(take((size_t)x.keycap * 4));
    x.ctr = reinterpret_cast<int *>(take(XC_NCTR * 4));
    CK(cudaMemsetAsync(buf.p, 0, bytes, st));
    CK(cudaMemsetAsync(x.slot_of, 0xff, LN * 4, st));
    CK(cudaMemsetAsync(x.key_of, 0xff, C * 4, st));
    std::vector<int> fl(C);
    for (size_t i = 0; i < C; i++) fl[i] = (int)(C - 1 - i);
    const int ctr[XC_NCTR] = {capacity, 0, 0, 0};
    const unsigned long long st0[XC_N] = {0, 0x9E3779B97F4A7C15ull, 0, 0, 0, 0, 0, 0};
    CK(cudaMemcpyAsync(x.free_list, fl.data(), C * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(x.ctr, ctr, sizeof(ctr), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(x.st, st0, sizeof(st0), cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
    return BT_OK;
}

// one layer of the device policy: lookup, then the slot copies from pinned host memory
static int xcache_layer_dev(bt_engine *e, int il, int T, cudaStream_t st) {
    const int K = (int)e->d.n_expert_used, NE = (int)e->d.n_expert;
    const Layer &l = e->L[il];
    const long long bytes = (long long)(l.gate.mat_bytes + l.up.mat_bytes + l.down.mat_bytes);
    timer_begin(e, "xcache_lookup");
    CK(launch_xcache_lookup(e->xd, il, e->sel_ids.as<int>(), T * K, e->x_slot_dev.as<int>() + (size_t)il * NE,
                            e->x_host_dev[il], e->x_pool.as<uint8_t>(), e->x_stride, bytes, e->x_bounce,
                            e->x_copies.as<XcCopy>(), e->x_ncopies.as<int>(), e->err.as<int>(), st));
    timer_end(e);
    timer_begin(e, "xcache_copy");
    CK(launch_xcache_copy(e->x_copies.as<XcCopy>(), e->x_ncopies.as<int>(), bytes, 2 * e->n_sm, st));
    timer_end(e);
    return BT_OK;
}

// The tensor-core gate/up of the grouped path: Q4_K gate and up, whole 128-row blocks, and
// shared memory for the chunk's operands.
// The gate/up input rows (a.fn, `rows` of them) as Q8_K rows for the tensor-core gate/up.
static cudaError_t stage_gateup_q8(bt_engine *e, ExpertArgs &a, int rows, cudaStream_t st, bool pdl) {
    a.q8_qs = e->q8_qs.as<int8_t>();
    a.q8_d = e->q8_d.as<float>();
    a.q8_bs = e->q8_bs.as<int>();
    return launch_q8_stage(a.fn, a.E, nullptr, nullptr, 0.0f, a.E, rows, e->q8_qs.as<int8_t>(), e->q8_d.as<float>(),
                           e->q8_bs.as<int>(), st, pdl);
}

static bool use_gateup_mma(const bt_engine *e, const Layer &l, size_t rows) {
    return e->mma && l.gate.type == T_Q4_K && l.up.type == T_Q4_K && e->d.n_ff_exp % 128 == 0 &&
           gateup_mma_smem_bytes((int)e->d.n_embd) <= (size_t)max_dynamic_smem() && rows <= e->q8_rows;
}

// The tensor-core down of the grouped path: a Q4_K or Q6_K down, output rows in whole 128-row
// blocks, and room in the Q8_K staging for `rows` SiLU-product rows.
static bool use_down_mma(const bt_engine *e, const Layer &l, size_t rows) {
    const int F = (int)e->d.n_ff_exp, nsb = F / 256;
    const size_t smem = l.down.type == T_Q4_K ? down_mma_smem_bytes(F)
                        : l.down.type == T_Q6_K ? down6_mma_smem_bytes(F) : (size_t)-1;
    return e->mma && F % 256 == 0 && nsb >= 1 && l.down.g.rpt * nsb <= 32 && l.down.g.tile_bytes % 16 == 0 &&
           e->d.n_embd % 128 == 0 && smem <= (size_t)max_dynamic_smem() && rows * (size_t)F <= e->q8_rows * e->q8_k;
}

static cudaError_t launch_down_tc(const ExpertArgs &a, int grid, cudaStream_t st, bool pdl) {
    return a.dtype == T_Q6_K ? launch_down6_mma(a, grid, st, pdl) : launch_down_mma(a, grid, st, pdl);
}

// The down input rows (a.act: `rows` (token, slot) rows of F SiLU products) as Q8_K rows.
static cudaError_t stage_down_q8(bt_engine *e, ExpertArgs &a, int rows, cudaStream_t st, bool pdl) {
    a.q8_qs = e->q8_qs.as<int8_t>();
    a.q8_d = e->q8_d.as<float>();
    a.q8_bs = e->q8_bs.as<int>();
    return launch_q8_stage(a.act, a.F, nullptr, nullptr, 0.0f, a.F, rows, e->q8_qs.as<int8_t>(), e->q8_d.as<float>(),
                           e->q8_bs.as<int>(), st, pdl);
}

// The routed experts of layer il for the T tokens of a step, on one GPU: the grouped kernels
// (T > MAX_T: each selected expert's weights once per step) or the per-token ones. Each token's
// selection comes from sel_ids / sel_w ([T][K], ascending ids) and its normalised row from e->fn;
// the weighted expert sum plus e->ffn_in (and the shared expert's rows, when given) goes to e->x.
static int launch_layer_experts(bt_engine *e, int il, int T, const int *sel_ids, const float *sel_w, const int *x_slot,
                                const float *shexp, cudaStream_t st, bool pdl) {
    const bt_model_desc &d = e->d;
    const int E = d.n_embd, K = d.n_expert_used, F = d.n_ff_exp, NE = d.n_expert;
    int *err = e->err.as<int>();
    const Layer &l = e->L[il];
    (void)F;
    (void)NE;
    if (T > MAX_T) {
            GroupArgs ga{};
            ga.sel_ids = sel_ids;
            ga.T = T;
            ga.K = K;
            ga.NE = NE;
            ga.g_count = e->g_count.as<int>();
            ga.g_off = e->g_off.as<int>();
            ga.g_list = e->g_list.as<int>();
            ga.g_active = e->g_active.as<int>();
            ga.g_nactive = e->g_nactive.as<int>();
            ga.g_chunk_e = e->g_chunk_e.as<int>();
            ga.g_chunk_r0 = e->g_chunk_r0.as<int>();
            ga.g_nchunks = e->g_nchunks.as<int>();
            timer_begin(e, "expert_group");
            CK(launch_group(ga, st, pdl));
            timer_end(e);
            ExpertArgs a{};
            a.gate = l.gate.buf.as<uint8_t>();
            a.up = l.up.buf.as<uint8_t>();
            a.down = l.down.buf.as<uint8_t>();
            a.gtype = l.gate.type;
            a.utype = l.up.type;
            a.dtype = l.down.type;
            a.g_nsb = l.gate.g.nsb;
            a.g_rpt = l.gate.g.rpt;
            a.g_S = l.gate.g.S;
            a.g_tile_bytes = l.gate.g.tile_bytes;
            a.g_n_tiles = (int)l.gate.g.n_tiles;
            a.u_tile_bytes = l.up.g.tile_bytes;
            a.g_expert_bytes = l.gate.mat_bytes;
            a.u_expert_bytes = l.up.mat_bytes;
            a.d_expert_bytes = l.down.mat_bytes;
            a.d_nsb = l.down.g.nsb;
            a.d_tile_bytes = l.down.g.tile_bytes;
            a.d_rpt = l.down.g.rpt;
            a.E = E;
            a.F = F;
            a.K = K;
            a.T = T;
            a.workers = (int)d.expert_workers;
            a.sel_ids = sel_ids;
            a.sel_w = sel_w;
            a.fn = e->fn.as<float>();
            a.act = e->act.as<float>();
            a.ffn_in = e->ffn_in.as<float>();
            a.x_out = e->x.as<float>();
            a.single = e->single.as<unsigned char>();
            a.err = err;
            a.g_count = ga.g_count;
            a.g_off = ga.g_off;
            a.g_list = ga.g_list;
            a.g_active = ga.g_active;
            a.g_nactive = ga.g_nactive;
            a.g_chunk_e = ga.g_chunk_e;
            a.g_chunk_r0 = ga.g_chunk_r0;
            a.g_nchunks = ga.g_nchunks;
            a.dpart = e->dpart.as<float>();
            a.row_div = K;  // list entry t*K + k uses token t's row
            a.slot_of = x_slot;
            a.pool = e->x_pool.as<uint8_t>();
            a.slot_stride = e->x_stride;
            a.shexp = shexp;
            const size_t cap = (size_t)max_dynamic_smem();
            a.slot_bytes = a.g_tile_bytes + a.u_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst_cap(a.slot_bytes, gateup_grouped_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes, cap);
            timer_begin(e, "expert_gateup");
            if (use_gateup_mma(e, l, (size_t)T)) {
                CK(stage_gateup_q8(e, a, T, st, pdl));
                CK(launch_gateup_mma(a, e->mma_grid ? e->mma_grid : e->n_sm, st, pdl));
            }
            else
                CK(launch_gateup_grouped(a, e->n_sm, st, pdl));
            timer_end(e);
            a.slot_bytes = down_group_rows(a) * a.d_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst_cap(a.slot_bytes, down_grouped_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes, cap);
            timer_begin(e, "expert_down");
            if (use_down_mma(e, l, (size_t)T * K)) {
                CK(stage_down_q8(e, a, T * K, st, pdl));
                CK(launch_down_tc(a, e->mma_grid ? e->mma_grid : e->n_sm, st, pdl));
            } else {
                CK(launch_down_grouped(a, e->n_sm, st, pdl));
            }
            timer_end(e);
            timer_begin(e, "expert_combine");
            CK(launch_down_combine(a, st, pdl));
            timer_end(e);
            }
        for (int t0 = 0; T <= MAX_T && t0 < T; t0 += MAX_T) {
            int tg = T - t0 < MAX_T ? T - t0 : MAX_T;
            ExpertArgs a{};
            a.gate = l.gate.buf.as<uint8_t>();
            a.up = l.up.buf.as<uint8_t>();
            a.down = l.down.buf.as<uint8_t>();
            a.gtype = l.gate.type;
            a.utype = l.up.type;
            a.dtype = l.down.type;
            a.g_nsb = l.gate.g.nsb;
            a.g_rpt = l.gate.g.rpt;
            a.g_S = l.gate.g.S;
            a.g_tile_bytes = l.gate.g.tile_bytes;
            a.g_n_tiles = (int)l.gate.g.n_tiles;
            a.u_tile_bytes = l.up.g.tile_bytes;
            a.g_expert_bytes = l.gate.mat_bytes;
            a.u_expert_bytes = l.up.mat_bytes;
            a.d_expert_bytes = l.down.mat_bytes;
            a.d_nsb = l.down.g.nsb;
            a.d_tile_bytes = l.down.g.tile_bytes;
            a.d_rpt = l.down.g.rpt;
            a.E = E;
            a.F = F;
            a.K = K;
            a.T = tg;
            a.workers = (int)d.expert_workers;
            a.sel_ids = sel_ids + (size_t)t0 * K;
            a.sel_w = sel_w + (size_t)t0 * K;
            a.fn = e->fn.as<float>() + (size_t)t0 * E;
            a.act = e->act.as<float>() + (size_t)t0 * K * F;
            a.ffn_in = e->ffn_in.as<float>() + (size_t)t0 * E;
            a.x_out = e->x.as<float>() + (size_t)t0 * E;
            a.single = e->single.as<unsigned char>() + t0;
            a.err = err;
            a.slot_of = x_slot;
            a.pool = e->x_pool.as<uint8_t>();
            a.slot_stride = e->x_stride;
            a.shexp = shexp ? shexp + (size_t)t0 * E : nullptr;
            if (e->prefetch && t0 == 0 && il + 1 < d.n_layer) {  // the next layer's q/k/v weights
                const Layer &n = e->L[il + 1];
                a.pf.ptr[0] = n.q.buf.p;
                a.pf.bytes[0] = n.q.buf.n;
                a.pf.ptr[1] = n.k.buf.p;
                a.pf.bytes[1] = n.k.buf.n;
                a.pf.ptr[2] = n.v.buf.p;
                a.pf.bytes[2] = n.v.buf.n;
                a.pf.n = 3;
            } else if (e->prefetch && t0 == 0) {  // the output head
                a.pf.ptr[0] = e->out.buf.p;
                a.pf.bytes[0] = e->out.buf.n < (64ull << 20) ? e->out.buf.n : (64ull << 20);
                a.pf.n = 1;
            }
            a.prefetch_down = e->prefetch ? 1 : 0;
            a.slot_bytes = a.g_tile_bytes + a.u_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst(a.slot_bytes, gateup_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes);
            timer_begin(e, "expert_gateup");
            CK(launch_gateup(a, grid_for(e, (long long)tg * K * a.g_n_tiles), st, pdl));
            timer_end(e);
            a.slot_bytes = K * a.d_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst(a.slot_bytes, down_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes);
            a.pf = PrefetchSpec{};
            a.prefetch_down = 0;
            timer_begin(e, "expert_down");
            CK(launch_down(a, grid_for(e, (long long)tg * E), st, pdl));
            timer_end(e);
        }
    return BT_OK;
}

static int launch_step(bt_engine *e, bt_kv *kv, const StepPlan &p, bool greedy) {
    if (e->ep_aborted) return fail(BT_ERR_TIMEOUT, "the expert-parallel communicator was aborted by an earlier failure");
    if (step_eligible(e, kv, p)) return launch_persistent_step(e, kv, p, greedy);
    const bt_model_desc &d = e->d;
    const int T = p.T, E = d.n_embd, H = d.n_head, HK = d.n_head_kv, D = d.head_dim;
    const int QW = H * D, KW = HK * D, K = d.n_expert_used, F = d.n_ff_exp, NE = d.n_expert;
    const int G = H / HK;
    cudaStream_t st = e->st;
    const bool pdl = e->pdl;
    int *err = e->err.as<int>();
    {
        EmbedArgs a{};
        a.table = e->embd.raw.as<uint8_t>();
        a.type = e->embd.type;
        a.E = E;
        a.V = d.n_vocab;
        a.T = T;
        a.tokens = e->tokens.as<int>();
        a.seq_of = e->seq_of.as<int>();
        a.local_idx = e->local_idx.as<int>();
        a.dev_len = kv->dev_len.as<int>();
        a.pos_of = e->pos_of.as<int>();
        a.x = e->x.as<float>();
        a.err = err;
        timer_begin(e, "embed");
        CK(launch_embed(a, st, pdl));
        timer_end(e);
    }
    for (uint32_t il = 0; il < d.n_layer; il++) {
        Layer &l = e->L[il];
        // while q/k/v run: pull this layer's KV pages, attn_output and router weights into L2
        PrefetchSpec pf_qkv{};
        pf_qkv.ptr[0] = l.o.buf.p;
        pf_qkv.bytes[0] = l.o.buf.n;
        pf_qkv.ptr[1] = l.gate_inp.p;
        pf_qkv.bytes[1] = l.gate_inp.n;
        pf_qkv.n = e->prefetch ? 2 : 0;
        if (e->prefetch && T <= MAX_T) {
            pf_qkv.kv = kv->pool.as<__half>();
            pf_qkv.block_table = kv->bt_dev.as<int>();
            pf_qkv.seq_of = e->seq_of.as<int>();
            pf_qkv.pos_of = e->pos_of.as<int>();
            pf_qkv.max_blocks = kv->max_blocks;
            pf_qkv.layer = (int)il;
            pf_qkv.n_blocks = kv->n_blocks;
            pf_qkv.HK = HK;
            pf_qkv.D = D;
            pf_qkv.T = T;
        }
        int qslot = l.q.g.tile_bytes > l.k.g.tile_bytes ? l.q.g.tile_bytes : l.k.g.tile_bytes;
        qslot = l.v.g.tile_bytes > qslot ? l.v.g.tile_bytes : qslot;
        const int qchunk = gemv_chunk(T, E, qslot);
        if (T > MAX_T) {
            const QMat *mats[3] = {&l.q, &l.k, &l.v};
            int offs[3] = {0, QW, QW + KW};
            int rr = run_gemv_batched(e, mats, offs, 3, e->x.as<float>(), E, l.attn_norm.as<float>(), E, T,
                                      e->qkv.as<float>(), QW + 2 * KW, nullptr, 0, "qkv_gemv", &pf_qkv);
            if (rr) return rr;
        }
        for (int t0 = 0; T <= MAX_T && t0 < T; t0 += qchunk) {
            int tg = T - t0 < qchunk ? T - t0 : qchunk;
            const QMat *mats[3] = {&l.q, &l.k, &l.v};
            int offs[3] = {0, QW, QW + KW};
            CK(run_gemv(e, mats, offs, 3, e->x.as<float>() + (size_t)t0 * E, E, nullptr, l.attn_norm.as<float>(), E, tg,
                        e->qkv.as<float>() + (size_t)t0 * (QW + 2 * KW), QW + 2 * KW, nullptr, 0, "qkv_gemv", nullptr,
                        t0 == 0 ? &pf_qkv : nullptr));
        }
        {
            QkvPostArgs a{};
            a.qkv = e->qkv.as<float>();
            a.qkv_stride = QW + 2 * KW;
            a.q_norm = l.q_norm.as<float>();
            a.k_norm = l.k_norm.as<float>();
            a.eps = d.rms_eps;
            a.rope = e->rope.as<float>();
            a.n_rot = d.n_rot;
            a.H = H;
            a.HK = HK;
            a.D = D;
            a.T = T;
            a.seq_of = e->seq_of.as<int>();
            a.pos_of = e->pos_of.as<int>();
            a.block_table = kv->bt_dev.as<int>();
            a.max_blocks = kv->max_blocks;
            a.layer = (int)il;
            a.n_blocks = kv->n_blocks;
            a.kv = kv->pool.as<__half>();
            a.q_out = e->qbuf.as<float>();
            timer_begin(e, "qkv_post");
            CK(launch_qkv_post(a, st, pdl));
            timer_end(e);
        }
        {
            AttnArgs a{};
            a.q = e->qbuf.as<float>();
            a.H = H;
            a.HK = HK;
            a.D = D;
            a.G = G;
            a.T = T;
            a.seq_of = e->seq_of.as<int>();
            a.pos_of = e->pos_of.as<int>();
            a.block_table = kv->bt_dev.as<int>();
            a.max_blocks = kv->max_blocks;
            a.layer = (int)il;
            a.n_blocks = kv->n_blocks;
            a.max_chunks = (int)((kv->max_positions + ATTN_CHUNK - 1) / ATTN_CHUNK);
            a.n_cta = e->n_sm * (e->attn_warp ? 4 : 3);  // resident CTAs per SM
            a.scale = 1.0f / sqrtf((float)D);
            a.part = e->part.as<float>();
            a.cnt = e->acnt.as<int>();
            a.out = e->att.as<float>();
            a.err = err;
            timer_begin(e, "attention");
            if (e->attn_warp)
                CK(launch_attn_warp(a, kv->tmap, st, pdl));
            else
                CK(launch_attn(a, kv->tmap, st, pdl));
            timer_end(e);
        }
        const int ochunk = gemv_chunk(T, QW, l.o.g.tile_bytes);
        if (T > MAX_T) {
            const QMat *mats[1] = {&l.o};
            int offs[1] = {0};
            int rr = run_gemv_batched(e, mats, offs, 1, e->att.as<float>(), QW, nullptr, QW, T, e->ffn_in.as<float>(), E,
                                      e->x.as<float>(), E, "attn_out_gemv", nullptr);
            if (rr) return rr;
        }
        for (int t0 = 0; T <= MAX_T && t0 < T; t0 += ochunk) {
            int tg = T - t0 < ochunk ? T - t0 : ochunk;
            const QMat *mats[1] = {&l.o};
            int offs[1] = {0};
            CK(run_gemv(e, mats, offs, 1, e->att.as<float>() + (size_t)t0 * QW, QW, nullptr, nullptr, QW, tg,
                        e->ffn_in.as<float>() + (size_t)t0 * E, E, e->x.as<float>() + (size_t)t0 * E, E, "attn_out_gemv"));
        }
        {
            RouterArgs a{};
            a.x = e->ffn_in.as<float>();
            a.norm_w = l.ffn_norm.as<float>();
            a.eps = d.rms_eps;
            a.E = E;
            a.Wr = l.gate_inp.as<float>();
            a.bias = l.gate_bias.p ? l.gate_bias.as<float>() : nullptr;
            a.NE = NE;
            a.K = K;
            a.T = T;
            a.rows_per_cta = 8;
            a.fn_out = e->fn.as<float>();
            a.logits = e->rlog.as<float>();
            a.cnt = e->rcnt.as<int>();
            a.topk_ids = e->dbg_ids.as<int>() + (size_t)il * e->TB * K;
            a.topk_w = e->dbg_w.as<float>() + (size_t)il * e->TB * K;
            a.sel_ids = e->sel_ids.as<int>();
            a.sel_w = e->sel_w.as<float>();
            timer_begin(e, "router");
            CK(launch_router(a, st, pdl));
            timer_end(e);
        }
        if (e->xcache) {
            int xr = e->xdev ? xcache_layer_dev(e, (int)il, T, st) : xcache_layer(e, (int)il, T);
            if (xr) return xr;
        }
        const int *x_slot = e->xcache ? e->x_slot_dev.as<int>() + (size_t)il * NE : nullptr;
        const float *shexp = nullptr;
        if (d.n_ff_shexp) {  // the shared expert on every token: gate|up GEMV, silu*up, down GEMV
            const int FS = (int)d.n_ff_shexp;
            const int ch = gemv_chunk(T, E, l.gate_sh.g.tile_bytes > l.up_sh.g.tile_bytes ? l.gate_sh.g.tile_bytes
                                                                                          : l.up_sh.g.tile_bytes);
            for (int t0 = 0; t0 < T; t0 += ch) {
                const int tg = T - t0 < ch ? T - t0 : ch;
                const QMat *mats[2] = {&l.gate_sh, &l.up_sh};
                int offs[2] = {0, FS};
                CK(run_gemv(e, mats, offs, 2, e->fn.as<float>() + (size_t)t0 * E, E, nullptr, nullptr, E, tg,
                            e->sh_gu.as<float>() + (size_t)t0 * 2 * FS, 2 * FS, nullptr, 0, "shexp_gateup_gemv"));
            }
            timer_begin(e, "shexp_act");
            CK(launch_shexp_act(e->sh_gu.as<float>(), e->sh_act.as<float>(), T, FS, st, pdl));
            timer_end(e);
            const int chd = gemv_chunk(T, FS, l.down_sh.g.tile_bytes);
            for (int t0 = 0; t0 < T; t0 += chd) {
                const int tg = T - t0 < chd ? T - t0 : chd;
                const QMat *mats[1] = {&l.down_sh};
                int offs[1] = {0};
                CK(run_gemv(e, mats, offs, 1, e->sh_act.as<float>() + (size_t)t0 * FS, FS, nullptr, nullptr, FS, tg,
                            e->sh_out.as<float>() + (size_t)t0 * E, E, nullptr, 0, "shexp_down_gemv"));
            }
            shexp = e->sh_out.as<float>();
        }
        if (e->ep) {  // expert parallelism: rows to the owning ranks, experts there, rows back
            const int S = step_cap(e) * K, n = e->ep_n, per = NE / n;
            const NcclApi *api = nccl_api();
            EpPackArgs pa{};
            pa.sel_ids = e->sel_ids.as<int>();
            pa.fn = e->fn.as<float>();
            pa.T = T;
            pa.K = K;
            pa.E = E;
            pa.ranks = n;
            pa.per = per;
            pa.slots = S;
            pa.send_meta = e->ep_send_meta.as<int>();
            pa.send_rows = e->ep_send_rows.as<float>();
            // the owners' gate/up reads Q8_K rows (tensor-core path): quantise the T token rows
            // here and send those, a quarter of the f32 bytes; the owner would stage the same bits
            const bool q8x = use_gateup_mma(e, l, (size_t)n * S) && (size_t)T <= e->q8_rows;
            const int nsb = E / 256;
            timer_begin(e, "ep_pack");
            if (q8x) {
                CK(stage_q8(e, e->fn.as<float>(), E, nullptr, nullptr, E, T));
                pa.q8_qs = e->q8_qs.as<int8_t>();
                pa.q8_d = e->q8_d.as<float>();
                pa.q8_bs = e->q8_bs.as<int>();
                pa.send_qs = e->ep_send_qs.as<int8_t>();
                pa.send_d = e->ep_send_d.as<float>();
                pa.send_bs = e->ep_send_bs.as<int>();
            }
            CK(launch_ep_pack(pa, st, pdl));
            timer_end(e);
            timer_begin(e, "ep_dispatch");
            NK(api->GroupStart());
            for (int r = 0; r < n; r++) {
                NK(api->Send(pa.send_meta + (size_t)r * S, S, ncclInt32, r, e->ep_comm, st));
                NK(api->Recv(e->ep_recv_meta.as<int>() + (size_t)r * S, S, ncclInt32, r, e->ep_comm, st));
                if (q8x) {
                    NK(api->Send(pa.send_qs + (size_t)r * S * E, (size_t)S * E, ncclInt8, r, e->ep_comm, st));
                    NK(api->Send(pa.send_d + (size_t)r * S * nsb, (size_t)S * nsb, ncclFloat32, r, e->ep_comm, st));
                    NK(api->Send(pa.send_bs + (size_t)r * S * nsb * 8, (size_t)S * nsb * 8, ncclInt32, r, e->ep_comm, st));
                    NK(api->Recv(e->ep_recv_qs.as<int8_t>() + (size_t)r * S * E, (size_t)S * E, ncclInt8, r, e->ep_comm,
                                 st));
                    NK(api->Recv(e->ep_recv_d.as<float>() + (size_t)r * S * nsb, (size_t)S * nsb, ncclFloat32, r,
                                 e->ep_comm, st));
                    NK(api->Recv(e->ep_recv_bs.as<int>() + (size_t)r * S * nsb * 8, (size_t)S * nsb * 8, ncclInt32, r,
                                 e->ep_comm, st));
                } else {
                    NK(api->Send(pa.send_rows + (size_t)r * S * E, (size_t)S * E, ncclFloat32, r, e->ep_comm, st));
                    NK(api->Recv(e->ep_recv_rows.as<float>() + (size_t)r * S * E, (size_t)S * E, ncclFloat32, r,
                                 e->ep_comm, st));
                }
            }
            NK(api->GroupEnd());
            timer_end(e);
            GroupArgs ga{};
            ga.sel_ids = e->ep_recv_meta.as<int>();
            ga.T = n * step_cap(e);
            ga.K = K;
            ga.NE = NE;
            ga.g_count = e->g_count.as<int>();
            ga.g_off = e->g_off.as<int>();
            ga.g_list = e->g_list.as<int>();
            ga.g_active = e->g_active.as<int>();
            ga.g_nactive = e->g_nactive.as<int>();
            ga.g_chunk_e = e->g_chunk_e.as<int>();
            ga.g_chunk_r0 = e->g_chunk_r0.as<int>();
            ga.g_nchunks = e->g_nchunks.as<int>();
            timer_begin(e, "expert_group");
            CK(launch_group(ga, st, false));
            timer_end(e);
            ExpertArgs a{};
            a.gate = l.gate.buf.as<uint8_t>();
            a.up = l.up.buf.as<uint8_t>();
            a.down = l.down.buf.as<uint8_t>();
            a.gtype = l.gate.type;
            a.utype = l.up.type;
            a.dtype = l.down.type;
            a.g_nsb = l.gate.g.nsb;
            a.g_rpt = l.gate.g.rpt;
            a.g_S = l.gate.g.S;
            a.g_tile_bytes = l.gate.g.tile_bytes;
            a.g_n_tiles = (int)l.gate.g.n_tiles;
            a.u_tile_bytes = l.up.g.tile_bytes;
            a.g_expert_bytes = l.gate.mat_bytes;
            a.u_expert_bytes = l.up.mat_bytes;
            a.d_expert_bytes = l.down.mat_bytes;
            a.d_nsb = l.down.g.nsb;
            a.d_tile_bytes = l.down.g.tile_bytes;
            a.d_rpt = l.down.g.rpt;
            a.E = E;
            a.F = F;
            a.K = K;
            a.T = T;
            a.workers = (int)d.expert_workers;
            a.err = err;
            a.g_count = ga.g_count;
            a.g_off = ga.g_off;
            a.g_list = ga.g_list;
            a.g_active = ga.g_active;
            a.g_nactive = ga.g_nactive;
            a.g_chunk_e = ga.g_chunk_e;
            a.g_chunk_r0 = ga.g_chunk_r0;
            a.g_nchunks = ga.g_nchunks;
            a.row_div = 1;  // received rows are indexed by their slot
            a.expert_base = e->ep_e0;  // this rank's experts only are resident
            a.fn = e->ep_recv_rows.as<float>();
            a.act = e->ep_act.as<float>();
            a.dpart = e->ep_dpart.as<float>();
            const size_t cap = (size_t)max_dynamic_smem();
            a.slot_bytes = a.g_tile_bytes + a.u_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst_cap(a.slot_bytes, gateup_grouped_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes, cap);
            timer_begin(e, "expert_gateup");
            if (q8x) {  // the received Q8_K rows are the B operand as they are
                a.q8_qs = e->ep_recv_qs.as<int8_t>();
                a.q8_d = e->ep_recv_d.as<float>();
                a.q8_bs = e->ep_recv_bs.as<int>();
                CK(launch_gateup_mma(a, e->mma_grid ? e->mma_grid : e->n_sm, st, pdl));
            } else if (use_gateup_mma(e, l, (size_t)n * S)) {
                CK(stage_gateup_q8(e, a, n * S, st, pdl));
                CK(launch_gateup_mma(a, e->mma_grid ? e->mma_grid : e->n_sm, st, pdl));
            }
            else
                CK(launch_gateup_grouped(a, e->n_sm, st, pdl));
            timer_end(e);
            a.slot_bytes = down_group_rows(a) * a.d_tile_bytes;
            a.nst = 1;
            a.nst = pick_nst_cap(a.slot_bytes, down_grouped_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes, cap);
            timer_begin(e, "expert_down");
            if (use_down_mma(e, l, (size_t)n * S)) {
                CK(stage_down_q8(e, a, n * S, st, pdl));
                CK(launch_down_tc(a, e->mma_grid ? e->mma_grid : e->n_sm, st, pdl));
            } else {
                CK(launch_down_grouped(a, e->n_sm, st, pdl));
            }
            timer_end(e);
            timer_begin(e, "ep_combine_exchange");
            NK(api->GroupStart());
            for (int r = 0; r < n; r++) {
                NK(api->Send(e->ep_dpart.as<float>() + (size_t)r * S * E, (size_t)S * E, ncclFloat32, r, e->ep_comm, st));
                NK(api->Recv(e->ep_ret.as<float>() + (size_t)r * S * E, (size_t)S * E, ncclFloat32, r, e->ep_comm, st));
            }
            NK(api->GroupEnd());
            timer_end(e);
            a.sel_ids = e->sel_ids.as<int>();
            a.sel_w = e->sel_w.as<float>();
            a.ffn_in = e->ffn_in.as<float>();
            a.x_out = e->x.as<float>();
            a.single = e->single.as<unsigned char>();
            a.dpart = e->ep_ret.as<float>();
            a.ep_ranks = n;
            a.ep_per = per;
            a.ep_slots = S;
            a.shexp = shexp;
            timer_begin(e, "expert_combine");
            CK(launch_down_combine(a, st, false));
            timer_end(e);
        } else {
            // (with the device cache the weights come from the copy kernel just before: the expert
            // kernels, which request weight tiles before their PDL wait, must not start early)
            int r_ = launch_layer_experts(e, il, T, e->sel_ids.as<int>(), e->sel_w.as<float>(), x_slot, shexp, st,
                                          pdl && !(e->xcache && e->xdev));
            if (r_) return r_;
        }
    }
    const int n_out = (int)p.x_rows.size();
    const bool head_mma = n_out > MAX_T && e->mma && mma6_fits(e->out) &&
                          gemv_mma6_smem_bytes(E) <= (size_t)max_dynamic_smem() && (size_t)n_out <= e->q8_rows;
    if (head_mma) {
        // more outputs than one dp4a launch carries: the Q6_K head on the tensor cores, with the
        // per-output argmax keys
        const QMat *mats[1] = {&e->out};
        int offs[1] = {0};
        timer_begin(e, "output_gemv");
        cudaError_t ce = stage_q8(e, e->x.as<float>(), E, e->x_rows.as<int>(), e->out_norm.as<float>(), E, n_out);
        if (ce == cudaSuccess) {
            const GemvArgs a = mma_args(e, mats, offs, 1, E, n_out, e->logits.as<float>() + (size_t)p.out_first * d.n_vocab,
                                        d.n_vocab, nullptr, 0, e->amax.as<unsigned long long>() + p.out_first);
            ce = launch_gemv_mma6(a, e->mma_grid ? e->mma_grid : e->n_sm, e->st, e->pdl);
        }
        timer_end(e);
        CK(ce);
    }
    for (int o0 = 0; !head_mma && o0 < n_out; o0 += MAX_T) {
        int og = n_out - o0 < MAX_T ? n_out - o0 : MAX_T;
        const QMat *mats[1] = {&e->out};
        int offs[1] = {0};
        CK(run_gemv(e, mats, offs, 1, e->x.as<float>(), E, e->x_rows.as<int>() + o0, e->out_norm.as<float>(), E, og,
                    e->logits.as<float>() + (size_t)(p.out_first + o0) * d.n_vocab, d.n_vocab, nullptr, 0, "output_gemv",
                    e->amax.as<unsigned long long>() + p.out_first + o0));
    }
    {
        StepEndArgs a{};
        a.logits = e->logits.as<float>();
        a.V = d.n_vocab;
        a.n_seqs = (int)p.st_seq.size();
        a.n_out = greedy ? (int)p.st_seq.size() : e->max_out;
        a.seq_ids = e->st_seq.as<int>();
        a.n_tok = e->st_ntok.as<int>();
        a.logit_row = e->st_lrow.as<int>();
        a.amax = e->amax.as<unsigned long long>();
        a.dev_len = kv->dev_len.as<int>();
        a.next_token = e->next_tok.as<int>();
        a.tokens_buf = greedy ? e->tokens.as<int>() : nullptr;
        a.gen_out = greedy ? e->gen_out.as<int>() : nullptr;
        a.gen_count = e->gen_count.as<int>();
        timer_begin(e, "step_end");
        CK(launch_step_end(a, st, pdl));
        timer_end(e);
    }
    return BT_OK;
}

// The device error word `h`, read back after the stream was waited for: nonzero clears it and
// fails the call.
static int err_word(bt_engine *e, int h) {
    if (h) {
        CK(cudaMemsetAsync(e->err.p, 0, 4, e->st));
        // a step that stopped early leaves its partial argmax keys behind (the step end clears them)
        CK(cudaMemsetAsync(e->amax.p, 0, (size_t)e->max_out * 8, e->st));
        CK(cudaStreamSynchronize(e->st));
        if (h & ERR_WAIT_TIMEOUT) return fail(BT_ERR_TIMEOUT, "a device wait ran out of time");
        return fail(BT_ERR_INVALID, "a kernel rejected an index (token id out of range?)");
    }
    return BT_OK;
}

static int check_err(bt_engine *e) {
    int local = 0;
    int *h = e->err_host ? e->err_host : &local;  // the single-op engines have no pinned staging
    CK(cudaMemcpyAsync(h, e->err.p, 4, cudaMemcpyDeviceToHost, e->st));
    int r = wait_stream(e);
    if (r) return r;
    return err_word(e, *h);
}

extern "C" int bt_forward(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *tokens,
                          const uint32_t *n_tokens, const uint32_t *pos_start, uint32_t n_seqs, float *logits_out) {
    if (!e || !kv || !seq_ids || !tokens || !n_tokens || !pos_start) return fail(BT_ERR_INVALID, "null argument");
    if (kv->e != e) return fail(BT_ERR_INVALID, "KV pool belongs to another engine");
    if (n_seqs == 0 || n_seqs > (uint32_t)e->max_out) return fail(BT_ERR_INVALID, "1..256 sequences per call");
    CK(cudaSetDevice(e->device));
    auto t0 = std::chrono::steady_clock::now();
    std::vector<char> seen(kv->max_seqs, 0);
    size_t total = 0;
    for (uint32_t i = 0; i < n_seqs; i++) {
        uint32_t s = seq_ids[i];
        if (s >= kv->max_seqs) return fail(BT_ERR_INVALID, "sequence id out of range");
        if (seen[s]) return fail(BT_ERR_INVALID, "a sequence appears twice in one call");
        seen[s] = 1;
        if (n_tokens[i] == 0) return fail(BT_ERR_INVALID, "a sequence has no tokens");
        if (pos_start[i] != kv->len[s]) return fail(BT_ERR_KV, "pos_start must equal the sequence's cache length");
        if ((uint64_t)kv->len[s] + n_tokens[i] > kv->max_positions)
            return fail(BT_ERR_KV, "context would exceed max_positions");
        total += n_tokens[i];
    }
    for (size_t i = 0; i < total; i++)
        if (tokens[i] >= e->d.n_vocab) return fail(BT_ERR_INVALID, "token id out of range");
    int r;
    for (uint32_t i = 0; i < n_seqs; i++)
        if ((r = kv_reserve(kv, seq_ids[i], kv->len[seq_ids[i]] + n_tokens[i]))) return r;
    if ((r = kv_sync(kv))) return r;
    // cut the concatenated tokens into steps of at most TB tokens
    size_t g = 0;
    uint32_t si = 0, ti = 0;  // current sequence, token within it
    while (g < total) {
        StepPlan p;
        std::map<int, int> seq_slot;
        while (p.T < step_cap(e) && g < total) {
            uint32_t s = seq_ids[si];
            p.tokens.push_back((int)tokens[g]);
            p.seq_of.push_back((int)s);
            auto it = seq_slot.find((int)s);
            int local = 0;
            if (it == seq_slot.end()) {
                seq_slot[(int)s] = (int)p.st_seq.size();
                p.st_seq.push_back((int)s);
                p.st_ntok.push_back(0);
                p.st_lrow.push_back(-1);
            } else {
                local = p.st_ntok[it->second];
            }
            int slot = seq_slot[(int)s];
            p.local_idx.push_back(local);
            p.single.push_back(n_tokens[si] == 1 ? 1 : 0);
            p.st_ntok[slot]++;
            if (ti + 1 == n_tokens[si]) {  // the sequence's last token: its logits row is si
                if (p.x_rows.empty()) p.out_first = (int)si;
                p.st_lrow[slot] = (int)si;
                p.x_rows.push_back(p.T);
            }
            p.T++;
            g++;
            ti++;
            if (ti == n_tokens[si]) {
                si++;
                ti = 0;
            }
        }
        if ((r = upload_plan(e, p))) return r;
        if ((r = launch_step(e, kv, p, false))) return r;
        e->last_T = p.T;
        e->last_first = g - p.T;
    }
    const size_t lbytes = (size_t)n_seqs * e->d.n_vocab * 4;
    cudaPointerAttributes pa{};
    const bool out_pinned = logits_out && cudaPointerGetAttributes(&pa, logits_out) == cudaSuccess &&
                            pa.type == cudaMemoryTypeHost;
    if (logits_out && !out_pinned) cudaGetLastError();  // (pageable memory: not an error)
    if (out_pinned) {
        // page-locked output (bt_host_alloc): the logits go straight into it, behind one wait
        CK(cudaMemcpyAsync(e->err_host, e->err.p, 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaMemcpyAsync(logits_out, e->logits.p, lbytes, cudaMemcpyDeviceToHost, e->st));
        if ((r = wait_stream(e))) return r;
        if ((r = err_word(e, *e->err_host))) return r;
    } else if (logits_out && n_seqs <= (uint32_t)STEP_MAX_T) {
        // error word and logits through pinned staging, behind one wait
        CK(cudaMemcpyAsync(e->err_host, e->err.p, 4, cudaMemcpyDeviceToHost, e->st));
        CK(cudaMemcpyAsync(e->logits_host, e->logits.p, lbytes, cudaMemcpyDeviceToHost, e->st));
        if ((r = wait_stream(e))) return r;
        if ((r = err_word(e, *e->err_host))) return r;
        memcpy(logits_out, e->logits_host, lbytes);
    } else {
        if ((r = check_err(e))) return r;
        if (logits_out) CK(cudaMemcpyAsync(logits_out, e->logits.p, lbytes, cudaMemcpyDeviceToHost, e->st));
        if ((r = wait_stream(e))) return r;
    }
    for (uint32_t i = 0; i < n_seqs; i++) {
        uint32_t s = seq_ids[i];
        kv->len[s] += n_tokens[i];
        for (auto &c : kv->layer_pos[s]) c = kv->len[s];
    }
    e->last_rows = (int)n_seqs;
    e->stats.forward_calls++;
    e->stats.tokens += total;
    e->stats.forward_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return BT_OK;
}

static int greedy_prepare(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *first_tokens,
                          uint32_t n_seqs, uint32_t n_steps, StepPlan &p) {
    if (!e || !kv || !seq_ids || !first_tokens) return fail(BT_ERR_INVALID, "null argument");
    if (kv->e != e) return fail(BT_ERR_INVALID, "KV pool belongs to another engine");
    if (n_seqs == 0 || n_seqs > (uint32_t)step_cap(e))
        return fail(BT_ERR_INVALID, "1..step-capacity sequences per greedy batch (64 under expert parallelism)");
    CK(cudaSetDevice(e->device));
    std::vector<char> seen(kv->max_seqs, 0);
    for (uint32_t i = 0; i < n_seqs; i++) {
        uint32_t s = seq_ids[i];
        if (s >= kv->max_seqs || seen[s]) return fail(BT_ERR_INVALID, "bad or repeated sequence id");
        seen[s] = 1;
        if ((uint64_t)kv->len[s] + n_steps > kv->max_positions) return fail(BT_ERR_KV, "context would exceed max_positions");
        if (first_tokens[i] >= e->d.n_vocab) return fail(BT_ERR_INVALID, "token id out of range");
    }
    int r;
    for (uint32_t i = 0; i < n_seqs; i++)
        if ((r = kv_reserve(kv, seq_ids[i], kv->len[seq_ids[i]] + n_steps))) return r;
    if ((r = kv_sync(kv))) return r;
    size_t need = (size_t)e->max_out * e->d.max_positions;
    if (e->gen_out.n < need * 4) {
        // the graphs hold the buffer's address: drop them before it moves
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        CK(e->gen_out.alloc(need * 4));
    }
    CK(cudaMemsetAsync(e->gen_count.p, 0, (size_t)e->max_out * 4, e->st));
    p.T = (int)n_seqs;
    for (uint32_t i = 0; i < n_seqs; i++) {
        p.tokens.push_back((int)first_tokens[i]);
        p.seq_of.push_back((int)seq_ids[i]);
        p.local_idx.push_back(0);
        p.single.push_back(1);
        p.st_seq.push_back((int)seq_ids[i]);
        p.st_ntok.push_back(1);
        p.st_lrow.push_back((int)i);
        p.x_rows.push_back((int)i);
    }
    p.out_first = 0;
    return upload_plan(e, p);
}

static int greedy_finish(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, uint32_t n_seqs, uint32_t n_steps,
                         uint32_t *tokens_out, float *last_logits) {
    int r = check_err(e);
    if (r) return r;
    if (tokens_out && n_steps)
        CK(cudaMemcpyAsync(tokens_out, e->gen_out.p, (size_t)n_steps * n_seqs * 4, cudaMemcpyDeviceToHost, e->st));
    if (last_logits && n_steps)
        CK(cudaMemcpyAsync(last_logits, e->logits.p, (size_t)n_seqs * e->d.n_vocab * 4, cudaMemcpyDeviceToHost, e->st));
    if ((r = wait_stream(e))) return r;
    for (uint32_t i = 0; i < n_seqs; i++) {
        uint32_t s = seq_ids[i];
        kv->len[s] += n_steps;
        for (auto &c : kv->layer_pos[s]) c = kv->len[s];
    }
    e->stats.tokens += (uint64_t)n_steps * n_seqs;
    if (n_steps) e->last_rows = (int)n_seqs;
    e->last_T = (int)n_seqs;
    e->last_first = 0;
    return BT_OK;
}

extern "C" int bt_generate_greedy(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *first_tokens,
                                  uint32_t n_seqs, uint32_t n_steps, uint32_t *tokens_out, float *last_logits) {
    auto t0 = std::chrono::steady_clock::now();
    StepPlan p;
    int r = greedy_prepare(e, kv, seq_ids, first_tokens, n_seqs, n_steps, p);
    if (r) return r;
    if (e->xcache) {  // a host decision in every layer: plain launches, no graph
        cudaEvent_t a, b;
        CK(cudaEventCreate(&a));
        CK(cudaEventCreate(&b));
        CK(cudaEventRecord(a, e->st));
        for (uint32_t s = 0; s < n_steps && !r; s++) r = launch_step(e, kv, p, true);
        CK(cudaEventRecord(b, e->st));
        if (!r) r = wait_stream(e);
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        if (r) return r;
        e->last_device_ms = ms;
        r = greedy_finish(e, kv, seq_ids, n_seqs, n_steps, tokens_out, last_logits);
        e->stats.forward_calls++;
        e->stats.forward_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        return r;
    }
    GraphKey key{kv, std::vector<uint32_t>(seq_ids, seq_ids + n_seqs)};
    auto it = e->graphs.find(key);
    if (it == e->graphs.end() && n_steps > 0) {
        cudaGraph_t graph;
        CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
        int lr = launch_step(e, kv, p, true);
        cudaError_t ce = cudaStreamEndCapture(e->st, &graph);
        if (lr) return lr;
        CK(ce);
        cudaGraphExec_t exec;
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        CK(ce);
        it = e->graphs.emplace(key, exec).first;
    }
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    CK(cudaEventRecord(a, e->st));
    for (uint32_t s = 0; s < n_steps; s++) CK(cudaGraphLaunch(it->second, e->st));
    CK(cudaEventRecord(b, e->st));
    if ((r = wait_stream(e))) {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        return r;
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    e->last_device_ms = ms;
    e->stats.graph_replays += n_steps;
    r = greedy_finish(e, kv, seq_ids, n_seqs, n_steps, tokens_out, last_logits);
    e->stats.forward_calls++;
    e->stats.forward_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return r;
}

// ------------------------------------------------------------------ isolated expert-FFN timing
// The routed experts' kernels alone, layer after layer over the whole model: T tokens a layer
// with a seeded selection of K distinct experts per token (ascending ids, random positive
// weights summing to 1) and seeded activation rows, through launch_layer_experts -- the kernels a
// decode step of T single tokens runs. Captured once as a CUDA graph of every layer, replayed
// once to warm up, then n_iters times between CUDA events.
extern "C" int bt_bench_experts(bt_engine *e, uint32_t T, uint32_t n_iters, uint64_t seed, uint32_t kernel,
                                double *ms_per_pass, uint64_t *bytes_per_pass, float *out_last) {
    if (!e || !ms_per_pass || !bytes_per_pass) return fail(BT_ERR_INVALID, "null argument");
    if (e->ep || e->xcache) return fail(BT_ERR_UNSUPPORTED, "the expert timing needs every expert resident on one GPU");
    if (T == 0 || (int)T > e->TB || n_iters == 0) return fail(BT_ERR_INVALID, "T must be 1..the step capacity, n_iters >= 1");
    if (kernel > 1) return fail(BT_ERR_INVALID, "kernel must be 0 (per-layer launches) or 1 (the stream kernel)");
    if (kernel == 1 && (int)T > STEP_MAX_T) return fail(BT_ERR_INVALID, "the stream kernel carries at most 4 tokens");
    CK(cudaSetDevice(e->device));
    const bt_model_desc &d = e->d;
    const int L = (int)d.n_layer, K = (int)d.n_expert_used, NE = (int)d.n_expert, E = (int)d.n_embd;
    const int F = (int)d.n_ff_exp;
    uint64_t st = seed ^ 0x5DEECE66Dull;
    auto next = [&st]() {  // splitmix64
        uint64_t z = (st += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    std::vector<int> sel((size_t)L * T * K);
    std::vector<float> w((size_t)L * T * K), fn((size_t)T * E);
    uint64_t bytes = 0;
    std::vector<int> perm(NE);
    for (int il = 0; il < L; il++) {
        std::vector<char> used(NE, 0);
        for (uint32_t t = 0; t < T; t++) {
            for (int i = 0; i < NE; i++) perm[i] = i;
            for (int k = 0; k < K; k++) {  // partial Fisher-Yates: K distinct experts
                const int j = k + (int)(next() % (uint64_t)(NE - k));
                std::swap(perm[k], perm[j]);
            }
            std::sort(perm.begin(), perm.begin() + K);
            float tot = 0.0f;
            for (int k = 0; k < K; k++) {
                const size_t o = ((size_t)il * T + t) * K + k;
                sel[o] = perm[k];
                used[perm[k]] = 1;
                w[o] = 0.05f + (float)(next() >> 40) / (float)(1ull << 24);
                tot += w[o];
            }
            for (int k = 0; k < K; k++) w[((size_t)il * T + t) * K + k] /= tot;
        }
        const Layer &l = e->L[il];
        for (int x = 0; x < NE; x++)
            if (used[x]) bytes += (uint64_t)(l.gate.mat_bytes + l.up.mat_bytes + l.down.mat_bytes);
    }
    for (auto &v : fn) v = (float)((int64_t)(next() >> 40) - (1ll << 23)) / (float)(1ll << 23);
    DevBuf dsel, dw, act_all, out_all;
    CK(dsel.alloc(sel.size() * 4));
    CK(dw.alloc(w.size() * 4));
    CK(cudaMemcpyAsync(dsel.p, sel.data(), sel.size() * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(dw.p, w.data(), w.size() * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->fn.p, fn.data(), fn.size() * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemsetAsync(e->ffn_in.p, 0, (size_t)T * E * 4, e->st));
    CK(cudaMemsetAsync(e->single.p, 1, T, e->st));
    ExpertStreamArgs xa{};
    int xs_grid = e->n_sm;
    if (kernel == 1) {
        if (!e->layer_dev.p) return fail(BT_ERR_UNSUPPORTED, "the stream kernel needs the device layer table");
        int slot = 0;
        for (int il = 0; il < L; il++) {
            const Layer &l = e->L[il];
            slot = std::max(slot, l.gate.g.tile_bytes + l.up.g.tile_bytes);
            slot = std::max(slot, K * l.down.g.tile_bytes);
            if (l.gate.g.rpt * l.gate.g.nsb > 32 || l.down.g.nsb > 32 || F % 256)
                return fail(BT_ERR_UNSUPPORTED, "the stream kernel needs 32-slot gate/up tiles and F % 256 == 0");
        }
        if ((int)((T * (uint32_t)E + (uint32_t)e->n_sm - 1) / (uint32_t)e->n_sm) > expert_stream_max_rows())
            return fail(BT_ERR_UNSUPPORTED, "the stream kernel's CTAs would own too many down rows");
        const size_t fixed = expert_stream_fixed_smem((int)T, E, K, F);
        // four consumer warps: two CTAs per SM, each within half the SM's shared memory; eight:
        // one CTA, 160 KB (the rest of the SM's memory stays L1 for the prefetched products)
        const int cons = e->stream_warps;
        const size_t cap = cons == 4 ? (size_t)112 * 1024
                           : e->stream_slots ? (size_t)max_dynamic_smem()
                                             : std::min<size_t>(160 * 1024, max_dynamic_smem());
        int nslot = cap > fixed ? (int)std::min<size_t>((cap - fixed) / (size_t)slot, (size_t)expert_stream_max_slots()) : 0;
        if (e->stream_slots) {
            if (e->stream_slots > nslot) return fail(BT_ERR_INVALID, "stream_slots: that many slots do not fit");
            nslot = e->stream_slots;
        }
        if (nslot < 2) return fail(BT_ERR_UNSUPPORTED, "the stream kernel's ring does not fit in shared memory");
        CK(act_all.alloc((size_t)L * T * K * F * 4));
        CK(out_all.alloc((size_t)L * T * E * 4));
        xa.layers = e->layer_dev.as<LayerDev>();
        xa.n_layer = L;
        xa.T = (int)T;
        xa.K = K;
        xa.E = E;
        xa.F = F;
        xa.workers = (int)d.expert_workers;
        xa.sel = dsel.as<int>();
        xa.wts = dw.as<float>();
        xa.xin = e->fn.as<float>();
        xa.xin_stride = 0;
        xa.act = act_all.as<float>();
        xa.out = out_all.as<float>();
        xa.bar = e->gbar.as<unsigned>();
        xa.err = e->err.as<int>();
        xa.wait_limit = WAIT_LIMIT_CYCLES;
        xa.nslot = nslot;
        xa.slot_bytes = slot;
        xa.consumers = cons;
        int per_sm = 0;
        CK(prepare_expert_stream(xa, &per_sm));
        if (per_sm < 1)
            return fail(BT_ERR_UNSUPPORTED, "the stream kernel does not fit an SM: " +
                                                std::to_string(expert_stream_fixed_smem((int)T, E, K, F) +
                                                               (size_t)nslot * slot) +
                                                " B of shared memory, " + std::to_string(expert_stream_regs()) +
                                                " registers per thread");
        xs_grid = per_sm * e->n_sm;
    }
    CK(cudaStreamSynchronize(e->st));
    const bool timing = e->timing;
    e->timing = false;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    int r = BT_OK;
    if (kernel == 1) {
        cudaError_t le = cudaMemsetAsync(xa.bar, 0, 4, e->st);
        if (le == cudaSuccess) le = launch_expert_stream(xa, xs_grid, e->st);
        if (le != cudaSuccess) r = fail(BT_ERR_CUDA, cudaGetErrorString(le));
    } else {
        for (int il = 0; il < L && r == BT_OK; il++)
            r = launch_layer_experts(e, il, (int)T, dsel.as<int>() + (size_t)il * T * K,
                                     dw.as<float>() + (size_t)il * T * K, nullptr, nullptr, e->st, e->pdl);
    }
    cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    e->timing = timing;
    if (r) {
        if (g) cudaGraphDestroy(g);
        return r;
    }
    CK(ce);
    ce = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    CK(ce);
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    ce = cudaGraphLaunch(ge, e->st);
    if (ce == cudaSuccess) ce = cudaEventRecord(e0, e->st);
    for (uint32_t i = 0; i < n_iters && ce == cudaSuccess; i++) ce = cudaGraphLaunch(ge, e->st);
    if (ce == cudaSuccess) ce = cudaEventRecord(e1, e->st);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(ge);
    CK(ce);
    if ((r = check_err(e))) return r;
    if (out_last) {
        const float *src = kernel == 1 ? out_all.as<float>() + (size_t)(L - 1) * T * E : e->x.as<float>();
        CK(cudaMemcpy(out_last, src, (size_t)T * E * 4, cudaMemcpyDeviceToHost));
    }
    *ms_per_pass = (double)ms / n_iters;
    *bytes_per_pass = bytes;
    return BT_OK;
}

extern "C" int bt_host_alloc(uint64_t bytes, void **out) {
    if (!out || bytes == 0) return fail(BT_ERR_INVALID, "bad argument");
    *out = nullptr;
    if (cudaHostAlloc(out, (size_t)bytes, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        *out = nullptr;
        return fail(BT_ERR_OOM, "page-locked host allocation failed");
    }
    return BT_OK;
}

extern "C" int bt_host_free(void *p) {
    if (p && cudaFreeHost(p) != cudaSuccess) {
        cudaGetLastError();
        return fail(BT_ERR_INVALID, "not a bt_host_alloc block");
    }
    return BT_OK;
}

// ------------------------------------------------------------------ sampling
extern "C" void bt_sampler_config_default(bt_sampler_config *c) {
    if (!c) return;
    memset(c, 0, sizeof *c);
    c->adaptive_p = -1.0f;  // SamplerConfig::default (sample.rs:183-222)
    c->adaptive_decay = 0.95f;
    c->top_p = 1.0f;
    c->repeat_penalty = 1.0f;
    c->repeat_last_n = 64;
    c->dry_base = 1.75f;
    c->dry_allowed_length = 2;
    c->typical_p = 1.0f;
    c->dynatemp_exponent = 1.0f;
    c->xtc_threshold = 0.1f;
    c->mirostat_tau = 5.0f;
    c->mirostat_eta = 0.1f;
    c->eos = -1;
}

extern "C" void bt_sampler_config_llamacpp(bt_sampler_config *c) {
    if (!c) return;
    bt_sampler_config_default(c);  // llamacpp_defaults (sample.rs:228-268)
    c->temperature = 0.8f;
    c->top_k = 40;
    c->top_p = 0.95f;
    c->min_p = 0.05f;
    c->repeat_penalty = 1.1f;
}

static float clamp_rs(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

extern "C" int bt_sampler_init(const bt_sampler_config *c, bt_sampler_state *st) {
    if (!c || !st) return fail(BT_ERR_INVALID, "null argument");
    st->rng = c->seed + 0x9E3779B97F4A7C15ull;  // Sampler::new (sample.rs:324-344)
    const float decay = clamp_rs(c->adaptive_decay, 0.0f, 0.99f);
    const float ap = (c->adaptive_p != c->adaptive_p || c->adaptive_p < 0.0f) ? 0.0f : c->adaptive_p;
    st->ap_weighted = ap / (1.0f - decay);
    st->ap_total = 1.0f / (1.0f - decay);
    st->mu = 2.0f * c->mirostat_tau;
    return BT_OK;
}

static_assert(sizeof(bt_sampler_state) == sizeof(SampState), "bt_sampler_state and SampState agree");

extern "C" int bt_sample(bt_engine *e, const bt_sampler_config *cfg, bt_sampler_state *states, uint32_t n_seqs,
                         const float *logits, const uint32_t *history, const uint32_t *history_len,
                         uint32_t *tokens_out) {
    if (!e || !cfg || !states || !tokens_out) return fail(BT_ERR_INVALID, "null argument");
    if (n_seqs == 0 || n_seqs > (uint32_t)e->max_out) return fail(BT_ERR_INVALID, "1..256 sequences per call");
    if (!logits && (int)n_seqs > e->last_rows)
        return fail(BT_ERR_INVALID, "no device logits for that many sequences: run bt_forward first or pass logits");
    if (cfg->chain && cfg->n_chain > (uint32_t)SAMP_MAX_CHAIN) return fail(BT_ERR_INVALID, "at most 32 sampler stages");
    if ((cfg->n_bias && (!cfg->bias_ids || !cfg->bias_values)) || (cfg->n_suppress && !cfg->suppress_ids) ||
        (cfg->n_dry_breakers && !cfg->dry_breakers))
        return fail(BT_ERR_INVALID, "a sampler list has a length but no array");
    SampParams P{};
    P.temperature = cfg->temperature;
    P.top_k = cfg->top_k;
    P.top_p = cfg->top_p;
    P.min_p = cfg->min_p;
    P.typical_p = cfg->typical_p;
    P.top_n_sigma = cfg->top_n_sigma;
    P.xtc_probability = cfg->xtc_probability;
    P.xtc_threshold = cfg->xtc_threshold;
    P.dynatemp_range = cfg->dynatemp_range;
    P.dynatemp_exponent = cfg->dynatemp_exponent;
    P.repeat_penalty = cfg->repeat_penalty;
    P.frequency_penalty = cfg->frequency_penalty;
    P.presence_penalty = cfg->presence_penalty;
    P.repeat_last_n = cfg->repeat_last_n;
    P.dry_multiplier = cfg->dry_multiplier;
    P.dry_base = cfg->dry_base;
    P.dry_allowed_length = cfg->dry_allowed_length;
    P.dry_penalty_last_n = cfg->dry_penalty_last_n;
    P.mirostat = cfg->mirostat;
    P.mirostat_tau = cfg->mirostat_tau;
    P.mirostat_eta = cfg->mirostat_eta;
    P.adaptive_p = cfg->adaptive_p;
    P.adaptive_decay = cfg->adaptive_decay;
    P.ignore_eos = cfg->ignore_eos;
    P.eos = cfg->eos;
    if (cfg->chain) {
        P.n_chain = (int)cfg->n_chain;
        for (uint32_t k = 0; k < cfg->n_chain; k++) {
            if (cfg->chain[k] < BT_STAGE_TOP_K || cfg->chain[k] > BT_STAGE_TEMPERATURE)
                return fail(BT_ERR_INVALID, "unknown sampler stage");
            P.chain[k] = cfg->chain[k];
        }
    } else {  // SamplerStage::default_chain (sample.rs:70-79)
        P.n_chain = 6;
        for (int k = 0; k < 6; k++) P.chain[k] = k;
    }
    P.n_bias = (int)cfg->n_bias;
    P.n_suppress = (int)cfg->n_suppress;
    P.n_breakers = (int)cfg->n_dry_breakers;
    P.greedy = cfg->temperature <= 0.0f && cfg->repeat_penalty == 1.0f && cfg->frequency_penalty == 0.0f &&
               cfg->presence_penalty == 0.0f && cfg->n_bias == 0 && !cfg->ignore_eos && cfg->mirostat == 0 &&
               cfg->dry_multiplier == 0.0f && cfg->adaptive_p < 0.0f && cfg->n_suppress == 0;
    const int V = (int)e->d.n_vocab;
    if ((uint64_t)n_seqs * (uint64_t)V > (uint64_t)INT32_MAX)
        return fail(BT_ERR_INVALID, "n_seqs * n_vocab must fit the sort's 31-bit item count");
    // The kernels count in int. Larger values mean the same as these bounds: a top_k at or
    // above the vocabulary keeps every candidate, a window longer than any history is the
    // whole history, and no repeat reaches an allowed length of 2^31 - 1.
    auto clamp31 = [](uint32_t x) { return x > (uint32_t)INT32_MAX ? (uint32_t)INT32_MAX : x; };
    P.top_k = P.top_k > (uint32_t)V ? (uint32_t)V : P.top_k;
    P.repeat_last_n = clamp31(P.repeat_last_n);
    P.dry_allowed_length = clamp31(P.dry_allowed_length);
    P.dry_penalty_last_n = clamp31(P.dry_penalty_last_n);
    // the lists, the histories and the states go up in one copy
    std::vector<uint32_t> off(n_seqs + 1, 0);
    for (uint32_t i = 0; i < n_seqs; i++) {
        const uint64_t next = (uint64_t)off[i] + (history_len ? history_len[i] : 0);
        if (next > (uint64_t)INT32_MAX) return fail(BT_ERR_INVALID, "the histories hold more than 2^31 - 1 tokens");
        off[i + 1] = (uint32_t)next;
    }
    if (off[n_seqs] && !history) return fail(BT_ERR_INVALID, "history lengths without a history");
    size_t at = 0;
    auto slot = [&](size_t bytes) {
        const size_t a = (at + 15) & ~(size_t)15;
        at = a + bytes;
        return a;
    };
    const size_t o_bid = slot(4ull * cfg->n_bias), o_bval = slot(4ull * cfg->n_bias);
    const size_t o_sup = slot(4ull * cfg->n_suppress), o_brk = slot(4ull * cfg->n_dry_breakers);
    const size_t o_hist = slot(4ull * off[n_seqs]), o_off = slot(4ull * (n_seqs + 1));
    const size_t o_st = slot(sizeof(SampState) * n_seqs), o_tok = slot(4ull * n_seqs), o_stat = slot(4ull * n_seqs);
    std::vector<uint8_t> host(at);
    auto put = [&](size_t o, const void *src, size_t bytes) {
        if (bytes) memcpy(host.data() + o, src, bytes);
    };
    put(o_bid, cfg->bias_ids, 4ull * cfg->n_bias);
    put(o_bval, cfg->bias_values, 4ull * cfg->n_bias);
    put(o_sup, cfg->suppress_ids, 4ull * cfg->n_suppress);
    put(o_brk, cfg->dry_breakers, 4ull * cfg->n_dry_breakers);
    put(o_hist, history, 4ull * off[n_seqs]);
    put(o_off, off.data(), 4ull * (n_seqs + 1));
    put(o_st, states, sizeof(SampState) * n_seqs);
    CK(cudaSetDevice(e->device));
    if (e->samp_aux.n < at) CK(e->samp_aux.alloc(at));
    const size_t need = sampler_scratch_bytes((int)n_seqs, V);
    if (e->samp_scratch.n < need) CK(e->samp_scratch.alloc(need));
    uint8_t *aux = e->samp_aux.as<uint8_t>();
    CK(cudaMemcpyAsync(aux, host.data(), at, cudaMemcpyHostToDevice, e->st));
    const float *rows = e->logits.as<float>();
    if (logits) {
        const size_t lb = (size_t)n_seqs * V * 4;
        if (e->samp_in.n < lb) CK(e->samp_in.alloc(lb));
        CK(cudaMemcpyAsync(e->samp_in.p, logits, lb, cudaMemcpyHostToDevice, e->st));
        rows = e->samp_in.as<float>();
    }
    SampLists L{};
    L.bias_ids = reinterpret_cast<const uint32_t *>(aux + o_bid);
    L.bias_values = reinterpret_cast<const float *>(aux + o_bval);
    L.suppress_ids = reinterpret_cast<const uint32_t *>(aux + o_sup);
    L.breakers = reinterpret_cast<const uint32_t *>(aux + o_brk);
    L.hist = reinterpret_cast<const uint32_t *>(aux + o_hist);
    L.hist_off = reinterpret_cast<const uint32_t *>(aux + o_off);
    auto *dst = reinterpret_cast<SampState *>(aux + o_st);
    auto *dtok = reinterpret_cast<uint32_t *>(aux + o_tok);
    auto *dstat = reinterpret_cast<int *>(aux + o_stat);
    CK(sampler_launch(e->st, P, L, rows, V, (int)n_seqs, e->samp_scratch.p, e->samp_scratch.n, dst, dtok, dstat));
    CK(cudaMemcpyAsync(host.data() + o_st, aux + o_st, o_stat + 4ull * n_seqs - o_st, cudaMemcpyDeviceToHost, e->st));
    int r = wait_stream(e);
    if (r) return r;
    const int *stat = reinterpret_cast<const int *>(host.data() + o_stat);
    for (uint32_t i = 0; i < n_seqs; i++)
        if (stat[i] == SAMP_ERR_TYPICAL_TOO_MANY)
            return fail(BT_ERR_UNSUPPORTED,
                        "typical_p over more than 4096 candidates: set top_k, or put top_p or min_p before it");
    memcpy(states, host.data() + o_st, sizeof(SampState) * n_seqs);
    memcpy(tokens_out, host.data() + o_tok, 4ull * n_seqs);
    return BT_OK;
}

extern "C" int bt_last_device_ms(const bt_engine *e, double *ms) {
    if (!e || !ms) return fail(BT_ERR_INVALID, "null argument");
    *ms = e->last_device_ms;
    return BT_OK;
}

extern "C" int bt_profile_decode(bt_engine *e, bt_kv *kv, const uint32_t *seq_ids, const uint32_t *first_tokens,
                                 uint32_t n_seqs, uint32_t n_steps, bt_kernel_time *out, uint32_t max_out,
                                 uint32_t *n_out) {
    StepPlan p;
    int r = greedy_prepare(e, kv, seq_ids, first_tokens, n_seqs, n_steps, p);
    if (r) return r;
    e->timers.clear();
    e->timing = true;
    bool pdl = e->pdl;
    e->pdl = false;  // serialised launches: each event pair brackets one kernel
    for (uint32_t s = 0; s < n_steps && !r; s++) {
        r = launch_step(e, kv, p, true);
        if (!r) r = wait_stream(e);
        timer_collect(e);
    }
    e->timing = false;
    e->pdl = pdl;
    if (r) return r;
    if ((r = greedy_finish(e, kv, seq_ids, n_seqs, n_steps, nullptr, nullptr))) return r;
    if (e->mega && (int)n_seqs <= STEP_MAX_T && n_steps > 0) {
        // one more step with the in-kernel timeline: per phase, the slowest CTA's work and the
        // barrier's release latency, averaged over layers
        const int grid = e->n_sm, L = (int)e->d.n_layer;
        const size_t rows = (size_t)(L + 1) * STEP_PHASES + 1;
        CK(e->trace.alloc(rows * (grid + 1) * 8));
        CK(cudaMemset(e->trace.p, 0, rows * (grid + 1) * 8));
        StepPlan q;
        if ((r = greedy_prepare(e, kv, seq_ids, first_tokens, n_seqs, 1, q))) return r;
        e->tracing = true;
        r = launch_step(e, kv, q, true);
        e->tracing = false;
        if (r) return r;
        CK(cudaStreamSynchronize(e->st));
        if ((r = greedy_finish(e, kv, seq_ids, n_seqs, 1, nullptr, nullptr))) return r;
        std::vector<unsigned long long> tr(rows * (grid + 1));
        CK(cudaMemcpy(tr.data(), e->trace.p, tr.size() * 8, cudaMemcpyDeviceToHost));
        const char *names[8] = {"ph0_qkv", "ph1_attn", "ph2_combine", "ph3_attn_out", "ph4_router",
                                "ph5_gateup", "ph6_down", "ph7_unused"};
        // points inside phases: slowest CTA, measured from the departure of the barrier before
        const char *pnames[8] = {"pt_qkv_staged", "pt_attn_item1", "pt_o_staged", "pt_router_staged",
                                 "pt_gateup_routed", "pt_gateup_units", "pt_down_units", "pt_unused"};
        const int point_after[8] = {-1, 0, 2, 3, -1, 4, 5, -1};  // barrier whose departure starts each point
        // cycle counters inside phases (max over warps, then over CTAs), as microseconds at the
        // SM clock the device reports
        int clk_khz = 0;
        cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, e->device);
        const char *cnames[8] = {"cyc_qkv_wait",    "cyc_qkv_compute",    "cyc_down_wait", "cyc_down_compute",
                                 "cyc_gateup_wait", "cyc_gateup_compute", "cyc_head_wait", "cyc_head_compute"};
        for (int l = 0; l <= L; l++)
            for (int k = 7; k <= 14; k++) {
                if ((l == L) != (k >= 13)) continue;  // the head's counters sit in the row after the layers
                const unsigned long long *row = tr.data() + ((size_t)l * STEP_PHASES + 8 + k) * (grid + 1);
                unsigned long long mx = 0;
                for (int c = 0; c < grid; c++) mx = row[c] > mx ? row[c] : mx;
                KernelTimer &w = e->timers[cnames[k - 7]];
                w.launches++;
                w.ms += clk_khz ? (double)mx / (double)clk_khz : 0.0;
            }
        for (int l = 0; l < L; l++) {
            for (int k = 0; k < 7; k++) {
                const unsigned long long *row = tr.data() + ((size_t)l * STEP_PHASES + 8 + k) * (grid + 1);
                unsigned long long mx = 0;
                for (int c = 0; c < grid; c++) mx = row[c] > mx ? row[c] : mx;
                if (!mx) continue;
                unsigned long long start;
                if (point_after[k] >= 0) {
                    const unsigned long long *b = tr.data() + ((size_t)l * STEP_PHASES + point_after[k]) * (grid + 1);
                    start = b[grid];
                    if (k == 2 && !start) start = tr[((size_t)l * STEP_PHASES + 1) * (grid + 1) + grid];
                } else if (k == 0) {
                    start = l == 0 ? tr[(rows - 1) * (grid + 1)] : tr[((size_t)(l - 1) * STEP_PHASES + 6) * (grid + 1) + grid];
                } else {  // k == 4: from the router barrier
                    start = tr[((size_t)l * STEP_PHASES + 4) * (grid + 1) + grid];
                }
                if (!start || mx < start) continue;
                KernelTimer &w = e->timers[pnames[k]];
                w.launches++;
                w.ms += (double)(mx - start) * 1e-6;
            }
        }
        // points inside a CTA's first attention item, from the departure of the barrier before it
        const char *anames[6] = {"pta_q_staged", "pta_tiles_landed", "pta_scores_max", "pta_softmax", "pta_pv",
                                 "pta_done"};
        for (int l = 0; l < L; l++) {
            const unsigned long long start = tr[((size_t)l * STEP_PHASES + 0) * (grid + 1) + grid];
            for (int k = 0; k < 6; k++) {
                const unsigned long long *row = tr.data() + ((size_t)l * STEP_PHASES + 8 + 16 + k) * (grid + 1);
                unsigned long long mx = 0;
                for (int c = 0; c < grid; c++) mx = row[c] > mx ? row[c] : mx;
                if (!start || mx < start) continue;
                KernelTimer &w = e->timers[anames[k]];
                w.launches++;
                w.ms += (double)(mx - start) * 1e-6;
            }
        }
        unsigned long long prev = tr[(rows - 1) * (grid + 1)];  // kernel start (CTA 0)
        for (int l = 0; l <= L; l++) {
            for (int ph = 0; ph < 8; ph++) {
                const unsigned long long *row = tr.data() + ((size_t)l * STEP_PHASES + ph) * (grid + 1);
                if (!row[grid]) continue;  // this barrier did not run (no combine, or past the head)
                unsigned long long mx = 0;
                for (int c = 0; c < grid; c++) mx = row[c] > mx ? row[c] : mx;
                std::string base = l == L ? std::string("ph_head") : std::string(names[ph]);
                KernelTimer &w = e->timers[base + "_work"];
                w.launches++;
                w.ms += (double)(mx - prev) * 1e-6;
                KernelTimer &b = e->timers[base + "_barrier"];
                b.launches++;
                b.ms += (double)(row[grid] - mx) * 1e-6;
                prev = row[grid];
            }
        }
    }
    uint32_t i = 0;
    for (auto &kt : e->timers) {
        if (i < max_out && out) {
            memset(&out[i], 0, sizeof(bt_kernel_time));
            strncpy(out[i].name, kt.first.c_str(), sizeof(out[i].name) - 1);
            out[i].launches = kt.second.launches;
            out[i].total_ms = kt.second.ms;
        }
        i++;
    }
    if (n_out) *n_out = i;
    return BT_OK;
}

extern "C" int bt_engine_set_router_bias(bt_engine *e, uint32_t layer, const float *bias, uint32_t n) {
    if (!e) return fail(BT_ERR_INVALID, "null engine");
    if (layer >= e->d.n_layer) return fail(BT_ERR_INVALID, "layer out of range");
    Layer &l = e->L[layer];
    if (!bias) {
        l.gate_bias = DevBuf();
    } else {
        if (n != e->d.n_expert) return fail(BT_ERR_INVALID, "the bias has one value per expert");
        CK(cudaSetDevice(e->device));
        CK(cudaStreamSynchronize(e->st));
        CK(l.gate_bias.alloc((size_t)n * 4));
        CK(cudaMemcpy(l.gate_bias.p, bias, (size_t)n * 4, cudaMemcpyHostToDevice));
    }
    for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);  // they hold the old pointers
    e->graphs.clear();
    return upload_layer_dev(e);
}

// ------------------------------------------------------------------ expert cache
extern "C" int bt_engine_enable_expert_cache(bt_engine *e, uint64_t cache_bytes, int policy) {
    if (!e) return fail(BT_ERR_INVALID, "null engine");
    if (e->ep) return fail(BT_ERR_UNSUPPORTED, "the expert cache and expert parallelism do not combine");
    if (policy != BT_XCACHE_LRU && policy != BT_XCACHE_FREQ) return fail(BT_ERR_INVALID, "unknown cache policy");
    const bt_model_desc &d = e->d;
    const int NE = (int)d.n_expert, K = (int)d.n_expert_used, L = (int)d.n_layer;
    if (e->xcache) {  // already host-resident: a new, empty cache of the given size and policy
        const long long cap = (long long)(cache_bytes / (uint64_t)e->x_stride);
        if (cap < 2 * K) return fail(BT_ERR_INVALID, "the cache must hold at least two steps' worth of experts (2 * top-k)");
        const int capacity = (int)(cap < (long long)L * NE ? cap : (long long)L * NE);
        CK(cudaStreamSynchronize(e->st));
        if (capacity != e->xpol.capacity()) CK(e->x_pool.alloc((size_t)(capacity + e->x_bounce) * e->x_stride));
        CK(cudaMemset(e->x_slot_dev.p, 0xff, (size_t)L * NE * 4));
        memset(e->x_slot_host, 0xff, (size_t)L * NE * 4);
        e->xpol = ExpertCachePolicy(policy, capacity, L, NE);
        e->xstats = XCacheStats();
        return xdev_init(e->xd_buf, e->xd, policy, capacity, L, NE, e->st);
    }
    long long stride = 0;
    for (int il = 0; il < L; il++) {
        const Layer &l = e->L[il];
        const long long b = (long long)(l.gate.mat_bytes + l.up.mat_bytes + l.down.mat_bytes);
        if (b > stride) stride = b;
    }
    stride = (stride + 127) & ~127ll;
    const long long cap = (long long)(cache_bytes / (uint64_t)stride);
    if (cap < 2 * K) return fail(BT_ERR_INVALID, "the cache must hold at least two steps' worth of experts (2 * top-k)");
    const int capacity = (int)(cap < (long long)L * NE ? cap : (long long)L * NE);
    const int bounce = NE < e->TB * K ? NE : e->TB * K;
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->st));
    // the experts to pinned host memory, one contiguous gate | up | down block per expert
    std::vector<uint8_t *> host(L, nullptr);
    auto undo = [&]() {
        for (uint8_t *h : host)
            if (h) cudaFreeHost(h);
    };
    for (int il = 0; il < L; il++) {
        const Layer &l = e->L[il];
        cudaError_t ce = cudaHostAlloc((void **)&host[il], (size_t)NE * stride, cudaHostAllocDefault);
        if (ce != cudaSuccess) {
            undo();
            return fail(BT_ERR_OOM, std::string("pinned host memory for the experts: ") + cudaGetErrorString(ce));
        }
        const QMat *mats[3] = {&l.gate, &l.up, &l.down};
        size_t off = 0;
        for (const QMat *m : mats) {
            ce = cudaMemcpy2D(host[il] + off, (size_t)stride, m->buf.p, (size_t)m->mat_bytes, (size_t)m->mat_bytes,
                              (size_t)NE, cudaMemcpyDeviceToHost);
            if (ce != cudaSuccess) {
                undo();
                return fail(BT_ERR_CUDA, std::string("expert copy to the host: ") + cudaGetErrorString(ce));
            }
            off += (size_t)m->mat_bytes;
        }
    }
    for (int il = 0; il < L; il++) {  // the device copies go: the pool replaces them
        Layer &l = e->L[il];
        l.gate.buf = DevBuf();
        l.up.buf = DevBuf();
        l.down.buf = DevBuf();
    }
    e->x_host = host;
    CK(e->x_pool.alloc((size_t)(capacity + bounce) * stride));
    CK(e->x_slot_dev.alloc((size_t)L * NE * 4));
    CK(cudaMemset(e->x_slot_dev.p, 0xff, (size_t)L * NE * 4));
    CK(cudaHostAlloc((void **)&e->x_sel_host, (size_t)e->TB * K * 4, cudaHostAllocDefault));
    CK(cudaHostAlloc((void **)&e->x_slot_host, (size_t)L * NE * 4, cudaHostAllocDefault));
    memset(e->x_slot_host, 0xff, (size_t)L * NE * 4);
    CK(cudaEventCreateWithFlags(&e->x_ev, cudaEventDisableTiming));
    e->xpol = ExpertCachePolicy(policy, capacity, L, NE);
    e->xstats = XCacheStats();
    e->x_stride = stride;
    e->x_bounce = bounce;
    e->x_host_dev.assign(L, nullptr);
    for (int il = 0; il < L; il++) {
        void *dp = nullptr;
        CK(cudaHostGetDevicePointer(&dp, host[il], 0));
        e->x_host_dev[il] = reinterpret_cast<const uint8_t *>(dp);
    }
    CK(e->x_host_devarr.alloc((size_t)L * sizeof(void *)));
    CK(cudaMemcpy(e->x_host_devarr.p, e->x_host_dev.data(), (size_t)L * sizeof(void *), cudaMemcpyHostToDevice));
    CK(e->x_copies.alloc((size_t)(e->TB * K + bounce) * sizeof(XcCopy)));
    CK(e->x_ncopies.alloc(16));
    CK(cudaMemset(e->x_ncopies.p, 0, 16));
    if (NE > XC_MAX_NE || e->TB * K > XC_MAX_SEL) e->xdev = false;  // beyond the device lookup's tables
    if (int xr = xdev_init(e->xd_buf, e->xd, policy, capacity, L, NE, e->st)) return xr;
    e->xcache = true;  // (the persistent step runs with it when the policy is on the device)
    for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
    e->graphs.clear();
    return BT_OK;
}

static void xcache_fill(const XCacheStats &s, int capacity, long long stride, bt_xcache_stats *out) {
    out->hits = s.hits;
    out->misses = s.misses;
    out->evictions = s.evictions;
    out->admissions = s.admissions;
    out->bypasses = s.bypasses;
    out->bytes_copied = s.bytes_copied;
    out->capacity_slots = (uint64_t)capacity;
    out->slot_bytes = (uint64_t)stride;
}

static int xdev_stats(const XcDev &x, XCacheStats &s) {
    unsigned long long v[XC_N];
    CK(cudaMemcpy(v, x.st, sizeof(v), cudaMemcpyDeviceToHost));
    s.hits = v[XC_HITS];
    s.misses = v[XC_MISSES];
    s.evictions = v[XC_EVICTIONS];
    s.admissions = v[XC_ADMISSIONS];
    s.bypasses = v[XC_BYPASSES];
    s.bytes_copied = v[XC_BYTES];
    return BT_OK;
}

extern "C" int bt_expert_cache_stats(const bt_engine *e, bt_xcache_stats *out) {
    if (!e || !out) return fail(BT_ERR_INVALID, "null argument");
    if (!e->xcache) return fail(BT_ERR_INVALID, "the expert cache is not enabled");
    XCacheStats s = e->xstats;
    if (e->xdev) {
        CK(cudaSetDevice(e->device));
        CK(cudaStreamSynchronize(e->st));
        if (int r = xdev_stats(e->xd, s)) return r;
    }
    xcache_fill(s, e->xpol.capacity(), e->x_stride, out);
    return BT_OK;
}

extern "C" int bt_expert_cache_simulate_device(int policy, uint32_t capacity, uint32_t n_layer, uint32_t n_expert,
                                               uint32_t n_sel, const int32_t *trace, uint32_t n_steps,
                                               bt_xcache_stats *out) {
    if (!trace || !out || !capacity || !n_layer || !n_expert || !n_sel)
        return fail(BT_ERR_INVALID, "bad argument");
    if (policy != BT_XCACHE_LRU && policy != BT_XCACHE_FREQ) return fail(BT_ERR_INVALID, "unknown cache policy");
    if (n_expert > (uint32_t)XC_MAX_NE || n_sel > (uint32_t)XC_MAX_SEL)
        return fail(BT_ERR_UNSUPPORTED, "more experts or selections than the device lookup takes");
    const size_t nt = (size_t)n_steps * n_layer * n_sel;
    for (size_t i = 0; i < nt; i++)
        if (trace[i] < 0 || (uint32_t)trace[i] >= n_expert) return fail(BT_ERR_INVALID, "expert id out of range");
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() { cudaStreamDestroy(s); }
    } guard{st};
    DevBuf buf, dtrace, rows, copies, nc, err;
    XcDev x;
    if (int r = xdev_init(buf, x, policy, (int)capacity, (int)n_layer, (int)n_expert, st)) return r;
    CK(dtrace.alloc(nt * 4 + 4));
    CK(rows.alloc((size_t)n_layer * n_expert * 4));
    CK(copies.alloc((size_t)n_sel * sizeof(XcCopy)));
    CK(nc.alloc(16));
    CK(err.alloc(16));
    CK(cudaMemsetAsync(err.p, 0, 16, st));
    CK(cudaMemcpyAsync(dtrace.p, trace, nt * 4, cudaMemcpyHostToDevice, st));
    for (uint32_t s = 0; s < n_steps; s++)
        for (uint32_t il = 0; il < n_layer; il++)
            CK(launch_xcache_lookup(x, (int)il, dtrace.as<int>() + ((size_t)s * n_layer + il) * n_sel, (int)n_sel,
                                    rows.as<int>() + (size_t)il * n_expert, nullptr, nullptr, 0, 0, (int)n_sel,
                                    copies.as<XcCopy>(), nc.as<int>(), err.as<int>(), st));
    CK(cudaStreamSynchronize(st));
    int herr = 0;
    CK(cudaMemcpy(&herr, err.p, 4, cudaMemcpyDeviceToHost));
    if (herr) return fail(BT_ERR_INVALID, "the device lookup rejected the trace");
    XCacheStats sres;
    if (int r = xdev_stats(x, sres)) return r;
    xcache_fill(sres, (int)capacity, 0, out);
    return BT_OK;
}

extern "C" int bt_expert_cache_simulate(int policy, uint32_t capacity, uint32_t n_layer, uint32_t n_expert,
                                        uint32_t n_sel, const int32_t *trace, uint32_t n_steps, bt_xcache_stats *out) {
    if (!trace || !out || !capacity || !n_layer || !n_expert || !n_sel)
        return fail(BT_ERR_INVALID, "bad argument");
    if (policy != BT_XCACHE_LRU && policy != BT_XCACHE_FREQ) return fail(BT_ERR_INVALID, "unknown cache policy");
    ExpertCachePolicy pol(policy, (int)capacity, (int)n_layer, (int)n_expert);
    XCacheStats st;
    std::vector<int> distinct, slot;
    std::vector<char> seen;
    std::unique_ptr<bool[]> copy(new bool[n_sel]);
    for (uint32_t s = 0; s < n_steps; s++)
        for (uint32_t il = 0; il < n_layer; il++) {
            const int32_t *sel = trace + ((size_t)s * n_layer + il) * n_sel;
            distinct.clear();
            seen.assign(n_expert, 0);
            for (uint32_t i = 0; i < n_sel; i++) {
                if (sel[i] < 0 || (uint32_t)sel[i] >= n_expert) return fail(BT_ERR_INVALID, "expert id out of range");
                if (!seen[sel[i]]) {
                    seen[sel[i]] = 1;
                    distinct.push_back(sel[i]);
                }
            }
            slot.resize(distinct.size());
            pol.lookup((int)il, distinct.data(), (int)distinct.size(), slot.data(), copy.get(), st);
        }
    xcache_fill(st, (int)capacity, 0, out);
    return BT_OK;
}

// ------------------------------------------------------------------ expert parallelism
extern "C" int bt_ep_unique_id(void *out, size_t nbytes) {
    if (!out || nbytes < sizeof(ncclUniqueId)) return fail(BT_ERR_INVALID, "the unique id needs 128 bytes");
    const NcclApi *api = nccl_api();
    if (!api) return fail(BT_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    NK(api->GetUniqueId(&id));
    memcpy(out, &id, sizeof(id));
    return BT_OK;
}

extern "C" int bt_engine_enable_ep(bt_engine *e, const void *unique_id, size_t nbytes, int rank, int n_ranks) {
    if (!e || !unique_id || nbytes < sizeof(ncclUniqueId)) return fail(BT_ERR_INVALID, "bad argument");
    if (n_ranks < 1 || rank < 0 || rank >= n_ranks) return fail(BT_ERR_INVALID, "rank out of range");
    if (e->ep) return fail(BT_ERR_INVALID, "expert parallelism is already enabled");
    if (e->xcache) return fail(BT_ERR_UNSUPPORTED, "the expert cache and expert parallelism do not combine");
    const bt_model_desc &d = e->d;
    if (d.n_expert % (uint32_t)n_ranks) return fail(BT_ERR_UNSUPPORTED, "the expert count must divide by the rank count");
    const NcclApi *api = nccl_api();
    if (!api) return fail(BT_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    CK(cudaSetDevice(e->device));
    const size_t S = (size_t)(EP_STEP_TOKENS < e->TB ? EP_STEP_TOKENS : e->TB) * d.n_expert_used, E = d.n_embd,
                 F = d.n_ff_exp, n = (size_t)n_ranks;
    CK(e->ep_send_meta.alloc(n * S * 4));
    CK(e->ep_recv_meta.alloc(n * S * 4));
    CK(e->ep_send_rows.alloc(n * S * E * 4));
    CK(e->ep_recv_rows.alloc(n * S * E * 4));
    CK(e->ep_send_qs.alloc(n * S * E));
    CK(e->ep_recv_qs.alloc(n * S * E));
    CK(e->ep_send_d.alloc(n * S * (E / 256) * 4));
    CK(e->ep_recv_d.alloc(n * S * (E / 256) * 4));
    CK(e->ep_send_bs.alloc(n * S * (E / 256) * 8 * 4));
    CK(e->ep_recv_bs.alloc(n * S * (E / 256) * 8 * 4));
    CK(alloc_q8(e, (size_t)n * S));
    CK(e->ep_act.alloc(n * S * F * 4));
    CK(e->ep_dpart.alloc(n * S * E * 4));
    CK(e->ep_ret.alloc(n * S * E * 4));
    CK(cudaMemsetAsync(e->ep_dpart.p, 0, n * S * E * 4, e->st));
    CK(cudaMemsetAsync(e->ep_send_meta.p, 0xff, n * S * 4, e->st));
    CK(e->g_list.alloc(n * S * 4));  // the grouped lists now cover every rank's slots
    CK(e->g_chunk_e.alloc((size_t)group_max_chunks((int)(n * S), (int)d.n_expert) * 4));
    CK(e->g_chunk_r0.alloc((size_t)group_max_chunks((int)(n * S), (int)d.n_expert) * 4));
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    ncclComm_t comm = nullptr;
    NK(api->CommInitRank(&comm, n_ranks, id, rank));
    e->ep_comm = comm;
    e->ep = true;
    e->ep_rank = rank;
    e->ep_n = n_ranks;
    // one exchange of the slot metadata now: NCCL connects the peers on first use, which
    // then happens outside any graph capture
    NK(api->GroupStart());
    for (int r = 0; r < n_ranks; r++) {
        NK(api->Send(e->ep_send_meta.as<int>() + (size_t)r * S, S, ncclInt32, r, comm, e->st));
        NK(api->Recv(e->ep_recv_meta.as<int>() + (size_t)r * S, S, ncclInt32, r, comm, e->st));
    }
    NK(api->GroupEnd());
    int wr = wait_stream(e);
    if (wr) return wr;
    // keep only this rank's experts in HBM (stream.rs:1422-1429 slices an expert tensor the same
    // way: expert e is bytes [e, e + 1) * size / n_expert): one layer at a time, so the extra
    // memory is one layer's share
    const int per = (int)(d.n_expert / (uint32_t)n_ranks), e0 = rank * per;
    for (uint32_t il = 0; il < d.n_layer; il++) {
        for (QMat *m : {&e->L[il].gate, &e->L[il].up, &e->L[il].down}) {
            DevBuf nb;
            CK(nb.alloc((size_t)per * m->mat_bytes));
            CK(cudaMemcpyAsync(nb.p, m->buf.as<uint8_t>() + (size_t)e0 * m->mat_bytes, (size_t)per * m->mat_bytes,
                               cudaMemcpyDeviceToDevice, e->st));
            CK(cudaStreamSynchronize(e->st));
            e->weight_bytes -= (uint64_t)(m->n_mats - per) * m->mat_bytes;
            std::swap(m->buf, nb);
            m->n_mats = per;
        }
    }
    e->ep_e0 = e0;
    e->ep_ne = per;
    e->stats.weight_bytes = e->weight_bytes;
    e->mega = false;  // the expert phase crosses ranks: per-phase kernels
    for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
    e->graphs.clear();
    return BT_OK;
}

extern "C" int bt_set_option(bt_engine *e, const char *name, int value) {
    if (!e || !name) return fail(BT_ERR_INVALID, "null argument");
    if (!strcmp(name, "prefetch")) {
        e->prefetch = value != 0;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "persistent")) {
        e->mega = value != 0;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "mma")) {
        e->mma = value != 0;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "attn_warp")) {
        e->attn_warp = value != 0;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "mma_grid")) {
        if (value < 0) return fail(BT_ERR_INVALID, "mma_grid must be >= 0");
        e->mma_grid = value;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "token_groups")) {
        e->token_groups = value ? 1 : 0;
        return BT_OK;
    }
    if (!strcmp(name, "mma_min_units")) {
        if (value < 1) return fail(BT_ERR_INVALID, "mma_min_units must be positive");
        e->mma_min_units = value;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "ep_timeout_ms")) {
        if (value < 1) return fail(BT_ERR_INVALID, "ep_timeout_ms must be positive");
        e->ep_timeout_ms = value;
        return BT_OK;
    }
    if (!strcmp(name, "wait_limit_us") || !strcmp(name, "fault_cta") || !strcmp(name, "fault_barrier") ||
        !strcmp(name, "fault_copy")) {
        if (value < 0) return fail(BT_ERR_INVALID, std::string(name) + " must be >= 0");
        (!strcmp(name, "wait_limit_us")   ? e->wait_limit_us
         : !strcmp(name, "fault_cta")     ? e->fault_cta
         : !strcmp(name, "fault_barrier") ? e->fault_barrier
                                          : e->fault_copy) = value;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);  // the values are baked into captured launches
        e->graphs.clear();
        return BT_OK;
    }
    if (!strcmp(name, "xcache_device")) {
        e->xdev = value != 0;
        if (!e->xcache) return BT_OK;
        if (e->d.n_expert > (uint32_t)XC_MAX_NE || e->TB * (int)e->d.n_expert_used > XC_MAX_SEL) e->xdev = false;
        // the two policies keep separate state: switching starts a new, empty cache
        return bt_engine_enable_expert_cache(e, (uint64_t)e->xpol.capacity() * (uint64_t)e->x_stride, e->xd.policy);
    }
    if (!strcmp(name, "stream_warps")) {
        if (value != 4 && value != 8) return fail(BT_ERR_INVALID, "stream_warps must be 4 or 8");
        e->stream_warps = value;
        return BT_OK;
    }
    if (!strcmp(name, "stream_slots")) {
        if (value < 0) return fail(BT_ERR_INVALID, "stream_slots must be >= 0");
        e->stream_slots = value;
        return BT_OK;
    }
    if (!strcmp(name, "pdl")) {
        e->pdl = value != 0;
        for (auto &g : e->graphs) cudaGraphExecDestroy(g.second);
        e->graphs.clear();
        return BT_OK;
    }
    return fail(BT_ERR_INVALID, std::string("unknown option ") + name);
}

// ------------------------------------------------------------------ parity hooks
extern "C" int bt_debug_topk(const bt_engine *e, uint32_t layer, uint32_t token, int32_t *ids, float *weights) {
    if (!e || !ids || !weights) return fail(BT_ERR_INVALID, "null argument");
    if (layer >= e->d.n_layer) return fail(BT_ERR_INVALID, "layer out of range");
    if (token < e->last_first || token >= e->last_first + e->last_T)
        return fail(BT_ERR_INVALID, "token is not in the last step of the last forward");
    const int K = e->d.n_expert_used;
    size_t off = ((size_t)layer * e->TB + (token - e->last_first)) * K;
    CK(cudaMemcpy(ids, e->dbg_ids.as<int>() + off, K * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(weights, e->dbg_w.as<float>() + off, K * 4, cudaMemcpyDeviceToHost));
    return BT_OK;
}

extern "C" int bt_debug_hidden(const bt_engine *e, uint32_t token, float *out) {
    if (!e || !out) return fail(BT_ERR_INVALID, "null argument");
    if (token < e->last_first || token >= e->last_first + e->last_T)
        return fail(BT_ERR_INVALID, "token is not in the last step of the last forward");
    CK(cudaMemcpy(out, e->x.as<float>() + (size_t)(token - e->last_first) * e->d.n_embd, e->d.n_embd * 4, cudaMemcpyDeviceToHost));
    return BT_OK;
}

extern "C" int bt_debug_dequant(uint32_t type, const void *bytes, uint64_t n, float *out) {
    if (!bytes || !out) return fail(BT_ERR_INVALID, "null argument");
    if (type != T_Q4_K && type != T_Q6_K) return fail(BT_ERR_UNSUPPORTED, "dequant hook covers Q4_K and Q6_K");
    if (n % 256) return fail(BT_ERR_INVALID, "a partial K-quant block");  // lib.rs:258-264
    if (n == 0) return BT_OK;
    long long rows = (long long)(n / 256);
    TileGeom g = tile_geom((int)type, rows, 256, 32);
    DevBuf raw, tiled, y;
    size_t rb = (size_t)rows * qk_block_bytes((int)type);
    CK(raw.alloc(rb));
    CK(tiled.alloc((size_t)g.n_tiles * g.tile_bytes));
    CK(y.alloc(n * 4));
    CK(cudaMemcpy(raw.p, bytes, rb, cudaMemcpyHostToDevice));
    CK(launch_repack((int)type, raw.as<uint8_t>(), rows, 256, 32, tiled.as<uint8_t>(), 1, 0));
    CK(launch_dequant_tiled((int)type, tiled.as<uint8_t>(), rows, 256, 32, y.as<float>(), 0));
    CK(cudaMemcpy(out, y.p, n * 4, cudaMemcpyDeviceToHost));
    return BT_OK;
}

extern "C" int bt_op_i8_mma(const uint8_t *a, const int8_t *b, uint32_t n, uint32_t k, int32_t *d) {
    if (!a || !b || !d) return fail(BT_ERR_INVALID, "null argument");
    if ((n != 8 && n != 16 && n != 32) || !k || k % 32 || k > 512) return fail(BT_ERR_INVALID, "n in {8, 16, 32}, k = 32..512");
    DevBuf ad, bd, dd, err;
    CK(ad.alloc((size_t)128 * k));
    CK(bd.alloc((size_t)n * k));
    CK(dd.alloc((size_t)128 * n * 4));
    CK(err.alloc(4));
    CK(cudaMemset(err.p, 0, 4));
    CK(cudaMemset(dd.p, 0, (size_t)128 * n * 4));
    CK(cudaMemcpy(ad.p, a, (size_t)128 * k, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(bd.p, b, (size_t)n * k, cudaMemcpyHostToDevice));
    CK(launch_i8_mma_probe(ad.as<uint8_t>(), bd.as<int8_t>(), dd.as<int32_t>(), (int)n, (int)k, err.as<int>(), 0));
    CK(cudaDeviceSynchronize());
    int h = 0;
    CK(cudaMemcpy(&h, err.p, 4, cudaMemcpyDeviceToHost));
    if (h) return fail(BT_ERR_TIMEOUT, "the MMA's completion wait ran out");
    CK(cudaMemcpy(d, dd.p, (size_t)128 * n * 4, cudaMemcpyDeviceToHost));
    return BT_OK;
}

extern "C" int bt_op_gemv(uint32_t type, const void *w_bytes, uint32_t rows, uint32_t cols, const float *x, uint32_t T,
                          float *y) {
    if (!w_bytes || !x || !y || !rows || !cols || !T) return fail(BT_ERR_INVALID, "bad argument");
    bt_engine tmp;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, dev));
    tmp.n_sm = prop.multiProcessorCount;
    tmp.device = dev;
    CK(init_kernel_attributes());
    CK(cudaStreamCreateWithFlags(&tmp.st, cudaStreamNonBlocking));
    tmp.pdl = false;
    QMat m;
    DevBuf staging, xd, yd;
    int r = ingest_qmat(&tmp, m, (int)type, rows, cols, 1, w_bytes, false, default_rpt(cols), false, staging);
    if (r) {
        cudaStreamDestroy(tmp.st);
        tmp.st = nullptr;
        return r;
    }
    CK(tmp.err.alloc(4));
    CK(cudaMemset(tmp.err.p, 0, 4));
    CK(xd.alloc((size_t)T * cols * 4));
    CK(yd.alloc((size_t)T * rows * 4));
    CK(cudaMemcpy(xd.p, x, (size_t)T * cols * 4, cudaMemcpyHostToDevice));
    for (uint32_t t0 = 0; t0 < T; t0 += MAX_T) {
        int tg = T - t0 < (uint32_t)MAX_T ? (int)(T - t0) : MAX_T;
        const QMat *mats[1] = {&m};
        int offs[1] = {0};
        CK(run_gemv(&tmp, mats, offs, 1, xd.as<float>() + (size_t)t0 * cols, cols, nullptr, nullptr, cols, tg,
                    yd.as<float>() + (size_t)t0 * rows, rows, nullptr, 0, "gemv"));
    }
    CK(cudaStreamSynchronize(tmp.st));
    r = check_err(&tmp);
    CK(cudaMemcpy(y, yd.p, (size_t)T * rows * 4, cudaMemcpyDeviceToHost));
    cudaStreamDestroy(tmp.st);
    tmp.st = nullptr;
    return r;
}

extern "C" int bt_engine_tensor_bytes(const bt_engine *ec, const char *name, void *host_out, uint64_t nbytes) {
    bt_engine *e = const_cast<bt_engine *>(ec);
    if (!e || !name || !host_out) return fail(BT_ERR_INVALID, "null argument");
    CK(cudaSetDevice(e->device));
    std::string n(name);
    const QMat *m = nullptr;
    const DevBuf *f = nullptr;
    if (n == "token_embd.weight") m = &e->embd;
    else if (n == "output.weight") m = &e->out;
    else if (n == "output_norm.weight") f = &e->out_norm;
    else if (n.rfind("blk.", 0) == 0) {
        size_t dot = n.find('.', 4);
        uint32_t il = (uint32_t)atoi(n.substr(4, dot - 4).c_str());
        if (il >= e->d.n_layer) return fail(BT_ERR_MISSING_TENSOR, "no tensor " + n);
        Layer &l = e->L[il];
        std::string s = n.substr(dot + 1);
        if (s == "attn_q.weight") m = &l.q;
        else if (s == "attn_k.weight") m = &l.k;
        else if (s == "attn_v.weight") m = &l.v;
        else if (s == "attn_output.weight") m = &l.o;
        else if (s == "ffn_gate_exps.weight" || s == "ffn_up_exps.weight" || s == "ffn_down_exps.weight") {
            if (e->ep_ne) return fail(BT_ERR_INVALID, "the engine holds only its own experts' share of " + n);
            m = s == "ffn_gate_exps.weight" ? &l.gate : s == "ffn_up_exps.weight" ? &l.up : &l.down;
        }
        else if (s == "ffn_gate_shexp.weight" && e->d.n_ff_shexp) m = &l.gate_sh;
        else if (s == "ffn_up_shexp.weight" && e->d.n_ff_shexp) m = &l.up_sh;
        else if (s == "ffn_down_shexp.weight" && e->d.n_ff_shexp) m = &l.down_sh;
        else if (s == "attn_norm.weight") f = &l.attn_norm;
        else if (s == "attn_q_norm.weight") f = &l.q_norm;
        else if (s == "attn_k_norm.weight") f = &l.k_norm;
        else if (s == "ffn_norm.weight") f = &l.ffn_norm;
        else if (s == "ffn_gate_inp.weight") f = &l.gate_inp;
        else if (s == "ffn_gate_inp.bias" && l.gate_bias.p) f = &l.gate_bias;
    }
    if (f) {
        if (nbytes != f->n) return fail(BT_ERR_INVALID, "size mismatch for " + n);
        CK(cudaMemcpy(host_out, f->p, nbytes, cudaMemcpyDeviceToHost));
        return BT_OK;
    }
    if (!m) return fail(BT_ERR_MISSING_TENSOR, "no tensor " + n);
    if (!m->buf.p) return fail(BT_ERR_UNSUPPORTED, n + " lives in the host expert cache");
    size_t raw = (size_t)m->n_mats * m->rows * (m->cols / 256) * qk_block_bytes(m->type);
    if (nbytes != raw) return fail(BT_ERR_INVALID, "size mismatch for " + n);
    DevBuf tmp;
    CK(tmp.alloc(raw));
    CK(launch_untile(m->type, m->buf.as<uint8_t>(), m->rows, m->cols, m->g.rpt, tmp.as<uint8_t>(), m->n_mats, e->st));
    CK(cudaMemcpyAsync(host_out, tmp.p, raw, cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    return BT_OK;
}

// ------------------------------------------------------------------ synthetic weights on the host
extern "C" int bt_synth_tensor(uint32_t type, uint64_t rows, uint64_t cols, uint64_t seed, uint64_t tensor_id,
                               float mean, float sigma, void *out) {
    if (!out) return fail(BT_ERR_INVALID, "null output");
    const uint64_t n = rows * cols;
    const int t = (int)type;
    if (t != T_F32 && t != T_F16 && t != T_Q4_K && t != T_Q6_K) return fail(BT_ERR_UNSUPPORTED, "unsupported type");
    if ((t == T_Q4_K || t == T_Q6_K) && (cols % 256)) return fail(BT_ERR_INVALID, "K-quant rows must be whole blocks");
    const uint64_t key = synth_key(seed, tensor_id);
    const float scale = synth_scale(sigma);
    const int eb = t == T_F32 ? 4 : (t == T_F16 ? 2 : 0);
    const int bb = synth_block_bytes(t);
    const long long nblk = (long long)((n + 255) / 256);
    uint8_t *o = reinterpret_cast<uint8_t *>(out);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nblk; i++) {
        uint8_t blk[1024];
        synth_block(t, key, (uint64_t)i * 256u, mean, scale, blk);
        long long left = (long long)n - i * 256;
        int nb = (eb && left < 256) ? (int)left * eb : bb;
        memcpy(o + (eb ? i * 256 * eb : i * bb), blk, (size_t)nb);
    }
    return BT_OK;
}

extern "C" uint64_t bt_tensor_id(const char *name) { return name ? name_id(name) : 0; }

// ------------------------------------------------------------------ allocation-free GEMV
// bt_op_gemv on caller-owned device buffers, with no allocation of any kind: the tiled copy of
// the weights and the error word live in a file-scope device array reserved when the module
// loads. Layout of the array: [0, 256) the error word (zeroed by every call on its stream),
// [256, BT_NOALLOC_SCRATCH_BYTES) the tiled matrix. One array per device, so calls on one
// device must not overlap.
static __device__ __align__(256) uint8_t g_noalloc_scratch[BT_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int NOALLOC_MAX_DEVICES = 64;
struct NoallocDevice {
    uint8_t *scratch = nullptr;
    int n_sm = 0;
    bool ready = false;
};
NoallocDevice g_noalloc[NOALLOC_MAX_DEVICES];
std::mutex g_noalloc_mu;
}  // namespace

extern "C" int bt_op_gemv_noalloc(uint32_t type, const void *w_dev, uint32_t rows, uint32_t cols, const float *x_dev,
                                  uint32_t T, float *y_dev, void *stream) {
    if (!w_dev || !x_dev || !y_dev || !rows || !cols || !T) return fail(BT_ERR_INVALID, "bad argument");
    if (type != T_Q4_K && type != T_Q6_K)
        return fail(BT_ERR_UNSUPPORTED, "bt_op_gemv_noalloc: the matrix must be Q4_K or Q6_K");
    if (cols % 256 || cols / 256 > 32)
        return fail(BT_ERR_UNSUPPORTED, "bt_op_gemv_noalloc: row length must be a multiple of 256 up to 8192");
    const int rpt = default_rpt(cols);
    const TileGeom g = tile_geom((int)type, rows, cols, rpt);
    const unsigned long long need = 256ull + (unsigned long long)g.n_tiles * (unsigned long long)g.tile_bytes;
    if (need > BT_NOALLOC_SCRATCH_BYTES)
        return fail(BT_ERR_INVALID, "bt_op_gemv_noalloc: the tiled matrix needs " + std::to_string(need) +
                                        " bytes of scratch; the static scratch holds " +
                                        std::to_string(BT_NOALLOC_SCRATCH_BYTES) + " (BT_NOALLOC_SCRATCH_BYTES)");
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(BT_ERR_INVALID, "bt_op_gemv_noalloc: device ordinal too large");
    NoallocDevice *nd = &g_noalloc[dev];
    {
        // one-time set-up on this device (the device is current): the scratch's address and the
        // kernels' shared-memory limits
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!nd->ready) {
            void *p = nullptr;
            CK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            CK(init_kernel_attributes());
            CK(cudaDeviceGetAttribute(&nd->n_sm, cudaDevAttrMultiProcessorCount, dev));
            nd->scratch = reinterpret_cast<uint8_t *>(p);
            nd->ready = true;
        }
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int *err = reinterpret_cast<int *>(nd->scratch);
    uint8_t *tiled = nd->scratch + 256;
    CK(cudaMemsetAsync(err, 0, sizeof(int), st));
    CK(launch_repack((int)type, reinterpret_cast<const uint8_t *>(w_dev), rows, cols, rpt, tiled, 1, st));
    GemvArgs a{};
    a.seg[0].w = tiled;
    a.seg[0].type = (int)type;
    a.seg[0].nsb = g.nsb;
    a.seg[0].rpt = g.rpt;
    a.seg[0].S = g.S;
    a.seg[0].tile_bytes = g.tile_bytes;
    a.seg[0].rows = (int)rows;
    a.seg[0].n_tiles = (int)g.n_tiles;
    a.seg[0].tile0 = 0;
    a.seg[0].out_off = 0;
    a.nseg = 1;
    a.total_tiles = (int)g.n_tiles;
    a.x_stride = cols;
    a.K = (int)cols;
    a.y_stride = rows;
    a.err = err;
    a.slot_bytes = g.tile_bytes;
    const int grid = g.n_tiles < nd->n_sm ? (int)g.n_tiles : nd->n_sm;
    for (uint32_t t0 = 0; t0 < T; t0 += MAX_T) {
        a.T = T - t0 < (uint32_t)MAX_T ? (int)(T - t0) : MAX_T;
        a.x = x_dev + (size_t)t0 * cols;
        a.y = y_dev + (size_t)t0 * rows;
        a.nst = 1;
        const size_t fixed = gemv_smem_bytes(a) - (size_t)GEMV_WARPS * a.slot_bytes;
        a.nst = pick_nst((size_t)a.slot_bytes, fixed);
        CK(launch_gemv(a, grid, st, false));
    }
    int h_err = 0;
    CK(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (h_err & ERR_WAIT_TIMEOUT) return fail(BT_ERR_TIMEOUT, "bt_op_gemv_noalloc: a bounded device wait ran out");
    if (h_err) return fail(BT_ERR_INVALID, "bt_op_gemv_noalloc: device error word " + std::to_string(h_err));
    return BT_OK;
}
