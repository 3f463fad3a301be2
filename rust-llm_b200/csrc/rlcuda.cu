// The C ABI (include/rlcuda.h): the device context that owns the caches,
// the scratch and the stream, argument checking with the reference's
// contract, and dispatch to the kernels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "rlcuda.h"
#include "tmap.h"

#define RL_VERSION_STRING "rlcuda 0.1 (sm_100a)"

struct rl_ctx {
    rl_config cfg{};
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    // caches (forward.rs:236-254)
    void *kv = nullptr;       // [n_full][2][n_kv][context][hd], f32 or bf16
    float *conv = nullptr;    // [n_linear][slots][conv_dim][kernel-1]
    float *ssm = nullptr;     // [n_linear][n_v][slots][s][s]
    // weights
    float *q_norm = nullptr, *k_norm = nullptr;              // [n_full][hd]
    float *conv1d = nullptr, *ssm_a = nullptr, *dt_bias = nullptr, *ssm_norm = nullptr;
    // scratch
    float *q_f32 = nullptr;
    __nv_bfloat16 *q_bf16 = nullptr;
    __nv_bfloat16 *gate_bf16 = nullptr;  // prefill: sigmoid(gate) staging
    float *part_o = nullptr, *part_ml = nullptr;
    int64_t part_rows = 0;    // (row, cluster) pairs the partial buffers hold
    int *counters = nullptr;  // [max_batch][n_kv][8] decode arrival counters
    float *rope_cs = nullptr, *rope_sn = nullptr;  // [context][n_rot/2]
    // bf16 caches: TMA map of the whole KV allocation as rows of head_dim
    CUtensorMap kv_map{};
    // bf16 caches: TMA map of the staged bf16 queries [max_batch][n_head][hd]
    CUtensorMap q_map{};
    CUtensorMap gate_map{};
    CUtensorMap ssm_map{};  // every layer's DeltaNet state, rows of d_state f32
    bool ssm_map_ok = false;
    // the chunk scan's operand maps (the tcgen05 scan runs when set)
    rl::DnScanMaps dn_scan_maps{};
    bool dn_scan_maps_ok = false;
    // chunked DeltaNet prefill scratch (slots == 1 and max_batch >= 64)
    __nv_bfloat16 *dn_qn = nullptr, *dn_kn = nullptr, *dn_vn = nullptr;
    __nv_bfloat16 *dn_qn_lo = nullptr, *dn_kn_lo = nullptr, *dn_vn_lo = nullptr;
    __nv_bfloat16 *dn_qn_l2 = nullptr, *dn_kn_l2 = nullptr;
    __nv_bfloat16 *dn_w_lo = nullptr, *dn_qp_lo = nullptr, *dn_kp_lo = nullptr, *dn_p_lo = nullptr;
    float *dn_lg = nullptr, *dn_bt = nullptr;
    __nv_bfloat16 *dn_w = nullptr, *dn_qp = nullptr, *dn_kp = nullptr, *dn_p = nullptr;
    float *dn_ut = nullptr, *dn_gc = nullptr, *dn_opre = nullptr;
    // the chunk scan beside the chunk-local kernel: per (value head, chunk)
    // ready flags, per head the epoch the flags count, the scan's stream and
    // the fork and join events
    int *dn_ready = nullptr, *dn_ready_epoch = nullptr;
    int *dn_local_next = nullptr;  // the chunk-local kernel's item counter
    int *dn_out_ready = nullptr;
    cudaStream_t dn_scan_stream = nullptr;
    cudaEvent_t dn_fork = nullptr, dn_join = nullptr;
    float *stage_raw = nullptr;  // the status word (64 B), then the staging
    float *stage = nullptr;   // staging for the *_host entry points
    size_t stage_floats = 0;
    // pinned host staging for the *_host entry points (calls of up to
    // hpin_rows rows): the status word, then the packed inputs and the
    // output.  Copies from and to the callers' own (usually pageable)
    // buffers are host memcpys; the device copies are asynchronous.
    void *hpin_base = nullptr;
    int *hstatus = nullptr;
    float *hpin = nullptr;
    int hpin_rows = 0;
    int *status = nullptr;    // device status word (rl::DEV_*)
    int pos = 0, live = 0;
    int64_t opt_splits = 0, opt_prefill_rows = 64, opt_chunk_rows = 64, opt_cluster = 0;
    int64_t opt_early_tiles = 2, opt_verify_tc = 1, opt_dn_rows = 1, opt_dn_overlap = 1,
            opt_dn_local_tc = 1;
    int64_t opt_wait_limit_us = 0;  // 0: rl::PEER_WAIT_LIMIT_NS
    int64_t opt_dn_scan_tc = 1;
    // RL_OPT_WALK_SPANS: [n_full][4] {first start, CTAs done, span sum, launches}
    unsigned long long *spans = nullptr;
    // rl_act_quantize's int8 activations (grown on demand) and their shape
    float *act_d = nullptr;
    int8_t *act_qs = nullptr;
    int16_t *act_bs = nullptr;
    size_t act_cap = 0;  // super-blocks the scratch holds
    int act_t = 0, act_k = 0;
    // resident clusters of the f32 decode kernel: [fused][log2 cluster size]
    int max_clusters[2][4] = {};
    // resident CTAs per SM of the bf16 walk: [fused]
    int mma_per_sm[2] = {};
    // the next bf16 decode may stream the cache early: the kernel just ahead
    // on the stream cannot be writing it
    bool early_ok = false;
    // the library kernel launched last on the stream: 1 = DeltaNet step of
    // layer prev_layer (its successor must not read that layer's state before
    // its grid-dependency wait), 0 = anything else
    int prev_dn = 0, prev_layer = -1;
    float theta_scale = 1.0f;
    // the cache holds sequence positions shard_lo .. shard_lo + context - 1
    // of a sequence of seq_context positions (rl_set_shard)
    int shard_lo = 0, seq_context = 0;
    // peer exchange of a split sequence (rl_exchange_*): this GPU's buffer,
    // the table of every GPU's buffer as addressed from here, the buffers
    // opened from other processes, the step's epoch and the arrival counter
    float *xbuf = nullptr;
    float **xpeers = nullptr;
    std::vector<void *> xopened;
    int xrank = 0, xworld = 0;
    unsigned xepoch = 0;          // steps published (host side; the kernels keep their own)
    unsigned *xepochs = nullptr;  // [n_head * 4] publishing CTAs' step counts, then
                                  // [n_head] merging CTAs' step counts
    bool xpublish = false;  // rl_full_attn_partial called by rl_split_publish
    std::string err;
    // per-kernel timing (rl_profile_*)
    bool prof_on = false;
    struct Pending {
        int kernel;
        cudaEvent_t a, b;
    };
    std::vector<cudaEvent_t> ev_pool;
    std::vector<Pending> pending;
    double prof_ms[RL_PROF_KERNELS] = {};
    int64_t prof_launches[RL_PROF_KERNELS] = {};
};

namespace {

thread_local std::string tl_err;

int fail(rl_ctx *ctx, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    else tl_err = buf;
    return code;
}

#define CK(ctx, call)                                                                      \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return fail((ctx), RL_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_),  \
                        __FILE__, __LINE__);                                               \
    } while (0)

size_t kv_elem(const rl_config &c) { return c.kv_dtype == RL_KV_BF16 ? 2 : 4; }
size_t conv_dim(const rl_config &c) {
    return (size_t)2 * c.n_k_heads * c.d_state + (size_t)c.n_v_heads * c.d_state;
}
size_t kv_layer_elems(const rl_config &c) {
    return (size_t)2 * c.n_head_kv * c.context * c.head_dim;
}
size_t conv_layer_floats(const rl_config &c) {
    return (size_t)c.slots * conv_dim(c) * (c.conv_kernel - 1);
}
size_t ssm_layer_floats(const rl_config &c) {
    return (size_t)c.n_v_heads * c.slots * c.d_state * c.d_state;
}

void *kv_layer(rl_ctx *x, int layer) {
    return (char *)x->kv + (size_t)layer * kv_layer_elems(x->cfg) * kv_elem(x->cfg);
}

cudaEvent_t take_event(rl_ctx *x) {
    if (!x->ev_pool.empty()) {
        cudaEvent_t e = x->ev_pool.back();
        x->ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Brackets one kernel launch: counts it, and with timing on records an
// event pair around it on the context's stream.
struct ProfScope {
    rl_ctx *x;
    int k;
    cudaEvent_t a = nullptr, b = nullptr;
    ProfScope(rl_ctx *x_, int k_) : x(x_), k(k_) {
        x->prof_launches[k] += 1;
        if (x->prof_on) {
            a = take_event(x);
            b = take_event(x);
            cudaEventRecord(a, x->stream);
        }
    }
    ~ProfScope() {
        if (a) {
            cudaEventRecord(b, x->stream);
            x->pending.push_back({k, a, b});
        }
    }
};

int drain_profile(rl_ctx *x) {
    if (x->pending.empty()) return RL_OK;
    cudaError_t e = cudaStreamSynchronize(x->stream);
    for (auto &p : x->pending) {
        float ms = 0.0f;
        if (e == cudaSuccess && cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess)
            x->prof_ms[p.kernel] += ms;
        x->ev_pool.push_back(p.a);
        x->ev_pool.push_back(p.b);
    }
    x->pending.clear();
    return e == cudaSuccess ? RL_OK : RL_ECUDA;
}

void free_all(rl_ctx *x) {
    for (auto &p : x->pending) {
        x->ev_pool.push_back(p.a);
        x->ev_pool.push_back(p.b);
    }
    x->pending.clear();
    for (cudaEvent_t e : x->ev_pool) cudaEventDestroy(e);
    x->ev_pool.clear();
    void *ps[] = {x->kv, x->conv, x->ssm, x->q_norm, x->k_norm, x->conv1d, x->ssm_a,
                  x->dt_bias, x->ssm_norm, x->q_f32, x->q_bf16, x->gate_bf16, x->part_o, x->part_ml,
                  x->counters, x->rope_cs, x->rope_sn, x->stage_raw,
                  x->dn_qn, x->dn_kn, x->dn_vn, x->dn_qn_lo, x->dn_kn_lo, x->dn_vn_lo, x->dn_qn_l2, x->dn_kn_l2, x->dn_w_lo, x->dn_qp_lo, x->dn_kp_lo, x->dn_p_lo, x->dn_lg, x->dn_bt, x->dn_w, x->dn_qp, x->dn_kp,
                  x->dn_p, x->dn_ut, x->dn_gc, x->dn_opre};
    for (void *p : ps)
        if (p) cudaFree(p);
    if (x->spans) cudaFree(x->spans);
    if (x->act_d) cudaFree(x->act_d);
    if (x->act_qs) cudaFree(x->act_qs);
    if (x->act_bs) cudaFree(x->act_bs);
    if (x->hpin_base) cudaFreeHost(x->hpin_base);
    if (x->dn_ready) cudaFree(x->dn_ready);
    if (x->dn_ready_epoch) cudaFree(x->dn_ready_epoch);
    if (x->dn_local_next) cudaFree(x->dn_local_next);
    if (x->dn_out_ready) cudaFree(x->dn_out_ready);
    if (x->dn_fork) cudaEventDestroy(x->dn_fork);
    if (x->dn_join) cudaEventDestroy(x->dn_join);
    if (x->dn_scan_stream) cudaStreamDestroy(x->dn_scan_stream);
    if (x->own_stream && x->stream) cudaStreamDestroy(x->stream);
}

template <typename T>
int alloc(rl_ctx *x, T **p, size_t elems) {
    if (elems == 0) elems = 1;
    cudaError_t e = cudaMalloc((void **)p, elems * sizeof(T));
    if (e != cudaSuccess) {
        *p = nullptr;
        return fail(x, RL_ENOMEM, "cudaMalloc of %zu bytes: %s", elems * sizeof(T),
                    cudaGetErrorString(e));
    }
    return RL_OK;
}

// Shapes the kernels are built for; anything else is refused up front.
int check_shapes(rl_ctx *x, const rl_config &c) {
    if (c.n_full < 0 || c.n_linear < 0 || c.context < 1 || c.slots < 1 || c.max_batch < 1)
        return fail(x, RL_EINVAL, "n_full, n_linear >= 0; context, slots, max_batch >= 1");
    if (c.kv_dtype != RL_KV_F32 && c.kv_dtype != RL_KV_BF16)
        return fail(x, RL_EINVAL, "kv_dtype %d is neither RL_KV_F32 nor RL_KV_BF16", c.kv_dtype);
    if (c.n_full > 0) {
        if (c.head_dim != 256 || c.n_head_kv < 1 || c.n_head != 4 * c.n_head_kv)
            return fail(x, RL_EUNSUPPORTED,
                        "full attention is built for head_dim 256 and 4 query heads per KV "
                        "head (got head_dim %d, %d/%d heads)",
                        c.head_dim, c.n_head, c.n_head_kv);
        if (c.n_rot < 0 || c.n_rot > c.head_dim || (c.n_rot & 1))
            return fail(x, RL_EINVAL, "n_rot must be even and at most head_dim");
        if (c.n_rot % 16)
            return fail(x, RL_EUNSUPPORTED,
                        "the kernels rotate whole 8-dim lanes: n_rot must be a multiple of 16 "
                        "(got %d)", c.n_rot);
    }
    if (c.n_linear > 0) {
        if (c.d_state != 128 || c.conv_kernel != 4 || c.n_k_heads < 1 ||
            c.n_v_heads % c.n_k_heads != 0 || c.n_v_heads / c.n_k_heads > rl::dn_max_group())
            return fail(x, RL_EUNSUPPORTED,
                        "the DeltaNet kernels are built for d_state 128, conv_kernel 4 and "
                        "n_v a multiple (at most %d) of n_k (got %d, %d, %d/%d)",
                        rl::dn_max_group(), c.d_state, c.conv_kernel, c.n_v_heads, c.n_k_heads);
    }
    return RL_OK;
}

// Host -> device copy ordered on the context's stream and finished before
// return (a synchronous cudaMemcpy runs on the legacy stream, which a
// non-blocking stream does not wait for).
cudaError_t h2d(rl_ctx *x, void *dst, const void *src, size_t bytes) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, x->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(x->stream);
    return e;
}

// Every layer's span slot back to {no start yet, 0 done, 0, 0}, once the
// stream has drained.
int reset_spans(rl_ctx *x) {
    std::vector<unsigned long long> h((size_t)x->cfg.n_full * 4, 0ull);
    for (int l = 0; l < x->cfg.n_full; ++l) h[4 * l] = ~0ull;
    CK(x, cudaStreamSynchronize(x->stream));
    CK(x, cudaMemcpy(x->spans, h.data(), h.size() * sizeof(h[0]), cudaMemcpyHostToDevice));
    return RL_OK;
}

// The end of a pinned host call: the status word and the output that follows
// it in the staging, back in one copy and one wait.
int finish_host_call(rl_ctx *x, size_t out_floats) {
    CK(x, cudaMemcpyAsync(x->hpin_base, x->stage_raw, 64 + out_floats * sizeof(float),
                          cudaMemcpyDeviceToHost, x->stream));
    CK(x, cudaStreamSynchronize(x->stream));
    const int st = *x->hstatus;
    if (st) {
        CK(x, cudaMemsetAsync(x->status, 0, sizeof(int), x->stream));
        if (st & rl::DEV_TIMEOUT)
            return fail(x, RL_ETIMEOUT, "a kernel's bounded wait gave up (status %d)", st);
        return fail(x, RL_EINVAL, "a kernel flagged a bad argument (status %d)", st);
    }
    return RL_OK;
}

int check_status(rl_ctx *x) {
    int st = 0;
    if (x->hstatus) {
        // through the pinned word: an asynchronous copy, then the one wait
        CK(x, cudaMemcpyAsync(x->hstatus, x->status, sizeof(int), cudaMemcpyDeviceToHost,
                              x->stream));
        CK(x, cudaStreamSynchronize(x->stream));
        st = *x->hstatus;
    } else {
        CK(x, cudaMemcpyAsync(&st, x->status, sizeof(int), cudaMemcpyDeviceToHost, x->stream));
        CK(x, cudaStreamSynchronize(x->stream));
    }
    if (st) {
        CK(x, cudaMemsetAsync(x->status, 0, sizeof(int), x->stream));
        if (st & rl::DEV_TIMEOUT)
            return fail(x, RL_ETIMEOUT, "a kernel's bounded wait gave up (status %d)", st);
        return fail(x, RL_EINVAL, "a kernel flagged a bad argument (status %d)", st);
    }
    return RL_OK;
}


// The bf16 split-KV walk and its merge for rows whose furthest row sees
// n_kv_max cached positions.  One wave of walk CTAs: as many splits per
// (KV head, row) as keep every resident slot busy, each a whole number of
// 64-position tiles.
int bf16_walk(rl_ctx *ctx, rl::DecodeArgs &d, int64_t n_kv_max, int64_t groups, int t,
              bool fused) {
    const int P = rl::decode_mma_positions_per_tile();
    const int64_t tiles = (n_kv_max + P - 1) / P;
    const int64_t resident = (int64_t)std::max(1, ctx->mma_per_sm[fused ? 1 : 0]) * ctx->num_sms;
    int64_t splits = std::max<int64_t>(1, resident / groups);
    if (ctx->opt_splits > 0) splits = std::min<int64_t>(splits, ctx->opt_splits);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, tiles));
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, ctx->part_rows / t));
    splits = std::min<int64_t>(splits, 512);
    d.chunk = (int)((tiles + splits - 1) / splits * P);
    d.n_splits = (int)splits;
    d.csize = 1;
    d.early_kv = fused && ctx->early_ok;
    d.early_tiles = (int)ctx->opt_early_tiles;
    if (ctx->spans && !d.rows) {
        const int64_t layer = d.k_row0 / (2 * (int64_t)ctx->cfg.n_head_kv * ctx->cfg.context);
        d.span = ctx->spans + 4 * layer;
    }
    {
        ProfScope ps(ctx, RL_PROF_DECODE);
        CK(ctx, rl::launch_decode_mma(d, ctx->kv_map, ctx->stream));
    }
    {
        ProfScope ps(ctx, RL_PROF_MERGE);
        CK(ctx, rl::launch_decode_combine(d, ctx->stream));
    }
    ctx->early_ok = fused;
    ctx->prev_dn = 0;
    return RL_OK;
}
// Tensor-core verify for t rows appended at pos (the kernel appends their
// keys and values and normalises and rotates the queries itself): one CTA
// per (key split, KV head), as many splits as one wave holds, each a whole
// number of 64-position tiles; the split merge applies the gate.
int verify_tc(rl_ctx *ctx, int layer, int pos, int t, const float *qg, const float *k,
              const float *v, float *out) {
    const rl_config &c = ctx->cfg;
    const int64_t tiles = ((int64_t)pos + t - 1) / 64 + 1;
    int64_t splits = std::max<int64_t>(1, ctx->num_sms / c.n_head_kv);
    if (ctx->opt_splits > 0) splits = std::min<int64_t>(splits, ctx->opt_splits);
    splits = std::min<int64_t>(splits, tiles);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, ctx->part_rows / t));
    splits = std::min<int64_t>(splits, 512);
    const int64_t per = (tiles + splits - 1) / splits;
    splits = (tiles + per - 1) / per;  // every split holds at least one tile
    rl::PrefillArgs pa{};
    pa.status = ctx->status;
    pa.t = t;
    pa.pos = pos;
    pa.n_head = c.n_head;
    pa.n_kv = c.n_head_kv;
    pa.context = c.context;
    pa.k_row0 = layer * 2 * c.n_head_kv * c.context;
    pa.v_row0 = pa.k_row0 + c.n_head_kv * c.context;
    pa.part_o = ctx->part_o;
    pa.part_ml = ctx->part_ml;
    pa.n_splits = (int)splits;
    pa.split_tiles = (int)per;
    pa.qg = qg;
    pa.q_norm = ctx->q_norm + (size_t)layer * c.head_dim;
    pa.rope_cs = ctx->rope_cs;
    pa.rope_sn = ctx->rope_sn;
    pa.eps = c.rms_eps;
    pa.k_in = k;
    pa.v_in = v;
    pa.k_norm = ctx->k_norm + (size_t)layer * c.head_dim;
    pa.k_cache = static_cast<__nv_bfloat16 *>(kv_layer(ctx, layer));
    pa.v_cache = pa.k_cache + (size_t)c.n_head_kv * c.context * c.head_dim;
    {
        ProfScope ps(ctx, RL_PROF_VERIFY);
        CK(ctx, rl::launch_verify_tc(pa, ctx->kv_map, ctx->stream));
    }
    rl::DecodeArgs d{};
    d.qg = qg;
    d.part_o = ctx->part_o;
    d.part_ml = ctx->part_ml;
    d.out = out;
    d.status = ctx->status;
    d.pos = pos;
    d.t = t;
    d.context = c.context;
    d.n_head = c.n_head;
    d.n_kv = c.n_head_kv;
    d.n_splits = (int)splits;
    d.kv_bf16 = true;
    d.part_out = nullptr;
    {
        ProfScope ps(ctx, RL_PROF_MERGE);
        CK(ctx, rl::launch_decode_combine(d, ctx->stream));
    }
    ctx->early_ok = false;
    ctx->prev_dn = 0;
    return RL_OK;
}
}  // namespace

void rl::set_thread_error(const char *msg) { tl_err = msg; }

extern "C" {

const char *rl_version(void) { return RL_VERSION_STRING; }

const char *rl_last_error(const rl_ctx *ctx) {
    return ctx ? ctx->err.c_str() : tl_err.c_str();
}

int rl_ctx_create(int device, const rl_config *cfg, rl_ctx **out) {
    if (!cfg || !out) return fail(nullptr, RL_EINVAL, "cfg and out must not be NULL");
    *out = nullptr;
    int code = check_shapes(nullptr, *cfg);
    if (code) return code;
    CK((rl_ctx *)nullptr, cudaSetDevice(device));
    rl_ctx *x = new rl_ctx();
    x->cfg = *cfg;
    // a batch longer than the context could never run (forward.rs:461)
    x->cfg.max_batch =
        std::max(1, std::min(std::max(x->cfg.max_batch, x->cfg.slots), x->cfg.context));
    x->device = device;
    x->seq_context = x->cfg.context;
    const rl_config &c = x->cfg;
    auto bail = [&](int code) {
        tl_err = x->err;
        free_all(x);
        delete x;
        return code;
    };
    if (cudaDeviceGetAttribute(&x->num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
        x->num_sms = 148;
    if (cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(x, RL_ECUDA, "cudaStreamCreate failed"));
    x->own_stream = true;
    if (rl::init_full_attn_kernels() != cudaSuccess || rl::init_dn_kernels() != cudaSuccess ||
        rl::init_decode_kernels() != cudaSuccess || rl::init_decode_mma_kernels() != cudaSuccess ||
        rl::init_prefill_kernels() != cudaSuccess || rl::init_dn_chunk_kernels() != cudaSuccess ||
        rl::init_matvec_kernel() != cudaSuccess ||
        rl::init_dn_rows_kernel() != cudaSuccess)
        return bail(fail(x, RL_ECUDA, "kernel attribute set-up failed"));
    for (int f = 0; f < 2; ++f) {
        for (int lc = 0; lc < 4; ++lc)
            x->max_clusters[f][lc] = rl::decode_max_active_clusters(false, f == 1, 1 << lc);
        x->mma_per_sm[f] = rl::decode_mma_max_active_ctas(f == 1);
    }
    const size_t hd = c.head_dim, nh = c.n_head, cd = conv_dim(c), s = c.d_state;
    const size_t mb = c.max_batch;
    if ((code = alloc(x, (char **)&x->kv, (size_t)c.n_full * kv_layer_elems(c) * kv_elem(c))) ||
        (code = alloc(x, &x->conv, (size_t)c.n_linear * conv_layer_floats(c))) ||
        (code = alloc(x, &x->ssm, (size_t)c.n_linear * ssm_layer_floats(c))) ||
        (code = alloc(x, &x->q_norm, (size_t)c.n_full * hd)) ||
        (code = alloc(x, &x->k_norm, (size_t)c.n_full * hd)) ||
        (code = alloc(x, &x->conv1d, (size_t)c.n_linear * cd * c.conv_kernel)) ||
        (code = alloc(x, &x->ssm_a, (size_t)c.n_linear * c.n_v_heads)) ||
        (code = alloc(x, &x->dt_bias, (size_t)c.n_linear * c.n_v_heads)) ||
        (code = alloc(x, &x->ssm_norm, (size_t)c.n_linear * s)))
        return bail(code);
    if (c.n_full > 0) {
        x->part_rows = std::max<int64_t>(mb, 4 * (int64_t)x->num_sms);
        if ((code = alloc(x, &x->q_f32, mb * nh * hd)) ||
            (code = alloc(x, &x->q_bf16, mb * nh * hd)) ||
            (code = alloc(x, &x->gate_bf16, c.kv_dtype == RL_KV_BF16 ? mb * nh * hd : 1)) ||
            (code = alloc(x, &x->part_o, (size_t)x->part_rows * nh * hd)) ||
            (code = alloc(x, &x->part_ml, (size_t)x->part_rows * nh * 8 * 2)) ||
            (code = alloc(x, &x->counters, (size_t)mb * c.n_head_kv * 8)))
            return bail(code);
        if (cudaMemset(x->counters, 0, (size_t)mb * c.n_head_kv * 8 * sizeof(int)) != cudaSuccess)
            return bail(fail(x, RL_ECUDA, "counter initialisation failed"));
        const size_t half = std::max(1, c.n_rot / 2);
        if ((code = alloc(x, &x->rope_cs, (size_t)c.context * half)) ||
            (code = alloc(x, &x->rope_sn, (size_t)c.context * half)))
            return bail(code);
        if (c.kv_dtype == RL_KV_BF16) {
            const uint64_t rows = (uint64_t)c.n_full * 2 * c.n_head_kv * c.context;
            if (rows >= (1ull << 31))
                return bail(fail(x, RL_EUNSUPPORTED, "a bf16 KV cache of %llu rows exceeds 2^31",
                                 (unsigned long long)rows));
            if (rl::encode_bf16_2d(&x->kv_map, x->kv, rows, c.head_dim, (uint64_t)c.head_dim * 2,
                                   rl::kDecodeBoxRows, rl::kDecodeBoxCols) != cudaSuccess)
                return bail(fail(x, RL_ECUDA, "encoding the KV tensor map failed"));
            if (rl::encode_bf16_3d(&x->q_map, x->q_bf16, c.head_dim, c.n_head, mb,
                                   (uint64_t)c.head_dim * 2, (uint64_t)c.head_dim * 2 * c.n_head,
                                   64, 1, rl::kPrefillQBoxRows) != cudaSuccess)
                return bail(fail(x, RL_ECUDA, "encoding the query tensor map failed"));
            if (rl::encode_bf16_3d(&x->gate_map, x->gate_bf16, c.head_dim, c.n_head, mb,
                                   (uint64_t)c.head_dim * 2, (uint64_t)c.head_dim * 2 * c.n_head,
                                   64, 1, rl::kPrefillQBoxRows) != cudaSuccess)
                return bail(fail(x, RL_ECUDA, "encoding the gate tensor map failed"));
        }
    }
    if (c.n_linear > 0 && c.d_state == 128) {
        // the rows kernel's tiles: 128 rows x 32 columns of one head's slot
        const uint64_t rows = (uint64_t)c.n_linear * c.n_v_heads * c.slots * s;
        x->ssm_map_ok = rows < (1ull << 31) &&
                        rl::encode_f32_2d(&x->ssm_map, x->ssm, rows, s, s * 4, 128, 32) ==
                            cudaSuccess;
    }
    if (c.n_linear > 0 && c.slots == 1 && mb >= 64) {
        const size_t nk = c.n_k_heads, nv = c.n_v_heads, nc = (mb + 63) / 64;
        if ((code = alloc(x, &x->dn_qn, mb * nk * s)) || (code = alloc(x, &x->dn_kn, mb * nk * s)) ||
            (code = alloc(x, &x->dn_qn_lo, mb * nk * s)) ||
            (code = alloc(x, &x->dn_kn_lo, mb * nk * s)) ||
            (code = alloc(x, &x->dn_qn_l2, mb * nk * s)) ||
            (code = alloc(x, &x->dn_kn_l2, mb * nk * s)) ||
            (code = alloc(x, &x->dn_vn_lo, mb * nv * s)) ||
            (code = alloc(x, &x->dn_w_lo, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_qp_lo, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_kp_lo, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_p_lo, nv * nc * 64 * 64)) ||
            (code = alloc(x, &x->dn_vn, mb * nv * s)) || (code = alloc(x, &x->dn_lg, mb * nv)) ||
            (code = alloc(x, &x->dn_bt, mb * nv)) || (code = alloc(x, &x->dn_w, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_qp, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_kp, nv * nc * 64 * s)) ||
            (code = alloc(x, &x->dn_p, nv * nc * 64 * 64)) ||
            (code = alloc(x, &x->dn_ut, nv * nc * 64 * s)) || (code = alloc(x, &x->dn_gc, nv * nc)) ||
            (code = alloc(x, &x->dn_opre, mb * nv * s)))
            return bail(code);
        const uint64_t rows = (uint64_t)nv * nc * 64;
        rl::DnScanMaps &m = x->dn_scan_maps;
        x->dn_scan_maps_ok =
            rows < (1ull << 31) &&
            rl::encode_bf16_2d(&m.w, x->dn_w, rows, s, s * 2, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.qh, x->dn_qp, rows, s, s * 2, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.ql, x->dn_qp_lo, rows, s, s * 2, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.kh, x->dn_kp, rows, s, s * 2, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.kl, x->dn_kp_lo, rows, s, s * 2, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.ph, x->dn_p, rows, 64, 128, 64, 64) == cudaSuccess &&
            rl::encode_bf16_2d(&m.pl, x->dn_p_lo, rows, 64, 128, 64, 64) == cudaSuccess;
        // the scan beside the chunk-local kernel, on a stream of the highest
        // priority so that its CTAs are placed ahead of the chunk-local ones
        int lo_prio = 0, hi_prio = 0;
        cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio);
        if ((code = alloc(x, &x->dn_ready, nv * nc)) ||
            (code = alloc(x, &x->dn_ready_epoch, nv)) ||
            (code = alloc(x, &x->dn_local_next, 1)) ||
            (code = alloc(x, &x->dn_out_ready, nv * nc)))
            return bail(code);
        if (cudaMemset(x->dn_ready, 0, nv * nc * sizeof(int)) != cudaSuccess ||
            cudaMemset(x->dn_ready_epoch, 0, nv * sizeof(int)) != cudaSuccess ||
            cudaStreamCreateWithPriority(&x->dn_scan_stream, cudaStreamNonBlocking, hi_prio) !=
                cudaSuccess ||
            cudaEventCreateWithFlags(&x->dn_fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&x->dn_join, cudaEventDisableTiming) != cudaSuccess)
            return bail(fail(x, RL_ECUDA, "the chunk scan's stream or events"));
    }
    // staging for the host entry points: the larger of the two paths' in+out
    const size_t full_io = mb * (2 * hd * nh + 2 * hd * c.n_head_kv + hd * nh);
    const size_t lin_io = mb * (cd + 2 * s * c.n_v_heads + 2 * c.n_v_heads);
    x->stage_floats = std::max(c.n_full ? full_io : 0, c.n_linear ? lin_io : 0);
    // the status word heads the staging, so that a host call's output and the
    // status behind it come back in one copy: [status, 64 B][output][inputs]
    if ((code = alloc(x, &x->stage_raw, x->stage_floats + 16))) return bail(code);
    x->status = reinterpret_cast<int *>(x->stage_raw);
    x->stage = x->stage_raw + 16;
    CK(x, cudaMemsetAsync(x->status, 0, sizeof(int), x->stream));
    {
        // pinned staging for calls of up to 64 rows (without it, the host
        // entry points copy from and to the callers' buffers directly)
        const int rows = (int)std::min<size_t>(mb, 64);
        const size_t bytes = 64 + (x->stage_floats / mb) * rows * sizeof(float);
        if (cudaMallocHost(&x->hpin_base, bytes) == cudaSuccess) {
            x->hstatus = static_cast<int *>(x->hpin_base);
            x->hpin = reinterpret_cast<float *>(static_cast<char *>(x->hpin_base) + 64);
            x->hpin_rows = rows;
        } else {
            x->hpin_base = nullptr;
            cudaGetLastError();
        }
    }
    // theta_scale = theta^(-2/n_rot), computed on the host exactly as
    // forward.rs:1853 does, so the device advances the same f32 angle
    x->theta_scale = c.n_rot > 0 ? std::pow(c.rope_theta, -2.0f / (float)c.n_rot) : 1.0f;
    if (c.n_full > 0) {
        if (rl::launch_rope_table(x->rope_cs, x->rope_sn, c.context, c.n_rot, x->theta_scale,
                                  x->stream) != cudaSuccess ||
            cudaStreamSynchronize(x->stream) != cudaSuccess)
            return bail(fail(x, RL_ECUDA, "RoPE table set-up failed"));
    }
    if ((code = rl_reset(x))) return bail(code);
    // unit norm weights until the caller sets its own
    if (c.n_full > 0 || c.n_linear > 0) {
        std::string ones;
        const size_t n = std::max(hd, s);
        float *h = new float[n];
        for (size_t i = 0; i < n; ++i) h[i] = 1.0f;
        for (int l = 0; l < c.n_full; ++l) {
            cudaMemcpy(x->q_norm + l * hd, h, hd * 4, cudaMemcpyHostToDevice);
            cudaMemcpy(x->k_norm + l * hd, h, hd * 4, cudaMemcpyHostToDevice);
        }
        for (int l = 0; l < c.n_linear; ++l)
            cudaMemcpy(x->ssm_norm + l * s, h, s * 4, cudaMemcpyHostToDevice);
        delete[] h;
        cudaMemset(x->conv1d, 0, (size_t)c.n_linear * cd * c.conv_kernel * 4);
        cudaMemset(x->ssm_a, 0, (size_t)c.n_linear * c.n_v_heads * 4);
        cudaMemset(x->dt_bias, 0, (size_t)c.n_linear * c.n_v_heads * 4);
        if (cudaDeviceSynchronize() != cudaSuccess)
            return bail(fail(x, RL_ECUDA, "weight initialisation failed"));
    }
    *out = x;
    return RL_OK;
}

void rl_ctx_destroy(rl_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (void *p : ctx->xopened) cudaIpcCloseMemHandle(p);
    if (ctx->xbuf) cudaFree(ctx->xbuf);
    if (ctx->xpeers) cudaFree(ctx->xpeers);
    if (ctx->xepochs) cudaFree(ctx->xepochs);
    free_all(ctx);
    delete ctx;
}

int rl_set_stream(rl_ctx *ctx, void *stream) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
    ctx->stream = (cudaStream_t)stream;
    ctx->own_stream = false;
    ctx->early_ok = false;
    return RL_OK;
}

void *rl_get_stream(const rl_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int rl_reset(rl_ctx *ctx) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaMemsetAsync(ctx->kv, 0, (size_t)c.n_full * kv_layer_elems(c) * kv_elem(c),
                            ctx->stream));
    CK(ctx, cudaMemsetAsync(ctx->conv, 0, (size_t)c.n_linear * conv_layer_floats(c) * 4,
                            ctx->stream));
    CK(ctx, cudaMemsetAsync(ctx->ssm, 0, (size_t)c.n_linear * ssm_layer_floats(c) * 4,
                            ctx->stream));
    CK(ctx, cudaMemsetAsync(ctx->status, 0, sizeof(int), ctx->stream));
    if (ctx->counters)
        CK(ctx, cudaMemsetAsync(ctx->counters, 0,
                                (size_t)c.max_batch * c.n_head_kv * 8 * sizeof(int), ctx->stream));
    ctx->pos = 0;
    ctx->live = 0;
    ctx->early_ok = false;
    return RL_OK;
}

int rl_set_weights_full(rl_ctx *ctx, int layer, const float *q_norm, const float *k_norm) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (layer < 0 || layer >= ctx->cfg.n_full || !q_norm || !k_norm)
        return fail(ctx, RL_EINVAL, "full layer %d of %d, or a NULL weight", layer, ctx->cfg.n_full);
    const size_t hd = ctx->cfg.head_dim;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, h2d(ctx, ctx->q_norm + layer * hd, q_norm, hd * 4));
    CK(ctx, h2d(ctx, ctx->k_norm + layer * hd, k_norm, hd * 4));
    return RL_OK;
}

int rl_set_weights_linear(rl_ctx *ctx, int layer, const float *conv1d, const float *ssm_a,
                          const float *dt_bias, const float *norm) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_linear || !conv1d || !ssm_a || !dt_bias || !norm)
        return fail(ctx, RL_EINVAL, "linear layer %d of %d, or a NULL weight", layer, c.n_linear);
    const size_t cw = conv_dim(c) * c.conv_kernel, nv = c.n_v_heads, s = c.d_state;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, h2d(ctx, ctx->conv1d + layer * cw, conv1d, cw * 4));
    CK(ctx, h2d(ctx, ctx->ssm_a + layer * nv, ssm_a, nv * 4));
    CK(ctx, h2d(ctx, ctx->dt_bias + layer * nv, dt_bias, nv * 4));
    CK(ctx, h2d(ctx, ctx->ssm_norm + layer * s, norm, s * 4));
    return RL_OK;
}

int rl_full_attn(rl_ctx *ctx, int layer, int pos, int t, const float *qg, const float *k,
                 const float *v, float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_full)
        return fail(ctx, RL_EINVAL, "full layer %d of %d", layer, c.n_full);
    if (t < 1 || t > c.max_batch)
        return fail(ctx, RL_EINVAL, "a batch of %d rows, but the scratch was sized for %d", t,
                    c.max_batch);
    if (pos < 0 || (int64_t)pos + t > c.context)
        return fail(ctx, RL_ECONTEXT, "context of %d tokens holds %d and cannot take %d more",
                    c.context, pos, t);
    if (!qg || !k || !v || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    if (((uintptr_t)qg | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15)
        return fail(ctx, RL_EINVAL, "qg, k, v and out must be 16-byte aligned");
    if (ctx->shard_lo != 0 || ctx->seq_context != c.context)
        return fail(ctx, RL_EINVAL,
                    "this context holds one shard of a split sequence: use rl_full_attn_partial");
    CK(ctx, cudaSetDevice(ctx->device));
    const bool bf16 = c.kv_dtype == RL_KV_BF16;
    const size_t half = (size_t)c.n_head_kv * c.context * c.head_dim * kv_elem(c);
    void *k_cache = kv_layer(ctx, layer);
    void *v_cache = (char *)k_cache + half;
    const bool fused = t == 1;
    const bool prefill = bf16 && ctx->opt_prefill_rows > 0 && t >= ctx->opt_prefill_rows;
    // a speculative-verify batch: its rows and the group's four query heads
    // share one tensor-core tile
    const bool verify = bf16 && !prefill && !fused && ctx->opt_verify_tc &&
                        t <= rl::kVerifyRows && c.n_head == 4 * c.n_head_kv && c.n_rot == 64;
    // the verify kernel appends the rows and normalises the queries itself
    if (verify) return verify_tc(ctx, layer, pos, t, qg, k, v, out);
    if (!fused) {
        // rows of a batch attend to each other's keys: append them all first
        rl::FullArgs a{};
        a.qg = qg;
        a.k = k;
        a.v = v;
        a.q_norm = ctx->q_norm + (size_t)layer * c.head_dim;
        a.k_norm = ctx->k_norm + (size_t)layer * c.head_dim;
        a.k_cache = k_cache;
        a.v_cache = v_cache;
        a.rope_cs = ctx->rope_cs;
        a.rope_sn = ctx->rope_sn;
        a.q_f32 = prefill ? nullptr : ctx->q_f32;
        a.q_bf16 = prefill ? ctx->q_bf16 : nullptr;
        a.gate_bf16 = prefill ? ctx->gate_bf16 : nullptr;
        a.t = t;
        a.pos = pos;
        a.n_head = c.n_head;
        a.n_kv = c.n_head_kv;
        a.hd = c.head_dim;
        a.context = c.context;
        a.n_rot = c.n_rot;
        a.theta_scale = ctx->theta_scale;
        a.eps = c.rms_eps;
        a.kv_bf16 = bf16;
        {
            ProfScope ps(ctx, RL_PROF_PROLOGUE);
            CK(ctx, rl::launch_full_prologue(a, ctx->stream));
        }
        if (prefill) {
            rl::PrefillArgs pa{};
            pa.out = out;
            pa.status = ctx->status;
            pa.t = t;
            pa.pos = pos;
            pa.n_head = c.n_head;
            pa.n_kv = c.n_head_kv;
            pa.context = c.context;
            pa.k_row0 = layer * 2 * c.n_head_kv * c.context;
            pa.v_row0 = pa.k_row0 + c.n_head_kv * c.context;
            {
                ProfScope ps(ctx, RL_PROF_PREFILL);
                CK(ctx, rl::launch_prefill(pa, ctx->q_map, ctx->kv_map, ctx->gate_map,
                                           ctx->stream));
            }
            ctx->early_ok = false;
            ctx->prev_dn = 0;
            return RL_OK;
        }
    }
    const int64_t n_kv_max = (int64_t)pos + t;
    const int64_t groups = (int64_t)c.n_head_kv * t;  // (KV head, row) pairs
    rl::DecodeArgs d{};
    d.qg = qg;
    d.k_in = k;
    d.v_in = v;
    d.q_f32 = ctx->q_f32;
    d.q_norm = ctx->q_norm + (size_t)layer * c.head_dim;
    d.k_norm = ctx->k_norm + (size_t)layer * c.head_dim;
    d.rope_cs = ctx->rope_cs;
    d.rope_sn = ctx->rope_sn;
    d.k_cache_v = k_cache;
    d.v_cache_v = v_cache;
    d.part_o = ctx->part_o;
    d.part_ml = ctx->part_ml;
    d.counters = ctx->counters;
    d.out = out;
    d.status = ctx->status;
    d.pos = pos;
    d.t = t;
    d.context = c.context;
    d.n_head = c.n_head;
    d.n_kv = c.n_head_kv;
    d.n_rot = c.n_rot;
    d.theta_scale = ctx->theta_scale;
    d.eps = c.rms_eps;
    d.kv_bf16 = bf16;
    d.fused = fused;
    d.k_row0 = layer * 2 * c.n_head_kv * c.context;
    d.v_row0 = d.k_row0 + c.n_head_kv * c.context;
    d.shard_lo = 0;
    d.part_out = nullptr;

    if (bf16) return bf16_walk(ctx, d, n_kv_max, groups, t, fused);

    // f32 caches: split-KV walk on the CUDA cores.  The (split, KV head, row)
    // CTAs of one launch must all be resident at once (one wave); the splits
    // of a (row, KV head) form clusters of csize CTAs.  Among cluster sizes
    // 8, 4, 2, 1, take the one that keeps the most CTAs resident, the larger
    // size on a tie (fewer partials for the cross-cluster merge).
    const int P = rl::decode_positions_per_tile(false);
    const int64_t tiles = (n_kv_max + P - 1) / P;
    int64_t splits = 0;
    int csize = 1;
    for (int lc = 3; lc >= 0; --lc) {
        const int cs = 1 << lc;
        if (ctx->opt_cluster > 0 && cs != ctx->opt_cluster) continue;
        int64_t per = (int64_t)ctx->max_clusters[fused ? 1 : 0][lc] / groups * cs;
        if (ctx->opt_splits > 0) per = std::min<int64_t>(per, ctx->opt_splits);
        per = std::min<int64_t>(per, (tiles + cs - 1) / cs * cs);
        per = std::min<int64_t>(per, (int64_t)cs * std::max<int64_t>(1, ctx->part_rows / t));
        per = std::min<int64_t>(per, (int64_t)cs * 64);  // the final merge holds 64 clusters
        per = per / cs * cs;
        // a smaller cluster only if it keeps at least 1/8 more CTAs resident:
        // larger clusters leave fewer partials for the cross-cluster merge
        if (per * 8 > splits * 9) splits = per, csize = cs;
    }
    if (splits < 1) {
        // more (KV head, row) pairs than resident CTAs: one split each, in waves
        splits = 1;
        csize = 1;
    }
    int64_t chunk = (n_kv_max + splits - 1) / splits;
    chunk = (chunk + P - 1) / P * P;
    d.chunk = (int)chunk;
    d.n_splits = (int)splits;
    d.csize = csize;
    d.early_kv = false;
    {
        ProfScope ps(ctx, RL_PROF_DECODE);
        CK(ctx, rl::launch_decode(d, ctx->stream));
    }
    ctx->early_ok = false;
    ctx->prev_dn = 0;
    return RL_OK;
}

int rl_set_shard(rl_ctx *ctx, int lo, int seq_context) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (c.kv_dtype != RL_KV_BF16 || c.n_full < 1)
        return fail(ctx, RL_EUNSUPPORTED, "a split sequence needs a bf16 KV cache");
    if (lo < 0 || seq_context < c.context || (int64_t)lo + c.context > seq_context)
        return fail(ctx, RL_EINVAL, "shard %d..%d does not lie inside a sequence of %d", lo,
                    lo + c.context, seq_context);
    CK(ctx, cudaSetDevice(ctx->device));
    if (seq_context != ctx->seq_context) {
        // the queries' RoPE angles are those of sequence positions
        const size_t half = std::max(1, c.n_rot / 2);
        float *cs = nullptr, *sn = nullptr;
        int code;
        if ((code = alloc(ctx, &cs, (size_t)seq_context * half)) ||
            (code = alloc(ctx, &sn, (size_t)seq_context * half))) {
            if (cs) cudaFree(cs);
            return code;
        }
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->rope_cs);
        cudaFree(ctx->rope_sn);
        ctx->rope_cs = cs;
        ctx->rope_sn = sn;
        CK(ctx, rl::launch_rope_table(cs, sn, seq_context, c.n_rot, ctx->theta_scale, ctx->stream));
        CK(ctx, cudaStreamSynchronize(ctx->stream));
    }
    ctx->shard_lo = lo;
    ctx->seq_context = seq_context;
    ctx->early_ok = false;
    return RL_OK;
}

int rl_full_attn_partial(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                         const float *v, float *partial) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_full)
        return fail(ctx, RL_EINVAL, "full layer %d of %d", layer, c.n_full);
    if (c.kv_dtype != RL_KV_BF16)
        return fail(ctx, RL_EUNSUPPORTED, "a split sequence needs a bf16 KV cache");
    if (pos < 0 || pos >= ctx->seq_context)
        return fail(ctx, RL_ECONTEXT, "position %d is outside the sequence of %d", pos,
                    ctx->seq_context);
    if (!qg || !k || !v || (!partial && !ctx->xpublish))
        return fail(ctx, RL_EINVAL, "NULL input or output");
    if (((uintptr_t)qg | (uintptr_t)k | (uintptr_t)v | (uintptr_t)partial) & 15)
        return fail(ctx, RL_EINVAL, "qg, k, v and partial must be 16-byte aligned");
    CK(ctx, cudaSetDevice(ctx->device));
    void *k_cache = kv_layer(ctx, layer);
    void *v_cache = (char *)k_cache + (size_t)c.n_head_kv * c.context * c.head_dim * kv_elem(c);
    rl::DecodeArgs d{};
    d.qg = qg;
    d.k_in = k;
    d.v_in = v;
    d.q_f32 = ctx->q_f32;
    d.q_norm = ctx->q_norm + (size_t)layer * c.head_dim;
    d.k_norm = ctx->k_norm + (size_t)layer * c.head_dim;
    d.rope_cs = ctx->rope_cs;
    d.rope_sn = ctx->rope_sn;
    d.k_cache_v = k_cache;
    d.v_cache_v = v_cache;
    d.part_o = ctx->part_o;
    d.part_ml = ctx->part_ml;
    d.counters = ctx->counters;
    d.out = nullptr;
    d.status = ctx->status;
    d.pos = pos;
    d.t = 1;
    d.context = c.context;
    d.n_head = c.n_head;
    d.n_kv = c.n_head_kv;
    d.n_rot = c.n_rot;
    d.theta_scale = ctx->theta_scale;
    d.eps = c.rms_eps;
    d.kv_bf16 = true;
    d.fused = true;
    d.k_row0 = layer * 2 * c.n_head_kv * c.context;
    d.v_row0 = d.k_row0 + c.n_head_kv * c.context;
    d.shard_lo = ctx->shard_lo;
    d.part_out = partial;
    if (ctx->xpublish) {
        ++ctx->xepoch;
        d.xpeers = ctx->xpeers;
        d.xrank = ctx->xrank;
        d.xworld = ctx->xworld;
        d.xepochs = ctx->xepochs;
    }
    const int64_t local = std::max<int64_t>(
        0, std::min<int64_t>((int64_t)pos + 1 - ctx->shard_lo, c.context));
    return bf16_walk(ctx, d, local, c.n_head_kv, 1, true);
}

int rl_exchange_init(rl_ctx *ctx, int rank, int world, void *handle_out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (world < 1 || rank < 0 || rank >= world || world > RL_EXCHANGE_MAX_GPUS)
        return fail(ctx, RL_EINVAL, "rank %d of %d (at most %d GPUs)", rank, world,
                    RL_EXCHANGE_MAX_GPUS);
    if (ctx->xbuf) return fail(ctx, RL_EINVAL, "the exchange is already set up");
    const rl_config &c = ctx->cfg;
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t bytes = rl::xbuf_bytes(world, c.n_head, c.head_dim);
    // its own allocation, so that its IPC handle names exactly this buffer
    CK(ctx, cudaMalloc(&ctx->xbuf, bytes));
    CK(ctx, cudaMemset(ctx->xbuf, 0, bytes));
    CK(ctx, cudaMalloc(&ctx->xepochs, sizeof(unsigned) * c.n_head * 5));
    CK(ctx, cudaMemset(ctx->xepochs, 0, sizeof(unsigned) * c.n_head * 5));
    CK(ctx, cudaMalloc(&ctx->xpeers, sizeof(float *) * world));
    ctx->xrank = rank;
    ctx->xworld = world;
    ctx->xepoch = 0;
    if (handle_out) {
        cudaIpcMemHandle_t h;
        CK(ctx, cudaIpcGetMemHandle(&h, ctx->xbuf));
        static_assert(sizeof(h) == RL_IPC_HANDLE_BYTES, "IPC handle size");
        memcpy(handle_out, &h, sizeof(h));
    }
    return RL_OK;
}

namespace {
int upload_peers(rl_ctx *ctx, const std::vector<float *> &ptrs) {
    CK(ctx, cudaMemcpy(ctx->xpeers, ptrs.data(), sizeof(float *) * ptrs.size(),
                       cudaMemcpyHostToDevice));
    return RL_OK;
}
}  // namespace

int rl_exchange_connect(rl_ctx *ctx, const void *handles) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!ctx->xbuf || !handles) return fail(ctx, RL_EINVAL, "rl_exchange_init first; handles");
    CK(ctx, cudaSetDevice(ctx->device));
    std::vector<float *> ptrs(ctx->xworld);
    for (int g = 0; g < ctx->xworld; ++g) {
        if (g == ctx->xrank) {
            ptrs[g] = ctx->xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + (size_t)g * RL_IPC_HANDLE_BYTES,
               sizeof(h));
        void *p = nullptr;
        CK(ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        ctx->xopened.push_back(p);
        ptrs[g] = static_cast<float *>(p);
    }
    return upload_peers(ctx, ptrs);
}

int rl_exchange_connect_ptrs(rl_ctx *ctx, const uint64_t *bufs) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!ctx->xbuf || !bufs) return fail(ctx, RL_EINVAL, "rl_exchange_init first; buffers");
    CK(ctx, cudaSetDevice(ctx->device));
    std::vector<float *> ptrs(ctx->xworld);
    for (int g = 0; g < ctx->xworld; ++g)
        ptrs[g] = g == ctx->xrank ? ctx->xbuf : reinterpret_cast<float *>(bufs[g]);
    return upload_peers(ctx, ptrs);
}

uint64_t rl_exchange_buffer(const rl_ctx *ctx) {
    return ctx ? reinterpret_cast<uint64_t>(ctx->xbuf) : 0;
}

int rl_split_publish(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                     const float *v) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!ctx->xbuf) return fail(ctx, RL_EINVAL, "rl_exchange_init and _connect first");
    // the walk and the merge of rl_full_attn_partial, the partial pushed to
    // every GPU's exchange slot instead of a caller's buffer
    ctx->xpublish = true;
    const int code = rl_full_attn_partial(ctx, layer, pos, qg, k, v, nullptr);
    ctx->xpublish = false;
    return code;
}

int rl_split_merge(rl_ctx *ctx, const float *qg, float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!ctx->xbuf || ctx->xepoch == 0)
        return fail(ctx, RL_EINVAL, "no partial published (rl_split_publish)");
    if (!qg || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    CK(ctx, cudaSetDevice(ctx->device));
    {
        ProfScope ps(ctx, RL_PROF_MERGE);
        const unsigned long long limit_ns =
            ctx->opt_wait_limit_us > 0 ? (unsigned long long)ctx->opt_wait_limit_us * 1000ull
                                       : rl::PEER_WAIT_LIMIT_NS;
        CK(ctx, rl::launch_peer_merge(reinterpret_cast<const unsigned long long *>(ctx->xbuf),
                                      ctx->xworld, ctx->cfg.n_head, qg, out,
                                      ctx->status, ctx->xepochs + 4 * ctx->cfg.n_head, limit_ns,
                                      ctx->stream));
    }
    ctx->prev_dn = 0;
    return RL_OK;
}

int rl_full_attn_split(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                       const float *v, float *out) {
    const int code = rl_split_publish(ctx, layer, pos, qg, k, v);
    return code != RL_OK ? code : rl_split_merge(ctx, qg, out);
}

// ---- batched decode over the contexts of many sequences -------------------
struct rl_batch {
    std::vector<rl_ctx *> ctxs;
    int n = 0, n_full = 0;
    rl::BatchRow *rows = nullptr;     // [n_full][n]
    CUtensorMap *maps = nullptr;      // [n], device copies of the contexts' maps
    float *part_o = nullptr, *part_ml = nullptr;
    int *counters = nullptr;          // [n][n_kv][8]
    int splits = 1;
};

void rl_batch_destroy(rl_batch *b) {
    if (!b) return;
    if (!b->ctxs.empty()) {
        cudaSetDevice(b->ctxs[0]->device);
        cudaStreamSynchronize(b->ctxs[0]->stream);
    }
    cudaFree(b->rows);
    cudaFree(b->maps);
    cudaFree(b->part_o);
    cudaFree(b->part_ml);
    cudaFree(b->counters);
    delete b;
}

int rl_batch_create(rl_ctx *const *ctxs, int n, rl_batch **out) {
    if (!ctxs || n < 1 || !out) return fail(nullptr, RL_EINVAL, "contexts, n >= 1 and out");
    *out = nullptr;
    rl_ctx *c0 = ctxs[0];
    if (!c0) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = c0->cfg;
    for (int i = 0; i < n; ++i) {
        const rl_ctx *x = ctxs[i];
        if (!x) return fail(nullptr, RL_EINVAL, "NULL context %d", i);
        const rl_config &ci = x->cfg;
        if (x->device != c0->device || ci.kv_dtype != RL_KV_BF16 || ci.n_full != c.n_full ||
            ci.n_head != c.n_head || ci.n_head_kv != c.n_head_kv || ci.head_dim != c.head_dim ||
            ci.n_rot != c.n_rot || ci.rms_eps != c.rms_eps || c.n_full < 1)
            return fail(c0, RL_EINVAL,
                        "context %d: a batch needs bf16 caches of the same shapes on one device",
                        i);
        if (x->shard_lo != 0 || x->seq_context != ci.context)
            return fail(c0, RL_EINVAL, "context %d holds a shard of a split sequence", i);
    }
    if (cudaSetDevice(c0->device) != cudaSuccess)
        return fail(c0, RL_ECUDA, "cudaSetDevice failed");
    rl_batch *b = new rl_batch();
    b->ctxs.assign(ctxs, ctxs + n);
    b->n = n;
    b->n_full = c.n_full;
    // splits per (sequence, KV head): about eight waves of walk CTAs in all
    const int64_t resident = (int64_t)std::max(1, c0->mma_per_sm[1]) * c0->num_sms;
    b->splits = (int)std::max<int64_t>(
        1, std::min<int64_t>(16, (8 * resident + (int64_t)c.n_head_kv * n - 1) /
                                     ((int64_t)c.n_head_kv * n)));
    const size_t rows_heads = (size_t)n * c.n_head;
    bool ok = cudaMalloc(&b->rows, sizeof(rl::BatchRow) * c.n_full * n) == cudaSuccess &&
              cudaMalloc(&b->maps, sizeof(CUtensorMap) * n) == cudaSuccess &&
              cudaMalloc(&b->part_o, sizeof(float) * rows_heads * b->splits * c.head_dim) ==
                  cudaSuccess &&
              cudaMalloc(&b->part_ml, sizeof(float) * rows_heads * b->splits * 2) == cudaSuccess &&
              cudaMalloc(&b->counters, sizeof(int) * n * c.n_head_kv * 8) == cudaSuccess &&
              cudaMemset(b->counters, 0, sizeof(int) * n * c.n_head_kv * 8) == cudaSuccess;
    if (ok) {
        std::vector<CUtensorMap> maps(n);
        std::vector<rl::BatchRow> rows((size_t)c.n_full * n);
        for (int i = 0; i < n; ++i) {
            rl_ctx *x = ctxs[i];
            maps[i] = x->kv_map;
            for (int l = 0; l < c.n_full; ++l) {
                rl::BatchRow &r = rows[(size_t)l * n + i];
                const rl_config &ci = x->cfg;
                r.map = b->maps + i;
                r.k_cache = kv_layer(x, l);
                r.v_cache = (char *)r.k_cache +
                            (size_t)ci.n_head_kv * ci.context * ci.head_dim * kv_elem(ci);
                r.q_norm = x->q_norm + (size_t)l * ci.head_dim;
                r.k_norm = x->k_norm + (size_t)l * ci.head_dim;
                r.rope_cs = x->rope_cs;
                r.rope_sn = x->rope_sn;
                r.context = ci.context;
                r.k_row0 = l * 2 * ci.n_head_kv * ci.context;
                r.v_row0 = r.k_row0 + ci.n_head_kv * ci.context;
            }
        }
        ok = cudaMemcpy(b->maps, maps.data(), sizeof(CUtensorMap) * n, cudaMemcpyHostToDevice) ==
                 cudaSuccess &&
             cudaMemcpy(b->rows, rows.data(), sizeof(rl::BatchRow) * rows.size(),
                        cudaMemcpyHostToDevice) == cudaSuccess;
    }
    if (!ok) {
        rl_batch_destroy(b);
        return fail(c0, RL_ENOMEM, "allocating the batch's %d rows failed", n);
    }
    *out = b;
    return RL_OK;
}

int rl_batch_full_attn(rl_batch *b, int layer, const int *pos, const float *qg, const float *k,
                       const float *v, float *out) {
    if (!b) return fail(nullptr, RL_EINVAL, "NULL batch");
    rl_ctx *ctx = b->ctxs[0];
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= b->n_full)
        return fail(ctx, RL_EINVAL, "full layer %d of %d", layer, b->n_full);
    if (!pos || !qg || !k || !v || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    if (((uintptr_t)qg | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15)
        return fail(ctx, RL_EINVAL, "qg, k, v and out must be 16-byte aligned");
    CK(ctx, cudaSetDevice(ctx->device));
    rl::DecodeArgs d{};
    d.qg = qg;
    d.k_in = k;
    d.v_in = v;
    d.part_o = b->part_o;
    d.part_ml = b->part_ml;
    d.counters = b->counters;
    d.out = out;
    d.status = ctx->status;
    d.pos = 0;
    d.t = b->n;
    d.context = c.context;
    d.n_head = c.n_head;
    d.n_kv = c.n_head_kv;
    d.n_rot = c.n_rot;
    d.theta_scale = ctx->theta_scale;
    d.eps = c.rms_eps;
    d.kv_bf16 = true;
    d.fused = true;
    d.rows = b->rows + (size_t)layer * b->n;
    d.batch_pos = pos;
    d.n_splits = b->splits;
    // each CTA's first tiles are its own; the rest come from the sequence's
    // counter, so CTAs of short and long sequences alike end near together
    d.chunk = 0;
    d.csize = 1;
    d.early_kv = false;
    d.early_tiles = (int)ctx->opt_early_tiles;
    {
        ProfScope ps(ctx, RL_PROF_DECODE);
        CK(ctx, rl::launch_decode_mma(d, ctx->kv_map, ctx->stream));
    }
    {
        ProfScope ps(ctx, RL_PROF_MERGE);
        CK(ctx, rl::launch_decode_combine(d, ctx->stream));
    }
    for (rl_ctx *x : b->ctxs) x->early_ok = false;
    return RL_OK;
}

int rl_merge_partials(rl_ctx *ctx, int n_parts, const float *parts, const float *qg,
                      float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (n_parts < 1 || !parts || !qg || !out)
        return fail(ctx, RL_EINVAL, "n_parts >= 1 and non-NULL buffers");
    CK(ctx, cudaSetDevice(ctx->device));
    {
        ProfScope ps(ctx, RL_PROF_MERGE);
        CK(ctx, rl::launch_merge_parts(parts, n_parts, ctx->cfg.n_head, qg, out, ctx->stream));
    }
    ctx->prev_dn = 0;
    return RL_OK;
}

int rl_full_attn_host(rl_ctx *ctx, int layer, int pos, int t, const float *qg, const float *k,
                      const float *v, float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (t < 1 || t > c.max_batch)
        return fail(ctx, RL_EINVAL, "a batch of %d rows, but the scratch was sized for %d", t,
                    c.max_batch);
    if (!qg || !k || !v || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t nqg = (size_t)t * 2 * c.head_dim * c.n_head;
    const size_t nk = (size_t)t * c.head_dim * c.n_head_kv;
    const size_t no = (size_t)t * c.head_dim * c.n_head;
    float *dout = ctx->stage, *dq = dout + no, *dk = dq + nqg, *dv = dk + nk;
    if (ctx->hpin && t <= ctx->hpin_rows) {
        // the inputs packed in the pinned staging in the device staging's
        // order (the previous call's copies have completed: every call ends
        // in a wait), one copy in; the status word and the output, one copy out
        float *hout = ctx->hpin, *hp = hout + no;
        std::memcpy(hp, qg, nqg * 4);
        std::memcpy(hp + nqg, k, nk * 4);
        std::memcpy(hp + nqg + nk, v, nk * 4);
        CK(ctx, cudaMemcpyAsync(dq, hp, (nqg + 2 * nk) * 4, cudaMemcpyHostToDevice, ctx->stream));
        int code = rl_full_attn(ctx, layer, pos, t, dq, dk, dv, dout);
        if (code) {
            cudaStreamSynchronize(ctx->stream);  // the staging's copy is done before reuse
            return code;
        }
        code = finish_host_call(ctx, no);
        std::memcpy(out, hout, no * 4);
        return code;
    }
    CK(ctx, cudaMemcpyAsync(dq, qg, nqg * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    int code = rl_full_attn(ctx, layer, pos, t, dq, dk, dv, dout);
    if (code) return code;
    CK(ctx, cudaMemcpyAsync(out, dout, no * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return check_status(ctx);
}

int rl_linear_attn(rl_ctx *ctx, int layer, int live, int t, const float *qkv, const float *z,
                   const float *alpha, const float *beta, float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_linear)
        return fail(ctx, RL_EINVAL, "linear layer %d of %d", layer, c.n_linear);
    if (t < 1 || t > c.max_batch)
        return fail(ctx, RL_EINVAL, "a batch of %d rows, but the scratch was sized for %d", t,
                    c.max_batch);
    if (live < 0 || live >= c.slots)
        return fail(ctx, RL_EINVAL, "live slot %d of a ring of %d", live, c.slots);
    if (!qkv || !z || !alpha || !beta || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    CK(ctx, cudaSetDevice(ctx->device));
    if (c.slots == 1 && ctx->dn_w && ctx->opt_chunk_rows > 0 && t >= ctx->opt_chunk_rows) {
        // chunked tensor-core prefill over the in-place state
        rl::DnChunkArgs d{};
        d.qkv = qkv;
        d.z = z;
        d.alpha = alpha;
        d.beta = beta;
        d.conv_state = ctx->conv + (size_t)layer * conv_layer_floats(c);
        d.ssm_state = ctx->ssm + (size_t)layer * ssm_layer_floats(c);
        d.conv1d = ctx->conv1d + (size_t)layer * conv_dim(c) * c.conv_kernel;
        d.ssm_a = ctx->ssm_a + (size_t)layer * c.n_v_heads;
        d.dt_bias = ctx->dt_bias + (size_t)layer * c.n_v_heads;
        d.norm = ctx->ssm_norm + (size_t)layer * c.d_state;
        d.out = out;
        d.qn = ctx->dn_qn;
        d.kn = ctx->dn_kn;
        d.qn_lo = ctx->dn_qn_lo;
        d.kn_lo = ctx->dn_kn_lo;
        d.qn_l2 = ctx->dn_qn_l2;
        d.kn_l2 = ctx->dn_kn_l2;
        d.vn_lo = ctx->dn_vn_lo;
        d.w_lo = ctx->dn_w_lo;
        d.qp_lo = ctx->dn_qp_lo;
        d.kp_lo = ctx->dn_kp_lo;
        d.p_lo = ctx->dn_p_lo;
        d.vn = ctx->dn_vn;
        d.lg = ctx->dn_lg;
        d.bt = ctx->dn_bt;
        d.w = ctx->dn_w;
        d.qp = ctx->dn_qp;
        d.kp = ctx->dn_kp;
        d.p = ctx->dn_p;
        d.ut = ctx->dn_ut;
        d.gc = ctx->dn_gc;
        d.opre = ctx->dn_opre;
        d.status = ctx->status;
        d.t = t;
        d.nc = (t + 63) / 64;
        d.n_k = c.n_k_heads;
        d.n_v = c.n_v_heads;
        d.live = live;
        d.slots = c.slots;
        d.eps = c.rms_eps;
        {
            ProfScope ps(ctx, RL_PROF_DN_CHUNK);
            const bool tc_scan = ctx->opt_dn_scan_tc && ctx->dn_scan_maps_ok;
            // the tcgen05 scan runs beside the chunk-local kernel
            const rl::DnOverlap ov{ctx->dn_scan_stream, ctx->dn_fork, ctx->dn_join};
            d.ready = tc_scan && ctx->opt_dn_overlap ? ctx->dn_ready : nullptr;
            d.ready_epoch = ctx->dn_ready_epoch;
            // beside the scan the chunk-local kernel gets the SMs the scan's n_v
            // CTAs leave
            d.local_ctas = std::max(1, ctx->num_sms - (d.ready ? c.n_v_heads : 0));
            d.local_next = ctx->dn_local_next;
            d.out_ready = d.ready ? ctx->dn_out_ready : nullptr;
            // the chunk-local kernel's tcgen05 form reads q and k by TMA, through
            // maps that end at this call's rows (the rows past them read as 0)
            rl::DnPlaneMaps pm;
            bool planes_ok = ctx->opt_dn_local_tc != 0;
            const uint64_t nk = c.n_k_heads, s = c.d_state;
            const __nv_bfloat16 *qp[3] = {ctx->dn_qn, ctx->dn_qn_lo, ctx->dn_qn_l2};
            const __nv_bfloat16 *kp[3] = {ctx->dn_kn, ctx->dn_kn_lo, ctx->dn_kn_l2};
            for (int x = 0; x < 3 && planes_ok; ++x)
                planes_ok = rl::encode_bf16_3d(&pm.q[x], qp[x], s, nk, (uint64_t)t, s * 2,
                                               nk * s * 2, 64, 1, 64) == cudaSuccess &&
                            rl::encode_bf16_3d(&pm.k[x], kp[x], s, nk, (uint64_t)t, s * 2,
                                               nk * s * 2, 64, 1, 64) == cudaSuccess;
            CK(ctx, rl::launch_dn_chunk(d, tc_scan ? &ctx->dn_scan_maps : nullptr, ctx->stream,
                                        tc_scan && ctx->opt_dn_overlap ? &ov : nullptr,
                                        planes_ok ? &pm : nullptr));
        }
        // a step of this layer right after must not read the state early
        ctx->prev_dn = 1;
        ctx->prev_layer = layer;
        return RL_OK;
    }
    rl::LinArgs a{};
    a.qkv = qkv;
    a.z = z;
    a.alpha = alpha;
    a.beta = beta;
    a.conv_state = ctx->conv + (size_t)layer * conv_layer_floats(c);
    a.ssm_state = ctx->ssm + (size_t)layer * ssm_layer_floats(c);
    a.conv1d = ctx->conv1d + (size_t)layer * conv_dim(c) * c.conv_kernel;
    a.ssm_a = ctx->ssm_a + (size_t)layer * c.n_v_heads;
    a.dt_bias = ctx->dt_bias + (size_t)layer * c.n_v_heads;
    a.norm = ctx->ssm_norm + (size_t)layer * c.d_state;
    a.out = out;
    a.status = ctx->status;
    a.t = t;
    a.slots = c.slots;
    a.live = live;
    a.s = c.d_state;
    a.n_k = c.n_k_heads;
    a.n_v = c.n_v_heads;
    a.kernel = c.conv_kernel;
    a.eps = c.rms_eps;
    a.early_state = !(ctx->prev_dn && ctx->prev_layer == layer);
    a.ssm_row0 = layer * c.n_v_heads * c.slots * c.d_state;
    {
        ProfScope ps(ctx, RL_PROF_DN_STEP);
        if (ctx->opt_dn_rows && ctx->ssm_map_ok && rl::dn_rows_fits(a))
            CK(ctx, rl::launch_dn_rows(a, ctx->ssm_map, ctx->stream));
        else
            CK(ctx, rl::launch_dn_step(a, ctx->stream));
    }
    ctx->prev_dn = 1;
    ctx->prev_layer = layer;
    return RL_OK;
}

int rl_linear_attn_host(rl_ctx *ctx, int layer, int live, int t, const float *qkv,
                        const float *z, const float *alpha, const float *beta, float *out) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (t < 1 || t > c.max_batch)
        return fail(ctx, RL_EINVAL, "a batch of %d rows, but the scratch was sized for %d", t,
                    c.max_batch);
    if (!qkv || !z || !alpha || !beta || !out) return fail(ctx, RL_EINVAL, "NULL input or output");
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t nx = (size_t)t * conv_dim(c), nz = (size_t)t * c.n_v_heads * c.d_state;
    const size_t ng = (size_t)t * c.n_v_heads;
    float *dout = ctx->stage, *dx = dout + nz, *dz = dx + nx, *da = dz + nz, *db = da + ng;
    if (ctx->hpin && t <= ctx->hpin_rows) {
        // as rl_full_attn_host: packed pinned inputs, one copy in, one out
        float *hout = ctx->hpin, *hp = hout + nz;
        std::memcpy(hp, qkv, nx * 4);
        std::memcpy(hp + nx, z, nz * 4);
        std::memcpy(hp + nx + nz, alpha, ng * 4);
        std::memcpy(hp + nx + nz + ng, beta, ng * 4);
        CK(ctx, cudaMemcpyAsync(dx, hp, (nx + nz + 2 * ng) * 4, cudaMemcpyHostToDevice,
                                ctx->stream));
        int code = rl_linear_attn(ctx, layer, live, t, dx, dz, da, db, dout);
        if (code) {
            cudaStreamSynchronize(ctx->stream);  // the staging's copy is done before reuse
            return code;
        }
        code = finish_host_call(ctx, nz);
        std::memcpy(out, hout, nz * 4);
        return code;
    }
    CK(ctx, cudaMemcpyAsync(dx, qkv, nx * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(dz, z, nz * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(da, alpha, ng * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(db, beta, ng * 4, cudaMemcpyHostToDevice, ctx->stream));
    int code = rl_linear_attn(ctx, layer, live, t, dx, dz, da, db, dout);
    if (code) return code;
    CK(ctx, cudaMemcpyAsync(out, dout, nz * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return check_status(ctx);
}

int rl_accept(rl_ctx *ctx, int rows) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (rows < 1)
        return fail(ctx, RL_EINVAL,
                    "a batch commits at least its first row; accept(%d) would leave the last "
                    "row of the batch live, not the state from before it",
                    rows);
    if ((int64_t)ctx->pos + rows > ctx->cfg.context)
        return fail(ctx, RL_ECONTEXT, "accept(%d) at pos %d runs past the context of %d", rows,
                    ctx->pos, ctx->cfg.context);
    ctx->pos += rows;
    ctx->live = (ctx->live + rows) % ctx->cfg.slots;
    return RL_OK;
}

int rl_pos(const rl_ctx *ctx) { return ctx ? ctx->pos : -1; }
int rl_live(const rl_ctx *ctx) { return ctx ? ctx->live : -1; }

int rl_sync(rl_ctx *ctx) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    return check_status(ctx);
}

// ---- projections ---------------------------------------------------------------

int rl_act_quantize(rl_ctx *ctx, const float *x, int t, int k) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!x || t < 1 || k < 1) return fail(ctx, RL_EINVAL, "x, t >= 1 and k >= 1 are required");
    if (((uintptr_t)x) & 15) return fail(ctx, RL_EINVAL, "x must be 16-byte aligned");
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t blocks = (size_t)t * ((k + 255) / 256);
    if (blocks > ctx->act_cap) {
        // grows once to the largest batch seen; a call that grows it allocates
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        if (ctx->act_d) cudaFree(ctx->act_d);
        if (ctx->act_qs) cudaFree(ctx->act_qs);
        if (ctx->act_bs) cudaFree(ctx->act_bs);
        ctx->act_d = nullptr, ctx->act_qs = nullptr, ctx->act_bs = nullptr, ctx->act_cap = 0;
        CK(ctx, cudaMalloc((void **)&ctx->act_d, blocks * sizeof(float)));
        CK(ctx, cudaMalloc((void **)&ctx->act_qs, blocks * 256));
        CK(ctx, cudaMalloc((void **)&ctx->act_bs, blocks * 16 * sizeof(int16_t)));
        ctx->act_cap = blocks;
    }
    CK(ctx, rl::launch_q8k_quantize(x, t, k, ctx->act_d, ctx->act_qs, ctx->act_bs, ctx->stream));
    ctx->act_t = t;
    ctx->act_k = k;
    ctx->early_ok = false;
    ctx->prev_dn = 0;
    return RL_OK;
}

namespace {
// The group's parts checked and packed (rows of k values each).
int make_group(rl_ctx *ctx, int k, int n, const int *types, const void *const *ws,
               const int *rows, float *const *outs, rl::MatvecGroup *g) {
    if (n < 1 || n > rl::kMatvecGroupMax || !types || !ws || !rows || !outs)
        return fail(ctx, RL_EINVAL, "a group of 1 to %d weights", rl::kMatvecGroupMax);
    *g = rl::MatvecGroup{};
    g->n = n;
    int64_t total = 0;
    for (int p = 0; p < n; ++p) {
        const size_t stride = rl::proj_row_bytes(types[p], k);
        if (stride == 0)
            return fail(ctx, RL_EUNSUPPORTED,
                        "weight type %d: Q4_K (12), Q6_K (14) and Q8_0 (8) only", types[p]);
        if (!ws[p] || !outs[p] || rows[p] < 1)
            return fail(ctx, RL_EINVAL, "weight %d: w, out and rows >= 1 are required", p);
        if (((uintptr_t)outs[p] & 3)) return fail(ctx, RL_EINVAL, "out must be 4-byte aligned");
        if (types[p] == 12 && ((uintptr_t)ws[p] & 15))
            return fail(ctx, RL_EINVAL,
                        "Q4_K rows are read in 16-byte pieces: w must be 16-byte aligned");
        if (stride + 30 > (size_t)rl::kMatvecRowSmemMax)
            return fail(ctx, RL_EUNSUPPORTED, "rows of %zu bytes: at most %d", stride,
                        rl::kMatvecRowSmemMax - 30);
        g->type[p] = types[p];
        g->rows[p] = rows[p];
        g->stride[p] = stride;
        g->w[p] = ws[p];
        g->out[p] = outs[p];
        total += rows[p];
    }
    if (total > (1 << 30)) return fail(ctx, RL_EINVAL, "too many rows in one group");
    return RL_OK;
}
}  // namespace

int rl_matvec_group(rl_ctx *ctx, int n, const int *types, const void *const *ws,
                    const int *rows, float *const *outs) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (ctx->act_k < 1) return fail(ctx, RL_EINVAL, "no activations quantized (rl_act_quantize)");
    rl::MatvecGroup g;
    const int code = make_group(ctx, ctx->act_k, n, types, ws, rows, outs, &g);
    if (code) return code;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, rl::launch_matvec_group(g, ctx->act_k, ctx->act_d, ctx->act_qs, ctx->act_bs, ctx->act_t,
                                    ctx->stream));
    ctx->early_ok = false;
    ctx->prev_dn = 0;
    return RL_OK;
}

int rl_matmul_group(rl_ctx *ctx, const float *x, int t, int k, int n, const int *types,
                    const void *const *ws, const int *rows, float *const *outs) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (!x || t < 1 || k < 1) return fail(ctx, RL_EINVAL, "x, t >= 1 and k >= 1 are required");
    if (((uintptr_t)x) & 15) return fail(ctx, RL_EINVAL, "x must be 16-byte aligned");
    rl::MatvecGroup g;
    int code = make_group(ctx, k, n, types, ws, rows, outs, &g);
    if (code) return code;
    size_t stride_max = 0;
    for (int p = 0; p < n; ++p) stride_max = std::max(stride_max, g.stride[p]);
    if (rl::matmul_group_smem(t, k, stride_max) > (size_t)rl::kMatmulSmemMax) {
        // too many activation rows to quantize in every CTA: two launches
        if ((code = rl_act_quantize(ctx, x, t, k))) return code;
        return rl_matvec_group(ctx, n, types, ws, rows, outs);
    }
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, rl::launch_matmul_group(g, x, t, k, ctx->stream));
    ctx->early_ok = false;
    ctx->prev_dn = 0;
    return RL_OK;
}

int rl_matvec(rl_ctx *ctx, int ggml_type, const void *w, int rows, float *out) {
    return rl_matvec_group(ctx, 1, &ggml_type, &w, &rows, &out);
}

int rl_set_option(rl_ctx *ctx, int option, int64_t value) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (value < 0) return fail(ctx, RL_EINVAL, "option values are >= 0");
    switch (option) {
    case RL_OPT_SPLITS: ctx->opt_splits = value; return RL_OK;
    case RL_OPT_PREFILL_ROWS: ctx->opt_prefill_rows = value; return RL_OK;
    case RL_OPT_CHUNK_ROWS: ctx->opt_chunk_rows = value; return RL_OK;
    case RL_OPT_VERIFY_TC:
        if (value > 1) return fail(ctx, RL_EINVAL, "verify option must be 0 or 1");
        ctx->opt_verify_tc = value;
        return RL_OK;
    case RL_OPT_DN_ROWS:
        if (value > 1) return fail(ctx, RL_EINVAL, "the rows-kernel option must be 0 or 1");
        ctx->opt_dn_rows = value;
        return RL_OK;
    case RL_OPT_EARLY_TILES:
        if (value < 1 || value > 3) return fail(ctx, RL_EINVAL, "early tiles must be 1, 2 or 3");
        ctx->opt_early_tiles = value;
        return RL_OK;
    case RL_OPT_CLUSTER:
        if (value != 0 && value != 1 && value != 2 && value != 4 && value != 8)
            return fail(ctx, RL_EINVAL, "cluster size must be 0 (automatic), 1, 2, 4 or 8");
        ctx->opt_cluster = value;
        return RL_OK;
    case RL_OPT_WAIT_LIMIT_US:
        if (value > 60000000)
            return fail(ctx, RL_EINVAL, "a wait limit above 60 s is not a limit");
        ctx->opt_wait_limit_us = value;
        return RL_OK;
    case RL_OPT_DN_SCAN_TC:
        if (value > 1) return fail(ctx, RL_EINVAL, "the scan option must be 0 or 1");
        ctx->opt_dn_scan_tc = value;
        return RL_OK;
    case RL_OPT_DN_OVERLAP:
        if (value > 1) return fail(ctx, RL_EINVAL, "the overlap option must be 0 or 1");
        ctx->opt_dn_overlap = value;
        return RL_OK;
    case RL_OPT_DN_LOCAL_TC:
        if (value > 1) return fail(ctx, RL_EINVAL, "the chunk-local option must be 0 or 1");
        ctx->opt_dn_local_tc = value;
        return RL_OK;
    case RL_OPT_WALK_SPANS:
        if (value > 1) return fail(ctx, RL_EINVAL, "the span option must be 0 or 1");
        CK(ctx, cudaSetDevice(ctx->device));
        if (value && !ctx->spans) {
            if (ctx->cfg.n_full < 1) return RL_OK;
            CK(ctx, cudaMalloc((void **)&ctx->spans,
                               (size_t)ctx->cfg.n_full * 4 * sizeof(unsigned long long)));
            return reset_spans(ctx);
        }
        if (!value && ctx->spans) {
            CK(ctx, cudaStreamSynchronize(ctx->stream));
            CK(ctx, cudaFree(ctx->spans));
            ctx->spans = nullptr;
        }
        return RL_OK;
    default: return fail(ctx, RL_EINVAL, "unknown option %d", option);
    }
}

int64_t rl_get_option(const rl_ctx *ctx, int option) {
    if (!ctx) return -1;
    switch (option) {
    case RL_OPT_SPLITS: return ctx->opt_splits;
    case RL_OPT_PREFILL_ROWS: return ctx->opt_prefill_rows;
    case RL_OPT_CHUNK_ROWS: return ctx->opt_chunk_rows;
    case RL_OPT_CLUSTER: return ctx->opt_cluster;
    case RL_OPT_EARLY_TILES: return ctx->opt_early_tiles;
    case RL_OPT_VERIFY_TC: return ctx->opt_verify_tc;
    case RL_OPT_DN_ROWS: return ctx->opt_dn_rows;
    case RL_OPT_WAIT_LIMIT_US: return ctx->opt_wait_limit_us;
    case RL_OPT_WALK_SPANS: return ctx->spans ? 1 : 0;
    case RL_OPT_DN_SCAN_TC: return ctx->opt_dn_scan_tc;
    case RL_OPT_DN_OVERLAP: return ctx->opt_dn_overlap;
    case RL_OPT_DN_LOCAL_TC: return ctx->opt_dn_local_tc;
    default: return -1;
    }
}

int rl_profile_enable(rl_ctx *ctx, int on) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    ctx->prof_on = on != 0;
    return RL_OK;
}

int rl_profile_read(rl_ctx *ctx, int kernel, double *total_ms, int64_t *launches) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    if (kernel < 0 || kernel >= RL_PROF_KERNELS)
        return fail(ctx, RL_EINVAL, "unknown kernel %d", kernel);
    CK(ctx, cudaSetDevice(ctx->device));
    if (kernel == RL_PROF_WALK_SPAN) {
        double ns = 0.0;
        int64_t n = 0;
        if (ctx->spans) {
            std::vector<unsigned long long> h((size_t)ctx->cfg.n_full * 4);
            CK(ctx, cudaStreamSynchronize(ctx->stream));
            CK(ctx, cudaMemcpy(h.data(), ctx->spans, h.size() * sizeof(h[0]),
                               cudaMemcpyDeviceToHost));
            for (int l = 0; l < ctx->cfg.n_full; ++l) {
                ns += (double)h[4 * l + 2];
                n += (int64_t)h[4 * l + 3];
            }
        }
        if (total_ms) *total_ms = ns * 1e-6;
        if (launches) *launches = n;
        return RL_OK;
    }
    if (drain_profile(ctx)) return fail(ctx, RL_ECUDA, "profile events could not be read");
    if (total_ms) *total_ms = ctx->prof_ms[kernel];
    if (launches) *launches = ctx->prof_launches[kernel];
    return RL_OK;
}

int rl_profile_reset(rl_ctx *ctx) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    CK(ctx, cudaSetDevice(ctx->device));
    drain_profile(ctx);
    for (int k = 0; k < RL_PROF_KERNELS; ++k) ctx->prof_ms[k] = 0.0, ctx->prof_launches[k] = 0;
    return ctx->spans ? reset_spans(ctx) : RL_OK;
}

// ---- state access ----------------------------------------------------------

static int kv_io(rl_ctx *ctx, int layer, int p0, int n, float *buf, int where, bool write) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_full || p0 < 0 || n < 1 || (int64_t)p0 + n > c.context || !buf)
        return fail(ctx, RL_EINVAL, "KV range %d+%d of layer %d is outside the cache", p0, n, layer);
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t elems = (size_t)2 * c.n_head_kv * n * c.head_dim;
    float *dev = buf;
    if (where == 0) CK(ctx, cudaMallocAsync((void **)&dev, elems * 4, ctx->stream));
    auto done = [&](int code) {
        if (where == 0) {
            cudaFreeAsync(dev, ctx->stream);
            cudaStreamSynchronize(ctx->stream);
        }
        return code;
    };
    if (write && where == 0)
        if (h2d(ctx, dev, buf, elems * 4) != cudaSuccess)
            return done(fail(ctx, RL_ECUDA, "copy of the KV rows failed"));
    void *kc = kv_layer(ctx, layer);
    void *vc = (char *)kc + (size_t)c.n_head_kv * c.context * c.head_dim * kv_elem(c);
    if (write) ctx->early_ok = false;
    cudaError_t e = write ? rl::launch_kv_fill(kc, vc, dev, c.n_head_kv, c.context, c.head_dim,
                                               p0, n, c.kv_dtype == RL_KV_BF16, ctx->stream)
                          : rl::launch_kv_read(kc, vc, dev, c.n_head_kv, c.context, c.head_dim,
                                               p0, n, c.kv_dtype == RL_KV_BF16, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess && !write && where == 0) {
        e = cudaMemcpyAsync(buf, dev, elems * 4, cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    }
    if (e != cudaSuccess) return done(fail(ctx, RL_ECUDA, "KV access: %s", cudaGetErrorString(e)));
    return done(RL_OK);
}

int rl_write_kv(rl_ctx *ctx, int layer, int p0, int n, const float *src, int where) {
    return kv_io(ctx, layer, p0, n, (float *)src, where, true);
}
int rl_read_kv(rl_ctx *ctx, int layer, int p0, int n, float *dst, int where) {
    return kv_io(ctx, layer, p0, n, dst, where, false);
}

static int state_io(rl_ctx *ctx, int layer, float *buf, int where, bool write, bool ssm) {
    if (!ctx) return fail(nullptr, RL_EINVAL, "NULL context");
    const rl_config &c = ctx->cfg;
    if (layer < 0 || layer >= c.n_linear || !buf)
        return fail(ctx, RL_EINVAL, "linear layer %d of %d", layer, c.n_linear);
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t n = ssm ? ssm_layer_floats(c) : conv_layer_floats(c);
    float *dev = (ssm ? ctx->ssm : ctx->conv) + (size_t)layer * n;
    const cudaMemcpyKind kind = write ? (where ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice)
                                      : (where ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost);
    CK(ctx, write ? cudaMemcpyAsync(dev, buf, n * 4, kind, ctx->stream)
                  : cudaMemcpyAsync(buf, dev, n * 4, kind, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    return RL_OK;
}

int rl_write_conv(rl_ctx *ctx, int layer, const float *src, int where) {
    return state_io(ctx, layer, (float *)src, where, true, false);
}
int rl_read_conv(rl_ctx *ctx, int layer, float *dst, int where) {
    return state_io(ctx, layer, dst, where, false, false);
}
int rl_write_ssm(rl_ctx *ctx, int layer, const float *src, int where) {
    return state_io(ctx, layer, (float *)src, where, true, true);
}
int rl_read_ssm(rl_ctx *ctx, int layer, float *dst, int where) {
    return state_io(ctx, layer, dst, where, false, true);
}

}  // extern "C"
