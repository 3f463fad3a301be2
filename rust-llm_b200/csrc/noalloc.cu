// rl_full_attn_noalloc: the full-attention step for callers that cannot
// allocate device memory.
//
// Who needs it.  A caller that plans every byte of device memory up front
// and must not allocate once tokens are flowing (a serving loop held to the
// reference runner's "the pass allocates nothing" guarantee), or a plug-in
// that runs inside another framework's memory budget and owns no context,
// cannot call cudaMalloc or hold an rl_ctx.  This entry point needs neither:
// the caller passes its own KV cache, weights, inputs and outputs, and the
// scratch the kernels need (normalised queries, split partials, arrival
// counters) lives in one file-scope __device__ array of RL_NOALLOC_SCRATCH_BYTES,
// which every GPU that loads the library holds until the process exits.
//
// It runs the multi-row path of rl_full_attn (prologue kernel, then the
// split-KV decode kernel reading the staged queries) with its scratch
// pointers aimed into that array.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "rlcuda.h"

namespace {

// The shared scratch.  Host code only ever sees this name as a host-side
// stand-in: its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) unsigned char noalloc_scratch[RL_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct DeviceState {
    bool ready = false;
    unsigned char *scratch = nullptr;  // device address of noalloc_scratch
    int num_sms = 0;
    int max_clusters[2][4] = {};       // [kv bf16][log2 cluster size], unfused kernel
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// Failures are described through rl_last_error(NULL), as for any call
// without a context.
int fail(int code, const char *msg) {
    rl::set_thread_error(msg);
    return code;
}

// First call on a device, with that device current: resolve the array's
// device address and the kernels' launch limits.
int setup(int device, DeviceState **out) {
    if (device < 0 || device >= kMaxDevices) return fail(RL_EINVAL, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState &d = g_dev[device];
    if (!d.ready) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scratch);
        if (e != cudaSuccess) return fail(RL_ECUDA, "cudaGetSymbolAddress of the scratch failed");
        if (rl::init_decode_kernels() != cudaSuccess)
            return fail(RL_ECUDA, "decode kernel attribute set-up failed");
        if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device) !=
            cudaSuccess)
            return fail(RL_ECUDA, "device query failed");
        for (int b = 0; b < 2; ++b)
            for (int lc = 0; lc < 4; ++lc)
                d.max_clusters[b][lc] = rl::decode_max_active_clusters(b == 1, false, 1 << lc);
        d.scratch = static_cast<unsigned char *>(p);
        d.ready = true;
    }
    *out = &d;
    return RL_OK;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// The array's last 256 bytes hold the status word the kernels OR a
// rl::DEV_* bit into when a bounded wait gives up.  It is sticky: calls
// never clear it; rl_noalloc_status reads and clears it.  The rest of the
// array is the per-call layout.
constexpr size_t kStatusOffset = RL_NOALLOC_SCRATCH_BYTES - 256;

}  // namespace

extern "C" int rl_full_attn_noalloc(const rl_config *cfg, void *stream, void *k_cache,
                                    void *v_cache, const float *q_norm, const float *k_norm,
                                    int pos, int t, const float *qg, const float *k,
                                    const float *v, float *out) {
    if (!cfg || !k_cache || !v_cache || !q_norm || !k_norm || !qg || !k || !v || !out)
        return fail(RL_EINVAL, "NULL argument");
    const rl_config &c = *cfg;
    if (c.head_dim != 256 || c.n_head_kv < 1 || c.n_head != 4 * c.n_head_kv)
        return fail(RL_EUNSUPPORTED, "built for head_dim 256 and 4 query heads per KV head");
    if (c.kv_dtype != RL_KV_F32 && c.kv_dtype != RL_KV_BF16)
        return fail(RL_EINVAL, "kv_dtype is neither RL_KV_F32 nor RL_KV_BF16");
    if (c.n_rot < 0 || c.n_rot > c.head_dim || (c.n_rot & 1))
        return fail(RL_EINVAL, "n_rot must be even and at most head_dim");
    if (c.n_rot % 16)
        return fail(RL_EINVAL,
                    "the kernels rotate whole 8-dim lanes: n_rot must be a multiple of 16");
    if (t < 1 || pos < 0 || (int64_t)pos + t > c.context)
        return fail(RL_ECONTEXT, "the rows do not fit the context");
    if (((uintptr_t)qg | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15)
        return fail(RL_EINVAL, "qg, k, v and out must be 16-byte aligned");
    // the prologue reads the norm weights as 16-byte vectors and the walks
    // read the caches with 16-byte loads and bulk copies
    if (((uintptr_t)q_norm | (uintptr_t)k_norm) & 15)
        return fail(RL_EINVAL, "q_norm and k_norm must be 16-byte aligned");
    if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15)
        return fail(RL_EINVAL, "k_cache and v_cache must be 16-byte aligned");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(RL_ECUDA, "cudaGetDevice failed");
    DeviceState *d = nullptr;
    int code = setup(device, &d);
    if (code) return code;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool bf16 = c.kv_dtype == RL_KV_BF16;
    const int hd = c.head_dim, nh = c.n_head, nkv = c.n_head_kv;

    // split-KV grid: one wave of resident clusters, as rl_full_attn sizes it
    const int64_t n_kv_max = (int64_t)pos + t;
    const int P = rl::decode_positions_per_tile(bf16);
    const int64_t tiles = (n_kv_max + P - 1) / P;
    const int64_t groups = (int64_t)nkv * t;
    int64_t splits = 0;
    int csize = 1;
    for (int lc = 3; lc >= 0; --lc) {
        const int cs = 1 << lc;
        int64_t per = (int64_t)d->max_clusters[bf16 ? 1 : 0][lc] / groups * cs;
        per = std::min<int64_t>(per, (tiles + cs - 1) / cs * cs);
        per = std::min<int64_t>(per, (int64_t)cs * 64);
        per = per / cs * cs;
        if (per * 8 > splits * 9) splits = per, csize = cs;
    }
    if (splits < 1) splits = 1, csize = 1;
    int64_t chunk = (n_kv_max + splits - 1) / splits;
    chunk = (chunk + P - 1) / P * P;
    const int64_t n_cl = splits / csize;

    // scratch layout: queries | cross-cluster partials | (max, sum) pairs | counters
    const size_t q_bytes = align256((size_t)t * nh * hd * sizeof(float));
    const size_t po_bytes = align256((size_t)t * nh * n_cl * hd * sizeof(float));
    const size_t pml_bytes = align256((size_t)t * nh * n_cl * 8 * 2 * sizeof(float));
    const size_t cnt_bytes = align256((size_t)t * nkv * 8 * sizeof(int));
    if (q_bytes + po_bytes + pml_bytes + cnt_bytes > kStatusOffset)
        return fail(RL_EINVAL,
                    "this call needs more scratch than RL_NOALLOC_SCRATCH_BYTES holds; use fewer "
                    "rows or rl_full_attn");
    unsigned char *base = d->scratch;
    float *q_f32 = reinterpret_cast<float *>(base);
    float *part_o = reinterpret_cast<float *>(base + q_bytes);
    float *part_ml = reinterpret_cast<float *>(base + q_bytes + po_bytes);
    int *counters = reinterpret_cast<int *>(base + q_bytes + po_bytes + pml_bytes);

    // the arrival counters must start at zero; a previous call that gave up
    // part-way could have left them otherwise
    if (cudaMemsetAsync(counters, 0, cnt_bytes, st) != cudaSuccess)
        return fail(RL_ECUDA, "clearing the counters failed");

    rl::FullArgs a{};
    a.qg = qg;
    a.k = k;
    a.v = v;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.q_f32 = q_f32;
    a.q_bf16 = nullptr;
    a.t = t;
    a.pos = pos;
    a.n_head = nh;
    a.n_kv = nkv;
    a.hd = hd;
    a.context = c.context;
    a.n_rot = c.n_rot;
    a.theta_scale = c.n_rot > 0 ? std::pow(c.rope_theta, -2.0f / (float)c.n_rot) : 1.0f;
    a.eps = c.rms_eps;
    a.kv_bf16 = bf16;
    if (rl::launch_full_prologue(a, st) != cudaSuccess) return fail(RL_ECUDA, "prologue launch failed");

    rl::DecodeArgs dd{};
    dd.qg = qg;
    dd.k_in = k;
    dd.v_in = v;
    dd.q_f32 = q_f32;
    dd.q_norm = q_norm;
    dd.k_norm = k_norm;
    dd.rope_cs = nullptr;
    dd.rope_sn = nullptr;
    dd.k_cache_v = k_cache;
    dd.v_cache_v = v_cache;
    dd.part_o = part_o;
    dd.part_ml = part_ml;
    dd.counters = counters;
    dd.out = out;
    dd.status = reinterpret_cast<int *>(base + kStatusOffset);
    dd.pos = pos;
    dd.t = t;
    dd.context = c.context;
    dd.n_head = nh;
    dd.n_kv = nkv;
    dd.chunk = (int)chunk;
    dd.n_splits = (int)splits;
    dd.csize = csize;
    dd.n_rot = c.n_rot;
    dd.theta_scale = a.theta_scale;
    dd.eps = c.rms_eps;
    dd.kv_bf16 = bf16;
    dd.fused = false;
    if (rl::launch_decode(dd, st) != cudaSuccess) return fail(RL_ECUDA, "decode launch failed");
    return RL_OK;
}

extern "C" int rl_noalloc_status(void *stream) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(RL_ECUDA, "cudaGetDevice failed");
    DeviceState *d = nullptr;
    int code = setup(device, &d);
    if (code) return code;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int *word = reinterpret_cast<int *>(d->scratch + kStatusOffset);
    int bits = 0;
    // read, then clear, in stream order behind the calls it reports on
    if (cudaMemcpyAsync(&bits, word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemsetAsync(word, 0, sizeof(int), st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(RL_ECUDA, "reading the no-alloc status word failed");
    if (bits & rl::DEV_TIMEOUT)
        return fail(RL_ETIMEOUT, "a kernel of an earlier rl_full_attn_noalloc call gave up a "
                                 "bounded wait; its output is not valid");
    if (bits) return fail(RL_EINVAL, "a kernel of an earlier rl_full_attn_noalloc call flagged "
                                     "a bad argument");
    return RL_OK;
}
