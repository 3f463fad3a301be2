// Gated DeltaNet, token-sequential step kernel for sm_100a.
//
// One fused kernel runs t sequential rows of a layer: the causal depthwise
// conv over the ring's history, SiLU, q/k L2 norm, the decay and beta gates,
// the delta rule on the 128x128 f32 state and the gated RMSNorm.  It is the
// decode step (t = 1), the speculative-verify pass (t rows writing t ring
// slots) and the exact token-sequential path for any t.
//
// Reference: Exec::linear_attn (crates/rust-llm/src/forward.rs:1530-1652),
// delta_net / delta_net_into (:1906-2010), depthwise_conv(_into) (:2018-2059),
// l2_norm_in_place (:1720-1727), softplus / sigmoid / silu (:1730-1743).
//
// Work split.  The state's output components j are independent of each other
// (each has its own sk_j, delta_j and readout o_j), so a value head's
// [i][j] state is split by columns over a cluster of S/JC CTAs, each holding
// its 128 x JC block in registers for the whole batch: 8 warps x 16 rows, one
// column per lane, every load a coalesced 128-byte row segment.  The value
// heads that share a key head (vh = kh + g*n_k) sit in one cluster of
// CL*GV CTAs: the only head-wide quantity, the gated RMSNorm's sum of squares
// over j, is exchanged through distributed shared memory, and one cluster
// barrier after the history is read lets the key head's single writer update
// the shared q/k conv history without racing the CTAs that read it.
//
// The kernel is launched as a programmatic dependent (PDL) of the kernel
// before it and triggers its own dependents as soon as its grid-dependency
// wait returns, so when a kernel starts, every kernel before the one just
// ahead of it has completed.  What the context owns and only this kernel
// writes (the state block and conv history of this layer) is therefore safe
// to load before the wait unless the kernel just ahead is a step of the same
// layer; the host passes `early_state` accordingly.  The conv weights and
// gate constants are loaded before the wait always (set once, synchronously);
// the row inputs are read, and every global write is made, after it.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace rl {
namespace dn {
constexpr int S = 128;          // d_state the kernel is built for
constexpr int JC = 32;          // state columns per CTA
constexpr int CL = S / JC;      // CTAs per value head (the cluster)
constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int RPW = S / WARPS;  // state rows per warp (16)
constexpr int HIST = 3;         // conv_kernel - 1
}  // namespace dn

// grid (CL * GV, n_k), cluster (CL * GV): blockIdx.x = grp * CL + cb
__global__ void __launch_bounds__(dn::THREADS, 1) dn_step_kernel(const LinArgs a) {
    using namespace dn;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float q_s[S], k_s[S], v_s[JC], d_s[JC];
    __shared__ float red[WARPS][JC];
    __shared__ double nred[WARPS];
    __shared__ double cl_part[2];

    const int n_k = a.n_k, n_v = a.n_v, slots = a.slots;
    const int cb = blockIdx.x % CL, grp = blockIdx.x / CL, kh = blockIdx.y;
    const int vh = kh + grp * n_k;  // so that vh % n_k == kh, as forward.rs:1602-1609
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int key_dim = n_k * S, d_inner = n_v * S, conv_dim = 2 * key_dim + d_inner;
    const int j0 = cb * JC, j = j0 + lane;
    const float scale = 1.0f / sqrtf((float)S);
    const float shrink = 1.0f / sqrtf((float)S);
    const float l2_eps = a.eps / (float)S;

    // channels: thread tid convolves q (tid < S) or k (tid >= S) channel of
    // key head kh; threads tid < JC also take value channel j0 + tid
    const int ch0 = tid < S ? kh * S + tid : key_dim + kh * S + (tid - S);
    const bool has_v = tid < JC;
    const int ch1 = 2 * key_dim + vh * S + j0 + tid;
    const bool write_qk = blockIdx.x == 0;  // one writer per key head
    float w0[4], h0[HIST], w1[4] = {0, 0, 0, 0}, h1[HIST] = {0, 0, 0};
#pragma unroll
    for (int e = 0; e < 4; ++e) w0[e] = a.conv1d[(size_t)ch0 * 4 + e];
    if (has_v) {
#pragma unroll
        for (int e = 0; e < 4; ++e) w1[e] = a.conv1d[(size_t)ch1 * 4 + e];
    }
    const float dt_bias = a.dt_bias[vh], ssm_a = a.ssm_a[vh];
    const float wnorm = a.norm[j];
    // state block, rows warp*RPW .. +RPW, column j, and the conv history,
    // both read from slot `live`
    float st[RPW];
    const float *hist_live = a.conv_state + (size_t)a.live * conv_dim * HIST;
    auto load_state = [&]() {
        const float *src = a.ssm_state + ((size_t)(vh * slots + a.live) * S) * S + j;
#pragma unroll
        for (int ii = 0; ii < RPW; ++ii) st[ii] = src[(size_t)(warp * RPW + ii) * S];
#pragma unroll
        for (int e = 0; e < HIST; ++e) h0[e] = hist_live[(size_t)ch0 * HIST + e];
        if (has_v) {
#pragma unroll
            for (int e = 0; e < HIST; ++e) h1[e] = hist_live[(size_t)ch1 * HIST + e];
        }
    };
    if (a.early_state) load_state();
    // the row inputs come from the kernel before; so does the right to write
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!a.early_state) load_state();
    // every CTA of the cluster holds the history it read; only now may the
    // writer overwrite slot `live` (slots == 1, or a batch that wraps the ring)
    cluster.sync();

    for (int r = 0; r < a.t; ++r) {
        const int to = (a.live + r + 1) % slots;
        // ---- conv (forward.rs:2018-2059: x*w[3] first, then history taps
        // in order) and SiLU
        const float *x = a.qkv + (size_t)r * conv_dim;
        const float x0 = x[ch0];
        float c0 = __fmul_rn(x0, w0[3]);
#pragma unroll
        for (int e = 0; e < HIST; ++e) c0 = __fadd_rn(c0, __fmul_rn(h0[e], w0[e]));
        h0[0] = h0[1];
        h0[1] = h0[2];
        h0[2] = x0;
        float c1 = 0.0f;
        if (has_v) {
            const float x1 = x[ch1];
            c1 = __fmul_rn(x1, w1[3]);
#pragma unroll
            for (int e = 0; e < HIST; ++e) c1 = __fadd_rn(c1, __fmul_rn(h1[e], w1[e]));
            h1[0] = h1[1];
            h1[1] = h1[2];
            h1[2] = x1;
        }
        if (slots > 1 || r == a.t - 1) {  // the history this row leaves behind
            float *hs = a.conv_state + (size_t)to * conv_dim * HIST;
            if (write_qk)
#pragma unroll
                for (int e = 0; e < HIST; ++e) hs[(size_t)ch0 * HIST + e] = h0[e];
            if (has_v)
#pragma unroll
                for (int e = 0; e < HIST; ++e) hs[(size_t)ch1 * HIST + e] = h1[e];
        }
        c0 = siluf_(c0);
        // ---- q/k L2 norm: warps 0-3 hold q, warps 4-7 hold k
        {
            double sq = warp_sum_d((double)__fmul_rn(c0, c0));
            if (lane == 0) nred[warp] = sq;
        }
        if (has_v) v_s[tid] = siluf_(c1);
        __syncthreads();
        {
            const int w0i = tid < S ? 0 : WARPS / 2;
            double sum = -0.0;
#pragma unroll
            for (int w = 0; w < WARPS / 2; ++w) sum += nred[w0i + w];
            const float sc = rms_scale_from_sum(sum, S, l2_eps);
            const float y = __fmul_rn(__fmul_rn(c0, sc), shrink);
            if (tid < S) q_s[tid] = y;
            else k_s[tid - S] = y;
        }
        // ---- gates (forward.rs:1530-1546, :1610)
        const float decay = __fmul_rn(softplusf_(__fadd_rn(a.alpha[(size_t)r * n_v + vh], dt_bias)), ssm_a);
        const float g = expf(decay);
        const float beta = sigmoidf_(a.beta[(size_t)r * n_v + vh]);
        __syncthreads();
        // ---- pass one: decay the state and contract it with k
        float acc = 0.0f;
#pragma unroll
        for (int ii = 0; ii < RPW; ++ii) {
            st[ii] = __fmul_rn(st[ii], g);
            acc = __fadd_rn(acc, __fmul_rn(st[ii], k_s[warp * RPW + ii]));
        }
        red[warp][lane] = acc;
        __syncthreads();
        if (warp == 0) {
            float sk = 0.0f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) sk = __fadd_rn(sk, red[w][lane]);
            d_s[lane] = __fmul_rn(__fsub_rn(v_s[lane], sk), beta);
        }
        __syncthreads();
        // ---- pass two: add the delta's outer product, read out against q
        const float dj = d_s[lane];
        float o = 0.0f;
#pragma unroll
        for (int ii = 0; ii < RPW; ++ii) {
            const int i = warp * RPW + ii;
            st[ii] = __fadd_rn(st[ii], __fmul_rn(dj, k_s[i]));
            o = __fadd_rn(o, __fmul_rn(st[ii], q_s[i]));
        }
        red[warp][lane] = o;
        if (slots > 1 || r == a.t - 1) {
            float *dst = a.ssm_state + ((size_t)(vh * slots + to) * S) * S + j;
#pragma unroll
            for (int ii = 0; ii < RPW; ++ii) dst[(size_t)(warp * RPW + ii) * S] = st[ii];
        }
        __syncthreads();
        // ---- gated RMSNorm over the head's S outputs (forward.rs:1642-1652)
        float oj = 0.0f;
        if (warp == 0) {
#pragma unroll
            for (int w = 0; w < WARPS; ++w) oj = __fadd_rn(oj, red[w][lane]);
            oj = __fmul_rn(oj, scale);
            const double sq = warp_sum_d((double)__fmul_rn(oj, oj));
            if (lane == 0) cl_part[r & 1] = sq;
        }
        cluster.sync();
        if (warp == 0) {
            double sum = -0.0;
#pragma unroll
            for (int c = 0; c < CL; ++c)
                sum += *cluster.map_shared_rank(&cl_part[r & 1], grp * CL + c);
            const float sc = rms_scale_from_sum(sum, S, a.eps);
            const float zz = a.z[(size_t)r * d_inner + (size_t)vh * S + j];
            a.out[(size_t)r * d_inner + (size_t)vh * S + j] =
                __fmul_rn(__fmul_rn(__fmul_rn(oj, sc), wnorm), siluf_(zz));
        }
    }
    cluster.sync();  // no CTA leaves while a peer may still read its cl_part
}

// Clusters of up to 16 CTAs (n_v / n_k up to 4) need the non-portable size.
cudaError_t init_dn_kernels() {
    return cudaFuncSetAttribute(dn_step_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

// Value heads per key head the kernel's cluster can hold.
int dn_max_group() { return 16 / dn::CL; }

cudaError_t launch_dn_step(const LinArgs &a, cudaStream_t st) {
    const int gv = a.n_v / a.n_k;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dn::CL * gv, a.n_k);
    cfg.blockDim = dim3(dn::THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = dn::CL * gv;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, dn_step_kernel, a);
}

}  // namespace rl
