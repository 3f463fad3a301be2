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
// Work split.  One CTA per value head holds the head's whole 128 x 128 f32
// state in registers for the batch: 16 warps, warp w takes the 32 columns
// 32*(w%4).. and the 32 rows 32*(w/4).., one column per lane, so every load
// and store is a coalesced 128-byte row segment.  The head-wide reductions
// (the q/k L2 norms, S^T k, S^T q and the gated RMSNorm's sum of squares)
// stay inside the CTA: shared memory and CTA barriers, five per row.  The
// value heads that share a key head (vh = kh + g*n_k) form a cluster only for
// the q/k conv history they share: each reads it, arrives on a split cluster
// barrier, and the single writer waits on that barrier just before it
// overwrites the history, by which time the others have long arrived.
//
// The kernel is launched as a programmatic dependent (PDL) of the kernel
// before it and triggers its own dependents as soon as its grid-dependency
// wait returns, so when a kernel starts, every kernel before the one just
// ahead of it has completed.  What the context owns and only this kernel
// writes (the state and conv history of this layer) is therefore safe to
// load before the wait unless the kernel just ahead is a step of the same
// layer; the host passes `early_state` accordingly.  The conv weights and
// gate constants are loaded before the wait always (set once, synchronously);
// the row inputs are read, and every global write is made, after it.
#include "common.cuh"
#include "kernels.h"

namespace rl {
namespace dn {
constexpr int S = 128;          // d_state the kernel is built for
constexpr int THREADS = 512;
constexpr int RG = 4;           // row groups (warps per column group)
constexpr int RPT = S / RG;     // state rows per thread (32)
constexpr int HIST = 3;         // conv_kernel - 1
}  // namespace dn

// grid (n_v / n_k, n_k), cluster (n_v / n_k): blockIdx.x = g, vh = kh + g*n_k
__global__ void __launch_bounds__(dn::THREADS, 1) dn_step_kernel(const LinArgs a) {
    using namespace dn;
    __shared__ float q_s[S], k_s[S], v_s[S];
    __shared__ float red_k[RG][S], red_q[RG][S];
    __shared__ double nred[8], ored[4];

    const int n_k = a.n_k, n_v = a.n_v, slots = a.slots;
    const int grp = blockIdx.x, kh = blockIdx.y;
    const int vh = kh + grp * n_k;  // so that vh % n_k == kh, as forward.rs:1602-1609
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cgrp = warp & 3, rg = warp >> 2;
    const int j = cgrp * 32 + lane, i0 = rg * RPT;
    const int key_dim = n_k * S, d_inner = n_v * S, conv_dim = 2 * key_dim + d_inner;
    const float scale = 1.0f / sqrtf((float)S);
    const float shrink = 1.0f / sqrtf((float)S);
    const float l2_eps = a.eps / (float)S;

    // conv channel of this thread: q (tid < 128) or k (< 256) of key head kh,
    // v (< 384) of value head vh; the q/k history has one writer per key head
    const bool conv_t = tid < 3 * S;
    const int ch = tid < S ? kh * S + tid
                 : tid < 2 * S ? key_dim + kh * S + (tid - S)
                               : 2 * key_dim + vh * S + (tid - 2 * S);
    const bool writes_hist = conv_t && (tid >= 2 * S || grp == 0);
    float w[4] = {0.0f, 0.0f, 0.0f, 0.0f}, h[HIST] = {0.0f, 0.0f, 0.0f};
    if (conv_t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = a.conv1d[(size_t)ch * 4 + e];
    }
    const float dt_bias = a.dt_bias[vh], ssm_a = a.ssm_a[vh];
    const float wnorm = a.norm[j];
    // the state block (rows i0.., column j) and the conv history, slot `live`
    float st[RPT];
    const float *hist_live = a.conv_state + (size_t)a.live * conv_dim * HIST;
    auto load_state = [&]() {
        const float *src = a.ssm_state + ((size_t)(vh * slots + a.live) * S + i0) * S + j;
#pragma unroll
        for (int ii = 0; ii < RPT; ++ii) st[ii] = src[(size_t)ii * S];
        if (conv_t) {
#pragma unroll
            for (int e = 0; e < HIST; ++e) h[e] = hist_live[(size_t)ch * HIST + e];
        }
        cluster_arrive_release();  // this CTA has read the shared history
    };
    if (a.early_state) load_state();
    // the row inputs come from the kernel before; so does the right to write
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!a.early_state) load_state();

    bool hist_released = false;
    for (int r = 0; r < a.t; ++r) {
        const int to = (a.live + r + 1) % slots;
        // ---- the row's inputs, issued together
        const float xin = conv_t ? a.qkv[(size_t)r * conv_dim + ch] : 0.0f;
        const float al = a.alpha[(size_t)r * n_v + vh], bl = a.beta[(size_t)r * n_v + vh];
        const float zz = rg == 0 ? a.z[(size_t)r * d_inner + (size_t)vh * S + j] : 0.0f;
        // ---- conv (forward.rs:2018-2059: x*w[3] first, then the history
        // taps in order) and SiLU
        float c = 0.0f;
        if (conv_t) {
            c = __fmul_rn(xin, w[3]);
#pragma unroll
            for (int e = 0; e < HIST; ++e) c = __fadd_rn(c, __fmul_rn(h[e], w[e]));
            h[0] = h[1];
            h[1] = h[2];
            h[2] = xin;
            c = siluf_(c);
        }
        if (slots > 1 || r == a.t - 1) {  // the history this row leaves behind
            if (!hist_released) {
                // every CTA of the cluster has read the history it shares
                cluster_wait_acquire();
                hist_released = true;
            }
            if (writes_hist) {
                float *hs = a.conv_state + (size_t)to * conv_dim * HIST + (size_t)ch * HIST;
#pragma unroll
                for (int e = 0; e < HIST; ++e) hs[e] = h[e];
            }
        }
        // ---- q/k L2 norm (warps 0-3 hold q, 4-7 hold k) and the gates
        // (forward.rs:1530-1546, :1610)
        if (warp < 8) {
            const double sq = warp_sum_d((double)__fmul_rn(c, c));
            if (lane == 0) nred[warp] = sq;
        }
        const float decay = __fmul_rn(softplusf_(__fadd_rn(al, dt_bias)), ssm_a);
        const float g = expf(decay);
        const float beta = sigmoidf_(bl);
        __syncthreads();
        if (warp < 8) {
            const int w0i = warp < 4 ? 0 : 4;
            double sum = -0.0;
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += nred[w0i + q];
            const float y = __fmul_rn(__fmul_rn(c, rms_scale_from_sum(sum, S, l2_eps)), shrink);
            if (warp < 4) q_s[tid] = y;
            else k_s[tid - S] = y;
        } else if (warp < 12) {
            v_s[tid - 2 * S] = c;
        }
        __syncthreads();
        // ---- pass one: decay the state and contract it with k
        float acc = 0.0f;
#pragma unroll
        for (int ii = 0; ii < RPT; ++ii) {
            st[ii] = __fmul_rn(st[ii], g);
            acc = __fadd_rn(acc, __fmul_rn(st[ii], k_s[i0 + ii]));
        }
        red_k[rg][j] = acc;
        __syncthreads();
        float sk = 0.0f;
#pragma unroll
        for (int q = 0; q < RG; ++q) sk = __fadd_rn(sk, red_k[q][j]);
        const float dj = __fmul_rn(__fsub_rn(v_s[j], sk), beta);
        // ---- pass two: add the delta's outer product, read out against q
        float o = 0.0f;
#pragma unroll
        for (int ii = 0; ii < RPT; ++ii) {
            st[ii] = __fadd_rn(st[ii], __fmul_rn(dj, k_s[i0 + ii]));
            o = __fadd_rn(o, __fmul_rn(st[ii], q_s[i0 + ii]));
        }
        red_q[rg][j] = o;
        // warps of row group 0 finish the readout; the others only arrive
        if (rg == 0) named_sync(1, THREADS);
        else named_arrive(1, THREADS);
        if (slots > 1 || r == a.t - 1) {
            float *dst = a.ssm_state + ((size_t)(vh * slots + to) * S + i0) * S + j;
#pragma unroll
            for (int ii = 0; ii < RPT; ++ii) dst[(size_t)ii * S] = st[ii];
        }
        // ---- gated RMSNorm over the head's S outputs (forward.rs:1642-1652)
        if (rg == 0) {
            float oj = 0.0f;
#pragma unroll
            for (int q = 0; q < RG; ++q) oj = __fadd_rn(oj, red_q[q][j]);
            oj = __fmul_rn(oj, scale);
            const double sq = warp_sum_d((double)__fmul_rn(oj, oj));
            if (lane == 0) ored[cgrp] = sq;
            named_sync(2, 4 * 32);
            double sum = -0.0;
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += ored[q];
            const float sc = rms_scale_from_sum(sum, S, a.eps);
            a.out[(size_t)r * d_inner + (size_t)vh * S + j] =
                __fmul_rn(__fmul_rn(__fmul_rn(oj, sc), wnorm), siluf_(zz));
        }
    }
}

cudaError_t init_dn_kernels() { return cudaSuccess; }

// Value heads per key head the kernel's cluster can hold (portable size).
int dn_max_group() { return 8; }

cudaError_t launch_dn_step(const LinArgs &a, cudaStream_t st) {
    const int gv = a.n_v / a.n_k;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gv, a.n_k);
    cfg.blockDim = dim3(dn::THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = gv;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, dn_step_kernel, a);
}

}  // namespace rl
