// Gated GQA full attention: the prologue of a multi-row call.
//
//   full_prologue_kernel   per-head q/k RMSNorm + partial RoPE, KV append of
//                          all t rows, f32 and/or bf16 staging of the
//                          queries, before the attention kernels read them
//
// Reference: the first half of Exec::full_attn's span
// (crates/rust-llm/src/forward.rs:1259-1292), rms_norm_in_place (:1690-1695)
// and rope (:1851-1862).  A single decode row does this inside the decode
// kernel instead (decode_attn.cu).
#include "common.cuh"
#include "kernels.h"

namespace rl {

// ---------------------------------------------------------------------------
// Prologue.  One warp per (row, head): heads [0, n_head) are queries, read
// from the query half of qg; heads [n_head, n_head + n_kv) are keys, whose
// warp also appends the value row.  Each lane holds 8 consecutive dims; the
// RMSNorm's sum of squares is an f64 warp sum (forward.rs:1697-1711) and the
// RoPE angles come from the per-context table, whose angles are advanced by
// repeated f32 multiplication as forward.rs:1855-1861 does.
// Eight consecutive cache elements in one or two 16-byte stores.
__device__ __forceinline__ void store8(float *dst, const float *x) {
    *reinterpret_cast<float4 *>(dst) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4 *>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
}
__device__ __forceinline__ uint32_t bf2_bits(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ void store8(__nv_bfloat16 *dst, const float *x) {
    uint4 u;
    u.x = bf2_bits(x[0], x[1]);
    u.y = bf2_bits(x[2], x[3]);
    u.z = bf2_bits(x[4], x[5]);
    u.w = bf2_bits(x[6], x[7]);
    *reinterpret_cast<uint4 *>(dst) = u;
}

// kv_only: the key heads alone (the verify kernel normalises its queries).
// Each launch waits for the grid ahead (a programmatic dependent launch
// makes that wait real) and then lets the next grid launch: when a kernel
// starts, every kernel before the one just ahead has completed.
template <typename KV>
__global__ void __launch_bounds__(256) full_prologue_kernel(const FullArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_heads = a.kv_only ? a.n_kv : a.n_head + a.n_kv;
    const int64_t item = (int64_t)blockIdx.x * 8 + warp;
    if (item >= (int64_t)a.t * n_heads) return;
    const int i = (int)(item / n_heads), p = a.pos + i;
    const int hh = (int)(item % n_heads) + (a.kv_only ? a.n_head : 0);
    const bool is_q = hh < a.n_head;
    constexpr int HD = 256;
    const float *src = is_q ? a.qg + ((size_t)i * a.n_head + hh) * 2 * HD
                            : a.k + ((size_t)i * a.n_kv + (hh - a.n_head)) * HD;
    const float *w = is_q ? a.q_norm : a.k_norm;
    const int half = a.n_rot / 2;
    const float *cs_row = a.rope_cs ? a.rope_cs + (size_t)p * half : nullptr;
    const float *sn_row = a.rope_sn ? a.rope_sn + (size_t)p * half : nullptr;
    float x[8], wv[8], c[8], sn[8], gt[8];
    float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
    if (is_q && a.gate_bf16) {
        g0 = *reinterpret_cast<const float4 *>(src + HD + lane * 8);
        g1 = *reinterpret_cast<const float4 *>(src + HD + lane * 8 + 4);
    }
    const float4 x0 = *reinterpret_cast<const float4 *>(src + lane * 8);
    const float4 x1 = *reinterpret_cast<const float4 *>(src + lane * 8 + 4);
    const float4 w0 = *reinterpret_cast<const float4 *>(w + lane * 8);
    const float4 w1 = *reinterpret_cast<const float4 *>(w + lane * 8 + 4);
    x[0] = x0.x, x[1] = x0.y, x[2] = x0.z, x[3] = x0.w, x[4] = x1.x, x[5] = x1.y, x[6] = x1.z, x[7] = x1.w;
    wv[0] = w0.x, wv[1] = w0.y, wv[2] = w0.z, wv[3] = w0.w, wv[4] = w1.x, wv[5] = w1.y, wv[6] = w1.z, wv[7] = w1.w;
    gt[0] = g0.x, gt[1] = g0.y, gt[2] = g0.z, gt[3] = g0.w, gt[4] = g1.x, gt[5] = g1.y, gt[6] = g1.z, gt[7] = g1.w;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        const int pr = d < half ? d : d - half;
        c[e] = 1.0f;
        sn[e] = 0.0f;
        if (d < a.n_rot) {
            if (a.rope_cs) {
                c[e] = cs_row[pr];
                sn[e] = sn_row[pr];
            } else {
                // no table (callers without a context): the same angle,
                // advanced by repeated f32 multiplication from theta = p
                float theta = (float)p;
                for (int jj = 0; jj < pr; ++jj) theta = __fmul_rn(theta, a.theta_scale);
                c[e] = cosf(theta);
                sn[e] = sinf(theta);
            }
        }
    }
    double sq = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) sq += (double)__fmul_rn(x[e], x[e]);
    sq = warp_sum_d(sq);
    const float scale = rms_scale_from_sum(sq, HD, a.eps);
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __fmul_rn(__fmul_rn(x[e], scale), wv[e]);
    // RoPE pairs dim d with d +- half: fetch the partner from the lane that
    // holds it (half is a multiple of 8, so the partner sits at the same e)
    const int lane_shift = half / 8;
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        const bool lo = d < half;
        const float up = __shfl_down_sync(0xffffffffu, y[e], lane_shift > 0 ? lane_shift : 1);
        const float dn = __shfl_up_sync(0xffffffffu, y[e], lane_shift > 0 ? lane_shift : 1);
        r[e] = y[e];
        if (d < a.n_rot)
            r[e] = lo ? __fsub_rn(__fmul_rn(y[e], c[e]), __fmul_rn(up, sn[e]))
                      : __fadd_rn(__fmul_rn(dn, sn[e]), __fmul_rn(y[e], c[e]));
    }
    if (is_q) {
        const size_t o = ((size_t)i * a.n_head + hh) * HD + lane * 8;
        if (a.q_f32) store8(a.q_f32 + o, r);
        if (a.q_bf16) store8(a.q_bf16 + o, r);
        if (a.gate_bf16) {
            // the output gate, sigmoid(g) (forward.rs:1327-1340), staged in
            // bf16 for the prefill kernel's epilogue
#pragma unroll
            for (int e = 0; e < 8; ++e) gt[e] = sigmoidf_(gt[e]);
            store8(a.gate_bf16 + o, gt);
        }
    } else {
        const int kh = hh - a.n_head;
        const size_t to = ((size_t)kh * a.context + p) * HD + lane * 8;
        const float *vsrc = a.v + ((size_t)i * a.n_kv + kh) * HD + lane * 8;
        const float4 v0 = *reinterpret_cast<const float4 *>(vsrc);
        const float4 v1 = *reinterpret_cast<const float4 *>(vsrc + 4);
        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        store8(static_cast<KV *>(a.k_cache) + to, r);
        store8(static_cast<KV *>(a.v_cache) + to, vv);
    }
}

// ---------------------------------------------------------------------------
// Host launchers.

cudaError_t launch_full_prologue(const FullArgs &a, cudaStream_t st) {
    if (a.hd != 256 || (a.n_rot % 16) != 0) return cudaErrorInvalidValue;
    const int64_t items = (int64_t)a.t * (a.kv_only ? a.n_kv : a.n_head + a.n_kv);
    const unsigned blocks = (unsigned)((items + 7) / 8);
    if (a.kv_bf16)
        full_prologue_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
    else
        full_prologue_kernel<float><<<blocks, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t init_full_attn_kernels() { return cudaSuccess; }

// One thread per position: the angle advanced by repeated f32
// multiplication from theta_0 = pos, exactly as forward.rs:1855-1861 does,
// and the cos and sin of each angle.
__global__ void rope_table_kernel(float *cs, float *sn, int context, int half,
                                  float theta_scale) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= context) return;
    float theta = (float)p;
    for (int i = 0; i < half; ++i) {
        cs[(size_t)p * half + i] = cosf(theta);
        sn[(size_t)p * half + i] = sinf(theta);
        theta = __fmul_rn(theta, theta_scale);
    }
}

cudaError_t launch_rope_table(float *cs, float *sn, int context, int n_rot, float theta_scale,
                              cudaStream_t st) {
    if (n_rot < 2) return cudaSuccess;
    rope_table_kernel<<<(context + 255) / 256, 256, 0, st>>>(cs, sn, context, n_rot / 2,
                                                             theta_scale);
    return cudaGetLastError();
}

}  // namespace rl
