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
#include <algorithm>

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
//
// The grid is a few blocks per SM and each warp walks the (row, head) items
// with a stride, loading the next item's row (and its gate or value row)
// while it works on the current one, so that two items' loads are in flight
// per warp: one item at a time left the kernel waiting on memory.
template <typename KV>
__global__ void __launch_bounds__(256, 3) full_prologue_kernel(const FullArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    constexpr int HD = 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_heads = a.kv_only ? a.n_kv : a.n_head + a.n_kv;
    const int head0 = a.kv_only ? a.n_head : 0;
    // t * n_heads stays far below 2^31 (the launcher checks), so the item
    // arithmetic is 32-bit: a 64-bit division is a long software routine
    const int n_items = a.t * n_heads, stride = (int)gridDim.x * 8;
    const int half = a.n_rot / 2;
    // the item's row (query or key, 8 dims a lane) and its second row (the
    // gate for a query when it is staged, the value for a key)
    auto load = [&](int item, float4 (&in)[4]) {
        const int i = item / n_heads, hh = item - i * n_heads + head0;
        const bool is_q = hh < a.n_head;
        const float *src = is_q ? a.qg + ((size_t)i * a.n_head + hh) * 2 * HD
                                : a.k + ((size_t)i * a.n_kv + (hh - a.n_head)) * HD;
        const float *src2 = is_q ? src + HD : a.v + ((size_t)i * a.n_kv + (hh - a.n_head)) * HD;
        in[0] = *reinterpret_cast<const float4 *>(src + lane * 8);
        in[1] = *reinterpret_cast<const float4 *>(src + lane * 8 + 4);
        if (!is_q || a.gate_bf16) {
            in[2] = *reinterpret_cast<const float4 *>(src2 + lane * 8);
            in[3] = *reinterpret_cast<const float4 *>(src2 + lane * 8 + 4);
        }
    };
    int item = (int)blockIdx.x * 8 + warp;
    if (item >= n_items) return;
    float4 cur[4], nxt[4];
    load(item, cur);
    for (; item < n_items; item += stride) {
        if (item + stride < n_items) load(item + stride, nxt);
        const int i = item / n_heads, p = a.pos + i;
        const int hh = item - i * n_heads + head0;
        const bool is_q = hh < a.n_head;
        const float *w = is_q ? a.q_norm : a.k_norm;
        float x[8], wv[8], c[8], sn[8], gt[8];
        x[0] = cur[0].x, x[1] = cur[0].y, x[2] = cur[0].z, x[3] = cur[0].w;
        x[4] = cur[1].x, x[5] = cur[1].y, x[6] = cur[1].z, x[7] = cur[1].w;
        gt[0] = cur[2].x, gt[1] = cur[2].y, gt[2] = cur[2].z, gt[3] = cur[2].w;
        gt[4] = cur[3].x, gt[5] = cur[3].y, gt[6] = cur[3].z, gt[7] = cur[3].w;
        const float4 w0 = *reinterpret_cast<const float4 *>(w + lane * 8);
        const float4 w1 = *reinterpret_cast<const float4 *>(w + lane * 8 + 4);
        wv[0] = w0.x, wv[1] = w0.y, wv[2] = w0.z, wv[3] = w0.w;
        wv[4] = w1.x, wv[5] = w1.y, wv[6] = w1.z, wv[7] = w1.w;
#pragma unroll
        for (int e = 0; e < 8; ++e) c[e] = 1.0f, sn[e] = 0.0f;
        if (lane * 8 < a.n_rot) {
            // the lane's 8 dims pair with table entries base .. base + 7
            // (half is a multiple of 8, so they do not straddle it)
            const int base = lane * 8 < half ? lane * 8 : lane * 8 - half;
            if (a.rope_cs) {
                const float *cs_row = a.rope_cs + (size_t)p * half + base;
                const float *sn_row = a.rope_sn + (size_t)p * half + base;
                const float4 c0 = *reinterpret_cast<const float4 *>(cs_row);
                const float4 c1 = *reinterpret_cast<const float4 *>(cs_row + 4);
                const float4 s0 = *reinterpret_cast<const float4 *>(sn_row);
                const float4 s1 = *reinterpret_cast<const float4 *>(sn_row + 4);
                c[0] = c0.x, c[1] = c0.y, c[2] = c0.z, c[3] = c0.w;
                c[4] = c1.x, c[5] = c1.y, c[6] = c1.z, c[7] = c1.w;
                sn[0] = s0.x, sn[1] = s0.y, sn[2] = s0.z, sn[3] = s0.w;
                sn[4] = s1.x, sn[5] = s1.y, sn[6] = s1.z, sn[7] = s1.w;
            } else {
                // no table (callers without a context): the same angle,
                // advanced by repeated f32 multiplication from theta = p
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float theta = (float)p;
                    for (int jj = 0; jj < base + e; ++jj) theta = __fmul_rn(theta, a.theta_scale);
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
        // RoPE pairs dim d with d +- half: fetch the partner from the lane
        // that holds it (half is a multiple of 8, so the partner sits at the
        // same e)
        const int lane_shift = half / 8;
        const bool lo = lane * 8 < half, rot = lane * 8 < a.n_rot;
        const int partner = rot ? (lo ? lane + lane_shift : lane - lane_shift) : lane;
        float r[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float other = __shfl_sync(0xffffffffu, y[e], partner);
            r[e] = y[e];
            if (rot)
                r[e] = lo ? __fsub_rn(__fmul_rn(y[e], c[e]), __fmul_rn(other, sn[e]))
                          : __fadd_rn(__fmul_rn(other, sn[e]), __fmul_rn(y[e], c[e]));
        }
        if (is_q) {
            const size_t o = ((size_t)i * a.n_head + hh) * HD + lane * 8;
            if (a.q_f32) store8(a.q_f32 + o, r);
            if (a.q_bf16) store8(a.q_bf16 + o, r);
            if (a.gate_bf16) {
                // the output gate, sigmoid(g) (forward.rs:1327-1340), staged
                // in bf16 for the prefill kernel's epilogue.  The hardware
                // exp2 and reciprocal are within a few f32 ulps of the exact
                // sigmoid, far below the bf16 rounding that follows; the
                // accurate library forms made this kernel issue-bound.
#pragma unroll
                for (int e = 0; e < 8; ++e) gt[e] = __fdividef(1.0f, 1.0f + __expf(-gt[e]));
                store8(a.gate_bf16 + o, gt);
            }
        } else {
            const int kh = hh - a.n_head;
            const size_t to = ((size_t)kh * a.context + p) * HD + lane * 8;
            store8(static_cast<KV *>(a.k_cache) + to, r);
            store8(static_cast<KV *>(a.v_cache) + to, gt);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) cur[q] = nxt[q];
    }
}

// ---------------------------------------------------------------------------
// Host launchers.

cudaError_t launch_full_prologue(const FullArgs &a, cudaStream_t st) {
    if (a.hd != 256 || (a.n_rot % 16) != 0) return cudaErrorInvalidValue;
    const int64_t items = (int64_t)a.t * (a.kv_only ? a.n_kv : a.n_head + a.n_kv);
    if (items >= (int64_t)1 << 30) return cudaErrorInvalidValue;
    // a few blocks per SM, each warp walking items with a stride
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned blocks = (unsigned)std::min<int64_t>((items + 7) / 8, (int64_t)sms * 3);
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
