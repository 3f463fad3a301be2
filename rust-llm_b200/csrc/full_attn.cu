// Gated GQA full attention: the prologue of a multi-row call.
//
//   full_prologue_kernel   per-head q/k RMSNorm + partial RoPE, KV append of
//                          all t rows, f32 (and optional bf16) staging of the
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
// Prologue.  Block (head, row): heads [0, n_head) are queries, read from the
// query half of qg; heads [n_head, n_head + n_kv) are keys.  One thread per
// dimension.
template <typename KV>
__global__ void full_prologue_kernel(const float *__restrict__ qg, const float *__restrict__ k,
                                     const float *__restrict__ v,
                                     const float *__restrict__ q_norm,
                                     const float *__restrict__ k_norm, KV *__restrict__ k_cache,
                                     KV *__restrict__ v_cache, float *__restrict__ q_out,
                                     __nv_bfloat16 *__restrict__ q_out_bf16, int pos, int n_head,
                                     int n_kv, int context, int n_rot, float theta_scale,
                                     float eps) {
    extern __shared__ float buf[];  // hd floats
    __shared__ double red[32];
    const int hd = blockDim.x, d = threadIdx.x;
    const int hh = blockIdx.x, i = blockIdx.y, p = pos + i;
    const bool is_q = hh < n_head;
    const float x = is_q ? qg[(size_t)i * 2 * hd * n_head + (size_t)hh * 2 * hd + d]
                         : k[(size_t)i * hd * n_kv + (size_t)(hh - n_head) * hd + d];
    const double sum = block_sum_d((double)__fmul_rn(x, x), red);
    const float scale = rms_scale_from_sum(sum, hd, eps);
    const float w = is_q ? q_norm[d] : k_norm[d];
    buf[d] = __fmul_rn(__fmul_rn(x, scale), w);
    __syncthreads();
    float y = buf[d];
    const int half = n_rot / 2;
    if (d < n_rot) {
        // the angle of pair (d mod half), advanced by repeated f32
        // multiplication exactly as forward.rs:1855-1861 does
        const int pr = d < half ? d : d - half;
        float theta = (float)p;
        for (int j = 0; j < pr; ++j) theta = __fmul_rn(theta, theta_scale);
        const float c = cosf(theta), s = sinf(theta);
        const float x0 = buf[pr], x1 = buf[pr + half];
        y = d < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                     : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    if (is_q) {
        const size_t o = ((size_t)i * n_head + hh) * hd + d;
        q_out[o] = y;
        if (q_out_bf16) q_out_bf16[o] = __float2bfloat16_rn(y);
    } else {
        const int kh = hh - n_head;
        const size_t to = ((size_t)kh * context + p) * hd + d;
        k_cache[to] = from_f32<KV>(y);
        v_cache[to] = from_f32<KV>(v[(size_t)i * hd * n_kv + (size_t)kh * hd + d]);
    }
}

// ---------------------------------------------------------------------------
// Host launchers.

template <typename KV>
static cudaError_t launch_prologue_t(const FullArgs &a, cudaStream_t st) {
    dim3 grid(a.n_head + a.n_kv, a.t);
    full_prologue_kernel<KV><<<grid, a.hd, a.hd * sizeof(float), st>>>(
        a.qg, a.k, a.v, a.q_norm, a.k_norm, (KV *)a.k_cache, (KV *)a.v_cache, a.q_f32, a.q_bf16,
        a.pos, a.n_head, a.n_kv, a.context, a.n_rot, a.theta_scale, a.eps);
    return cudaGetLastError();
}

cudaError_t launch_full_prologue(const FullArgs &a, cudaStream_t st) {
    return a.kv_bf16 ? launch_prologue_t<__nv_bfloat16>(a, st) : launch_prologue_t<float>(a, st);
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
