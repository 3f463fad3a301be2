// Gated GQA full attention on sm_100a: the CUDA-core path.
//
//   full_prologue_kernel   per-head q/k RMSNorm + partial RoPE, KV append,
//                          f32 (and optional bf16) staging of the queries
//   decode_split_kernel    split-KV flash decoding: one CTA per (split, KV
//                          head, query row) walks its KV range once for all
//                          GROUP query heads of the KV head, K/V tiles staged
//                          by bulk TMA copies through a 3-stage mbarrier ring
//   decode_merge_kernel    log-sum-exp merge of the splits, sigmoid output
//                          gate, head-major -> token-major transpose
//
// The reference is Exec::full_attn (crates/rust-llm/src/forward.rs:1259-1340)
// with attend_batch (:1783-1826), softmax (:1831-1842) and rope (:1851-1862).
// Where the reference materialises a score row and runs one softmax over it,
// this runs an online (running max / running sum) softmax per split and
// merges the splits: the same function, rounded differently, checked against
// the oracle at 1e-4 relative.
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
// Split-KV decode.
namespace dec {
constexpr int HD = 256;     // head dimension the kernel is built for
constexpr int GROUP = 4;    // query heads per KV head
constexpr int WARPS = 4;    // == GROUP: warp h runs head h's softmax
constexpr int THREADS = WARPS * 32;
constexpr int STAGES = 3;
constexpr float LOG2E = 1.4426950408889634f;
}  // namespace dec

template <typename KV>
struct DecTraits;
template <>
struct DecTraits<__nv_bfloat16> {
    static constexpr int P = 32;    // positions per tile: 16 KB of K, 16 KB of V
    static constexpr int EPC = 8;   // elements per 16-byte chunk
};
template <>
struct DecTraits<float> {
    static constexpr int P = 16;
    static constexpr int EPC = 4;
};

template <typename KV>
constexpr size_t dec_smem_bytes() {
    return (size_t)dec::STAGES * 2 * DecTraits<KV>::P * dec::HD * sizeof(KV);
}

// 16 bytes of KV elements widened to f32.
__device__ __forceinline__ void chunk_to_f32(const uint4 &w, float *f, __nv_bfloat16 *) {
    bf16x8_to_f32(w, f);
}
__device__ __forceinline__ void chunk_to_f32(const uint4 &w, float *f, float *) {
    f[0] = __uint_as_float(w.x);
    f[1] = __uint_as_float(w.y);
    f[2] = __uint_as_float(w.z);
    f[3] = __uint_as_float(w.w);
}

template <typename KV>
__global__ void __launch_bounds__(dec::THREADS, 2)
    decode_split_kernel(const float *__restrict__ q, const KV *__restrict__ k_cache,
                        const KV *__restrict__ v_cache, float *__restrict__ part_o,
                        float *__restrict__ part_ml, int pos, int context, int n_head,
                        int chunk, int n_splits, int *status) {
    using namespace dec;
    constexpr int P = DecTraits<KV>::P;
    constexpr int EPC = DecTraits<KV>::EPC;
    constexpr int NCH = 16 / EPC;           // 16-byte chunks per lane in QK (16 dims)
    constexpr int PV_CH = HD / (32 * EPC);  // 16-byte chunks per lane in PV
    constexpr int PV_D = PV_CH * EPC;       // dims per lane in PV (8)
    constexpr int ROW = HD * sizeof(KV);    // bytes per cached position

    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[STAGES];
    __shared__ float scores[GROUP][P];
    __shared__ __align__(16) float wts[P][GROUP];
    __shared__ float alpha_s[GROUP];

    const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_kv = pos + row + 1;  // causal: row attends over pos+row+1 keys
    const int p_begin = split * chunk;
    const int p_end = min(p_begin + chunk, n_kv);
    const size_t head0 = (size_t)row * n_head + (size_t)kh * GROUP;
    float *po = part_o + (head0 * n_splits + split) * HD;  // + h * n_splits * HD
    float *pml = part_ml + (head0 * n_splits + split) * 2;

    if (p_begin >= p_end) {  // an empty split (only rows before the last)
        for (int e = tid; e < GROUP * HD; e += THREADS)
            po[(size_t)(e / HD) * n_splits * HD + e % HD] = 0.0f;
        if (tid < GROUP) {
            pml[(size_t)tid * n_splits * 2] = -INFINITY;
            pml[(size_t)tid * n_splits * 2 + 1] = 0.0f;
        }
        return;
    }
    const int n_tiles = (p_end - p_begin + P - 1) / P;
    const KV *kbase = k_cache + ((size_t)kh * context + p_begin) * HD;
    const KV *vbase = v_cache + ((size_t)kh * context + p_begin) * HD;
    KV *stage_k[STAGES], *stage_v[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
        stage_k[s] = reinterpret_cast<KV *>(smem) + (size_t)s * 2 * P * HD;
        stage_v[s] = stage_k[s] + P * HD;
    }

    auto issue = [&](int tile) {
        const int s = tile % STAGES;
        const int rows = min(P, p_end - p_begin - tile * P);
        const uint32_t bytes = (uint32_t)rows * ROW;
        mbar_arrive_expect_tx(&bars[s], 2 * bytes);
        bulk_g2s(stage_k[s], kbase + (size_t)tile * P * HD, bytes, &bars[s]);
        bulk_g2s(stage_v[s], vbase + (size_t)tile * P * HD, bytes, &bars[s]);
    };

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int t = 0; t < min(STAGES, n_tiles); ++t) issue(t);

    // Queries for QK: lane (sub, part) covers chunks part + 16*c of a row.
    const int part = lane & 15, sub = lane >> 4;
    float qr[GROUP][NCH * EPC];
#pragma unroll
    for (int h = 0; h < GROUP; ++h)
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const float *src = q + (head0 + h) * HD + (part + 16 * c) * EPC;
#pragma unroll
            for (int e = 0; e < EPC; e += 4) {
                const float4 f = *reinterpret_cast<const float4 *>(src + e);
                qr[h][c * EPC + e] = f.x;
                qr[h][c * EPC + e + 1] = f.y;
                qr[h][c * EPC + e + 2] = f.z;
                qr[h][c * EPC + e + 3] = f.w;
            }
        }
    const float qk_scale = (1.0f / 16.0f) * LOG2E;  // 1/sqrt(256), in log2 units

    float acc[GROUP][PV_D];
#pragma unroll
    for (int h = 0; h < GROUP; ++h)
#pragma unroll
        for (int e = 0; e < PV_D; ++e) acc[h][e] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;  // meaningful in warp h == head h
    bool ok = true;
    int issued_until = 0, failed_at = 0;

    for (int t = 0; t < n_tiles; ++t) {
        const int s = t % STAGES;
        const bool landed = mbar_wait(&bars[s], (t / STAGES) & 1, status);
        const KV *K = stage_k[s];
        const KV *V = stage_v[s];
        const int base = p_begin + t * P;
        const int valid = min(P, p_end - base);

        // ---- scores: two positions per warp step, 16 lanes per position
#pragma unroll
        for (int st = 0; st < P / WARPS / 2; ++st) {
            const int p = warp * (P / WARPS) + 2 * st + sub;
            float a[GROUP];
#pragma unroll
            for (int h = 0; h < GROUP; ++h) a[h] = 0.0f;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const uint4 w = *reinterpret_cast<const uint4 *>(K + p * HD + (part + 16 * c) * EPC);
                float kf[EPC];
                chunk_to_f32(w, kf, (KV *)nullptr);
#pragma unroll
                for (int e = 0; e < EPC; ++e)
#pragma unroll
                    for (int h = 0; h < GROUP; ++h) a[h] = fmaf(qr[h][c * EPC + e], kf[e], a[h]);
            }
            // reduce-scatter over the 16 lanes of the position: 5 shuffles
            const bool b3 = part & 8, b2 = part & 4;
            const float keep0 = b3 ? a[2] : a[0], keep1 = b3 ? a[3] : a[1];
            const float send0 = b3 ? a[0] : a[2], send1 = b3 ? a[1] : a[3];
            const float y0 = keep0 + __shfl_xor_sync(0xffffffffu, send0, 8);
            const float y1 = keep1 + __shfl_xor_sync(0xffffffffu, send1, 8);
            float z = (b2 ? y1 : y0) + __shfl_xor_sync(0xffffffffu, b2 ? y0 : y1, 4);
            z += __shfl_xor_sync(0xffffffffu, z, 2);
            z += __shfl_xor_sync(0xffffffffu, z, 1);
            if ((part & 3) == 0) scores[(part >> 2) & 3][p] = p < valid ? z * qk_scale : -INFINITY;
        }
        // every thread agrees on giving up, so none is left at a barrier
        if (!__syncthreads_and(landed)) {
            ok = false;
            issued_until = min(n_tiles, STAGES + max(0, t - 1));
            failed_at = t;
            break;
        }
        // the stage read by the previous tile is free now: refill it
        if (tid == 0 && t >= 1 && t - 1 + STAGES < n_tiles) issue(t - 1 + STAGES);

        // ---- online softmax, warp h for head h
        {
            const int h = warp;
            const float sv = lane < P ? scores[h][lane] : -INFINITY;
            const float m_new = fmaxf(m_run, warp_max(sv));
            const float al = exp2f(m_run - m_new);
            const float pv = exp2f(sv - m_new);
            const float ps = warp_sum(pv);
            l_run = fmaf(l_run, al, ps);
            m_run = m_new;
            if (lane < P) wts[lane][h] = pv;
            if (lane == 0) alpha_s[h] = al;
        }
        __syncthreads();

        // ---- weighted values: warp w takes P/WARPS positions, lane 8 dims
        {
            float al[GROUP];
#pragma unroll
            for (int h = 0; h < GROUP; ++h) al[h] = alpha_s[h];
#pragma unroll
            for (int h = 0; h < GROUP; ++h)
#pragma unroll
                for (int e = 0; e < PV_D; ++e) acc[h][e] *= al[h];
            const int p0 = warp * (P / WARPS);
            const int p1 = min(p0 + P / WARPS, valid);
            for (int p = p0; p < p1; ++p) {
                const float4 w4 = *reinterpret_cast<const float4 *>(&wts[p][0]);
                const float wv[GROUP] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int c = 0; c < PV_CH; ++c) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(V + p * HD + (lane + 32 * c) * EPC);
                    float vf[EPC];
                    chunk_to_f32(w, vf, (KV *)nullptr);
#pragma unroll
                    for (int e = 0; e < EPC; ++e)
#pragma unroll
                        for (int h = 0; h < GROUP; ++h)
                            acc[h][c * EPC + e] = fmaf(wv[h], vf[e], acc[h][c * EPC + e]);
                }
            }
        }
    }
    if (!ok) {
        // give the copies still in flight a bounded chance to land before the
        // shared memory they target is released
        for (int u = failed_at; u < issued_until; ++u)
            mbar_wait(&bars[u % STAGES], (u / STAGES) & 1, status);
        return;
    }
    __syncthreads();  // every stage consumed: reuse the ring for the reduction
    float *red = reinterpret_cast<float *>(smem);  // [WARPS][GROUP][HD]
#pragma unroll
    for (int h = 0; h < GROUP; ++h)
#pragma unroll
        for (int c = 0; c < PV_CH; ++c)
#pragma unroll
            for (int e = 0; e < EPC; e += 4)
                *reinterpret_cast<float4 *>(&red[(warp * GROUP + h) * HD + (lane + 32 * c) * EPC + e]) =
                    make_float4(acc[h][c * EPC + e], acc[h][c * EPC + e + 1],
                                acc[h][c * EPC + e + 2], acc[h][c * EPC + e + 3]);
    __syncthreads();
    for (int e = tid; e < GROUP * HD; e += THREADS) {
        float sum = red[e];
#pragma unroll
        for (int w = 1; w < WARPS; ++w) sum += red[w * GROUP * HD + e];
        po[(size_t)(e / HD) * n_splits * HD + e % HD] = sum;
    }
    if (lane == 0) {
        pml[(size_t)warp * n_splits * 2] = m_run;
        pml[(size_t)warp * n_splits * 2 + 1] = l_run;
    }
}

// ---------------------------------------------------------------------------
// Merge.  Block (head, row), one thread per dimension.
__global__ void decode_merge_kernel(const float *__restrict__ part_o,
                                    const float *__restrict__ part_ml,
                                    const float *__restrict__ qg, float *__restrict__ out,
                                    int n_head, int n_splits) {
    extern __shared__ float wsplit[];  // n_splits weights
    __shared__ float red[32];
    __shared__ float s_max, s_l;
    const int hd = blockDim.x, d = threadIdx.x, h = blockIdx.x, row = blockIdx.y;
    const size_t hr = (size_t)row * n_head + h;
    const float *ml = part_ml + hr * n_splits * 2;
    float m = -INFINITY;
    for (int s = d; s < n_splits; s += hd) m = fmaxf(m, ml[2 * s]);
    m = warp_max(m);
    if ((d & 31) == 0) red[d >> 5] = m;
    __syncthreads();
    if (d == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < (hd >> 5); ++w) mm = fmaxf(mm, red[w]);
        s_max = mm;
    }
    __syncthreads();
    const float M = s_max;
    float l = 0.0f;
    for (int s = d; s < n_splits; s += hd) {
        const float w = exp2f(ml[2 * s] - M);
        wsplit[s] = w;
        l = fmaf(w, ml[2 * s + 1], l);
    }
    l = warp_sum(l);
    __syncthreads();
    if ((d & 31) == 0) red[d >> 5] = l;
    __syncthreads();
    if (d == 0) {
        float ll = 0.0f;
        for (int w = 0; w < (hd >> 5); ++w) ll += red[w];
        s_l = ll;
    }
    __syncthreads();
    const float *o = part_o + hr * n_splits * hd + d;
    float acc = 0.0f;
    for (int s = 0; s < n_splits; ++s) acc = fmaf(wsplit[s], o[(size_t)s * hd], acc);
    const float attn = acc / s_l;
    const float g = qg[(size_t)row * 2 * hd * n_head + (size_t)h * 2 * hd + hd + d];
    out[(size_t)row * hd * n_head + (size_t)h * hd + d] = attn * sigmoidf_(g);
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

int decode_tile_positions(bool kv_bf16) {
    return kv_bf16 ? DecTraits<__nv_bfloat16>::P : DecTraits<float>::P;
}

template <typename KV>
static cudaError_t launch_decode_t(const FullArgs &a, int chunk, int n_splits, cudaStream_t st) {
    constexpr size_t smem = dec_smem_bytes<KV>();
    dim3 grid(n_splits, a.n_kv, a.t);
    decode_split_kernel<KV><<<grid, dec::THREADS, smem, st>>>(
        a.q_f32, (const KV *)a.k_cache, (const KV *)a.v_cache, a.part_o, a.part_ml, a.pos,
        a.context, a.n_head, chunk, n_splits, a.status);
    return cudaGetLastError();
}

cudaError_t init_full_attn_kernels() {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<__nv_bfloat16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)dec_smem_bytes<__nv_bfloat16>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(decode_split_kernel<float>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)dec_smem_bytes<float>());
}

cudaError_t launch_decode_split(const FullArgs &a, int chunk, int n_splits, cudaStream_t st) {
    return a.kv_bf16 ? launch_decode_t<__nv_bfloat16>(a, chunk, n_splits, st)
                     : launch_decode_t<float>(a, chunk, n_splits, st);
}

cudaError_t launch_decode_merge(const FullArgs &a, int n_splits, cudaStream_t st) {
    dim3 grid(a.n_head, a.t);
    decode_merge_kernel<<<grid, a.hd, n_splits * sizeof(float), st>>>(
        a.part_o, a.part_ml, a.qg, a.out, a.n_head, n_splits);
    return cudaGetLastError();
}

}  // namespace rl
