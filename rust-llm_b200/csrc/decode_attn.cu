// Split-KV flash decoding for the gated GQA layers, sm_100a, CUDA cores.
//
// One CTA per (KV split, KV head, query row) walks its range of the cache
// once for all GROUP query heads of the KV head.  Warp roles:
//   warp 4       producer: one lane issues the bulk TMA copies of K and V
//                tiles into a STAGES-deep ring, gated by full/empty mbarriers
//   warps 0..3   consumers: each owns a quarter of every tile's positions and
//                keeps its own online softmax (running max and sum per head)
//                and its own f32 accumulators, so the loop has no block-wide
//                barrier; the four warps are merged once at the end.
// Scores: 16 lanes per position, 16 dims per lane, packed f32x2 FMAs, a
// 5-shuffle reduce-scatter that leaves head h's score in the lanes of
// quarter h.  Values: 32 lanes x 8 dims per position, f32x2 FMAs.
//
// The splits of one (row, KV head) form clusters of C CTAs that merge their
// partial (max, sum, output) triples through distributed shared memory, each
// rank merging a slice of the head dimension.  With more than one cluster
// the merged slices go to global memory and the last cluster to arrive on a
// slice (an atomic counter) merges that slice across clusters.  The sigmoid
// output gate and the head-major -> token-major transpose are applied there,
// so the whole step is this one kernel; for a single decode row the q/k
// RMSNorm, partial RoPE and the KV append are fused in as well (FUSED).
//
// Reference: attend_batch / softmax / rope and the gate of Exec::full_attn
// (crates/rust-llm/src/forward.rs:1259-1340, :1783-1862).  The reference keeps
// whole score rows and one softmax; this online, split form is the same
// function with different rounding, checked against the oracle at 1e-4.
#include <cooperative_groups.h>

#include "common.cuh"
#include "decode_merge.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace rl {
namespace dec2 {
constexpr int HD = 256;
constexpr int GROUP = 4;
constexpr int CWARPS = 4;                  // consumer warps (== GROUP)
constexpr int THREADS = (CWARPS + 1) * 32; // + one producer warp
constexpr int STAGES = 3;
constexpr float LOG2E = 1.4426950408889634f;
}  // namespace dec2

template <typename KV>
struct Dec2Traits;
template <>
struct Dec2Traits<__nv_bfloat16> {
    static constexpr int P = 32;   // positions per tile (16 KB of K + 16 KB of V)
    static constexpr int EPC = 8;  // KV elements per 16-byte chunk
};
template <>
struct Dec2Traits<float> {
    static constexpr int P = 16;
    static constexpr int EPC = 4;
};

template <typename KV>
constexpr size_t dec2_stage_bytes() {
    return (size_t)2 * Dec2Traits<KV>::P * dec2::HD * sizeof(KV);
}
template <typename KV>
constexpr size_t dec2_smem_bytes() {
    return (size_t)dec2::STAGES * dec2_stage_bytes<KV>();
}

// 16 bytes of KV elements widened to f32 pairs.
__device__ __forceinline__ void chunk_to_f2(const uint4 &w, float2 *f, const __nv_bfloat16 *) {
    f[0] = make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u));
    f[1] = make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
    f[2] = make_float2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u));
    f[3] = make_float2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u));
}
__device__ __forceinline__ void chunk_to_f2(const uint4 &w, float2 *f, const float *) {
    f[0] = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
    f[1] = make_float2(__uint_as_float(w.z), __uint_as_float(w.w));
}


template <typename KV, bool FUSED>
__global__ void __launch_bounds__(dec2::THREADS, 2) decode_kernel(const DecodeArgs a) {
    using namespace dec2;
    constexpr int P = Dec2Traits<KV>::P;
    constexpr int EPC = Dec2Traits<KV>::EPC;
    constexpr int NCH = 16 / EPC;           // QK: 16-byte chunks per lane (16 dims)
    constexpr int PV_CH = HD / (32 * EPC);  // PV: 16-byte chunks per lane (8 dims)
    constexpr int PPW = P / CWARPS;         // positions per warp per tile
    constexpr int ROW = HD * sizeof(KV);

    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES];
    __shared__ __align__(16) float q_s[GROUP][HD];
    __shared__ __align__(16) KV newk_s[HD], newv_s[HD];
    __shared__ __align__(16) float kf_s[HD];
    __shared__ float rope_cs[128], rope_sn[128];
    __shared__ __align__(16) float wbuf[CWARPS][PPW][GROUP];
    __shared__ __align__(16) float abuf[CWARPS][GROUP];
    __shared__ float cta_m[GROUP], cta_l[GROUP];
    __shared__ int flag_s;

    const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
    const int C = a.csize;
    const int crank = split % C, cl = split / C, n_cl = a.n_splits / C;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos_row = a.pos + row;       // this row's own position
    const int n_kv = pos_row + 1;          // causal: keys 0..pos_row
    const int p_begin = split * a.chunk;
    const int p_end = min(p_begin + a.chunk, n_kv);
    const int n_tiles = p_end > p_begin ? (p_end - p_begin + P - 1) / P : 0;
    const int head0 = row * a.n_head + kh * GROUP;  // (row, first query head)
    KV *const k_cache = static_cast<KV *>(a.k_cache_v);
    KV *const v_cache = static_cast<KV *>(a.v_cache_v);
    const KV *kbase = k_cache + ((size_t)kh * a.context + p_begin) * HD;
    const KV *vbase = v_cache + ((size_t)kh * a.context + p_begin) * HD;
    const bool covers_new = FUSED && p_begin <= pos_row && pos_row < p_end;
    KV *stages = reinterpret_cast<KV *>(smem);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], CWARPS);
        }
        flag_s = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // per-warp online softmax state: lanes of quarter h track head h
    float m_run = -INFINITY, l_run = 0.0f;
    float2 acc[GROUP][4];
#pragma unroll
    for (int h = 0; h < GROUP; ++h)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] = make_float2(0.0f, 0.0f);
    bool ok = true;

    if (warp == CWARPS) {
        // ---------------- producer ----------------
        if (lane == 0) {
            for (int j = 0; j < n_tiles; ++j) {
                const int s = j % STAGES;
                if (j >= STAGES && !mbar_wait(&empty_bar[s], ((j / STAGES) - 1) & 1, a.status)) {
                    atomicOr(&flag_s, 1);
                    break;
                }
                const int rows = min(P, p_end - p_begin - j * P);
                const uint32_t bytes = (uint32_t)rows * ROW;
                KV *sk = stages + (size_t)s * 2 * P * HD;
                mbar_arrive_expect_tx(&full_bar[s], 2 * bytes);
                bulk_g2s(sk, kbase + (size_t)j * P * HD, bytes, &full_bar[s]);
                bulk_g2s(sk + P * HD, vbase + (size_t)j * P * HD, bytes, &full_bar[s]);
            }
        }
    } else {
        // ---------------- consumers ----------------
        if (FUSED) {
            // q/k RMSNorm + RoPE for this KV head's query heads, computed
            // while the first tiles are in flight, with this position's
            // angles from the context's table
            float x[8];
            const float *src = a.qg + (size_t)(head0 + warp) * 2 * HD + lane * 8;
#pragma unroll
            for (int e = 0; e < 8; e += 4) {
                const float4 f = *reinterpret_cast<const float4 *>(src + e);
                x[e] = f.x, x[e + 1] = f.y, x[e + 2] = f.z, x[e + 3] = f.w;
            }
            const int half = a.n_rot / 2;
            for (int i = tid; i < half; i += 32 * CWARPS) {
                rope_cs[i] = a.rope_cs[(size_t)pos_row * half + i];
                rope_sn[i] = a.rope_sn[(size_t)pos_row * half + i];
            }
            consumer_bar();
            warp_norm_rope<dec2::HD>(x, a.q_norm, q_s[warp], rope_cs, rope_sn, a.n_rot, a.eps, lane);
            if (covers_new && warp < 2) {
                // warp 0: the new key (normed, rotated); warp 1: the new value.
                // Both are rounded to the cache's type, stored to the cache
                // and kept in shared memory for the tile that holds them.
                const float *in = (warp == 0 ? a.k_in : a.v_in) + (size_t)row * a.n_kv * HD +
                                  (size_t)kh * HD + lane * 8;
#pragma unroll
                for (int e = 0; e < 8; e += 4) {
                    const float4 f = *reinterpret_cast<const float4 *>(in + e);
                    x[e] = f.x, x[e + 1] = f.y, x[e + 2] = f.z, x[e + 3] = f.w;
                }
                float y[8];
                if (warp == 0) {
                    warp_norm_rope<dec2::HD>(x, a.k_norm, kf_s, rope_cs, rope_sn, a.n_rot, a.eps, lane);
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = kf_s[lane * 8 + e];
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = x[e];
                }
                KV *cache = (warp == 0 ? k_cache : v_cache) +
                            ((size_t)kh * a.context + pos_row) * HD + lane * 8;
                KV *keep = (warp == 0 ? newk_s : newv_s) + lane * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const KV r = from_f32<KV>(y[e]);
                    cache[e] = r;
                    keep[e] = r;
                }
            }
            consumer_bar();
        }
        // queries for QK: lane (sub, part) covers chunks part + 16*c of a row
        const int part = lane & 15, sub = lane >> 4;
        float2 qr[GROUP][8];
#pragma unroll
        for (int h = 0; h < GROUP; ++h)
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const float *src = FUSED ? &q_s[h][(part + 16 * c) * EPC]
                                         : a.q_f32 + (size_t)(head0 + h) * HD + (part + 16 * c) * EPC;
#pragma unroll
                for (int e = 0; e < EPC; e += 4) {
                    const float4 f = *reinterpret_cast<const float4 *>(src + e);
                    qr[h][(c * EPC + e) / 2] = make_float2(f.x, f.y);
                    qr[h][(c * EPC + e) / 2 + 1] = make_float2(f.z, f.w);
                }
            }
        const float qk_scale = (1.0f / 16.0f) * LOG2E;  // 1/sqrt(256), in log2 units
        const int hq = (part >> 2) & 3;                     // head this lane's scores belong to
        const int pw0 = warp * PPW;

        for (int j = 0; j < n_tiles; ++j) {
            const int s = j % STAGES;
            // the warp gives up as one, so no lane is left at a shuffle
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[s], (j / STAGES) & 1, a.status))) {
                ok = false;
                break;
            }
            const KV *K = stages + (size_t)s * 2 * P * HD;
            const KV *V = K + P * HD;
            const int base = p_begin + j * P;
            const int valid = min(P, p_end - base);
            // ---- scores
            float sc[PPW / 2];
#pragma unroll
            for (int st = 0; st < PPW / 2; ++st) {
                const int p = pw0 + 2 * st + sub;
                const KV *krow = (FUSED && base + p == pos_row) ? newk_s : K + p * HD;
                float2 a2[GROUP];
#pragma unroll
                for (int h = 0; h < GROUP; ++h) a2[h] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(krow + (part + 16 * c) * EPC);
                    float2 kf[EPC / 2];
                    chunk_to_f2(w, kf, (const KV *)nullptr);
#pragma unroll
                    for (int e = 0; e < EPC / 2; ++e)
#pragma unroll
                        for (int h = 0; h < GROUP; ++h)
                            a2[h] = __ffma2_rn(qr[h][c * EPC / 2 + e], kf[e], a2[h]);
                }
                float av[GROUP];
#pragma unroll
                for (int h = 0; h < GROUP; ++h) av[h] = a2[h].x + a2[h].y;
                const bool b3 = part & 8, b2 = part & 4;
                const float keep0 = b3 ? av[2] : av[0], keep1 = b3 ? av[3] : av[1];
                const float send0 = b3 ? av[0] : av[2], send1 = b3 ? av[1] : av[3];
                const float y0 = keep0 + __shfl_xor_sync(0xffffffffu, send0, 8);
                const float y1 = keep1 + __shfl_xor_sync(0xffffffffu, send1, 8);
                float z = (b2 ? y1 : y0) + __shfl_xor_sync(0xffffffffu, b2 ? y0 : y1, 4);
                z += __shfl_xor_sync(0xffffffffu, z, 2);
                z += __shfl_xor_sync(0xffffffffu, z, 1);
                sc[st] = p < valid ? z * qk_scale : -INFINITY;
            }
            // ---- online softmax over this warp's positions, head hq
            float mx = sc[0];
#pragma unroll
            for (int st = 1; st < PPW / 2; ++st) mx = fmaxf(mx, sc[st]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float m_new = fmaxf(m_run, mx);
            const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
            float ps = 0.0f;
#pragma unroll
            for (int st = 0; st < PPW / 2; ++st) {
                const float pv = m_new == -INFINITY ? 0.0f : exp2f(sc[st] - m_new);
                ps += pv;
                if ((part & 3) == 0) wbuf[warp][2 * st + sub][hq] = pv;
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l_run = fmaf(l_run, alpha, ps);
            m_run = m_new;
            if ((part & 3) == 0 && sub == 0) abuf[warp][hq] = alpha;
            __syncwarp();
            // ---- weighted values
            {
                const float4 al4 = *reinterpret_cast<const float4 *>(abuf[warp]);
                const float al[GROUP] = {al4.x, al4.y, al4.z, al4.w};
#pragma unroll
                for (int h = 0; h < GROUP; ++h) {
                    const float2 a2 = make_float2(al[h], al[h]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[h][e] = __fmul2_rn(acc[h][e], a2);
                }
#pragma unroll
                for (int q = 0; q < PPW; ++q) {
                    const int p = pw0 + q;
                    if (p < valid) {
                        const float4 w4 = *reinterpret_cast<const float4 *>(wbuf[warp][q]);
                        const float wv[GROUP] = {w4.x, w4.y, w4.z, w4.w};
                        const KV *vrow = (FUSED && base + p == pos_row) ? newv_s : V + p * HD;
#pragma unroll
                        for (int c = 0; c < PV_CH; ++c) {
                            const uint4 w = *reinterpret_cast<const uint4 *>(vrow + (lane + 32 * c) * EPC);
                            float2 vf[EPC / 2];
                            chunk_to_f2(w, vf, (const KV *)nullptr);
#pragma unroll
                            for (int e = 0; e < EPC / 2; ++e)
#pragma unroll
                                for (int h = 0; h < GROUP; ++h)
                                    acc[h][c * EPC / 2 + e] = __ffma2_rn(
                                        make_float2(wv[h], wv[h]), vf[e], acc[h][c * EPC / 2 + e]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
        }
    }

    // ---------------- merge the four consumer warps ----------------
    __syncthreads();  // every tile consumed: the stage ring is free
    if (!ok) atomicOr(&flag_s, 1);
    float *red_o = reinterpret_cast<float *>(smem);            // [CWARPS][GROUP][HD]
    float *red_ml = red_o + CWARPS * GROUP * HD;               // [CWARPS][GROUP][2]
    float *cta_o = red_ml + CWARPS * GROUP * 2;                // [GROUP][HD]
    if (warp < CWARPS) {
#pragma unroll
        for (int h = 0; h < GROUP; ++h)
#pragma unroll
            for (int c = 0; c < PV_CH; ++c)
#pragma unroll
                for (int e = 0; e < EPC; e += 4) {
                    const float2 lo = acc[h][(c * EPC + e) / 2], hi = acc[h][(c * EPC + e) / 2 + 1];
                    *reinterpret_cast<float4 *>(
                        &red_o[(warp * GROUP + h) * HD + (lane + 32 * c) * EPC + e]) =
                        make_float4(lo.x, lo.y, hi.x, hi.y);
                }
        const int part = lane & 15;
        if ((part & 3) == 0 && lane < 16) {
            red_ml[(warp * GROUP + (part >> 2)) * 2] = m_run;
            red_ml[(warp * GROUP + (part >> 2)) * 2 + 1] = l_run;
        }
    }
    __syncthreads();
    decode_merge<HD, GROUP, CWARPS, THREADS>(cluster, a, red_o, red_ml, cta_o, cta_m, cta_l,
                                             flag_s, head0, kh, row, crank, cl, n_cl, C, tid);
}

template <typename KV, bool FUSED>
static cudaError_t launch_t(const DecodeArgs &a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.n_kv, a.t);
    cfg.blockDim = dim3(dec2::THREADS);
    cfg.dynamicSmemBytes = dec2_smem_bytes<KV>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_kernel<KV, FUSED>, a);
}

cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t st) {
    if (a.kv_bf16)
        return a.fused ? launch_t<__nv_bfloat16, true>(a, st) : launch_t<__nv_bfloat16, false>(a, st);
    return a.fused ? launch_t<float, true>(a, st) : launch_t<float, false>(a, st);
}

template <typename KV, bool FUSED>
static cudaError_t set_attr() {
    return cudaFuncSetAttribute(decode_kernel<KV, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)dec2_smem_bytes<KV>());
}

cudaError_t init_decode_kernels() {
    cudaError_t e;
    if ((e = set_attr<__nv_bfloat16, true>()) != cudaSuccess) return e;
    if ((e = set_attr<__nv_bfloat16, false>()) != cudaSuccess) return e;
    if ((e = set_attr<float, true>()) != cudaSuccess) return e;
    return set_attr<float, false>();
}

// Clusters of `csize` decode CTAs that can be resident at once on this
// device (0 if the configuration cannot launch).
int decode_max_active_clusters(bool kv_bf16, bool fused, int csize) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csize * 64, 1, 1);
    cfg.blockDim = dim3(dec2::THREADS);
    cfg.dynamicSmemBytes =
        kv_bf16 ? dec2_smem_bytes<__nv_bfloat16>() : dec2_smem_bytes<float>();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    cudaError_t e;
    if (kv_bf16)
        e = fused ? cudaOccupancyMaxActiveClusters(&n, decode_kernel<__nv_bfloat16, true>, &cfg)
                  : cudaOccupancyMaxActiveClusters(&n, decode_kernel<__nv_bfloat16, false>, &cfg);
    else
        e = fused ? cudaOccupancyMaxActiveClusters(&n, decode_kernel<float, true>, &cfg)
                  : cudaOccupancyMaxActiveClusters(&n, decode_kernel<float, false>, &cfg);
    return e == cudaSuccess ? n : 0;
}

int decode_positions_per_tile(bool kv_bf16) {
    return kv_bf16 ? Dec2Traits<__nv_bfloat16>::P : Dec2Traits<float>::P;
}

}  // namespace rl
