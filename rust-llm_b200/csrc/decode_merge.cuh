// Shared tail of the split-KV decode kernels: merge the consumer warps'
// partial softmax states, merge the cluster's splits through distributed
// shared memory (each rank one slice of the head dimension), and, with more
// than one cluster, let the last cluster to finish a slice merge that slice
// across clusters from global memory and apply the sigmoid output gate.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace rl {

// RMSNorm (f64 sum of f32 squares, forward.rs:1697-1711) and partial RoPE
// from the angle table of one 256-wide head by one warp; the result lands in
// `dst` (shared).  x holds the lane's 8 consecutive inputs.
template <int HD>
__device__ __forceinline__ void warp_norm_rope(const float *x, const float *w, float *dst,
                                               const float *cs, const float *sn, int n_rot,
                                               float eps, int lane) {
    double sq = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) sq += (double)__fmul_rn(x[e], x[e]);
    sq = warp_sum_d(sq);
    const float scale = rms_scale_from_sum(sq, HD, eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane * 8 + e] = __fmul_rn(__fmul_rn(x[e], scale), w[lane * 8 + e]);
    __syncwarp();
    const int half = n_rot / 2;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        y[e] = dst[d];
        if (d < n_rot) {
            const int pr = d < half ? d : d - half;
            const float c = cs[pr], s = sn[pr];
            const float x0 = dst[pr], x1 = dst[pr + half];
            y[e] = d < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                            : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    }
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane * 8 + e] = y[e];
    __syncwarp();
}


// red_o [CWARPS][GROUP][HD] and red_ml [CWARPS][GROUP][2] hold every consumer
// warp's unnormalised output and (max, sum), already written; cta_o
// ([GROUP][HD]), cta_m, cta_l ([GROUP]) are this CTA's shared scratch for
// the merged state.  All THREADS threads of every CTA of the cluster call it.
template <int HD, int GROUP, int CWARPS, int THREADS>
__device__ __forceinline__ void decode_merge(cooperative_groups::cluster_group &cluster,
                                             const DecodeArgs &a, const float *red_o,
                                             const float *red_ml, float *cta_o, float *cta_m,
                                             float *cta_l, int flag, int head0, int kh,
                                             int row, int crank, int cl, int n_cl, int C,
                                             int tid) {
    __syncthreads();
    __shared__ float wscale[CWARPS][GROUP];
    if (tid < GROUP) {
        float M = -INFINITY;
        for (int w = 0; w < CWARPS; ++w) M = fmaxf(M, red_ml[(w * GROUP + tid) * 2]);
        float L = 0.0f;
        for (int w = 0; w < CWARPS; ++w) {
            const float mw = red_ml[(w * GROUP + tid) * 2];
            const float sc = mw == -INFINITY ? 0.0f : exp2f(mw - M);
            wscale[w][tid] = sc;
            L = fmaf(red_ml[(w * GROUP + tid) * 2 + 1], sc, L);
        }
        cta_m[tid] = M;
        cta_l[tid] = L;
    }
    __syncthreads();
    for (int e4 = tid; e4 < GROUP * HD / 4; e4 += THREADS) {
        const int h = e4 / (HD / 4);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) {
            const float sc = wscale[w][h];
            const float4 r = reinterpret_cast<const float4 *>(red_o)[w * GROUP * HD / 4 + e4];
            o.x = fmaf(r.x, sc, o.x), o.y = fmaf(r.y, sc, o.y);
            o.z = fmaf(r.z, sc, o.z), o.w = fmaf(r.w, sc, o.w);
        }
        reinterpret_cast<float4 *>(cta_o)[e4] = o;
    }

    // ---------------- merge the cluster's splits through DSMEM ----------------
    cluster.sync();
    const int ds = HD / C;          // this rank's slice of the head dimension
    const int d0 = crank * ds;
    float *gout_o = a.part_o;       // [row][head][cluster][HD]
    float *gout_ml = a.part_ml;     // [row][head][cluster][C][2]
    __shared__ float rscale[8][GROUP], cl_M[GROUP], cl_L[GROUP];
    if (tid < GROUP) {
        float mr[8], lr[8];
        float M = -INFINITY;
        for (int r = 0; r < C; ++r) {
            mr[r] = *cluster.map_shared_rank(&cta_m[tid], r);
            lr[r] = *cluster.map_shared_rank(&cta_l[tid], r);
            M = fmaxf(M, mr[r]);
        }
        float L = 0.0f;
        for (int r = 0; r < C; ++r) {
            const float sc = mr[r] == -INFINITY ? 0.0f : exp2f(mr[r] - M);
            rscale[r][tid] = sc;
            L = fmaf(lr[r], sc, L);
        }
        cl_M[tid] = M;
        cl_L[tid] = L;
    }
    __syncthreads();
    for (int e4 = tid; e4 < GROUP * ds / 4; e4 += THREADS) {
        const int h = e4 / (ds / 4), d = d0 + (e4 % (ds / 4)) * 4;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < C; ++r) {
            const float sc = rscale[r][h];
            const float4 v = *reinterpret_cast<const float4 *>(
                cluster.map_shared_rank(&cta_o[h * HD + d], r));
            o.x = fmaf(v.x, sc, o.x), o.y = fmaf(v.y, sc, o.y);
            o.z = fmaf(v.z, sc, o.z), o.w = fmaf(v.w, sc, o.w);
        }
        const int hh = head0 + h;  // (row, query head)
        if (n_cl == 1) {
            const float L = cl_L[h];
            const float *g = a.qg + (size_t)hh * 2 * HD + HD + d;
            float *dst = a.out + (size_t)hh * HD + d;
            dst[0] = (o.x / L) * sigmoidf_(g[0]);
            dst[1] = (o.y / L) * sigmoidf_(g[1]);
            dst[2] = (o.z / L) * sigmoidf_(g[2]);
            dst[3] = (o.w / L) * sigmoidf_(g[3]);
        } else {
            *reinterpret_cast<float4 *>(&gout_o[((size_t)hh * n_cl + cl) * HD + d]) = o;
            if (e4 % (ds / 4) == 0) {
                gout_ml[(((size_t)hh * n_cl + cl) * C + crank) * 2] = cl_M[h];
                gout_ml[(((size_t)hh * n_cl + cl) * C + crank) * 2 + 1] = cl_L[h];
            }
        }
    }
    cluster.sync();  // peers are done reading this CTA's shared memory
    if (n_cl == 1) {
        if (flag && tid == 0) atomicOr(a.status, DEV_TIMEOUT);
        return;
    }

    // ---------------- last cluster to finish a slice merges it ----------------
    __threadfence();
    __syncthreads();
    __shared__ int last_s;
    int *counter = a.counters + ((size_t)row * a.n_kv + kh) * 8 + crank;
    if (tid == 0) last_s = atomicAdd(counter, 1) == n_cl - 1;
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    // one thread per (head, 4 dims) of the slice; every load below is
    // independent of the others, so they are all in flight at once
    __shared__ float fscale[GROUP][64];  // per-cluster weights, n_cl <= 64
    __shared__ float fL[GROUP];
    if (tid < GROUP) {
        const float *ml = gout_ml + (size_t)(head0 + tid) * n_cl * C * 2 + crank * 2;
        float M = -INFINITY;
        for (int c = 0; c < n_cl; ++c) M = fmaxf(M, __ldcg(ml + (size_t)c * C * 2));
        float L = 0.0f;
        for (int c = 0; c < n_cl; ++c) {
            const float mc = __ldcg(ml + (size_t)c * C * 2);
            const float sc = mc == -INFINITY ? 0.0f : exp2f(mc - M);
            fscale[tid][c] = sc;
            L = fmaf(__ldcg(ml + (size_t)c * C * 2 + 1), sc, L);
        }
        fL[tid] = L;
    }
    __syncthreads();
    for (int e4 = tid; e4 < GROUP * ds / 4; e4 += THREADS) {
        const int h = e4 / (ds / 4), d = d0 + (e4 % (ds / 4)) * 4;
        const int hh = head0 + h;
        const float4 *src = reinterpret_cast<const float4 *>(gout_o + (size_t)hh * n_cl * HD + d);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int c = 0; c < n_cl; ++c) {
            const float4 v = __ldcg(src + (size_t)c * HD / 4);
            const float sc = fscale[h][c];
            o.x = fmaf(v.x, sc, o.x), o.y = fmaf(v.y, sc, o.y);
            o.z = fmaf(v.z, sc, o.z), o.w = fmaf(v.w, sc, o.w);
        }
        const float L = fL[h];
        const float *g = a.qg + (size_t)hh * 2 * HD + HD + d;
        float *dst = a.out + (size_t)hh * HD + d;
        dst[0] = (o.x / L) * sigmoidf_(g[0]);
        dst[1] = (o.y / L) * sigmoidf_(g[1]);
        dst[2] = (o.z / L) * sigmoidf_(g[2]);
        dst[3] = (o.w / L) * sigmoidf_(g[3]);
    }
    if (tid == 0) {
        *counter = 0;  // ready for the next launch (and the next graph replay)
        if (flag) atomicOr(a.status, DEV_TIMEOUT);
    }
}

}  // namespace rl
