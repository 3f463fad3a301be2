// KV cache fill and read-back in f32, for tests, checkpoints and benchmark
// set-up (rl_write_kv / rl_read_kv).  src/dst are [2][n_kv][n][hd] f32; the
// cache is [n_kv][context][hd] per half, f32 or bf16.
#include "common.cuh"
#include "kernels.h"

namespace rl {

template <typename KV>
__global__ void kv_fill_kernel(KV *__restrict__ k_cache, KV *__restrict__ v_cache,
                               const float *__restrict__ src, int n_kv, int context, int hd,
                               int p0, int n) {
    const size_t per_half = (size_t)n_kv * n * hd;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < 2 * per_half;
         e += (size_t)gridDim.x * blockDim.x) {
        const size_t w = e % per_half;
        const int h = (int)(w / ((size_t)n * hd));
        const size_t rem = w % ((size_t)n * hd);
        const size_t to = ((size_t)h * context + p0) * hd + rem;
        (e < per_half ? k_cache : v_cache)[to] = from_f32<KV>(src[e]);
    }
}

template <typename KV>
__global__ void kv_read_kernel(const KV *__restrict__ k_cache, const KV *__restrict__ v_cache,
                               float *__restrict__ dst, int n_kv, int context, int hd, int p0,
                               int n) {
    const size_t per_half = (size_t)n_kv * n * hd;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < 2 * per_half;
         e += (size_t)gridDim.x * blockDim.x) {
        const size_t w = e % per_half;
        const int h = (int)(w / ((size_t)n * hd));
        const size_t rem = w % ((size_t)n * hd);
        const size_t from = ((size_t)h * context + p0) * hd + rem;
        dst[e] = (float)(e < per_half ? k_cache : v_cache)[from];
    }
}

cudaError_t launch_kv_fill(void *k_cache, void *v_cache, const float *src, int n_kv,
                           int context, int hd, int p0, int n, bool kv_bf16, cudaStream_t st) {
    const int blocks = 148 * 8, threads = 256;
    if (kv_bf16)
        kv_fill_kernel<<<blocks, threads, 0, st>>>((__nv_bfloat16 *)k_cache,
                                                   (__nv_bfloat16 *)v_cache, src, n_kv, context,
                                                   hd, p0, n);
    else
        kv_fill_kernel<<<blocks, threads, 0, st>>>((float *)k_cache, (float *)v_cache, src, n_kv,
                                                   context, hd, p0, n);
    return cudaGetLastError();
}

cudaError_t launch_kv_read(const void *k_cache, const void *v_cache, float *dst, int n_kv,
                           int context, int hd, int p0, int n, bool kv_bf16, cudaStream_t st) {
    const int blocks = 148 * 8, threads = 256;
    if (kv_bf16)
        kv_read_kernel<<<blocks, threads, 0, st>>>((const __nv_bfloat16 *)k_cache,
                                                   (const __nv_bfloat16 *)v_cache, dst, n_kv,
                                                   context, hd, p0, n);
    else
        kv_read_kernel<<<blocks, threads, 0, st>>>((const float *)k_cache, (const float *)v_cache,
                                                   dst, n_kv, context, hd, p0, n);
    return cudaGetLastError();
}

}  // namespace rl
