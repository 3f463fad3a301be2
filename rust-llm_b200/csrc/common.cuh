// Shared device helpers for the sm_100a attention kernels: bf16 unpacking,
// mbarrier + bulk-copy (TMA) wrappers, bounded waits, block reductions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rl {

// Device status bits, OR-ed into the context's status word by a kernel that
// had to give up; rl_sync() turns them into RL_ETIMEOUT / RL_EINVAL.
constexpr int DEV_TIMEOUT = 1;
constexpr int DEV_BAD_ARG = 2;

// A bounded wait gives up after this many SM clocks (about a second at the
// B200's 1.0-2.0 GHz), sets DEV_TIMEOUT and lets the kernel return.
constexpr long long WAIT_LIMIT_CYCLES = 2000000000ll;
// The default limit, in nanoseconds, of a wait on another GPU's flag (the
// context option RL_OPT_WAIT_LIMIT_US overrides it).
constexpr unsigned long long PEER_WAIT_LIMIT_NS = 1000000000ull;

// A value with its step's epoch in one 64-bit store (single-copy atomic at
// system scope), to another GPU's memory or this one's.
__device__ __forceinline__ void xstore(unsigned long long *dst, float v, unsigned epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
}

// The global nanosecond timer (the same on every SM of the GPU).
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most WAIT_LIMIT_CYCLES.
// Returns false (and flags DEV_TIMEOUT) when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > WAIT_LIMIT_CYCLES) {
            atomicOr(status, DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier 1 over the 128 threads of warps 0-3 (the consumer warps of
// the decode kernels; their producer warp does not take part).
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// ---- bulk copies (TMA, non-tensor) ---------------------------------------
// One contiguous global -> shared copy completing on `bar`.  Both addresses
// 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- tensor copies (TMA, tiled) --------------------------------------------
// One box of a 2-D tensor map, global -> shared, completing on `bar`.  The
// map is a __grid_constant__ kernel parameter.  x (the innermost
// coordinate, in elements) must keep x * element size a multiple of 16
// bytes; y may be any row.  No multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// One box of a 2-D tensor map, shared -> global, in this thread's current
// bulk group; the same x rule as the load (x * element size a multiple of
// 16 bytes), and x, y never negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *src) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_u32(src))
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's most recent bulk groups have still
// to read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until this thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Brings `bytes` (a multiple of 16, 16-byte aligned) of global memory into
// L2 without waiting for it.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a box written
// with the 128-byte swizzle (rows of 128 bytes, box base 1024-byte aligned).
__device__ __forceinline__ uint32_t swz128(int r, int c) {
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// ---- bf16 ----------------------------------------------------------------
// Eight bf16 in a 16-byte word, widened to f32 exactly.
__device__ __forceinline__ void bf16x8_to_f32(const uint4 &w, float *f) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(u[i] << 16);
        f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) {
    return x;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// ---- warp / block reductions ---------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block in f64 (the reference accumulates squares in f64).
// `red` holds blockDim.x/32 doubles.  Every thread gets the total.
__device__ __forceinline__ double block_sum_d(double v, double *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = -0.0;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

// The reference's rms_scale (forward.rs:1697-1711) from an f64 sum of f32
// squares: the mean rounded to f32, an f32 root and reciprocal.
__device__ __forceinline__ float rms_scale_from_sum(double sum, int n, float eps) {
    // sum / n; for a power-of-two n the product with the exact reciprocal is
    // the same rounding and avoids a double division
    const double mean_d = (n & (n - 1)) == 0 ? sum * (1.0 / (double)n) : sum / (double)n;
    const float mean = static_cast<float>(mean_d);
    return 1.0f / sqrtf(__fadd_rn(mean, eps));
}

// The same scale with the hardware reciprocal square root (within 2 ulp of
// 1 / sqrt), for norms on a kernel's critical path; n a power of two.
__device__ __forceinline__ float rms_scale_fast(double sum, int n, float eps) {
    const float mean = static_cast<float>(sum * (1.0 / (double)n));
    return rsqrtf(__fadd_rn(mean, eps));
}

// Programmatic dependent launch: wait for the grid ahead on the stream to
// complete (its writes visible); let the next grid on the stream launch.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Named barrier `id` (1..15) over `n` threads (a multiple of 32).
__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Split-phase cluster barrier: every thread of every CTA of the cluster
// arrives (release), then waits (acquire) before the next arrive.
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store one double into the same shared variable of cluster CTA `rank`,
// completing 8 bytes of transaction on that CTA's copy of mbarrier `bar`
// (no fence: the receiver learns of it from its own barrier).
__device__ __forceinline__ void st_async_cluster_f64(const void *local, const uint64_t *bar,
                                                     int rank, double v) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    uint32_t ra, rb;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(b), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f64 [%0], %1, [%2];" ::
                     "r"(ra), "d"(v), "r"(rb)
                 : "memory");
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplusf_(float x) {
    return x > 20.0f ? x : log1pf(expf(x));
}

}  // namespace rl

namespace rl {
// Reads a value stored by xstore once it carries `epoch`, waiting until
// `start + limit_ns` at most (then `late` is set and the value is whatever
// is there).
__device__ __forceinline__ float xload(const unsigned long long *src, unsigned epoch,
                                       unsigned long long start, unsigned long long limit_ns,
                                       bool &late) {
    unsigned long long w;
    while (true) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
        if ((unsigned)(w >> 32) == epoch || late) break;
        if (globaltimer_ns() - start > limit_ns) {
            late = true;
            break;
        }
        __nanosleep(20);
    }
    return __uint_as_float((unsigned)w);
}
}  // namespace rl

namespace rl {
// A flag another CTA of the same GPU publishes once its global writes are
// done: st.release.gpu after every writer's fence and a CTA barrier on the
// writing side; ld.acquire.gpu here.  Waits until the flag holds `value`,
// for PEER_WAIT_LIMIT_NS at most on the global timer; a wait that gives up
// flags DEV_TIMEOUT and returns false.
__device__ __forceinline__ void st_release_gpu(int *p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add_gpu(int *p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool wait_flag_gpu(const int *flag, int value, int *status) {
    if (ld_acquire_gpu(flag) == value) return true;
    const unsigned long long start = globaltimer_ns();
    while (ld_acquire_gpu(flag) != value) {
        if (globaltimer_ns() - start > PEER_WAIT_LIMIT_NS) {
            atomicOr(status, DEV_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}
}  // namespace rl

namespace rl {
// A tiled TMA load of a 3-D box at (x, y, z), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y,
                                            int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
}  // namespace rl
