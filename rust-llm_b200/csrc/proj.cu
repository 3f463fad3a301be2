// The projections either side of the attention path on the device, sm_100a:
// activations quantized to int8 per 256-value super-block, then each weight
// row (Q4_K, Q6_K or Q8_0 blocks, the GGUF layouts) dotted with them in
// integer arithmetic and the blocks' scales applied in f32, block by block in
// order.  This is the reference's scalar kernel tier, value for value:
//   Activations::quantize_batch   crates/llm-core/src/quant.rs:337-372
//   q4k_dot_scalar / q6k_dot_scalar / q80_dot_scalar
//                                 crates/llm-core/src/kernels/mod.rs:245-320
// The integer sums are exact whatever their order, and every f32 operation
// is the reference's, in its order and without contraction, so a row's
// result is the scalar tier's bit for bit.  The rows are HBM-bound at decode
// sizes: one warp per weight row, the row's blocks streamed once, all of a
// batch's activation rows dotted against them while they are in registers.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace rl {
namespace pj {
constexpr int QK = 256;            // super-block
constexpr int Q4K_BYTES = 144, Q6K_BYTES = 210, Q80_BYTES = 34;
}  // namespace pj

// ---- activation quantization -------------------------------------------------
// One warp per (row, super-block); lane l takes values 8l .. 8l+7.  amax is a
// max (exact in any order); d = amax / 127 and the inverse 127 / amax are the
// reference's two f32 divisions; q = round(x * inverse), ties away from zero,
// clamped to +-127; the tail past k is zero; bsums are exact.
__global__ void __launch_bounds__(256) q8k_quantize_kernel(const float *x, int k, int t, int nb,
                                                           float *d, int8_t *qs, int16_t *bs) {
    // x comes from the kernel ahead; the scratch it writes was last read by
    // the matvecs ahead, which have completed once this wait returns
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= t * nb) return;
    const int row = item / nb, b = item % nb;
    const float *src = x + (size_t)row * k + (size_t)b * pj::QK + lane * 8;
    const int n = min(pj::QK, k - b * pj::QK) - lane * 8;  // this lane's values inside k
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = e < n ? src[e] : 0.0f;
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
    amax = warp_max(amax);
    const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    int q[8];
    int s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        float r = roundf(__fmul_rn(v[e], id));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[e] = (int)r;
        s += q[e];
    }
    uint2 packed;
    packed.x = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)q[3] << 24);
    packed.y = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)q[7] << 24);
    *reinterpret_cast<uint2 *>(qs + (size_t)item * pj::QK + lane * 8) = packed;
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // 16 values: lanes 2g, 2g + 1
    if (!(lane & 1)) bs[(size_t)item * 16 + lane / 2] = (int16_t)s;
    if (lane == 0) d[item] = __fdiv_rn(amax, 127.0f);
}

// ---- dots ------------------------------------------------------------------------
__device__ __forceinline__ float f16_at(const uint8_t *p) {
    const uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
    return __half2float(__ushort_as_half(h));
}
// Sum over the 8 lanes of a group (lane bits 0-2); exact for integers.
__device__ __forceinline__ int sum8(int v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    return v;
}
__device__ __forceinline__ int sum32(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// 32 bytes of int8 activations, as 8 packed words
__device__ __forceinline__ void act32(const int8_t *p, int (&a)[8]) {
    const int4 x = *reinterpret_cast<const int4 *>(p), y = *reinterpret_cast<const int4 *>(p + 16);
    a[0] = x.x, a[1] = x.y, a[2] = x.z, a[3] = x.w, a[4] = y.x, a[5] = y.y, a[6] = y.z, a[7] = y.w;
}

// Q4_K super-block (d, dmin, 12 bytes of 6-bit scales and mins, 128 bytes of
// nibbles) at b (shared memory) against activation block ab: lane e of the
// block's 8-lane group takes sub-block e (32 weights: the low nibbles of
// bytes (e/2)*32 .. +31 for even e, the high ones for odd).  Returns the
// term ad * (d * isum - dmin * imin) on every lane of the group.
__device__ __forceinline__ float q4k_term(const uint8_t *b, float ad, const int8_t *aq,
                                          const int16_t *bsum, int e, int swz) {
    const uint8_t *scales = b + 4;
    int sc, m;
    if (e < 4) {
        sc = scales[e] & 63;
        m = scales[e + 4] & 63;
    } else {
        sc = (scales[e + 4] & 0xF) | ((scales[e - 4] >> 6) << 4);
        m = (scales[e + 4] >> 4) | ((scales[e] >> 6) << 4);
    }
    const uint4 *wq = reinterpret_cast<const uint4 *>(b + 16 + (e >> 1) * 32);
    const uint4 w0 = wq[0], w1 = wq[1];
    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    int a[8];
    act32(aq + (e ^ swz) * 32, a);
    const int sh = (e & 1) * 4;
    int dot = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) dot = __dp4a((int)((wv[i] >> sh) & 0x0F0F0F0Fu), a[i], dot);
    const int isum = sum8(sc * dot);
    const int imin = sum8(m * ((int)bsum[2 * e] + (int)bsum[2 * e + 1]));
    const float d = f16_at(b), dmin = f16_at(b + 2);
    return __fmul_rn(ad, __fsub_rn(__fmul_rn(d, (float)isum), __fmul_rn(dmin, (float)imin)));
}

// Q6_K super-block (ql 128, qh 64, int8 scales 16, d) at b: lane e of the group
// takes the 32 values e*32 .. e*32+31 (h = e / 4, g = e % 4), whose scales are
// sc[h*8 + 2g] for the first 16 and sc[h*8 + 2g + 1] for the rest.
__device__ __forceinline__ float q6k_term(const uint8_t *b, float ad, const int8_t *aq, int e,
                                          int swz) {
    const int h = e >> 2, g = e & 3;
    const uint8_t *ql = b + h * 64 + (g & 1) * 32, *qh = b + 128 + h * 32;
    int a[8];
    act32(aq + (e ^ swz) * 32, a);
    int dot0 = 0, dot1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = (uint32_t)ql[4 * i] | ((uint32_t)ql[4 * i + 1] << 8) |
                            ((uint32_t)ql[4 * i + 2] << 16) | ((uint32_t)ql[4 * i + 3] << 24);
        const uint32_t hi = (uint32_t)qh[4 * i] | ((uint32_t)qh[4 * i + 1] << 8) |
                            ((uint32_t)qh[4 * i + 2] << 16) | ((uint32_t)qh[4 * i + 3] << 24);
        const uint32_t low = (lo >> ((g >> 1) * 4)) & 0x0F0F0F0Fu;
        const uint32_t high = ((hi >> (2 * g)) & 0x03030303u) << 4;
        const int q = (int)__vsub4(low | high, 0x20202020u);  // (low | high) - 32 per byte
        if (i < 4) dot0 = __dp4a(q, a[i], dot0);
        else dot1 = __dp4a(q, a[i], dot1);
    }
    const int s0 = (int8_t)b[192 + h * 8 + 2 * g], s1 = (int8_t)b[192 + h * 8 + 2 * g + 1];
    const int isum = sum8(s0 * dot0 + s1 * dot1);
    return __fmul_rn(__fmul_rn(ad, f16_at(b + 208)), (float)isum);
}

__device__ __forceinline__ void pj_cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void pj_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pj_cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copies `bytes` from global p (any alignment) into shared s (16-byte
// aligned) plus p's offset within 16 bytes: the whole 16-byte pieces inside
// the range as asynchronous copies in this lane's current group (commit and
// wait before reading them), the ends by bytes, in place on return.  Returns
// the row's start in s.
__device__ __forceinline__ const uint8_t *stage_row_async(uint8_t *s, const uint8_t *p,
                                                          size_t bytes, int lane) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(p), a1 = a0 + bytes;
    const uintptr_t v0 = (a0 + 15) & ~(uintptr_t)15, v1 = a1 & ~(uintptr_t)15;
    const int off = (int)(a0 & 15);
    if (v0 < v1) {
        for (uintptr_t a = v0 + 16 * lane; a < v1; a += 16 * 32)
            pj_cp_async16(s + off + (a - a0), reinterpret_cast<const void *>(a));
    }
    const uintptr_t head_end = v0 < a1 ? v0 : a1;
    for (uintptr_t a = a0 + lane; a < head_end; a += 32) s[off + (a - a0)] = *reinterpret_cast<const uint8_t *>(a);
    for (uintptr_t a = (v1 > head_end ? v1 : head_end) + lane; a < a1; a += 32)
        s[off + (a - a0)] = *reinterpret_cast<const uint8_t *>(a);
    return s + off;
}

// One weight row against t activation rows: the row staged at `row`
// (shared memory), the activations' d / quants / block sums at ad / aq / abs_
// (global or shared memory, [t][nb], [t][nb][256], [t][nb][16]).  The warp's
// four 8-lane groups take four super-blocks at a time (lane e of a group
// sub-block e); lane 0 adds their terms to the running f32 sum in block
// order, and writes out[tt * rows + r].  SWZ: the activations sit in the
// one-launch kernel's shared memory, where 32-byte unit u of block b is
// stored at unit u ^ (b & 7).
template <bool SWZ>
__device__ __forceinline__ void row_dots(const uint8_t *row, int type, int k, int nb,
                                         const float *ad, const int8_t *aq, const int16_t *abs_,
                                         int t, int rows, int r, float *out, int lane) {
    const int grp = lane >> 3, e = lane & 7;
    for (int tt = 0; tt < t; ++tt) {
        const float *adt = ad + (size_t)tt * nb;
        const int8_t *aqt = aq + (size_t)tt * nb * pj::QK;
        float sum = 0.0f;
        if (type == 8) {
            // Q8_0: lane l takes blocks l, l + 32, ...; each block's term is
            // independent, the sum over them sequential in block order
            const int n32 = (k + 31) / 32;
            for (int i0 = 0; i0 < n32; i0 += 32) {
                const int ib = i0 + lane;
                float term = 0.0f;
                if (ib < n32) {
                    const uint8_t *b = row + (size_t)ib * pj::Q80_BYTES;
                    const int blk = ib / 8;
                    const int8_t *qa =
                        aqt + (size_t)blk * pj::QK + ((ib % 8) ^ (SWZ ? blk & 7 : 0)) * 32;
                    int dot = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int w = (int)((uint32_t)b[2 + 4 * i] | ((uint32_t)b[3 + 4 * i] << 8) |
                                            ((uint32_t)b[4 + 4 * i] << 16) |
                                            ((uint32_t)b[5 + 4 * i] << 24));
                        dot = __dp4a(w, *reinterpret_cast<const int *>(qa + 4 * i), dot);
                    }
                    term = __fmul_rn(__fmul_rn(f16_at(b), adt[blk]), (float)dot);
                }
                const int n = min(32, n32 - i0);
                for (int i = 0; i < n; ++i) {
                    const float v = __shfl_sync(0xffffffffu, term, i);
                    if (lane == 0) sum = __fadd_rn(sum, v);
                }
            }
        } else {
            for (int ib0 = 0; ib0 < nb; ib0 += 4) {
                // every lane runs a block (the group shuffles take all 32
                // lanes); a group past the row's end repeats the last block
                // and its term is dropped
                const int ib = min(ib0 + grp, nb - 1);
                const size_t ab = (size_t)tt * nb + ib;
                const int swz = SWZ ? ib & 7 : 0;
                float term = type == 12 ? q4k_term(row + (size_t)ib * pj::Q4K_BYTES, ad[ab],
                                                   aq + ab * pj::QK, abs_ + ab * 16, e, swz)
                                        : q6k_term(row + (size_t)ib * pj::Q6K_BYTES, ad[ab],
                                                   aq + ab * pj::QK, e, swz);
                if (ib0 + grp >= nb) term = 0.0f;
                const int n = min(4, nb - ib0);
                for (int i = 0; i < n; ++i) {
                    const float v = __shfl_sync(0xffffffffu, term, 8 * i);
                    if (lane == 0) sum = __fadd_rn(sum, v);
                }
            }
        }
        if (lane == 0) out[(size_t)tt * rows + r] = sum;
    }
}

// Q4_K rows with one lane per super-block: lane l takes block b = l % nb of
// row j = l / nb (32 / nb rows a warp) when nb <= 32, else blocks l, l + 32,
// ... of one row.  The lane runs the whole block's integer dot (eight
// sub-blocks of 32 weights, dp4a) and its f32 term alone, so no shuffle
// reduction is spent on a block; the row's terms are then added in block
// order by the row's first lane, as the reference adds them.  The rows are
// staged contiguously at `span` (shared memory, 16-byte aligned, `stride`
// bytes apart); the activations sit in shared memory in the swizzled layout
// (32-byte unit u of block b at unit u ^ (b & 7)).
__device__ __forceinline__ float q4k_block(const uint8_t *blk, int ab, int bsw, const float *ad,
                                           const int8_t *aq, const int16_t *abs_) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, 12 scale bytes
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    auto byte_at = [](uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFF); };
    const int8_t *a = aq + (size_t)ab * pj::QK;
    const uint32_t *bs = reinterpret_cast<const uint32_t *>(abs_ + (size_t)ab * 16);
    int isum = 0, imin = 0;
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
        // the 32 nibble bytes that sub-blocks 2pr (low nibbles) and 2pr + 1
        // (high nibbles) share
        const uint4 w0 = *reinterpret_cast<const uint4 *>(blk + 16 + pr * 32);
        const uint4 w1 = *reinterpret_cast<const uint4 *>(blk + 32 + pr * 32);
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = 2 * pr + h;
            int sc, m;
            if (e < 4) {
                sc = byte_at(e < 4 ? s0 : s1, e & 3) & 63;
                m = byte_at(s1, e & 3) & 63;
            } else {
                sc = (byte_at(s2, e & 3) & 0xF) | ((byte_at(s0, e & 3) >> 6) << 4);
                m = (byte_at(s2, e & 3) >> 4) | ((byte_at(s1, e & 3) >> 6) << 4);
            }
            const int8_t *au = a + ((e ^ bsw) * 32);
            const int4 x = *reinterpret_cast<const int4 *>(au), y = *reinterpret_cast<const int4 *>(au + 16);
            const int av[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = __dp4a((int)((wv[i] >> (4 * h)) & 0x0F0F0F0Fu), av[i], dot);
            isum += sc * dot;
            const uint32_t pair = bs[e];  // block sums 2e and 2e + 1 (int16 each)
            imin += m * ((int)(int16_t)(pair & 0xFFFF) + (int)(int16_t)(pair >> 16));
        }
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    return __fmul_rn(ad[ab], __fsub_rn(__fmul_rn(d, (float)isum), __fmul_rn(dmin, (float)imin)));
}

__device__ __forceinline__ void q4k_lane_rows(const uint8_t *span, size_t stride, int nr, int nb,
                                              const float *ad, const int8_t *aq,
                                              const int16_t *abs_, int t, int rows, int r0,
                                              float *out, int lane) {
    if (nb <= 32) {
        const int j = lane / nb, b = lane - j * nb;
        const bool live = j < nr;
        const int first = j * nb;  // the row's first lane
        const uint8_t *blk = span + (size_t)(live ? j : 0) * stride + (size_t)b * pj::Q4K_BYTES;
        for (int tt = 0; tt < t; ++tt) {
            float term = 0.0f;
            if (live) term = q4k_block(blk, tt * nb + b, b & 7, ad, aq, abs_);
            float sum = 0.0f;
            for (int i = 0; i < nb; ++i) {
                const float v = __shfl_sync(0xffffffffu, term, min(first + i, 31));
                if (live && b == 0) sum = __fadd_rn(sum, v);
            }
            if (live && b == 0) out[(size_t)tt * rows + r0 + j] = sum;
        }
    } else {
        // one row (nr == 1): lane l takes blocks l + 32 i, lane 0 adds them
        // in block order
        constexpr int kMaxPasses = 8;  // nb <= 256: k <= 65536
        for (int tt = 0; tt < t; ++tt) {
            float term[kMaxPasses];
#pragma unroll
            for (int i = 0; i < kMaxPasses; ++i) {
                const int b = lane + 32 * i;
                term[i] = b < nb ? q4k_block(span + (size_t)b * pj::Q4K_BYTES, tt * nb + b, b & 7,
                                             ad, aq, abs_)
                                 : 0.0f;
            }
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < kMaxPasses; ++i) {
                const int n = min(32, nb - 32 * i);
                for (int l = 0; l < n; ++l) {
                    const float v = __shfl_sync(0xffffffffu, term[i], l);
                    if (lane == 0) sum = __fadd_rn(sum, v);
                }
            }
            if (lane == 0) out[(size_t)tt * rows + r0] = sum;
        }
    }
}

// Weight row `gr` of the group: its part, its row within the part, its bytes.
struct GroupRow {
    int p, r;
    const uint8_t *bytes;
};
__device__ __forceinline__ GroupRow group_row(const MatvecGroup &g, int gr) {
    int p = 0;
    while (p < g.n && gr >= g.rows[p]) gr -= g.rows[p++];
    GroupRow out{p, gr, nullptr};
    if (p < g.n) out.bytes = static_cast<const uint8_t *>(g.w[p]) + (size_t)gr * g.stride[p];
    return out;
}

// One warp per weight row against activations already quantized (by
// q8k_quantize_kernel).  Launched as a programmatic dependent: the row is
// staged before the wait for the kernel ahead (the quantization), since the
// weights do not depend on it.
constexpr int kMvWarps = 4;
__global__ void __launch_bounds__(kMvWarps * 32)
    matvec_group_kernel(const __grid_constant__ MatvecGroup g, int k, int nb, const float *ad,
                        const int8_t *aq, const int16_t *abs_, int t, int row_smem) {
    extern __shared__ __align__(16) uint8_t mv_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const GroupRow gr = group_row(g, blockIdx.x * kMvWarps + warp);
    const bool live = gr.p < g.n;
    const uint8_t *row = nullptr;
    // asynchronous copies: every piece of the row in flight at once
    if (live) row = stage_row_async(mv_smem + warp * row_smem, gr.bytes, g.stride[gr.p], lane);
    pj_cp_commit();
    grid_dep_wait();    // the activations are quantized
    grid_dep_launch();  // the next kernel may start staging its own weights
    pj_cp_wait<0>();
    __syncwarp();
    if (!live) return;
    row_dots<false>(row, g.type[gr.p], k, nb, ad, aq, abs_, t, g.rows[gr.p], gr.r, g.out[gr.p],
                    lane);
}

// Exec::matmul_group in one launch.  Each warp owns a span of consecutive
// rows of one part of the group (rpw rows: 32 / nb of them for Q4_K, whose
// lanes take one super-block each; one row for the other types) and stages
// the span in shared memory by asynchronous copies before the programmatic-
// dependency wait, since the weights do not depend on the kernel ahead, so
// the grid streams its weights while that kernel finishes.  After the wait
// every CTA quantizes the t activation rows into its shared memory (the same
// bits in every CTA: the quantization is a function of the values alone), in
// the swizzled layout the block lanes read without bank conflicts.
constexpr int kMmWarps = 8;
__global__ void __launch_bounds__(kMmWarps * 32)
    matmul_group_kernel(const __grid_constant__ MatvecGroup g, const float *x, int k, int nb,
                        int t, int span_smem) {
    extern __shared__ __align__(16) uint8_t mm_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int items = t * nb;
    int8_t *aq = reinterpret_cast<int8_t *>(mm_smem);
    float *ad = reinterpret_cast<float *>(mm_smem + (size_t)items * pj::QK);
    int16_t *abs_ = reinterpret_cast<int16_t *>(mm_smem + (size_t)items * (pj::QK + 4));
    uint8_t *span_s = mm_smem + (((size_t)items * (pj::QK + 4 + 32) + 15) / 16 * 16) +
                      (size_t)warp * span_smem;
    // this warp's part and rows
    const int gw = (int)blockIdx.x * kMmWarps + warp;
    int p = 0;
    while (p < g.n && gw >= g.wfirst[p + 1]) ++p;
    const bool live = p < g.n;
    int r0 = 0, nr = 0;
    const uint8_t *span = nullptr;
    if (live) {
        r0 = (gw - g.wfirst[p]) * g.rpw[p];
        nr = min(g.rpw[p], g.rows[p] - r0);
        span = stage_row_async(span_s, static_cast<const uint8_t *>(g.w[p]) + (size_t)r0 * g.stride[p],
                               (size_t)nr * g.stride[p], lane);
    }
    pj_cp_commit();
    grid_dep_wait();    // x comes from the kernel ahead
    grid_dep_launch();  // the next kernel may start staging its own weights
    // the activations, as q8k_quantize_kernel quantizes them, 32-byte unit u
    // of block b stored at unit u ^ (b & 7)
    for (int item = warp; item < items; item += kMmWarps) {
        const int rr = item / nb, b = item % nb;
        const float *src = x + (size_t)rr * k + (size_t)b * pj::QK + lane * 8;
        const int n = min(pj::QK, k - b * pj::QK) - lane * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = i < n ? src[i] : 0.0f;
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = warp_max(amax);
        const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        int q[8], sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float f = roundf(__fmul_rn(v[i], id));
            f = fminf(fmaxf(f, -127.0f), 127.0f);
            q[i] = (int)f;
            sum += q[i];
        }
        uint2 packed;
        packed.x = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)q[3] << 24);
        packed.y = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)q[7] << 24);
        const int unit = (lane >> 2) ^ (b & 7);
        *reinterpret_cast<uint2 *>(aq + (size_t)item * pj::QK + unit * 32 + (lane & 3) * 8) = packed;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (!(lane & 1)) abs_[(size_t)item * 16 + lane / 2] = (int16_t)sum;
        if (lane == 0) ad[item] = __fdiv_rn(amax, 127.0f);
    }
    __syncthreads();
    pj_cp_wait<0>();  // this warp's rows
    __syncwarp();
    if (!live) return;
    if (g.type[p] == 12) {
        q4k_lane_rows(span, g.stride[p], nr, nb, ad, aq, abs_, t, g.rows[p], r0, g.out[p], lane);
    } else {
        for (int j = 0; j < nr; ++j)
            row_dots<true>(span + (size_t)j * g.stride[p], g.type[p], k, nb, ad, aq, abs_, t,
                           g.rows[p], r0 + j, g.out[p], lane);
    }
}

size_t proj_row_bytes(int ggml_type, int k) {
    switch (ggml_type) {
    case 12: return (size_t)((k + 255) / 256) * pj::Q4K_BYTES;
    case 14: return (size_t)((k + 255) / 256) * pj::Q6K_BYTES;
    case 8: return (size_t)((k + 31) / 32) * pj::Q80_BYTES;
    default: return 0;
    }
}

cudaError_t launch_q8k_quantize(const float *x, int t, int k, float *d, int8_t *qs, int16_t *bs,
                                cudaStream_t st) {
    const int nb = (k + pj::QK - 1) / pj::QK;
    const int items = t * nb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((items + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, q8k_quantize_kernel, x, k, t, nb, d, qs, bs);
}

cudaError_t init_matvec_kernel() {
    cudaError_t e = cudaFuncSetAttribute(matvec_group_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kMvWarps * kMatvecRowSmemMax);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(matmul_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMatmulSmemMax);
    return e;
}

// Rows per warp of a part in the one-launch kernel: as many Q4_K rows as
// give every lane a super-block, one row of the other types.
static int rows_per_warp(int type, int nb) { return type == 12 && nb <= 32 ? 32 / nb : 1; }
// A warp's span in shared memory: its rows plus the first one's offset
// within 16 bytes, in whole 16-byte pieces.
static size_t span_bytes(size_t bytes) { return (bytes + 15 + 15) / 16 * 16; }
static size_t act_smem(int t, int k) {
    const size_t items = (size_t)t * ((k + pj::QK - 1) / pj::QK);
    return (items * (pj::QK + 4 + 32) + 15) / 16 * 16;
}
// The most shared memory a one-launch group of rows up to stride_max bytes
// may need (a Q4_K span holds at most 32 super-blocks).
size_t matmul_group_smem(int t, int k, size_t stride_max) {
    const size_t span = span_bytes(std::max(stride_max, (size_t)32 * pj::Q4K_BYTES));
    return act_smem(t, k) + (size_t)kMmWarps * span;
}

cudaError_t launch_matmul_group(const MatvecGroup &g_in, const float *x, int t, int k,
                                cudaStream_t st) {
    const int nb = (k + pj::QK - 1) / pj::QK;
    MatvecGroup g = g_in;
    size_t span_max = 0;
    g.wfirst[0] = 0;
    for (int p = 0; p < g.n; ++p) {
        g.rpw[p] = rows_per_warp(g.type[p], nb);
        g.wfirst[p + 1] = g.wfirst[p] + (g.rows[p] + g.rpw[p] - 1) / g.rpw[p];
        span_max = std::max(span_max, span_bytes((size_t)g.rpw[p] * g.stride[p]));
    }
    const size_t smem = act_smem(t, k) + (size_t)kMmWarps * span_max;
    if (smem > (size_t)kMatmulSmemMax) return cudaErrorInvalidValue;
    const int warps = g.wfirst[g.n];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max(1, (warps + kMmWarps - 1) / kMmWarps));
    cfg.blockDim = dim3(kMmWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, matmul_group_kernel, g, x, k, nb, t, (int)span_max);
}

cudaError_t launch_matvec_group(const MatvecGroup &g, int k, const float *d, const int8_t *qs,
                                const int16_t *bs, int t, cudaStream_t st) {
    const int nb = (k + pj::QK - 1) / pj::QK;
    int total = 0;
    size_t stride_max = 0;
    for (int p = 0; p < g.n; ++p) total += g.rows[p], stride_max = max(stride_max, g.stride[p]);
    // a row plus its offset within 16 bytes, in whole 16-byte pieces
    const int row_smem = (int)((stride_max + 15 + 15) / 16 * 16);
    if (row_smem > kMatvecRowSmemMax) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((total + kMvWarps - 1) / kMvWarps);
    cfg.blockDim = dim3(kMvWarps * 32);
    cfg.dynamicSmemBytes = (size_t)kMvWarps * row_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, matvec_group_kernel, g, k, nb, d, qs, bs, t, row_smem);
}

}  // namespace rl
