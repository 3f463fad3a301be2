// Gated DeltaNet prefill in chunks of 64 tokens on the tensor cores, sm_100a.
//
// The reference runs the delta rule one token at a time (forward.rs:1906-1950):
//   S <- g_t S;  d = beta_t (v_t - S^T k_t);  S += k_t d^T;  o_t = S^T q_t / sqrt(128)
// With gamma_t the product of the decays since the chunk start and S_0 the
// state before the chunk, that recurrence unrolls to (rows = tokens):
//   (I + L) U = diag(beta) (V - diag(gamma) K S_0),  L[t][s] = beta_t gamma_t/gamma_s k_t.k_s (s < t)
//   O   = diag(gamma) Q S_0 + (Q K^T o Mgamma) U,   Mgamma[t][s] = gamma_t/gamma_s (s <= t)
//   S_C = gamma_C S_0 + K^T diag(gamma_C/gamma) U
// so with T = (I + L)^-1, Ut = T diag(beta) V and W = T diag(beta gamma) K,
// U = Ut - W S_0: every product is a small dense GEMM.  Four kernels:
//   dn_prep_kernel        per 8 tokens: causal conv + SiLU, q/k L2 norm, gates
//                         (forward.rs:1530-1584, :2018-2059, :1720-1727)
//   dn_chunk_local_kernel per (value head, chunk), all in parallel: K K^T and
//                         Q K^T on mma.sync, T by forward substitution (f32),
//                         Ut and W on mma.sync, P = Q K^T o Mgamma,
//                         Q' = gamma Q, K' = gamma_C/gamma K
//   dn_chunk_scan_kernel  per (value head, 32 state columns): the 64 chunks in
//                         order, state in f32, U = Ut - W S and S = gamma_C S
//                         + K'^T U on eight warps, O = Q' S + P U on eight more
// Every operand of every product is a bf16 pair x = hi + lo (a 16-bit
// mantissa) and every product is the three mma.sync terms hi*hi + hi*lo +
// lo*hi with f32 accumulation: the gated RMSNorm that follows normalises each
// head, so a head whose readout nearly cancels needs its relative error
// small, and single bf16 operands (8 bits) are not enough for that.  Q K^T
// goes further: q and k are bf16 triples (24 bits) and it takes six terms.
//   dn_out_kernel         per token: gated RMSNorm times SiLU(z) (:1642-1652);
//                         dn_hist_kernel leaves the last three raw inputs as the
//                         conv history (the reference's history after the batch)
// The state columns are independent of each other in the recurrence, so the
// scan splits each head's 128 x 128 state over 4 CTAs.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tc.cuh"

namespace rl {
namespace dc {
constexpr int S = 128;     // d_state
constexpr int C = 64;      // chunk length
constexpr int LDB = 136;   // padded bf16 row (272 B: ldmatrix rows in distinct bank groups)
constexpr int LDP = 72;    // padded bf16 row of a 64-wide matrix (144 B)
constexpr int LDF = 65;    // padded f32 row of a 64-wide matrix
constexpr int JC = 32;     // state columns per scan CTA
constexpr int SCAN_THREADS = 512;  // chunk scan: 8 chain warps + 8 output warps
constexpr int GROUP_THREADS = 256;
constexpr int LOCAL_THREADS = 512;  // chunk-local CTA: 16 warps
constexpr int LOCAL_WARPS = LOCAL_THREADS / 32;
// the chunk-local products are cut into 4 row blocks of 16 times
// LOCAL_WARPS / 4 column blocks, one per warp
constexpr int QK_COLS = C * 4 / LOCAL_WARPS;  // K K^T, Q K^T columns per warp
constexpr int UW_COLS = S * 4 / LOCAL_WARPS;  // Ut, W columns per warp
}  // namespace dc

// ---------------------------------------------------------------------------
// SiLU from the hardware exp2 and an approximate divide: within a few f32
// ulps of x / (1 + e^-x), far inside the bf16-pair products that follow
// (the accurate library forms made the prep and output kernels issue-bound).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// dn_prep_kernel: grid (t / PREP_TOKENS, groups / 8), 8 warps; one warp per
// (PREP_TOKENS tokens, group of 128 channels: a q head, a k head or a v
// head), 4 channels per lane.
__device__ __forceinline__ void store_pair4(__nv_bfloat16 *hi, __nv_bfloat16 *lo, const float *y) {
    uint2 h, l;
    h.x = pack_bf16(y[0], y[1]);
    h.y = pack_bf16(y[2], y[3]);
    l.x = pack_bf16(y[0] - bf16_hi(y[0]), y[1] - bf16_hi(y[1]));
    l.y = pack_bf16(y[2] - bf16_hi(y[2]), y[3] - bf16_hi(y[3]));
    *reinterpret_cast<uint2 *>(hi) = h;
    *reinterpret_cast<uint2 *>(lo) = l;
}
// The bf16 triple (hi, lo, l2) of four values: x = hi + lo + l2 to 24 bits.
__device__ __forceinline__ void store_triple4(__nv_bfloat16 *hi, __nv_bfloat16 *lo,
                                              __nv_bfloat16 *l2, const float *y) {
    store_pair4(hi, lo, y);
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float h = bf16_hi(y[e]);
        r[e] = (y[e] - h) - bf16_hi(y[e] - h);
    }
    uint2 w;
    w.x = pack_bf16(r[0], r[1]);
    w.y = pack_bf16(r[2], r[3]);
    *reinterpret_cast<uint2 *>(l2) = w;
}

// One warp per (8 consecutive tokens, group of 128 channels): the group's
// conv weights are loaded once and the three-token history slides along in
// registers.
constexpr int PREP_TOKENS = 8;
__global__ void __launch_bounds__(256, 3) dn_prep_kernel(const DnChunkArgs a) {
    using namespace dc;
    const int lane = threadIdx.x & 31;
    const int i0 = blockIdx.x * PREP_TOKENS, g = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (a.out_ready && blockIdx.y == 0) {
        // the output kernel of this call waits for the scan to count these up
        const int f = blockIdx.x * blockDim.x + threadIdx.x;
        if (f < a.n_v * a.nc) a.out_ready[f] = 0;
    }
    // the chunk-local kernel after this one claims its items from zero
    if (a.local_next && blockIdx.x == 0 && threadIdx.x == 0 && blockIdx.y == 0) *a.local_next = 0;
    const int n_groups = 2 * a.n_k + a.n_v;
    if (g >= n_groups) return;
    const int key_dim = a.n_k * S, conv_dim = 2 * key_dim + a.n_v * S;
    const int ch = g * S + lane * 4;
    float4 w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = *reinterpret_cast<const float4 *>(a.conv1d + (size_t)(ch + e) * 4);
    // h[j] = input of token i - 3 + j (the saved history before the batch)
    float h[3][4];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int src = i0 - 3 + j;
        if (src >= 0) {
            const float4 v = *reinterpret_cast<const float4 *>(a.qkv + (size_t)src * conv_dim + ch);
            h[j][0] = v.x, h[j][1] = v.y, h[j][2] = v.z, h[j][3] = v.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) h[j][e] = a.conv_state[(size_t)(ch + e) * 3 + (src + 3)];
        }
    }
    // a v head's gates, one token a lane: their loads go out with the rows'
    const bool is_v = g >= 2 * a.n_k;
    const int vh = g - 2 * a.n_k;
    float gx = 0.0f, gb = 0.0f;
    if (is_v && lane < PREP_TOKENS && i0 + lane < a.t) {
        gx = __fadd_rn(a.alpha[(size_t)(i0 + lane) * a.n_v + vh], a.dt_bias[vh]);
        gb = a.beta[(size_t)(i0 + lane) * a.n_v + vh];
    }
    float4 xin[PREP_TOKENS];
#pragma unroll
    for (int tt = 0; tt < PREP_TOKENS; ++tt)
        xin[tt] = i0 + tt < a.t
                      ? *reinterpret_cast<const float4 *>(a.qkv + (size_t)(i0 + tt) * conv_dim + ch)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    // the causal conv and SiLU of every token first, so that the q/k heads'
    // norm reductions below run side by side
    float y[PREP_TOKENS][4];
#pragma unroll
    for (int tt = 0; tt < PREP_TOKENS; ++tt) {
        const float xs[4] = {xin[tt].x, xin[tt].y, xin[tt].z, xin[tt].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            // forward.rs:2018-2031: x * w[3] first, then the history taps in order
            float c = __fmul_rn(xs[e], w[e].w);
            c = __fadd_rn(c, __fmul_rn(h[0][e], w[e].x));
            c = __fadd_rn(c, __fmul_rn(h[1][e], w[e].y));
            c = __fadd_rn(c, __fmul_rn(h[2][e], w[e].z));
            y[tt][e] = silu_fast(c);
            h[0][e] = h[1][e];
            h[1][e] = h[2][e];
            h[2][e] = xs[e];
        }
    }
    const int n_tok = min(PREP_TOKENS, a.t - i0);
    if (!is_v) {
        // L2 norm: rms_scale with eps/n, then 1/sqrt(n) (forward.rs:1720-1727);
        // each token's sum is the same butterfly, the tokens' interleaved
        double sq[PREP_TOKENS];
#pragma unroll
        for (int tt = 0; tt < PREP_TOKENS; ++tt) {
            sq[tt] = 0.0;
#pragma unroll
            for (int e = 0; e < 4; ++e) sq[tt] += (double)__fmul_rn(y[tt][e], y[tt][e]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int tt = 0; tt < PREP_TOKENS; ++tt)
                sq[tt] += __shfl_xor_sync(0xffffffffu, sq[tt], o);
        const float shrink = 1.0f / sqrtf((float)S);
        const bool is_q = g < a.n_k;
#pragma unroll
        for (int tt = 0; tt < PREP_TOKENS; ++tt) {
            if (tt >= n_tok) break;  // warp-uniform
            const float sc = rms_scale_fast(sq[tt], S, a.eps / (float)S);
            float yn[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) yn[e] = __fmul_rn(__fmul_rn(y[tt][e], sc), shrink);
            const size_t o = ((size_t)(i0 + tt) * a.n_k + (is_q ? g : g - a.n_k)) * S + lane * 4;
            store_triple4((is_q ? a.qn : a.kn) + o, (is_q ? a.qn_lo : a.kn_lo) + o,
                          (is_q ? a.qn_l2 : a.kn_l2) + o, yn);
        }
    } else {
#pragma unroll
        for (int tt = 0; tt < PREP_TOKENS; ++tt) {
            if (tt >= n_tok) break;  // warp-uniform
            const size_t o = ((size_t)(i0 + tt) * a.n_v + vh) * S + lane * 4;
            store_pair4(a.vn + o, a.vn_lo + o, y[tt]);
        }
        if (lane < n_tok) {
            // gates (forward.rs:1530-1546): log decay and beta, token i0 + lane
            // (hardware exp2 / log2)
            const size_t o = (size_t)(i0 + lane) * a.n_v + vh;
            const float sp = gx > 20.0f ? gx : __logf(1.0f + __expf(gx));
            a.lg[o] = __fmul_rn(sp, a.ssm_a[vh]);
            a.bt[o] = __fdividef(1.0f, 1.0f + __expf(-gb));
        }
    }
}

// ---------------------------------------------------------------------------
// Fragment loaders for m16n8k16 (A row-major [m][k], B given as rows [n][k]).
__device__ __forceinline__ void ld_a(const __nv_bfloat16 *base, int ld, int m0, int k0, int lane,
                                     uint32_t (&a)[4]) {
    const int r = m0 + (lane & 7) + ((lane >> 3) & 1) * 8, c = k0 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(base + r * ld + c), a);
}
// B fragments of two n-tiles (n0, n0 + 8) from a matrix stored as rows n with k contiguous
__device__ __forceinline__ void ld_b2(const __nv_bfloat16 *base, int ld, int n0, int k0, int lane,
                                      uint32_t (&b)[4]) {
    const int r = n0 + (lane & 7) + (lane >> 4) * 8, c = k0 + ((lane >> 3) & 1) * 8;
    ldsm_x4(smem_u32(base + r * ld + c), b);
}
// B fragments of two n-tiles from a matrix stored as rows k with n contiguous
__device__ __forceinline__ void ld_b2_t(const __nv_bfloat16 *base, int ld, int n0, int k0,
                                        int lane, uint32_t (&b)[4]) {
    const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n0 + (lane >> 4) * 8;
    ldsm_x4_t(smem_u32(base + r * ld + c), b);
}
// A fragment (m rows m0.., k cols k0..) of A = X^T, X stored as rows k with m contiguous
__device__ __forceinline__ void ld_a_t(const __nv_bfloat16 *base, int ld, int m0, int k0,
                                       int lane, uint32_t (&a)[4]) {
    const int r = k0 + (lane & 7) + (lane >> 4) * 8, c = m0 + ((lane >> 3) & 1) * 8;
    ldsm_x4_t(smem_u32(base + r * ld + c), a);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// m16n8k16 fragments of f32 matrices in shared memory (row stride ld), each
// split into a bf16 pair: A is the 16 x 16 block at (m0, k0), B the 16 x 8
// block at (k0, n0).
__device__ __forceinline__ void frag_a_f32(const float *base, int ld, int m0, int k0, int lane,
                                           uint32_t (&hi)[4], uint32_t (&lo)[4]) {
    const int g = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int r = m0 + g + (q & 1) * 8, c = k0 + t2 + (q >> 1) * 8;
        const float x0 = base[r * ld + c], x1 = base[r * ld + c + 1];
        hi[q] = pack_bf16(x0, x1);
        lo[q] = pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
    }
}
__device__ __forceinline__ void frag_b_f32(const float *base, int ld, int k0, int n0, int lane,
                                           uint32_t (&hi)[2], uint32_t (&lo)[2]) {
    const int g = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int k = k0 + t2 + q * 8, n = n0 + g;
        const float x0 = base[k * ld + n], x1 = base[(k + 1) * ld + n];
        hi[q] = pack_bf16(x0, x1);
        lo[q] = pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
    }
}
// d += a * b over bf16 pairs: hi*hi + hi*lo + lo*hi
__device__ __forceinline__ void mma3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                     const uint32_t (&bh)[2], const uint32_t (&bl)[2]) {
    mma_16816(d, ah, bh[0], bh[1]);
    mma_16816(d, ah, bl[0], bl[1]);
    mma_16816(d, al, bh[0], bh[1]);
}

// 16 bytes, or zeros when `valid` is false (the source is not read)
__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// dn_chunk_local_kernel: items (value head, chunk), LOCAL_THREADS threads
// (16 warps: row block warp % 4 of 16 rows, column block warp / 4 in the
// product phases); a CTA per item, or (the tcgen05 form) one per SM looping.
struct LocalSmem {
    __nv_bfloat16 k[dc::C][dc::LDB], q[dc::C][dc::LDB], v[dc::C][dc::LDB];
    __nv_bfloat16 kl[dc::C][dc::LDB], ql[dc::C][dc::LDB], vl[dc::C][dc::LDB];  // low halves
    float kk[dc::C][dc::LDF], qk[dc::C][dc::LDF], t[dc::C][dc::LDF], x[dc::C][dc::LDF];
    union {
        struct {
            __nv_bfloat16 ta_hi[dc::C][dc::LDP], ta_lo[dc::C][dc::LDP];  // T diag(beta)
            __nv_bfloat16 tb_hi[dc::C][dc::LDP], tb_lo[dc::C][dc::LDP];  // T diag(beta gamma)
        };
        // the third terms of q and k, read by Q K^T only (before T exists)
        struct {
            __nv_bfloat16 q2[dc::C][dc::LDB], k2[dc::C][dc::LDB];
        };
    };
    float cum[dc::C], beta[dc::C];
    int next[2];  // the item after this one, by the item's parity
};

// The tcgen05 form's layout (1024-byte aligned).  q and k arrive by TMA as
// 64-token x 64-channel boxes with the 128-byte swizzle, in 16 KiB blocks of
// (plane, channel box): K's 64 rows, then Q's, so that a block is the
// 128-row A operand [K; Q] of K K^T and Q K^T stacked, and its first half
// the B operand K.  The planes' third terms are read by that product only,
// so T's pairs and the T inversion's scratch reuse their space.
struct LocalSmemTc {
    unsigned char hl[2][2][16384];  // [hi, lo][channel box]
    union {
        unsigned char l2[2][16384];  // [channel box], the third terms
        float x[dc::C][dc::LDF];
        struct {
            __nv_bfloat16 ta_hi[dc::C][dc::LDP], ta_lo[dc::C][dc::LDP];  // T diag(beta)
            __nv_bfloat16 tb_hi[dc::C][dc::LDP], tb_lo[dc::C][dc::LDP];  // T diag(beta gamma)
        };
    };
    __nv_bfloat16 v[dc::C][dc::LDB], vl[dc::C][dc::LDB];
    float kk[dc::C][dc::LDF], qk[dc::C][dc::LDF], t[dc::C][dc::LDF];
    float cum[dc::C], beta[dc::C];
    uint64_t qk_full, mma_done;
    uint32_t tmem_base;
    int next[2];  // the item after this one, by the item's parity
};
static_assert(sizeof(LocalSmemTc) + 1024 <= 227 * 1024, "the tcgen05 chunk-local layout fits");
constexpr uint32_t QK_BLOCK = 16384, Q_HALF = 8192;

// The tcgen05 form's plane x (0 hi, 1 lo, 2 third term) of k (q: + Q_HALF),
// channel box cb
template <typename Sm>
__device__ __forceinline__ unsigned char *qk_block(Sm &sm, int x, int cb) {
    return x < 2 ? sm.hl[x][cb] : sm.l2[cb];
}
// B fragments of two n-tiles (channels n0, n0 + 8) from a swizzled plane
// stored as rows k (tokens) with n (channels) contiguous, as ld_b2_t reads a
// padded one
__device__ __forceinline__ void ld_b2_t_swz(const unsigned char *box0, int n0, int k0, int lane,
                                            uint32_t (&b)[4]) {
    const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n0 + (lane >> 4) * 8;
    ldsm_x4_t(smem_u32(box0 + (c >> 6) * QK_BLOCK + swz128(r, (c & 63) >> 3)), b);
}

template <bool TC>
__global__ void __launch_bounds__(dc::LOCAL_THREADS)
    dn_chunk_local_kernel(const DnChunkArgs a, const __grid_constant__ DnPlaneMaps pm) {
    using namespace dc;
    using Sm = std::conditional_t<TC, LocalSmemTc, LocalSmem>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *base =
        TC ? smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023) : smem_raw;
    Sm &sm = *reinterpret_cast<Sm *>(base);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if constexpr (TC) {
        if (tid == 0) {
            mbar_init(&sm.qk_full, 1);
            mbar_init(&sm.mma_done, 1);
            fence_barrier_init();
        }
        if (warp == 0) {
            tc::tmem_alloc(&sm.tmem_base, 64);
            tc::tmem_relinquish();
        }
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
    }
    // The items (value head, chunk) in chunk-major order.  The tcgen05 form
    // runs one CTA per SM the kernel gets, each looping with no launch
    // between items: its first item is its block index, each later one is
    // claimed from a counter while the one before runs, so that the chunks
    // finish in order (an overlapped scan waits for them in that order) and a
    // CTA that falls behind takes fewer.
    const int n_items = a.n_v * a.nc;
    int item = blockIdx.x;
#pragma unroll 1
    for (int it = 0; item < n_items; ++it) {
        const int vh = item % a.n_v, ck = item / a.n_v, kh = vh % a.n_k;
        const uint32_t par = it & 1;  // the mbarriers' phase of this item
        // the epoch this call's scan waits for (its scan advances it only after
        // this item's flag is up)
        const int ready_value = a.ready ? a.ready_epoch[vh] + 1 : 0;
        const int t0 = ck * C, rows = min(C, a.t - t0);

        // ---- operands of the chunk (rows past the batch are zero): every copy
        // in flight at once, q and k first (the first products), v after them
        // (needed only for Ut, after T)
        if constexpr (TC) {
            // q and k by TMA (the maps end at the call's rows, so the rows past
            // them read as zero), into the stacked blocks
            if (tid == 0) {
                mbar_arrive_expect_tx(&sm.qk_full, 12 * Q_HALF);
#pragma unroll 1
                for (int x = 0; x < 3; ++x)
#pragma unroll 1
                    for (int cb = 0; cb < 2; ++cb) {
                        unsigned char *blk = qk_block(sm, x, cb);
                        tma_load_3d(blk, &pm.k[x], cb * 64, kh, t0, &sm.qk_full);
                        tma_load_3d(blk + Q_HALF, &pm.q[x], cb * 64, kh, t0, &sm.qk_full);
                    }
            }
        } else {
#pragma unroll 2
            for (int e = tid; e < C * (S / 8); e += LOCAL_THREADS) {
                const int r = e / (S / 8), c8 = (e % (S / 8)) * 8;
                const bool ok = r < rows;
                const size_t ko = ((size_t)(t0 + (ok ? r : 0)) * a.n_k + kh) * S + c8;
                cp_async16_zfill(&sm.k[r][c8], a.kn + ko, ok);
                cp_async16_zfill(&sm.q[r][c8], a.qn + ko, ok);
                cp_async16_zfill(&sm.kl[r][c8], a.kn_lo + ko, ok);
                cp_async16_zfill(&sm.ql[r][c8], a.qn_lo + ko, ok);
                cp_async16_zfill(&sm.k2[r][c8], a.kn_l2 + ko, ok);
                cp_async16_zfill(&sm.q2[r][c8], a.qn_l2 + ko, ok);
            }
            cp_async_commit();
        }
#pragma unroll 2
        for (int e = tid; e < C * (S / 8); e += LOCAL_THREADS) {
            const int r = e / (S / 8), c8 = (e % (S / 8)) * 8;
            const bool ok = r < rows;
            const size_t vo = ((size_t)(t0 + (ok ? r : 0)) * a.n_v + vh) * S + c8;
            cp_async16_zfill(&sm.v[r][c8], a.vn + vo, ok);
            cp_async16_zfill(&sm.vl[r][c8], a.vn_lo + vo, ok);
        }
        cp_async_commit();
        if (tid == 64)  // a warp with nothing else waiting on it here
            sm.next[(it + 1) & 1] = a.local_next ? (int)gridDim.x + atomicAdd(a.local_next, 1)
                                                 : item + (int)gridDim.x;
        if (warp == 0) {
            // cumulative log decay, gamma_t = exp(cum[t]): lane l holds tokens
            // 2l and 2l + 1, an inclusive scan over the pairs' sums
            const int ta = 2 * lane, tb = ta + 1;
            const float la = ta < rows ? a.lg[(size_t)(t0 + ta) * a.n_v + vh] : 0.0f;
            const float lb = tb < rows ? a.lg[(size_t)(t0 + tb) * a.n_v + vh] : 0.0f;
            float inc = la + lb;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            sm.cum[tb] = inc;
            sm.cum[ta] = inc - lb;
            sm.beta[ta] = ta < rows ? a.bt[(size_t)(t0 + ta) * a.n_v + vh] : 0.0f;
            sm.beta[tb] = tb < rows ? a.bt[(size_t)(t0 + tb) * a.n_v + vh] : 0.0f;
        }
        if constexpr (!TC) {
            cp_async_wait<1>();  // q and k (v may still be in flight)
            __syncthreads();
        }
        // Q' = gamma Q and K' = gamma_C / gamma K as bf16 pairs, 8 consecutive
        // elements a thread (16-byte stores); needs cum and the q/k planes
        const size_t blk = (size_t)vh * a.nc + ck;
        auto write_qk_prime = [&]() {
            const float cum_c = sm.cum[C - 1];
            __nv_bfloat16 *qp_out = a.qp + blk * C * S, *kp_out = a.kp + blk * C * S;
            __nv_bfloat16 *qpl_out = a.qp_lo + blk * C * S, *kpl_out = a.kp_lo + blk * C * S;
#pragma unroll 2
            for (int e8 = tid; e8 < C * S / 8; e8 += LOCAL_THREADS) {
                const int r = e8 / (S / 8), c0 = (e8 % (S / 8)) * 8;
                const float gq = __expf(sm.cum[r]), gk = __expf(cum_c - sm.cum[r]);
                uint4 qh, ql, kh4, kl4;
                if constexpr (TC) {
                    const uint32_t so = (c0 >> 6) * QK_BLOCK + swz128(r, (c0 & 63) >> 3);
                    qh = *reinterpret_cast<const uint4 *>(sm.hl[0][0] + so + Q_HALF);
                    ql = *reinterpret_cast<const uint4 *>(sm.hl[1][0] + so + Q_HALF);
                    kh4 = *reinterpret_cast<const uint4 *>(sm.hl[0][0] + so);
                    kl4 = *reinterpret_cast<const uint4 *>(sm.hl[1][0] + so);
                } else {
                    qh = *reinterpret_cast<const uint4 *>(&sm.q[r][c0]);
                    ql = *reinterpret_cast<const uint4 *>(&sm.ql[r][c0]);
                    kh4 = *reinterpret_cast<const uint4 *>(&sm.k[r][c0]);
                    kl4 = *reinterpret_cast<const uint4 *>(&sm.kl[r][c0]);
                }
                const __nv_bfloat162 *qh2 = reinterpret_cast<const __nv_bfloat162 *>(&qh);
                const __nv_bfloat162 *ql2 = reinterpret_cast<const __nv_bfloat162 *>(&ql);
                const __nv_bfloat162 *kh2 = reinterpret_cast<const __nv_bfloat162 *>(&kh4);
                const __nv_bfloat162 *kl2 = reinterpret_cast<const __nv_bfloat162 *>(&kl4);
                uint32_t xh[4], xl[4], yh[4], yl[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 qa = __bfloat1622float2(qh2[k]), qb = __bfloat1622float2(ql2[k]);
                    const float2 ka = __bfloat1622float2(kh2[k]), kb = __bfloat1622float2(kl2[k]);
                    const float x0 = (qa.x + qb.x) * gq, x1 = (qa.y + qb.y) * gq;
                    const float y0 = (ka.x + kb.x) * gk, y1 = (ka.y + kb.y) * gk;
                    xh[k] = pack_bf16(x0, x1);
                    xl[k] = pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
                    yh[k] = pack_bf16(y0, y1);
                    yl[k] = pack_bf16(y0 - bf16_hi(y0), y1 - bf16_hi(y1));
                }
                const size_t o = (size_t)r * S + c0;
                *reinterpret_cast<uint4 *>(qp_out + o) = make_uint4(xh[0], xh[1], xh[2], xh[3]);
                *reinterpret_cast<uint4 *>(qpl_out + o) = make_uint4(xl[0], xl[1], xl[2], xl[3]);
                *reinterpret_cast<uint4 *>(kp_out + o) = make_uint4(yh[0], yh[1], yh[2], yh[3]);
                *reinterpret_cast<uint4 *>(kpl_out + o) = make_uint4(yl[0], yl[1], yl[2], yl[3]);
            }
        };
        // ---- K K^T as hi*hi + hi*lo + lo*hi of the bf16 pairs, and Q K^T of
        // the bf16 triples (hi*hi + hi*lo + lo*hi + lo*lo + hi*l2 + l2*hi): the
        // readout P U of a token whose state has all but decayed away cancels
        // down to the q.k products of its own chunk, and the per-head gated norm
        // that follows magnifies their error; pairs (16 bits) measured 1.3e-2 of
        // such a head's output at 4096 tokens, triples stay at the f32 level
        if constexpr (TC) {
            // one tcgen05 chain: [K; Q]_xa K_xb^T over the six (xa, xb) plane
            // pairs Q K^T takes (hi hi, hi lo, hi l2, lo hi, lo lo, l2 hi); the
            // accumulator's rows 0-63 are K K^T (to six terms), 64-127 Q K^T.
            // The chain keeps the tensor pipe busy for ~2,400 cycles: warp 15
            // issues it while every warp writes Q' and K' from the same planes,
            // then warps 0-3 read the products back.  The barrier after the
            // planes land also publishes cum and beta.
            const bool okq = mbar_wait(&sm.qk_full, par, a.status);
            __syncthreads();
            if (tid == LOCAL_THREADS - 32) {
                if (okq) {
                    tc::fence_after_sync();
                    constexpr uint32_t id = tc::idesc_bf16(128, 64, false);
                    const int xa[6] = {0, 0, 0, 1, 1, 2}, xb[6] = {0, 1, 2, 0, 1, 0};
#pragma unroll
                    for (int p = 0; p < 6; ++p) {
                        const uint64_t ad =
                            tc::smem_desc(smem_u32(qk_block(sm, xa[p], 0)), 16, 1024);
                        const uint64_t bd =
                            tc::smem_desc(smem_u32(qk_block(sm, xb[p], 0)), 16, 1024);
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            // a 16-channel step is 32 bytes inside a box, the next
                            // box the next block
                            const uint64_t step = ((kk >> 2) * QK_BLOCK + (kk & 3) * 32) >> 4;
                            tc::mma_ss(sm.tmem_base, ad + step, bd + step, id, p > 0 || kk > 0);
                        }
                    }
                    tc::commit(&sm.mma_done);
                } else {
                    mbar_arrive(&sm.mma_done);  // flagged; the readers go on
                }
            }
            write_qk_prime();
            if (warp < 4) {
                // warp w reads tensor-memory lanes 32w .. 32w + 31: rows of K K^T
                // (w < 2) or of Q K^T
                mbar_wait(&sm.mma_done, par, a.status);
                tc::fence_after_sync();
                uint32_t r0[32], r1[32];
                const uint32_t taddr = sm.tmem_base + ((uint32_t)(warp * 32) << 16);
                tc::ld32(taddr, r0);
                tc::ld32(taddr + 32, r1);
                tc::wait_ld();
                const int row = warp * 32 + lane;
                float *dst = row < C ? &sm.kk[row][0] : &sm.qk[row - C][0];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    dst[c] = __uint_as_float(r0[c]);
                    dst[32 + c] = __uint_as_float(r1[c]);
                }
            }
        } else {
            // warp: rows 16 * (warp % 4), columns QK_COLS * (warp / 4) ..
            constexpr int NT = QK_COLS / 8;
            const int rw = (warp & 3) * 16, cn = (warp >> 2) * QK_COLS;
            float dk[NT][4], dq[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) dk[n][e] = dq[n][e] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < S / 16; ++ks) {
                uint32_t ak[4], aq[4], akl[4], aql[4], aq2[4];
                ld_a(&sm.k[0][0], LDB, rw, ks * 16, lane, ak);
                ld_a(&sm.q[0][0], LDB, rw, ks * 16, lane, aq);
                ld_a(&sm.kl[0][0], LDB, rw, ks * 16, lane, akl);
                ld_a(&sm.ql[0][0], LDB, rw, ks * 16, lane, aql);
                ld_a(&sm.q2[0][0], LDB, rw, ks * 16, lane, aq2);
#pragma unroll
                for (int np = 0; np < NT / 2; ++np) {
                    uint32_t b[4], bl[4], b2[4];
                    ld_b2(&sm.k[0][0], LDB, cn + np * 16, ks * 16, lane, b);
                    ld_b2(&sm.kl[0][0], LDB, cn + np * 16, ks * 16, lane, bl);
                    ld_b2(&sm.k2[0][0], LDB, cn + np * 16, ks * 16, lane, b2);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        mma_16816(dk[2 * np + h], ak, b[2 * h], b[2 * h + 1]);
                        mma_16816(dk[2 * np + h], ak, bl[2 * h], bl[2 * h + 1]);
                        mma_16816(dk[2 * np + h], akl, b[2 * h], b[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aq, b[2 * h], b[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aq, bl[2 * h], bl[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aql, b[2 * h], b[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aql, bl[2 * h], bl[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aq, b2[2 * h], b2[2 * h + 1]);
                        mma_16816(dq[2 * np + h], aq2, b[2 * h], b[2 * h + 1]);
                    }
                }
            }
            const int r0 = rw + (lane >> 2), c0 = cn + (lane & 3) * 2;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                sm.kk[r0][n * 8 + c0] = dk[n][0];
                sm.kk[r0][n * 8 + c0 + 1] = dk[n][1];
                sm.kk[r0 + 8][n * 8 + c0] = dk[n][2];
                sm.kk[r0 + 8][n * 8 + c0 + 1] = dk[n][3];
                sm.qk[r0][n * 8 + c0] = dq[n][0];
                sm.qk[r0][n * 8 + c0 + 1] = dq[n][1];
                sm.qk[r0 + 8][n * 8 + c0] = dq[n][2];
                sm.qk[r0 + 8][n * 8 + c0 + 1] = dq[n][3];
            }
        }
        __syncthreads();
        // ---- P = Q K^T o Mgamma (s <= t), and in the mma.sync form Q' and K'
        // (the tcgen05 form wrote them beside its products): written now, so
        // that the stores drain while T is built (8 consecutive elements a
        // thread: 16-byte stores)
        __nv_bfloat16 *p_out = a.p + blk * C * C, *pl_out = a.p_lo + blk * C * C;
#pragma unroll 2
        for (int e8 = tid; e8 < C * C / 8; e8 += LOCAL_THREADS) {
            const int r = e8 / (C / 8), s0 = (e8 % (C / 8)) * 8;
            const float cr = sm.cum[r];
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int sa = s0 + 2 * k, sb = sa + 1;
                const float x0 = sa <= r ? sm.qk[r][sa] * __expf(cr - sm.cum[sa]) : 0.0f;
                const float x1 = sb <= r ? sm.qk[r][sb] * __expf(cr - sm.cum[sb]) : 0.0f;
                hi[k] = pack_bf16(x0, x1);
                lo[k] = pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
            }
            *reinterpret_cast<uint4 *>(p_out + r * C + s0) =
                make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4 *>(pl_out + r * C + s0) =
                make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        const float cum_c = sm.cum[C - 1];
        if constexpr (!TC) write_qk_prime();
        if (tid == 0) a.gc[blk] = __expf(cum_c);
        // ---- L (in place over kk) and T = (I + L)^-1, one column per thread
        {
            // this thread's column s is fixed (the CTA is a multiple of C)
            const int s = tid & (C - 1);
            const float cs = sm.cum[s];
#pragma unroll 4
            for (int r = tid / C; r < C; r += LOCAL_THREADS / C) {
                sm.kk[r][s] = s < r ? sm.beta[r] * __expf(sm.cum[r] - cs) * sm.kk[r][s] : 0.0f;
                sm.t[r][s] = 0.0f;
            }
        }
        __syncthreads();
        // T = (I + L)^-1 in 16 x 16 blocks: the four diagonal blocks by forward
        // substitution (one column per thread), then the blocks below the
        // diagonal, one diagonal at a time: T_ij = -T_ii sum_{j<=k<i} L_ik T_kj
        if (tid < C) {
            // column s of diagonal block b0, in registers (entries above the
            // diagonal are zero, so the sums may run over every m < r)
            const int b0 = (tid >> 4) * 16, s = tid & 15;
            float tc[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float acc = 0.0f;
#pragma unroll
                for (int m = 0; m < r; ++m) acc = fmaf(sm.kk[b0 + r][b0 + m], tc[m], acc);
                tc[r] = r == s ? 1.0f : (r > s ? -acc : 0.0f);
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) sm.t[b0 + r][b0 + s] = tc[r];
        }
        __syncthreads();
        // the blocks below the diagonal, one diagonal dg at a time: warp j < 4 -
        // dg takes block (i, j) = (j + dg, j), X = sum_{j <= k < i} L_ik T_kj and
        // then T_ij = -T_ii X, both on the tensor cores as bf16 pairs
#pragma unroll 1
        for (int dg = 1; dg < 4; ++dg) {
            if (warp < 4 - dg) {
                const int bj = warp, bi = warp + dg;
                const int g = lane >> 2, t2 = (lane & 3) * 2;
                float x[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                for (int kb = bj; kb < bi; ++kb) {
                    uint32_t ah[4], al[4];
                    frag_a_f32(&sm.kk[0][0], LDF, 16 * bi, 16 * kb, lane, ah, al);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        uint32_t bh[2], bl[2];
                        frag_b_f32(&sm.t[0][0], LDF, 16 * kb, 16 * bj + 8 * nt, lane, bh, bl);
                        mma3(x[nt], ah, al, bh, bl);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    sm.x[16 * bi + g][16 * bj + 8 * nt + t2] = x[nt][0];
                    sm.x[16 * bi + g][16 * bj + 8 * nt + t2 + 1] = x[nt][1];
                    sm.x[16 * bi + g + 8][16 * bj + 8 * nt + t2] = x[nt][2];
                    sm.x[16 * bi + g + 8][16 * bj + 8 * nt + t2 + 1] = x[nt][3];
                }
                __syncwarp();
                uint32_t ah[4], al[4];
                frag_a_f32(&sm.t[0][0], LDF, 16 * bi, 16 * bi, lane, ah, al);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    uint32_t bh[2], bl[2];
                    frag_b_f32(&sm.x[0][0], LDF, 16 * bi, 16 * bj + 8 * nt, lane, bh, bl);
                    float y[4] = {0.f, 0.f, 0.f, 0.f};
                    mma3(y, ah, al, bh, bl);
                    sm.t[16 * bi + g][16 * bj + 8 * nt + t2] = -y[0];
                    sm.t[16 * bi + g][16 * bj + 8 * nt + t2 + 1] = -y[1];
                    sm.t[16 * bi + g + 8][16 * bj + 8 * nt + t2] = -y[2];
                    sm.t[16 * bi + g + 8][16 * bj + 8 * nt + t2 + 1] = -y[3];
                }
            }
            __syncthreads();
        }
        // ---- T diag(beta) and T diag(beta gamma) as bf16 pairs
        {
            // this thread's column s is fixed (the CTA is a multiple of C)
            const int s = tid & (C - 1);
            const float bs = sm.beta[s], gs = __expf(sm.cum[s]);
#pragma unroll 4
            for (int r = tid / C; r < C; r += LOCAL_THREADS / C) {
                const float x = sm.t[r][s] * bs;
                const float y = x * gs;
                const float xh = bf16_hi(x), yh = bf16_hi(y);
                sm.ta_hi[r][s] = __float2bfloat16_rn(x);
                sm.ta_lo[r][s] = __float2bfloat16_rn(x - xh);
                sm.tb_hi[r][s] = __float2bfloat16_rn(y);
                sm.tb_lo[r][s] = __float2bfloat16_rn(y - yh);
            }
        }
        cp_async_wait<0>();  // v
        __syncthreads();
        // ---- Ut = T diag(beta) V and W = T diag(beta gamma) K (warp: 16 rows,
        // UW_COLS columns)
        float *ut_out = a.ut + blk * C * S;
        __nv_bfloat16 *w_out = a.w + blk * C * S, *wl_out = a.w_lo + blk * C * S;
        const int r0 = (warp & 3) * 16 + (lane >> 2), c0 = (lane & 3) * 2;
        {
            constexpr int NT = UW_COLS / 8;
            const int cb = (warp >> 2) * UW_COLS;  // this warp's first output column
            float du[NT][4], dw[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) du[n][e] = dw[n][e] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
                uint32_t ah[4], al[4], bh[4], bl[4];
                ld_a(&sm.ta_hi[0][0], LDP, (warp & 3) * 16, ks * 16, lane, ah);
                ld_a(&sm.ta_lo[0][0], LDP, (warp & 3) * 16, ks * 16, lane, al);
                ld_a(&sm.tb_hi[0][0], LDP, (warp & 3) * 16, ks * 16, lane, bh);
                ld_a(&sm.tb_lo[0][0], LDP, (warp & 3) * 16, ks * 16, lane, bl);
#pragma unroll
                for (int np = 0; np < NT / 2; ++np) {
                    const int n0 = cb + np * 16;
                    uint32_t vh_[4], vl_[4], kh_[4], kl_[4];
                    ld_b2_t(&sm.v[0][0], LDB, n0, ks * 16, lane, vh_);
                    ld_b2_t(&sm.vl[0][0], LDB, n0, ks * 16, lane, vl_);
                    if constexpr (TC) {
                        ld_b2_t_swz(sm.hl[0][0], n0, ks * 16, lane, kh_);
                        ld_b2_t_swz(sm.hl[1][0], n0, ks * 16, lane, kl_);
                    } else {
                        ld_b2_t(&sm.k[0][0], LDB, n0, ks * 16, lane, kh_);
                        ld_b2_t(&sm.kl[0][0], LDB, n0, ks * 16, lane, kl_);
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        mma_16816(du[2 * np + h], ah, vh_[2 * h], vh_[2 * h + 1]);
                        mma_16816(du[2 * np + h], ah, vl_[2 * h], vl_[2 * h + 1]);
                        mma_16816(du[2 * np + h], al, vh_[2 * h], vh_[2 * h + 1]);
                        mma_16816(dw[2 * np + h], bh, kh_[2 * h], kh_[2 * h + 1]);
                        mma_16816(dw[2 * np + h], bh, kl_[2 * h], kl_[2 * h + 1]);
                        mma_16816(dw[2 * np + h], bl, kh_[2 * h], kh_[2 * h + 1]);
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int col = cb + n * 8 + c0;
                *reinterpret_cast<float2 *>(ut_out + r0 * S + col) =
                    make_float2(du[n][0], du[n][1]);
                *reinterpret_cast<float2 *>(ut_out + (r0 + 8) * S + col) =
                    make_float2(du[n][2], du[n][3]);
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    const float x0 = dw[n][2 * e2], x1 = dw[n][2 * e2 + 1];
                    const size_t o = (size_t)(r0 + 8 * e2) * S + col;
                    *reinterpret_cast<uint32_t *>(w_out + o) = pack_bf16(x0, x1);
                    if (a.w_lo_out)  // only the mma.sync scan reads W's low half
                        *reinterpret_cast<uint32_t *>(wl_out + o) =
                            pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
                }
            }
        }
        // every thread is done with this item's shared memory and tensor memory
        // (the next item's copies overwrite them) and has stored its outputs
        if constexpr (TC) tc::fence_before_sync();
        __syncthreads();
        if constexpr (TC) tc::fence_after_sync();
        // The barrier orders every thread's stores before warp 1's, and a
        // release is cumulative: once the flag is seen at GPU scope, so is
        // everything its writer had seen (the semaphore pattern).  Warp 1 waits
        // for the stores to land while thread 0 sends the next item's loads.
        if (a.ready && tid == 32) st_release_gpu(a.ready + (size_t)vh * a.nc + ck, ready_value);
        item = sm.next[(it + 1) & 1];
    }
    if constexpr (TC) {
        if (warp == 0) tc::tmem_dealloc(sm.tmem_base, 64);
    }
}

// ---------------------------------------------------------------------------
// dn_chunk_scan_kernel: grid (S / JC, n_v), 512 threads.  The chunks in
// order; this CTA owns state columns j0 .. j0 + 31 of value head vh.  Warps
// 0-7 run the U/S chain and fetch the next chunk's W and Ut (once U is done)
// and K' (once S is); warps 8-15 compute the output and fetch the next Q' and
// P.  S and U are kept as bf16 pairs in row-major [k][n] form (the B
// operands, read with transposing ldmatrix), written with packed 4-byte
// stores.
constexpr int LDU = dc::JC + 8;  // padded bf16 row of a 32-column matrix (80 B)
struct ScanSmem {
    __nv_bfloat16 w[2][dc::C][dc::LDB], qp[2][dc::C][dc::LDB], kp[2][dc::C][dc::LDB];  // [hi, lo]
    __nv_bfloat16 p[2][dc::C][dc::LDP];
    float ut[dc::C][dc::JC];
    float s[dc::S][dc::JC + 1];                 // the state block, f32
    __nv_bfloat16 st[2][2][dc::S][LDU];         // S [buffer][hi, lo] as [i][j]
    __nv_bfloat16 up[2][2][dc::C][LDU];         // U [buffer][hi, lo] as [t][j]
};

// W (hi, lo) and this CTA's 32 columns of Ut for chunk block `blk`, 16-byte
// asynchronous copies from every thread
__device__ __forceinline__ void scan_load_wu(ScanSmem &sm, const DnChunkArgs &a, size_t blk,
                                             int j0, int tid) {
    using namespace dc;
    const __nv_bfloat16 *w = a.w + blk * C * S, *wl = a.w_lo + blk * C * S;
    for (int e = tid; e < C * (S / 8); e += GROUP_THREADS) {
        const int r = e / (S / 8), c8 = (e % (S / 8)) * 8;
        cp_async16(&sm.w[0][r][c8], w + r * S + c8);
        cp_async16(&sm.w[1][r][c8], wl + r * S + c8);
    }
    const float *ut = a.ut + blk * C * S;
    for (int e = tid; e < C * (JC / 4); e += GROUP_THREADS) {
        const int r = e / (JC / 4), c4 = (e % (JC / 4)) * 4;
        cp_async16(&sm.ut[r][c4], ut + r * S + j0 + c4);
    }
}
// K' (hi, lo) for chunk block `blk`
__device__ __forceinline__ void scan_load_k(ScanSmem &sm, const DnChunkArgs &a, size_t blk,
                                            int tid) {
    using namespace dc;
    const __nv_bfloat16 *kp = a.kp + blk * C * S, *kpl = a.kp_lo + blk * C * S;
    for (int e = tid; e < C * (S / 8); e += GROUP_THREADS) {
        const int r = e / (S / 8), c8 = (e % (S / 8)) * 8;
        cp_async16(&sm.kp[0][r][c8], kp + r * S + c8);
        cp_async16(&sm.kp[1][r][c8], kpl + r * S + c8);
    }
}
// Q' and P (hi, lo) for chunk block `blk`
__device__ __forceinline__ void scan_load_qp(ScanSmem &sm, const DnChunkArgs &a, size_t blk,
                                             int tid) {
    using namespace dc;
    const __nv_bfloat16 *qp = a.qp + blk * C * S, *qpl = a.qp_lo + blk * C * S;
    for (int e = tid; e < C * (S / 8); e += GROUP_THREADS) {
        const int r = e / (S / 8), c8 = (e % (S / 8)) * 8;
        cp_async16(&sm.qp[0][r][c8], qp + r * S + c8);
        cp_async16(&sm.qp[1][r][c8], qpl + r * S + c8);
    }
    const __nv_bfloat16 *p = a.p + blk * C * C, *pl = a.p_lo + blk * C * C;
    for (int e = tid; e < C * (C / 8); e += GROUP_THREADS) {
        const int r = e / (C / 8), c8 = (e % (C / 8)) * 8;
        cp_async16(&sm.p[0][r][c8], p + r * C + c8);
        cp_async16(&sm.p[1][r][c8], pl + r * C + c8);
    }
}

// d += A B with A (16 rows from m0) given as a bf16 pair in row-major [m][k]
// smem and B (NP pairs of n-tiles from n0, 16 NP columns) as a pair of
// row-major [k][n] matrices; three terms: hi*hi + hi*lo + lo*hi, over k from
// 0 to K.
template <int K, int NP>
__device__ __forceinline__ void mma3_rows(float (&d)[2 * NP][4], const __nv_bfloat16 *ah,
                                          const __nv_bfloat16 *al, int lda, int m0,
                                          const __nv_bfloat16 *bh, const __nv_bfloat16 *bl,
                                          int ldb, int n0, int lane) {
#pragma unroll
    for (int ks = 0; ks < K / 16; ++ks) {
        uint32_t xh[4], xl[4];
        ld_a(ah, lda, m0, ks * 16, lane, xh);
        ld_a(al, lda, m0, ks * 16, lane, xl);
#pragma unroll
        for (int np = 0; np < NP; ++np) {
            uint32_t yh[4], yl[4];
            ld_b2_t(bh, ldb, n0 + np * 16, ks * 16, lane, yh);
            ld_b2_t(bl, ldb, n0 + np * 16, ks * 16, lane, yl);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                mma_16816(d[2 * np + h], xh, yh[2 * h], yh[2 * h + 1]);
                mma_16816(d[2 * np + h], xh, yl[2 * h], yl[2 * h + 1]);
                mma_16816(d[2 * np + h], xl, yh[2 * h], yh[2 * h + 1]);
            }
        }
    }
}

__global__ void __launch_bounds__(dc::SCAN_THREADS, 1) dn_chunk_scan_kernel(const DnChunkArgs a) {
    using namespace dc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ScanSmem &sm = *reinterpret_cast<ScanSmem *>(smem_raw);
    const int j0 = blockIdx.x * JC, vh = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31;
    // warps 0-7 run the chain U_c = Ut - W S_{c-1}, S_c = gamma S_{c-1} + K'^T U_c;
    // warps 8-15 the output O_c = Q' S_{c-1} + P U_c, which nothing later needs,
    // while the chain goes on with S_c and U_{c+1} (U is double-buffered; S_{c+1}
    // waits until O_c has read S_{c-1}, whose buffer it takes).  Named
    // barriers: 1 the chain warps, 2 the output warps, 3 U_c ready (the chain
    // arrives, the output warps wait), 4 O_c done (the other way).
    const bool chain = tid < GROUP_THREADS;
    const int ltid = chain ? tid : tid - GROUP_THREADS, lwarp = ltid >> 5;
    const int g = lane >> 2, c0 = (lane & 3) * 2;
    const float scale = 1.0f / sqrtf((float)S);
    float *state = a.ssm_state + (size_t)vh * a.slots * S * S + (size_t)a.live * S * S;
    const size_t blk0 = (size_t)vh * a.nc;
    const int wm = (lwarp & 3) * 16, wn = (lwarp >> 2) * 16;  // U and O: 16 x 16 per warp

    if (chain) {
        scan_load_wu(sm, a, blk0, j0, ltid);
        cp_async_commit();
        scan_load_k(sm, a, blk0, ltid);
        cp_async_commit();
        for (int e = ltid; e < S * JC / 2; e += GROUP_THREADS) {
            const int i = e / (JC / 2), j = (e % (JC / 2)) * 2;
            const float2 x = *reinterpret_cast<const float2 *>(state + (size_t)i * S + j0 + j);
            sm.s[i][j] = x.x;
            sm.s[i][j + 1] = x.y;
            *reinterpret_cast<uint32_t *>(&sm.st[0][0][i][j]) = pack_bf16(x.x, x.y);
            *reinterpret_cast<uint32_t *>(&sm.st[0][1][i][j]) =
                pack_bf16(x.x - bf16_hi(x.x), x.y - bf16_hi(x.y));
        }
        for (int ck = 0; ck < a.nc; ++ck) {
            const int cur = ck & 1, nxt = cur ^ 1, ub = ck & 1;
            const bool more = ck + 1 < a.nc;
            // W and Ut of this chunk have landed (its K' may be in flight);
            // the state of the step before is in place
            cp_async_wait<1>();
            named_sync(1, GROUP_THREADS);
            // ---- U = Ut - W S (warp: rows 16 (w % 4).., columns 16 (w / 4)..)
        {
            float d[2][4] = {};
            mma3_rows<S, 1>(d, &sm.w[0][0][0], &sm.w[1][0][0], LDB, wm, &sm.st[cur][0][0][0],
                            &sm.st[cur][1][0][0], LDU, wn, lane);
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    const int r = wm + g + e2 * 8, c = wn + n * 8 + c0;
                    const float u0 = sm.ut[r][c] - d[n][2 * e2];
                    const float u1 = sm.ut[r][c + 1] - d[n][2 * e2 + 1];
                    *reinterpret_cast<uint32_t *>(&sm.up[ub][0][r][c]) = pack_bf16(u0, u1);
                    *reinterpret_cast<uint32_t *>(&sm.up[ub][1][r][c]) =
                        pack_bf16(u0 - bf16_hi(u0), u1 - bf16_hi(u1));
                }
        }
            named_sync(1, GROUP_THREADS);  // U is complete, W and Ut used up
            // S_c takes the buffer of S_{c-2}, and U_{c+1} that of U_{c-1}: the
            // output of the chunk before must have read both.  Waiting for it
            // here, before U_c is announced, also keeps the two barriers in
            // strict alternation: the output warps cannot arrive for O_c
            // before this wait has taken their arrival for O_{c-1}.
            if (ck > 0) named_sync(4, SCAN_THREADS);
            named_arrive(3, SCAN_THREADS);  // U_c and S_{c-1} for the output warps
            if (more) scan_load_wu(sm, a, blk0 + ck + 1, j0, ltid);
            cp_async_commit();
            cp_async_wait<1>();  // this chunk's K'
            named_sync(1, GROUP_THREADS);
        // ---- S = gamma_C S + K'^T U (warp: state rows 16w.., 32 columns)
        {
            const float gc = a.gc[blk0 + ck];
            const int m0 = lwarp * 16;
            float d[4][4] = {};
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
                uint32_t xh[4], xl[4];
                ld_a_t(&sm.kp[0][0][0], LDB, m0, ks * 16, lane, xh);
                ld_a_t(&sm.kp[1][0][0], LDB, m0, ks * 16, lane, xl);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t yh[4], yl[4];
                    ld_b2_t(&sm.up[ub][0][0][0], LDU, np * 16, ks * 16, lane, yh);
                    ld_b2_t(&sm.up[ub][1][0][0], LDU, np * 16, ks * 16, lane, yl);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        mma_16816(d[2 * np + h], xh, yh[2 * h], yh[2 * h + 1]);
                        mma_16816(d[2 * np + h], xh, yl[2 * h], yl[2 * h + 1]);
                        mma_16816(d[2 * np + h], xl, yh[2 * h], yh[2 * h + 1]);
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    const int i = m0 + g + e2 * 8, j = n * 8 + c0;
                    const float x0 = fmaf(gc, sm.s[i][j], d[n][2 * e2]);
                    const float x1 = fmaf(gc, sm.s[i][j + 1], d[n][2 * e2 + 1]);
                    sm.s[i][j] = x0;
                    sm.s[i][j + 1] = x1;
                    *reinterpret_cast<uint32_t *>(&sm.st[nxt][0][i][j]) = pack_bf16(x0, x1);
                    *reinterpret_cast<uint32_t *>(&sm.st[nxt][1][i][j]) =
                        pack_bf16(x0 - bf16_hi(x0), x1 - bf16_hi(x1));
                }
        }
            named_sync(1, GROUP_THREADS);  // K' used up
            if (more) scan_load_k(sm, a, blk0 + ck + 1, ltid);
            cp_async_commit();
        }
        named_sync(4, SCAN_THREADS);  // the last chunk's output is done
        cp_async_wait<0>();
        for (int e = ltid; e < S * JC; e += GROUP_THREADS) {
            const int i = e / JC, j = e % JC;
            state[(size_t)i * S + j0 + j] = sm.s[i][j];
        }
    } else {
        scan_load_qp(sm, a, blk0, ltid);
        cp_async_commit();
        for (int ck = 0; ck < a.nc; ++ck) {
            const int cur = ck & 1, ub = ck & 1;
            const bool more = ck + 1 < a.nc;
            named_sync(3, SCAN_THREADS);  // U_c and S_{c-1} are in place
            cp_async_wait<0>();           // this chunk's Q' and P
            named_sync(2, GROUP_THREADS);
        // ---- O = Q' S + P U (warp: rows 16 (w % 4).., columns 16 (w / 4)..)
        {
            float d[2][4] = {};
            mma3_rows<S, 1>(d, &sm.qp[0][0][0], &sm.qp[1][0][0], LDB, wm, &sm.st[cur][0][0][0],
                            &sm.st[cur][1][0][0], LDU, wn, lane);
            mma3_rows<C, 1>(d, &sm.p[0][0][0], &sm.p[1][0][0], LDP, wm, &sm.up[ub][0][0][0],
                            &sm.up[ub][1][0][0], LDU, wn, lane);
            const int r0 = wm + g;
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
                const int r = r0 + e2 * 8, tok = ck * C + r;
                if (tok < a.t) {
                    float *dst = a.opre + ((size_t)tok * a.n_v + vh) * S + j0 + wn;
#pragma unroll
                    for (int n = 0; n < 2; ++n)
                        *reinterpret_cast<float2 *>(dst + n * 8 + c0) =
                            make_float2(d[n][2 * e2] * scale, d[n][2 * e2 + 1] * scale);
                }
            }
        }
            named_sync(2, GROUP_THREADS);  // Q' and P used up
            named_arrive(4, SCAN_THREADS);  // O_c done
            if (more) scan_load_qp(sm, a, blk0 + ck + 1, ltid);
            cp_async_commit();
        }
    }
}

// ---------------------------------------------------------------------------
// dn_out_kernel: grid (t, n_v / 4), 4 warps, one (token, value head) each:
// heads = rms_norm(o; norm, eps) * silu(z) (forward.rs:1642-1652).
__global__ void __launch_bounds__(128) dn_out_kernel(const DnChunkArgs a) {
    using namespace dc;
    const int i = blockIdx.x, vh = blockIdx.y * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (vh >= a.n_v) return;
    const size_t off = ((size_t)i * a.n_v + vh) * S + lane * 4;
    const float4 z = *reinterpret_cast<const float4 *>(a.z + off);
    const float4 w = *reinterpret_cast<const float4 *>(a.norm + lane * 4);
    if (a.out_ready) {
        // beside the scan: its rows of this chunk are stored once its four
        // readout warps have counted in
        if (lane == 0) wait_flag_gpu(a.out_ready + (size_t)vh * a.nc + i / C, 4, a.status);
        __syncwarp();
    }
    const float4 o = *reinterpret_cast<const float4 *>(a.opre + off);
    double sq = (double)__fmul_rn(o.x, o.x) + (double)__fmul_rn(o.y, o.y) +
                (double)__fmul_rn(o.z, o.z) + (double)__fmul_rn(o.w, o.w);
    sq = warp_sum_d(sq);
    const float sc = rms_scale_fast(sq, S, a.eps);
    float4 y;
    y.x = __fmul_rn(__fmul_rn(__fmul_rn(o.x, sc), w.x), silu_fast(z.x));
    y.y = __fmul_rn(__fmul_rn(__fmul_rn(o.y, sc), w.y), silu_fast(z.y));
    y.z = __fmul_rn(__fmul_rn(__fmul_rn(o.z, sc), w.z), silu_fast(z.z));
    y.w = __fmul_rn(__fmul_rn(__fmul_rn(o.w, sc), w.w), silu_fast(z.w));
    *reinterpret_cast<float4 *>(a.out + off) = y;
}

// The conv history after the batch: the last three raw inputs, newest last
// (for a batch shorter than three, the oldest entries come from the history
// before it).
__global__ void dn_hist_kernel(const DnChunkArgs a) {
    const int conv_dim = 2 * a.n_k * dc::S + a.n_v * dc::S;
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= conv_dim) return;
    float *h = a.conv_state + (size_t)ch * 3;
    float old[3] = {h[0], h[1], h[2]};
    float nw[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int src = a.t - 3 + j;
        nw[j] = src >= 0 ? a.qkv[(size_t)src * conv_dim + ch] : old[src + 3];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) h[j] = nw[j];
}

cudaError_t init_dn_chunk_kernels() {
    cudaError_t e = cudaFuncSetAttribute(dn_chunk_local_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(LocalSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dn_chunk_local_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(LocalSmemTc) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(ScanSmem));
    if (e == cudaSuccess) e = init_dn_scan_tc_kernel();
    // With lazy module loading a kernel is loaded at its first launch, and
    // loading waits for the device.  The overlapped prefill launches the
    // chunk-local, output and history kernels while the scan spins on the
    // chunks' ready flags, so a first launch there would wait for a scan that
    // waits for it: load every kernel of the path here, before any scan runs.
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, dn_prep_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, dn_out_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, dn_hist_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, dn_chunk_local_kernel<false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, dn_chunk_local_kernel<true>);
    return e;
}

cudaError_t launch_dn_chunk(const DnChunkArgs &a_in, const DnScanMaps *scan_maps, cudaStream_t st,
                            const DnOverlap *overlap, const DnPlaneMaps *planes) {
    using namespace dc;
    DnChunkArgs a = a_in;
    a.w_lo_out = scan_maps == nullptr;
    // the tcgen05 form: one CTA per SM it gets, looping over the items; the
    // mma.sync form: a CTA per item
    const int n_items = a.n_v * a.nc;
    auto launch_local = [&](const DnChunkArgs &la) {
        if (planes) {
            const int grid = la.local_ctas > 0 && la.local_ctas < n_items ? la.local_ctas : n_items;
            dn_chunk_local_kernel<true>
                <<<grid, LOCAL_THREADS, sizeof(LocalSmemTc) + 1024, st>>>(la, *planes);
        } else {
            dn_chunk_local_kernel<false>
                <<<n_items, LOCAL_THREADS, sizeof(LocalSmem), st>>>(la, DnPlaneMaps{});
        }
    };
    dn_prep_kernel<<<dim3((a.t + PREP_TOKENS - 1) / PREP_TOKENS, (2 * a.n_k + a.n_v + 7) / 8), 256, 0,
                     st>>>(a);
    const int conv_dim = 2 * a.n_k * S + a.n_v * S;
    if (scan_maps && overlap && a.ready) {
        // the scan beside the chunk-local kernel: it starts once the prep
        // kernel is done and walks each head's chunks as their flags go up.
        // The output kernel follows the chunk-local kernel on the context's
        // stream, beside the scan's last chunks: an output warp waits for its
        // chunk's rows of the scan (out_ready).  The history kernel (it reads
        // only the raw rows) follows the scan on its stream, and the
        // context's stream then joins the scan's.
        cudaStream_t ss = overlap->scan_stream;
        cudaError_t e = cudaEventRecord(overlap->fork, st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ss, overlap->fork, 0);
        if (e == cudaSuccess) e = launch_dn_scan_tc(a, *scan_maps, ss);
        if (e != cudaSuccess) return e;
        launch_local(a);
        dn_out_kernel<<<dim3(a.t, (a.n_v + 3) / 4), 128, 0, st>>>(a);
        dn_hist_kernel<<<(conv_dim + 255) / 256, 256, 0, ss>>>(a);
        e = cudaEventRecord(overlap->join, ss);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, overlap->join, 0);
        if (e != cudaSuccess) return e;
        return cudaGetLastError();
    } else if (scan_maps) {
        a.ready = nullptr;
        launch_local(a);
        const cudaError_t e = launch_dn_scan_tc(a, *scan_maps, st);
        if (e != cudaSuccess) return e;
    } else {
        a.ready = nullptr;
        launch_local(a);
        dn_chunk_scan_kernel<<<dim3(S / JC, a.n_v), SCAN_THREADS, sizeof(ScanSmem), st>>>(a);
    }
    dn_out_kernel<<<dim3(a.t, (a.n_v + 3) / 4), 128, 0, st>>>(a);
    dn_hist_kernel<<<(conv_dim + 255) / 256, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace rl
