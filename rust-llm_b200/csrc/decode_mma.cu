// Split-KV flash decoding over a bf16 KV cache, sm_100a: K/V tiles staged by
// TMA tensor copies, both dot products on the tensor cores (mma.sync
// m16n8k16, bf16 in, f32 accumulate).
//
// The step is bound by HBM: every cached position is read once (1 KiB of K
// and V per KV head) and used by the four query heads of its group.  What
// keeps it at the memory roofline:
//   - copies are TMA boxes of 64 positions x 64 dims (8 KiB, 128-byte
//     swizzle): one tile of 64 positions is 4 K boxes + 4 V boxes, 64 KiB,
//     in a 3-deep ring per CTA.  Row-sized (512 B) bulk copies issue too
//     slowly to keep one SM's share of HBM in flight;
//   - the swizzle puts the 8 rows an ldmatrix reads in 8 different bank
//     groups, so the stage needs no padding and one copy fills it;
//   - the two dot products are m16n8k16 chains (~2 instructions per
//     position and head instead of ~25 on the CUDA cores), leaving the
//     consumer warps idle most of the time;
//   - the fused prologue issues all of its small loads (query, gate, norm
//     weights, RoPE row) before using any of them.
//
// Precision: the queries and the softmax weights enter the MMAs as a bf16
// pair hi + lo (hi = bf16(x), lo = bf16(x - hi)), a 16-bit mantissa; keys and
// values are already bf16 in the cache.  So S^T = K [q_hi | q_lo]^T and
// O^T = V^T [p_hi | p_lo]^T are each one m16n8k16 chain whose 8 columns hold
// the 4 heads' hi parts and lo parts, summed afterwards.  Residual error is
// ~1e-5 relative, inside the 1e-4 bar.
//
// Shape of the work: one CTA per (KV split, KV head, query row), one CTA per
// SM, one wave; a tile is 64 positions, 16 per consumer warp (the M of
// S^T).  A single producer lane keeps STAGES tiles in flight behind
// full/empty mbarriers.  Each CTA merges its four warps and writes one
// partial (max, sum, unnormalised output) per query head; a second small
// kernel (decode_combine_kernel) merges the splits and applies the sigmoid
// output gate.  For one decode row the q/k norm, RoPE and KV append are fused
// into the walk.
//
// Both kernels are launched as programmatic dependents of the kernel before
// them (PDL), and each triggers its own dependents only after its grid-
// dependency wait has returned (the merge right after it, the walk at its
// end).  So when a kernel starts, every kernel but the one just ahead of it
// has completed, and the one just ahead has passed its wait.  The walk's producer may start streaming this layer's cache before
// the previous kernel has finished (`early_kv`, set by the host when the
// kernel just ahead cannot be writing this cache: a merge, a DeltaNet step,
// or nothing since a synchronous write); every read of the step's inputs and
// every global write waits for the previous grid first.
//
// Reference: attend_batch / softmax of Exec::full_attn
// (crates/rust-llm/src/forward.rs:1783-1842) and its gate (:1327-1340).
#include "common.cuh"
#include "kernels.h"
#include "rlcuda.h"
#include "mma.cuh"

namespace rl {
namespace dm {
constexpr int kStaticRounds = 2;  // tiles per CTA dealt by index before the counter
constexpr int HD = 256;
constexpr int GROUP = 4;
constexpr int CWARPS = 4;
constexpr int THREADS = (CWARPS + 1) * 32;
constexpr int STAGES = 3;
constexpr int P = 16 * CWARPS;                  // positions per tile
constexpr int BOX_COLS = kDecodeBoxCols;        // dims per box (128 bytes)
constexpr int NBOX = HD / BOX_COLS;             // boxes per 256-dim row block
constexpr int BOX_BYTES = P * BOX_COLS * 2;     // 8 KiB
constexpr int HALF_BYTES = NBOX * BOX_BYTES;    // K (or V) part of a stage
constexpr int STAGE_BYTES = 2 * HALF_BYTES;     // 64 KiB
constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024;  // + alignment slack
constexpr float LOG2E = 1.4426950408889634f;
static_assert(kDecodeBoxRows == P, "one box row per tile position");
static_assert((size_t)STAGES * STAGE_BYTES >=
                  (size_t)(CWARPS * GROUP * HD + CWARPS * GROUP * 2 + GROUP * HD) * 4,
              "the merge scratch reuses the stage ring");
}  // namespace dm

// One lane's share (8 consecutive dims) of a 256-wide head before RMSNorm
// and RoPE, with every global load issued before any is used.
struct LaneHead {
    float x[8], w[8], c[8], s[8];
};

__device__ __forceinline__ void load4(float *dst, const float *src) {
    const float4 f = *reinterpret_cast<const float4 *>(src);
    dst[0] = f.x, dst[1] = f.y, dst[2] = f.z, dst[3] = f.w;
}

__device__ __forceinline__ void load_lane_head(LaneHead &h, const float *x, const float *w,
                                               const float *cs_row, const float *sn_row,
                                               int n_rot, int lane) {
    load4(h.x, x + lane * 8);
    load4(h.x + 4, x + lane * 8 + 4);
    load4(h.w, w + lane * 8);
    load4(h.w + 4, w + lane * 8 + 4);
    const int half = n_rot / 2;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        const int pr = d < half ? d : d - half;
        h.c[e] = d < n_rot ? cs_row[pr] : 1.0f;
        h.s[e] = d < n_rot ? sn_row[pr] : 0.0f;
    }
}

// RMSNorm (f64 sum of f32 squares, forward.rs:1697-1711) then partial RoPE
// (forward.rs:1851-1862) of one head by one warp; the result lands in `dst`
// (shared, 256 floats).
__device__ __forceinline__ void lane_norm_rope(const LaneHead &h, float *dst, int n_rot, float eps,
                                               int lane) {
    double sq = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) sq += (double)__fmul_rn(h.x[e], h.x[e]);
    sq = warp_sum_d(sq);
    const float scale = rms_scale_from_sum(sq, dm::HD, eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane * 8 + e] = __fmul_rn(__fmul_rn(h.x[e], scale), h.w[e]);
    __syncwarp();
    const int half = n_rot / 2;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        y[e] = dst[d];
        if (d < n_rot) {
            const int pr = d < half ? d : d - half;
            const float x0 = dst[pr], x1 = dst[pr + half];
            y[e] = d < half ? __fsub_rn(__fmul_rn(x0, h.c[e]), __fmul_rn(x1, h.s[e]))
                            : __fadd_rn(__fmul_rn(x0, h.s[e]), __fmul_rn(x1, h.c[e]));
        }
    }
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane * 8 + e] = y[e];
    __syncwarp();
}

template <bool FUSED>
__global__ void __launch_bounds__(dm::THREADS, 1)
    decode_mma_kernel(const __grid_constant__ DecodeArgs a, const __grid_constant__ CUtensorMap kv_map) {
    using namespace dm;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], ready_bar;
    __shared__ __align__(16) float q_s[GROUP][HD];
    __shared__ __align__(16) __nv_bfloat16 newk_s[HD], newv_s[HD];
    __shared__ __align__(16) float kf_s[HD];
    __shared__ __align__(16) __nv_bfloat16 pbuf[CWARPS][8][16];  // P^T per warp: [col][pos]
    __shared__ int flag_s;
    __shared__ int tile_s[STAGES];  // tile index in each stage, -1: no more tiles

    // the swizzled boxes want a 1024-byte aligned base
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (a.span && tid == 0) atomicMin(a.span, globaltimer_ns());
    // a batch row is its own sequence with its own cache and tensor map
    const BatchRow *br = a.rows ? a.rows + row : nullptr;
    const int pos_row = br ? a.batch_pos[row] : a.pos + row;  // sequence position of this row
    const int ctx_row = br ? br->context : a.context;
    const CUtensorMap *map = br ? br->map : &kv_map;
    // this cache holds sequence positions shard_lo .. shard_lo + context - 1
    const int loc_row = pos_row - a.shard_lo;  // the row's cache index (may lie outside)
    const int n_kv = max(0, min(loc_row + 1, ctx_row));  // cached positions the row sees
    const int n_all = (n_kv + P - 1) / P;   // tiles of this row
    const int n_split = a.n_splits;          // CTAs sharing them
    const int head0 = row * a.n_head + kh * GROUP;
    __nv_bfloat16 *const k_cache = static_cast<__nv_bfloat16 *>(br ? br->k_cache : a.k_cache_v);
    __nv_bfloat16 *const v_cache = static_cast<__nv_bfloat16 *>(br ? br->v_cache : a.v_cache_v);
    const float *const q_norm = br ? br->q_norm : a.q_norm;
    const float *const k_norm = br ? br->k_norm : a.k_norm;
    // every CTA of a KV head builds the appended row (any of them may draw
    // the tile holding it); split 0 writes it to the cache
    const bool builds_new = FUSED && loc_row >= 0 && loc_row < ctx_row;
    const bool writes_new = builds_new && split == 0;
    const float *cs_row = (br ? br->rope_cs : a.rope_cs) + (size_t)pos_row * (a.n_rot / 2);
    const float *sn_row = (br ? br->rope_sn : a.rope_sn) + (size_t)pos_row * (a.n_rot / 2);
    const float *kv_in = (warp == 0 ? a.k_in : a.v_in) + (size_t)row * a.n_kv * HD + (size_t)kh * HD;
    if (FUSED && warp < CWARPS && lane < 8) {
        // warm L2 with this step's small inputs while the previous grid
        // finishes; the values themselves are read after the wait
        const float *q = a.qg + (size_t)(head0 + warp) * 2 * HD;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(q + lane * 32));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(q_norm + lane * 32));
        if (warp < 2) asm volatile("prefetch.global.L2 [%0];" ::"l"(kv_in + lane * 32));
        if (warp == 0 && lane == 0) {
            asm volatile("prefetch.global.L2 [%0];" ::"l"(cs_row));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(sn_row));
        }
        if (warp == 1) asm volatile("prefetch.global.L2 [%0];" ::"l"(k_norm + lane * 32));
    }

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], CWARPS);
        }
        mbar_init(&ready_bar, CWARPS);
        flag_s = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // per-lane softmax state for heads hb, hb+1 (hb = (lane & 1) * 2)
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    float o[16][4];
#pragma unroll
    for (int mt = 0; mt < 16; ++mt)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[mt][c] = 0.0f;
    bool ok = true;

    if (warp == CWARPS) {
        // ---------------- producer: one lane, 8 tensor boxes per tile ----------------
        // Tiles are dealt to the row's CTAs: the first kStaticRounds rounds
        // by index (split, split + n_split, ...), the rest from an atomic
        // counter, so the CTAs finish within about one tile of each other
        // whatever bandwidth each SM gets.  Every CTA ends with exactly one
        // draw past the end; the last such draw resets the counter for the
        // next launch.
        if (lane == 0) {
            prefetch_tensormap(map);
            if (!a.early_kv) grid_dep_wait();
            int *counter = a.counters + ((size_t)row * a.n_kv + kh) * 8;
            const int n_dyn = max(0, n_all - kStaticRounds * n_split);
            const int krow = (br ? br->k_row0 : a.k_row0) + kh * ctx_row;
            const int vrow = (br ? br->v_row0 : a.v_row0) + kh * ctx_row;
            const int early = max(1, min(a.early_tiles, STAGES));
            int issued = 0, round = 0, tile = split;
            bool stopped = false;
            while (true) {
                if (round >= kStaticRounds || tile >= n_all) {
                    const int t = atomicAdd(counter, 1);
                    if (t >= n_dyn) {
                        if (t == n_dyn + n_split - 1) atomicExch(counter, 0);
                        break;
                    }
                    tile = kStaticRounds * n_split + t;
                }
                const int s = issued % STAGES;
                if ((issued == early && !mbar_wait(&ready_bar, 0, a.status)) ||
                    (issued >= STAGES &&
                     !mbar_wait(&empty_bar[s], ((issued / STAGES) - 1) & 1, a.status))) {
                    flag_s = 1;
                    stopped = true;
                    break;
                }
                tile_s[s] = tile;
                mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
                unsigned char *st = smem + (size_t)s * STAGE_BYTES;
#pragma unroll
                for (int b = 0; b < NBOX; ++b) {
                    tma_load_2d(st + b * BOX_BYTES, map, b * BOX_COLS, krow + tile * P,
                                &full_bar[s]);
                    tma_load_2d(st + HALF_BYTES + b * BOX_BYTES, map, b * BOX_COLS,
                                vrow + tile * P, &full_bar[s]);
                }
                ++issued;
                ++round;
                tile += n_split;
            }
            // tell the consumers there is nothing more: an arrival without
            // bytes on the next stage, whose tile index reads -1
            const int s = issued % STAGES;
            if (!stopped && (issued < STAGES ||
                             mbar_wait(&empty_bar[s], ((issued / STAGES) - 1) & 1, a.status))) {
                tile_s[s] = -1;
                mbar_arrive(&full_bar[s]);
            } else {
                flag_s = 1;
                // a consumer gave up: every copy this CTA started lands before
                // its shared memory is released
                for (int j = max(0, issued - STAGES); j < issued; ++j)
                    mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, a.status);
            }
        }
    } else {
        // ---------------- consumers ----------------
        grid_dep_wait();  // the step's inputs come from the kernel before
        if (FUSED) {
            LaneHead hq, hk;
            load_lane_head(hq, a.qg + (size_t)(head0 + warp) * 2 * HD, q_norm, cs_row, sn_row,
                           a.n_rot, lane);
            if (builds_new && warp < 2)
                load_lane_head(hk, kv_in, k_norm, cs_row, sn_row, a.n_rot, lane);
            lane_norm_rope(hq, q_s[warp], a.n_rot, a.eps, lane);
            if (builds_new && warp < 2) {
                float y[8];
                if (warp == 0) {
                    lane_norm_rope(hk, kf_s, a.n_rot, a.eps, lane);
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = kf_s[lane * 8 + e];
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = hk.x[e];
                }
                __nv_bfloat16 *cache = (warp == 0 ? k_cache : v_cache) +
                                       ((size_t)kh * ctx_row + loc_row) * HD + lane * 8;
                __nv_bfloat16 *keep = (warp == 0 ? newk_s : newv_s) + lane * 8;
                uint4 packed;
                packed.x = pack_bf16(y[0], y[1]);
                packed.y = pack_bf16(y[2], y[3]);
                packed.z = pack_bf16(y[4], y[5]);
                packed.w = pack_bf16(y[6], y[7]);
                *reinterpret_cast<uint4 *>(keep) = packed;
                if (writes_new) {
                    *reinterpret_cast<uint4 *>(cache) = packed;
                    // visible GPU-wide before this grid's trigger, so a later
                    // walk that streams early reads the appended row
                    __threadfence();
                }
            }
            consumer_bar();
        }
        // B fragments of [q_hi | q_lo]^T: column n = lane/4 (heads 0-3 hi,
        // 4-7 lo), rows (dims) ks*16 + (lane%4)*2 + {0, 1} and + 8
        uint32_t qf[16][2];
        {
            const int n = lane >> 2, kb = (lane & 3) * 2, hq = n & 3;
            const bool lo = n >= 4;
            const float *qrow = FUSED ? q_s[hq] : a.q_f32 + (size_t)(head0 + hq) * HD;
#pragma unroll
            for (int ks = 0; ks < 16; ++ks)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int d = ks * 16 + hf * 8 + kb;
                    const float2 xv = *reinterpret_cast<const float2 *>(qrow + d);
                    float x0 = xv.x, x1 = xv.y;
                    if (lo) x0 = x0 - bf16_hi(x0), x1 = x1 - bf16_hi(x1);
                    qf[ks][hf] = pack_bf16(x0, x1);
                }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready_bar);           // inputs consumed
        const float qk_scale = (1.0f / 16.0f) * LOG2E;  // 1/sqrt(256), in log2 units
        const int wrow0 = warp * 16;                      // this warp's rows of a tile
        const uint32_t smem0 = smem_u32(smem);
        // ldmatrix rows: K (A = K rows, chunk k_c of each 16-dim step) and
        // V^T (A = V rows transposed)
        const int k_r = (lane & 7) + ((lane >> 3) & 1) * 8, k_c = lane >> 4;
        const int v_r = (lane >> 4) * 8 + (lane & 7), v_c = (lane >> 3) & 1;

        for (int j = 0;; ++j) {
            const int s = j % STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[s], (j / STAGES) & 1, a.status))) {
                ok = false;
                break;
            }
            const int tile = tile_s[s];
            if (tile < 0) break;
            const int base = tile * P;
            const int vw = max(0, min(16, n_kv - base - wrow0));  // valid rows of this warp
            const uint32_t kst = smem0 + s * STAGE_BYTES;
            const uint32_t vst = kst + HALF_BYTES;
            bool patched = false;
            if (builds_new && loc_row >= base + wrow0 && loc_row < base + wrow0 + 16) {
                // the appended row is in this warp's block: the copy may have
                // read it before it was written, so put the fresh one in place
                const int r = loc_row - base;
                const int b = lane >> 3, c = lane & 7;
                unsigned char *st = smem + (size_t)s * STAGE_BYTES;
                *reinterpret_cast<uint4 *>(st + b * BOX_BYTES + swz128(r, c)) =
                    reinterpret_cast<const uint4 *>(newk_s)[lane];
                *reinterpret_cast<uint4 *>(st + HALF_BYTES + b * BOX_BYTES + swz128(r, c)) =
                    reinterpret_cast<const uint4 *>(newv_s)[lane];
                __syncwarp();
                patched = true;
            }
            if (vw > 0) {
                // ---- S^T = K q^T over 16 dims per MMA; rows past vw read row 0
                float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const int kr = wrow0 + (k_r < vw ? k_r : 0);
#pragma unroll
                for (int ks = 0; ks < 16; ++ks) {
                    const int ch = 2 * ks + k_c;  // 16-byte chunk of the 512-byte row
                    uint32_t fa[4];
                    ldsm_x4(kst + (ch >> 3) * BOX_BYTES + swz128(kr, ch & 7), fa);
                    mma_16816(sacc, fa, qf[ks][0], qf[ks][1]);
                }
                // hi + lo columns: lane^2 holds the other half of the same heads
#pragma unroll
                for (int c = 0; c < 4; ++c) sacc[c] += __shfl_xor_sync(0xffffffffu, sacc[c], 2);
                const int p0 = lane >> 2, p1 = p0 + 8;
                float sv[4];
                sv[0] = p0 < vw ? sacc[0] * qk_scale : -INFINITY;
                sv[1] = p0 < vw ? sacc[1] * qk_scale : -INFINITY;
                sv[2] = p1 < vw ? sacc[2] * qk_scale : -INFINITY;
                sv[3] = p1 < vw ? sacc[3] * qk_scale : -INFINITY;
                // ---- online softmax over the warp's 16 positions, heads hb, hb+1
                float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
                const float al0 = exp2f(m_run[0] - mn0), al1 = exp2f(m_run[1] - mn1);
                const float pv0 = exp2f(sv[0] - mn0), pv1 = exp2f(sv[1] - mn1);
                const float pv2 = exp2f(sv[2] - mn0), pv3 = exp2f(sv[3] - mn1);
                l_run[0] = fmaf(l_run[0], al0, pv0 + pv2);
                l_run[1] = fmaf(l_run[1], al1, pv1 + pv3);
                m_run[0] = mn0;
                m_run[1] = mn1;
                // ---- P^T as the B operand of the second MMA, through shared
                if ((lane & 2) == 0) {
                    const int hb = (lane & 1) * 2;
                    __nv_bfloat16 *pb = &pbuf[warp][0][0];
                    const float pv[4] = {pv0, pv1, pv2, pv3};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int h = hb + (c & 1), p = (c < 2) ? p0 : p1;
                        const float hi = bf16_hi(pv[c]);
                        pb[h * 16 + p] = __float2bfloat16_rn(pv[c]);
                        pb[(h + 4) * 16 + p] = __float2bfloat16_rn(pv[c] - hi);
                    }
                }
                __syncwarp();
                const uint32_t b0 =
                    *reinterpret_cast<const uint32_t *>(&pbuf[warp][lane >> 2][(lane & 3) * 2]);
                const uint32_t b1 =
                    *reinterpret_cast<const uint32_t *>(&pbuf[warp][lane >> 2][(lane & 3) * 2 + 8]);
                // ---- rescale, then O^T += V^T P^T, 16 dims per MMA
                if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
                    for (int mt = 0; mt < 16; ++mt) {
                        o[mt][0] *= al0, o[mt][1] *= al1;
                        o[mt][2] *= al0, o[mt][3] *= al1;
                    }
                }
                const int vr = wrow0 + (v_r < vw ? v_r : 0);
#pragma unroll
                for (int mt = 0; mt < 16; ++mt) {
                    const int ch = 2 * mt + v_c;
                    uint32_t fa[4];
                    ldsm_x4_t(vst + (ch >> 3) * BOX_BYTES + swz128(vr, ch & 7), fa);
                    mma_16816(o[mt], fa, b0, b1);
                }
                __syncwarp();
            }
            if (patched) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
        }
    }

    // ---------------- merge the four warps, write this split's partial ----------------
    __syncthreads();  // every tile consumed: the stage ring is free
    if (!ok) atomicOr(&flag_s, 1);
    float *red_o = reinterpret_cast<float *>(smem);   // [CWARPS][GROUP][HD]
    float *red_ml = red_o + CWARPS * GROUP * HD;      // [CWARPS][GROUP][2]
    if (warp < CWARPS) {
        // l: sum the lanes' partial sums over positions (lanes with the same
        // lane & 3); O: hi column + lo column (lane ^ 2)
        float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, off);
            l1 += __shfl_xor_sync(0xffffffffu, l1, off);
        }
#pragma unroll
        for (int mt = 0; mt < 16; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) o[mt][c] += __shfl_xor_sync(0xffffffffu, o[mt][c], 2);
        if ((lane & 2) == 0) {
            const int hb = (lane & 1) * 2, dr = lane >> 2;
#pragma unroll
            for (int mt = 0; mt < 16; ++mt) {
                red_o[(warp * GROUP + hb) * HD + mt * 16 + dr] = o[mt][0];
                red_o[(warp * GROUP + hb + 1) * HD + mt * 16 + dr] = o[mt][1];
                red_o[(warp * GROUP + hb) * HD + mt * 16 + dr + 8] = o[mt][2];
                red_o[(warp * GROUP + hb + 1) * HD + mt * 16 + dr + 8] = o[mt][3];
            }
            if (lane < 2) {
                red_ml[(warp * GROUP + hb) * 2] = m_run[0];
                red_ml[(warp * GROUP + hb) * 2 + 1] = l0;
                red_ml[(warp * GROUP + hb + 1) * 2] = m_run[1];
                red_ml[(warp * GROUP + hb + 1) * 2 + 1] = l1;
            }
        }
    }
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
        // partial (max, sum) of query head head0 + tid for this split
        float2 *pml = reinterpret_cast<float2 *>(a.part_ml);
        pml[(size_t)(head0 + tid) * a.n_splits + split] = make_float2(M, L);
    }
    __syncthreads();
    for (int e4 = tid; e4 < GROUP * HD / 4; e4 += THREADS) {
        const int h = e4 / (HD / 4), d4 = e4 % (HD / 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) {
            const float sc = wscale[w][h];
            const float4 r = reinterpret_cast<const float4 *>(red_o)[w * GROUP * HD / 4 + e4];
            acc.x = fmaf(r.x, sc, acc.x), acc.y = fmaf(r.y, sc, acc.y);
            acc.z = fmaf(r.z, sc, acc.z), acc.w = fmaf(r.w, sc, acc.w);
        }
        reinterpret_cast<float4 *>(a.part_o + ((size_t)(head0 + h) * a.n_splits + split) * HD)[d4] =
            acc;
    }
    if (tid == 0 && flag_s) atomicOr(a.status, DEV_TIMEOUT);
    // triggered last: a merge resident for the whole walk slowed it down
    __syncthreads();
    if (a.span && tid == 0) {
        // the launch's span: from its first CTA's start to its last CTA's end
        const unsigned long long now = globaltimer_ns();
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        if (atomicAdd(a.span + 1, 1ull) == total - 1) {
            const unsigned long long t0 = atomicAdd(a.span, 0ull);
            atomicAdd(a.span + 2, now - t0);
            atomicAdd(a.span + 3, 1ull);
            atomicExch(a.span, ~0ull);
            atomicExch(a.span + 1, 0ull);
        }
    }
    grid_dep_launch();
}

// Merges the splits of one (row, query head) for a 64-dim slice and applies
// the sigmoid output gate (forward.rs:1327-1340).  Block: 64 dims x 8 split
// lanes; each thread issues its partial loads in predicated batches of 8, so
// a merge of up to 64 splits is one round trip to L2.
constexpr int kCombineDims = 64, kCombineLanes = 8, kCombineBatch = 8, kCombineMaxSplits = 512;
__global__ void __launch_bounds__(kCombineDims *kCombineLanes)
    decode_combine_kernel(const __grid_constant__ DecodeArgs a) {
    grid_dep_wait();    // the walk's partials are complete and visible
    grid_dep_launch();  // the next kernel may be scheduled while this merge runs
    __shared__ float sc_s[kCombineMaxSplits], m_s[kCombineMaxSplits], l_s[kCombineMaxSplits];
    __shared__ float red[kCombineLanes][kCombineDims];
    __shared__ float L_s;
    const int hh = blockIdx.x;  // row * n_head + head
    const int tx = threadIdx.x % kCombineDims, ty = threadIdx.x / kCombineDims;
    const int d = blockIdx.y * kCombineDims + tx;
    const int S = a.n_splits;
    const float gate = a.qg[(size_t)hh * 2 * dm::HD + dm::HD + d];
    // a split sequence's publish: this CTA's own step count (only this CTA
    // touches its word, and only after every thread has read it)
    const int xcta = hh * gridDim.y + blockIdx.y;
    const unsigned xE = a.xpeers ? a.xepochs[xcta] + 1 : 0u;
    const float2 *ml = reinterpret_cast<const float2 *>(a.part_ml) + (size_t)hh * S;
    const float *po = a.part_o + (size_t)hh * S * dm::HD + d;
    // the first batch of partials goes out with the (max, sum) loads
    float v[kCombineBatch];
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i) {
        const int s = ty + i * kCombineLanes;
        v[i] = s < S ? __ldcg(po + (size_t)s * dm::HD) : 0.0f;
    }
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const float2 x = __ldcg(&ml[s]);
        m_s[s] = x.x;
        l_s[s] = x.y;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        // one warp: the max over the splits, each split's weight, the sum
        const int lane = threadIdx.x;
        float M = -INFINITY;
        for (int s = lane; s < S; s += 32) M = fmaxf(M, m_s[s]);
        M = warp_max(M);
        float L = 0.0f;
        for (int s = lane; s < S; s += 32) {
            const float sc = m_s[s] == -INFINITY ? 0.0f : exp2f(m_s[s] - M);
            sc_s[s] = sc;
            L = fmaf(l_s[s], sc, L);
        }
        L = warp_sum(L);
        if (lane == 0) L_s = L;
    }
    __syncthreads();
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i) {
        const int s = ty + i * kCombineLanes;
        if (s < S) acc = fmaf(v[i], sc_s[s], acc);
    }
    for (int s0 = kCombineBatch * kCombineLanes; s0 < S; s0 += kCombineBatch * kCombineLanes) {
#pragma unroll
        for (int i = 0; i < kCombineBatch; ++i) {
            const int s = s0 + ty + i * kCombineLanes;
            v[i] = s < S ? __ldcg(po + (size_t)s * dm::HD) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kCombineBatch; ++i) {
            const int s = s0 + ty + i * kCombineLanes;
            if (s < S) acc = fmaf(v[i], sc_s[s], acc);
        }
    }
    red[ty][tx] = acc;
    __syncthreads();
    if (ty == 0) {
        float o = 0.0f;
#pragma unroll
        for (int y = 0; y < kCombineLanes; ++y) o += red[y][tx];
        if (a.part_out || a.xpeers) {
            // one shard of a sequence split across GPUs: this GPU's partial
            // (unnormalised output, max in log2 units, sum) for the merge,
            // into the caller's buffer or into every GPU's exchange slot
            float M = -INFINITY;
            if (blockIdx.y == 0 && tx == 0)
                for (int s = 0; s < S; ++s) M = fmaxf(M, m_s[s]);
            if (a.part_out) {
                float *po_out = a.part_out + (size_t)hh * (dm::HD + 2);
                po_out[d] = o;
                if (blockIdx.y == 0 && tx == 0) {
                    po_out[dm::HD] = M;
                    po_out[dm::HD + 1] = L_s;
                }
            } else {
                // every value goes to every GPU's slot with the step's epoch in
                // the same 64-bit store, so the reader checks each value itself
                // and no fence or flag is needed
                for (int g = 0; g < a.xworld; ++g) {
                    unsigned long long *dst =
                        reinterpret_cast<unsigned long long *>(a.xpeers[g]) +
                        (((size_t)(xE & 1) * a.xworld + a.xrank) * gridDim.x + hh) * (dm::HD + 2);
                    xstore(dst + d, o, xE);
                    if (blockIdx.y == 0 && tx == 0) {
                        xstore(dst + dm::HD, M, xE);
                        xstore(dst + dm::HD + 1, L_s, xE);
                    }
                }
            }
        } else {
            a.out[(size_t)hh * dm::HD + d] = (o / L_s) * sigmoidf_(gate);
        }
    }
    if (a.xpeers) {
        __syncthreads();  // every thread has read this CTA's step count
        if (threadIdx.x == 0) a.xepochs[xcta] = xE;
    }
}

// The merge of a split sequence's partials from this GPU's exchange buffer,
// where every GPU stored each value with the step's epoch beside it: one CTA
// per (row, head), one thread per dim.  It launches as soon as the publishing
// merge ahead of it has started and needs no flag: thread d waits (bounded)
// until every GPU's value d of this head carries the step's epoch (the CTA's
// own count of steps), threads 0.. and 32.. the same for the GPUs' (max,
// sum).  Reference: the softmax over all positions (forward.rs:1831-1842)
// reassembled by the log-sum-exp rule, then the gate (:1327-1340).
__global__ void __launch_bounds__(256) peer_merge_kernel(const unsigned long long *xbuf,
                                                         int world, int rows_heads,
                                                         const float *qg, float *out, int *status,
                                                         unsigned *epochs,
                                                         unsigned long long limit_ns) {
    grid_dep_launch();  // the next layer's walk may start streaming meanwhile
    __shared__ float m_s[RL_EXCHANGE_MAX_GPUS], l_s[RL_EXCHANGE_MAX_GPUS];
    const int hh = blockIdx.x, d = threadIdx.x;
    const unsigned E = epochs[hh] + 1;  // written last by this CTA's previous step
    const size_t stride = (size_t)rows_heads * (dm::HD + 2);
    const unsigned long long *p0 = xbuf + (size_t)(E & 1) * world * stride + (size_t)hh * (dm::HD + 2);
    const unsigned long long start = globaltimer_ns();
    bool late = false;
    if ((d & 31) < world && d < 64) {
        const int g = d & 31;
        const float v = xload(p0 + g * stride + dm::HD + (d >> 5), E, start, limit_ns, late);
        (d < 32 ? m_s : l_s)[g] = v;
    }
    // every GPU's value d in flight at once (one round trip for all of them,
    // where polling them in turn took one each), then a bounded wait for any
    // that did not yet carry the step's epoch
    unsigned long long w[RL_EXCHANGE_MAX_GPUS];
#pragma unroll
    for (int g = 0; g < RL_EXCHANGE_MAX_GPUS; ++g)
        if (g < world)
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];"
                         : "=l"(w[g])
                         : "l"(p0 + g * stride + d)
                         : "memory");
    float vals[RL_EXCHANGE_MAX_GPUS];
#pragma unroll
    for (int g = 0; g < RL_EXCHANGE_MAX_GPUS; ++g)
        if (g < world)
            vals[g] = (unsigned)(w[g] >> 32) == E
                          ? __uint_as_float((unsigned)w[g])
                          : xload(p0 + g * stride + d, E, start, limit_ns, late);
    if (__syncthreads_or(late) && d == 0) atomicOr(status, DEV_TIMEOUT);
    float M = -INFINITY;
    for (int g = 0; g < world; ++g) M = fmaxf(M, m_s[g]);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int g = 0; g < RL_EXCHANGE_MAX_GPUS; ++g) {
        if (g < world) {
            const float sc = m_s[g] == -INFINITY ? 0.0f : exp2f(m_s[g] - M);
            L = fmaf(l_s[g], sc, L);
            o = fmaf(vals[g], sc, o);
        }
    }
    const float gate = qg[(size_t)hh * 2 * dm::HD + dm::HD + d];
    out[(size_t)hh * dm::HD + d] = (o / L) * sigmoidf_(gate);
    __syncthreads();
    if (d == 0) epochs[hh] = E;
}

cudaError_t launch_peer_merge(const unsigned long long *xbuf, int world, int rows_heads,
                              const float *qg, float *out, int *status, unsigned *epochs,
                              unsigned long long limit_ns, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows_heads);
    cfg.blockDim = dim3(dm::HD);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, peer_merge_kernel, xbuf, world, rows_heads, qg, out, status,
                              epochs, limit_ns);
}

// Merges the partials of a sequence split across GPUs, gathered as
// parts [n_parts][rows * n_head][hd + 2] (unnormalised output, max in log2
// units, sum), with the same log-sum-exp merge, then applies the sigmoid
// output gate (forward.rs:1327-1340).  One CTA per (row, head), one thread
// per dim.
__global__ void __launch_bounds__(256) merge_parts_kernel(const float *parts, int n_parts,
                                                          int rows_heads, const float *qg,
                                                          float *out) {
    const int hh = blockIdx.x, d = threadIdx.x;
    const size_t stride = (size_t)rows_heads * (dm::HD + 2);
    const float *p0 = parts + (size_t)hh * (dm::HD + 2);
    float M = -INFINITY;
    for (int g = 0; g < n_parts; ++g) M = fmaxf(M, p0[g * stride + dm::HD]);
    float L = 0.0f, o = 0.0f;
    for (int g = 0; g < n_parts; ++g) {
        const float *pg = p0 + g * stride;
        const float m = pg[dm::HD];
        const float sc = m == -INFINITY ? 0.0f : exp2f(m - M);
        L = fmaf(pg[dm::HD + 1], sc, L);
        o = fmaf(pg[d], sc, o);
    }
    const float gate = qg[(size_t)hh * 2 * dm::HD + dm::HD + d];
    out[(size_t)hh * dm::HD + d] = (o / L) * sigmoidf_(gate);
}

cudaError_t launch_merge_parts(const float *parts, int n_parts, int rows_heads, const float *qg,
                               float *out, cudaStream_t st) {
    merge_parts_kernel<<<rows_heads, dm::HD, 0, st>>>(parts, n_parts, rows_heads, qg, out);
    return cudaGetLastError();
}

template <bool FUSED>
static cudaError_t launch_mma_t(const DecodeArgs &a, const CUtensorMap &map, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.n_kv, a.t);
    cfg.blockDim = dim3(dm::THREADS);
    cfg.dynamicSmemBytes = dm::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_mma_kernel<FUSED>, a, map);
}

cudaError_t launch_decode_mma(const DecodeArgs &a, const CUtensorMap &kv_map, cudaStream_t st) {
    if (a.n_splits > kCombineMaxSplits) return cudaErrorInvalidValue;
    return a.fused ? launch_mma_t<true>(a, kv_map, st) : launch_mma_t<false>(a, kv_map, st);
}

cudaError_t launch_decode_combine(const DecodeArgs &a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_head * a.t, dm::HD / kCombineDims);
    cfg.blockDim = dim3(kCombineDims * kCombineLanes);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_combine_kernel, a);
}

cudaError_t init_decode_mma_kernels() {
    cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dm::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(decode_mma_kernel<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dm::SMEM);
    // the merge asks for the walk's shared-memory split, so a walk CTA of the
    // next layer can join it on the same SM without reconfiguring the SM
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(decode_combine_kernel,
                                 cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return e;
}

int decode_mma_max_active_ctas(bool fused) {
    int per_sm = 0;
    const cudaError_t e =
        fused ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mma_kernel<true>,
                                                              dm::THREADS, dm::SMEM)
              : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mma_kernel<false>,
                                                              dm::THREADS, dm::SMEM);
    return e == cudaSuccess ? per_sm : 0;
}

int decode_mma_positions_per_tile() { return dm::P; }

}  // namespace rl
