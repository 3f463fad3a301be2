// Causal prefill attention for the gated GQA layers on the fifth-generation
// tensor cores (tcgen05 + tensor memory), bf16 in, f32 accumulate, sm_100a.
//
// One CTA per (128-row query tile, query head).  Warp roles:
//   warps 0,10  TMA producers: warp 0 the query tile once (4 boxes of 128
//               rows x 64 dims) and then K tiles of 64 positions (4 boxes of
//               64 x 64), warp 10 the V tiles, each into its own 2-slot ring
//               (a K slot frees when its Q K^T is done, a V slot when its P V
//               is); 128-byte swizzle throughout
//   warp 1      tensor-memory allocator and the single MMA-issuing thread:
//               S_j = Q K_j^T (M 128, N 64, K 256: 16 MMAs) into one of two
//               S buffers, then O += P_{j-1} V_{j-1} (M 128, N 256, K 64: 4
//               MMAs) with P read from tensor memory, so the next tile's
//               Q K^T runs while the softmax works on this one
//   warps 2-9   softmax and epilogue, two threads per query row (each half
//               of the tile's columns and of O): S from tensor memory, causal
//               mask on the diagonal tiles, the row max exchanged through
//               shared memory, online softmax in log2 units with a lazy
//               rescale (O is corrected only when a row's max grows by more
//               than 2^12), P written back as bf16 over the S buffer; at the
//               end O / l times the sigmoid output gate (staged in bf16 by
//               the prologue, loaded by TMA over the query tile once the last
//               Q K^T is done), to global memory in whole 128-byte rows
// Tensor memory (512 columns): O in columns 0-255, S buffers at 256 and 320;
// P_j aliases the first 32 columns of its S buffer.  MMAs of one thread run
// in issue order, so Q K^T of tile j+2 (same S buffer) cannot overtake the
// P V of tile j that reads P_j.
//
// Reference: attend_batch / softmax over the causal prefix
// (crates/rust-llm/src/forward.rs:1783-1842) and the gate (:1327-1340); the
// queries and the appended keys come from the multi-row prologue
// (full_attn.cu), which applies the norms and RoPE (:1259-1292).
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace rl {
namespace pf {
constexpr int HD = 256;
constexpr int BM = 128;          // query rows per CTA
constexpr int BN = 64;           // key positions per tile
constexpr int THREADS = 352;     // 11 warps
constexpr int Q_BOX = BM * 128;  // 16 KiB: 128 rows x 64 dims
constexpr int KV_BOX = BN * 128; // 8 KiB: 64 rows x 64 dims
constexpr int Q_BYTES = 4 * Q_BOX;
constexpr int KV_HALF = 4 * KV_BOX;  // K (or V) of one tile
constexpr int STAGE = 2 * KV_HALF;
constexpr int SMEM = Q_BYTES + 2 * STAGE + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 0, S_COL = 256;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 12.0f;  // P up to 2^12: no range issue in bf16 or f32
}  // namespace pf

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y,
                                            int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// VERIFY: the multi-row verify form.  The CTA is (key split, KV head); tile
// row r is draft row r % 32 of query head 4 * kv_head + r / 32, so the four
// heads that share a KV head read its tiles once; the CTA walks only its
// split's key tiles and writes an unnormalised partial (O, max, sum) per
// (row, head) for the split merge, which applies the gate.
template <bool VERIFY>
__global__ void __launch_bounds__(pf::THREADS, 1)
    prefill_kernel(const __grid_constant__ PrefillArgs a, const __grid_constant__ CUtensorMap q_map,
                   const __grid_constant__ CUtensorMap kv_map,
                   const __grid_constant__ CUtensorMap gate_map) {
    using namespace pf;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t q_full, k_full[2], v_full[2], k_empty[2], v_empty[2],
        s_full[2], p_full[2], o_ready, o_final, g_full;
    __shared__ uint32_t tmem_base_s;
    __shared__ int flag_s;
    __shared__ float red_m[2][2][BM], red_l[2][BM];  // the two halves of each row
    // the halves meet on mbarriers (bounded waits), not named barriers, so a
    // warp that gives up cannot leave its partner waiting for good
    __shared__ __align__(8) uint64_t mx_bar[2], l_bar;

    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int head, kh, q0, j0, n_kt, split = 0;
    if constexpr (VERIFY) {
        kh = blockIdx.x % a.n_kv;
        split = blockIdx.x / a.n_kv;
        head = kh * 4;  // the group's first query head
        q0 = 0;
        const int n_tiles = (a.pos + a.t - 1) / BN + 1;
        j0 = split * a.split_tiles;
        n_kt = max(0, min(n_tiles, j0 + a.split_tiles) - j0);
    } else {
        // heaviest query tiles first: they have the most key tiles
        const int n_qt = (a.t + BM - 1) / BM;
        const int qt = n_qt - 1 - (int)(blockIdx.x / a.n_head);
        head = blockIdx.x % a.n_head;
        kh = head / (a.n_head / a.n_kv);
        q0 = qt * BM;
        const int q_last = min(a.t, q0 + BM) - 1;  // last valid row of the tile
        j0 = 0;
        n_kt = (a.pos + q_last) / BN + 1;           // key tiles the tile needs
    }
    const uint32_t sbase = smem_u32(smem);

    if (tid == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 8);
        }
        mbar_init(&o_ready, 1);
        mbar_init(&o_final, 1);
        mbar_init(&g_full, 1);
        mbar_init(&mx_bar[0], 256);
        mbar_init(&mx_bar[1], 256);
        mbar_init(&l_bar, 256);
        flag_s = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_base_s, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0 || warp == 10) {
        // ---------------- TMA producers ----------------
        // warp 0: the query tile, then K tiles (a slot frees when its Q K^T is
        // done); warp 10: V tiles (a slot frees when its P V is done).  Two
        // warps, so K runs ahead of V by as much as the slots allow.
        if (lane == 0) {
            const bool is_k = warp == 0;
            if (is_k) {
                prefetch_tensormap(&q_map);
                prefetch_tensormap(&kv_map);
                mbar_arrive_expect_tx(&q_full, Q_BYTES);
                if constexpr (VERIFY) {
                    // 32-row boxes: head g of the group lands in tile rows
                    // 32g..32g+31 (rows past t are computed and never stored)
                    for (int g = 0; g < 4; ++g)
                        for (int b = 0; b < 4; ++b)
                            tma_load_3d(smem + b * Q_BOX + g * 32 * 128, &q_map, b * 64, head + g,
                                        0, &q_full);
                } else {
                    for (int b = 0; b < 4; ++b)
                        tma_load_3d(smem + b * Q_BOX, &q_map, b * 64, head, q0, &q_full);
                }
            }
            const int row0 = (is_k ? a.k_row0 : a.v_row0) + kh * a.context;
            uint64_t *full = is_k ? k_full : v_full, *empty = is_k ? k_empty : v_empty;
            int issued = 0;
            for (int j = 0; j < n_kt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&empty[s], ((j >> 1) - 1) & 1, a.status)) {
                    flag_s = 1;
                    break;
                }
                unsigned char *st = smem + Q_BYTES + s * STAGE + (is_k ? 0 : KV_HALF);
                mbar_arrive_expect_tx(&full[s], KV_HALF);
                for (int b = 0; b < 4; ++b)
                    tma_load_2d(st + b * KV_BOX, &kv_map, b * 64, row0 + (j0 + j) * BN, &full[s]);
                issued = j + 1;
            }
            if (!VERIFY && is_k && issued == n_kt) {
                // the last Q K^T done, the query tile is free: the output gate
                // (sigmoid, bf16, staged by the prologue) takes its place
                if (mbar_wait(&k_empty[(n_kt - 1) & 1], ((n_kt - 1) >> 1) & 1, a.status)) {
                    prefetch_tensormap(&gate_map);
                    mbar_arrive_expect_tx(&g_full, Q_BYTES);
                    for (int b = 0; b < 4; ++b)
                        tma_load_3d(smem + b * Q_BOX, &gate_map, b * 64, head, q0, &g_full);
                    mbar_wait(&g_full, 0, a.status);
                } else {
                    flag_s = 1;
                }
            }
            // everything started has landed before the CTA releases its memory
            if (is_k) mbar_wait(&q_full, 0, a.status);
            for (int j = max(0, issued - 2); j < issued; ++j)
                mbar_wait(&full[j & 1], (j >> 1) & 1, a.status);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t id_qk = tc::idesc_bf16(BM, BN, false);
            constexpr uint32_t id_pv = tc::idesc_bf16(BM, HD, true);
            bool ok = mbar_wait(&q_full, 0, a.status);
            tc::fence_after_sync();
            for (int j = 0; ok && j <= n_kt; ++j) {
                if (j < n_kt) {
                    const int s = j & 1;
                    if (!mbar_wait(&k_full[s], (j >> 1) & 1, a.status)) { ok = false; break; }
                    tc::fence_after_sync();
                    const uint32_t kst = sbase + Q_BYTES + s * STAGE;
                    const uint32_t d = tmem + S_COL + s * BN;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (kk & 3) * 32;  // 16 dims inside a 64-dim box
                        const uint64_t da = tc::smem_desc(sbase + (kk >> 2) * Q_BOX + off, 16, 1024);
                        const uint64_t db = tc::smem_desc(kst + (kk >> 2) * KV_BOX + off, 16, 1024);
                        tc::mma_ss(d, da, db, id_qk, kk > 0);
                    }
                    tc::commit(&s_full[s]);
                    tc::commit(&k_empty[s]);
                }
                if (j >= 1) {
                    const int jj = j - 1, s = jj & 1;
                    if (!mbar_wait(&p_full[s], (jj >> 1) & 1, a.status) ||
                        !mbar_wait(&v_full[s], (jj >> 1) & 1, a.status)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t vst = sbase + Q_BYTES + s * STAGE + KV_HALF;
                    const uint32_t p = tmem + S_COL + s * BN;
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk) {
                        const uint64_t db = tc::smem_desc(vst + kk * 16 * 128, KV_BOX, 1024);
                        tc::mma_ts(tmem + O_COL, p + kk * 8, db, id_pv, jj > 0 || kk > 0);
                    }
                    tc::commit(&v_empty[s]);
                    tc::commit(&o_ready);
                }
            }
            if (!ok) flag_s = 1;
            // o_final completes when every MMA issued above is done; the
            // tensor memory is not released before that
            tc::commit(&o_final);
            mbar_wait(&o_final, 0, a.status);
        }
    } else {
        // ---------------- softmax + epilogue: two threads per query row ----------------
        // warps 2-5 take S columns 0-31 of each tile and O columns 0-127,
        // warps 6-9 columns 32-63 and O columns 128-255; warps w and w+4 share
        // the tensor-memory lane quarter w % 4, i.e. the same 32 rows
        const int quarter = warp & 3;
        const int h = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        // absolute position of this row (verify: draft row `lane` of head
        // head + quarter)
        const int qa = a.pos + (VERIFY ? lane : q0 + r);
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const float scale = (1.0f / 16.0f) * LOG2E;
        const int first_masked = (a.pos + q0) / BN;  // earliest tile a row of the CTA masks
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_kt; ++j) {
            const int s = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[s], (j >> 1) & 1, a.status))) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t sc = tmem + lane_off + S_COL + s * BN;
            uint32_t u[32];
            tc::ld32(sc + 32 * h, u);
            tc::wait_ld();
            const int kv0 = (j0 + j) * BN + 32 * h;
            if (j0 + j >= first_masked) {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    if (kv0 + c > qa) u[c] = __float_as_uint(-INFINITY);
            }
            float mx0 = __uint_as_float(u[0]), mx1 = __uint_as_float(u[1]);
#pragma unroll
            for (int c = 2; c < 32; c += 2) {
                mx0 = fmaxf(mx0, __uint_as_float(u[c]));
                mx1 = fmaxf(mx1, __uint_as_float(u[c + 1]));
            }
            // the row's max over both halves (scores scale by a positive
            // constant): post this half's, then compute P optimistically with
            // the running max while the partner's arrives; only a row whose
            // max grows past the lazy threshold (rare) redoes the exponentials
            red_m[j & 1][h][r] = fmaxf(mx0, mx1);
            mbar_arrive(&mx_bar[j & 1]);
            uint32_t pk[16];
            float ps0 = 0.0f, ps1 = 0.0f;
            auto exps = [&](float m) {
                ps0 = 0.0f;
                ps1 = 0.0f;
                // a row with every key so far masked (a verify split past
                // the row) has m = -inf: its P is 0, not NaN
                const float neg_m = m == -INFINITY ? 0.0f : -m;
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const float p0 = ex2_approx(fmaf(__uint_as_float(u[2 * c]), scale, neg_m));
                    const float p1 = ex2_approx(fmaf(__uint_as_float(u[2 * c + 1]), scale, neg_m));
                    ps0 += p0;
                    ps1 += p1;
                    __nv_bfloat162 hh = __floats2bfloat162_rn(p0, p1);
                    pk[c] = *reinterpret_cast<uint32_t *>(&hh);
                }
            };
            exps(m_run);
            if (!__all_sync(0xffffffffu, mbar_wait(&mx_bar[j & 1], (j >> 1) & 1, a.status))) {
                ok = false;
                break;
            }
            const float mt = fmaxf(red_m[j & 1][0][r], red_m[j & 1][1][r]) * scale;
            const bool grow = mt > m_run + RESCALE_LOG2;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? mt : m_run;
                const float corr = m_run == -INFINITY ? 0.0f : exp2f(m_run - m_new);
                if (j > 0) {
                    // O holds tiles < j: wait for the last P V, then correct
                    // this thread's half of the row
                    if (!__all_sync(0xffffffffu, mbar_wait(&o_ready, (j - 1) & 1, a.status))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t oc = tmem + lane_off + O_COL + 128 * h;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t o[32];
                        tc::ld32(oc + c * 32, o);
                        tc::wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                        tc::st32(oc + c * 32, o);
                    }
                    tc::wait_st();
                }
                l_run *= corr;
                m_run = m_new;
                exps(m_run);
            }
            l_run += ps0 + ps1;
            tc::st16(sc + 16 * h, pk);
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[s]);
        }
        // ---- epilogue: O / l * sigmoid(gate), this thread's 128 columns
        if (ok && !__all_sync(0xffffffffu, mbar_wait(&o_final, 0, a.status))) ok = false;
        if (!ok) flag_s = 1;
        red_l[h][r] = l_run;
        mbar_arrive(&l_bar);
        if (!__all_sync(0xffffffffu, mbar_wait(&l_bar, 0, a.status))) ok = false;
        tc::fence_after_sync();
        const float l_row = red_l[0][r] + red_l[1][r];
        const float inv_l = 1.0f / l_row;
        if constexpr (VERIFY) {
            // the split's (max, sum) of draft row `lane`, head head + quarter
            if (h == 0 && lane < a.t && ok)
                reinterpret_cast<float2 *>(a.part_ml)[((size_t)lane * a.n_head + head + quarter) *
                                                          a.n_splits + split] =
                    make_float2(m_run, l_row);
        } else {
            if (ok && !__all_sync(0xffffffffu, mbar_wait(&g_full, 0, a.status))) ok = false;
        }
        // O / l times the gate (verify: O as it stands) goes through shared
        // memory (the K/V ring, idle now) so that the output stores are whole
        // 128-byte rows per warp: per 32-column chunk, each thread parks its
        // row's values, then each warp walks its 32 rows with lane = column
        const uint32_t oc = tmem + lane_off + O_COL + 128 * h;
        float *stage = reinterpret_cast<float *>(smem + Q_BYTES) + h * (BM * 33);
        // valid rows of this warp
        const int n_rows = VERIFY ? min(32, a.t) : max(0, min(32, a.t - (q0 + quarter * 32)));
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::ld32(oc + c * 32, o);
            tc::wait_ld();
            const int col0 = 128 * h + 32 * c;
            if constexpr (VERIFY) {
#pragma unroll
                for (int e = 0; e < 32; ++e) stage[r * 33 + e] = __uint_as_float(o[e]);
            } else {
                // the row's 32 gate values: 64 bytes of a swizzled 128-byte box row
                const unsigned char *gbox = smem + (col0 >> 6) * Q_BOX;
                uint4 gw[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    gw[k] = *reinterpret_cast<const uint4 *>(gbox +
                                                             swz128(r, ((col0 & 63) >> 3) + k));
                const __nv_bfloat16 *gb = reinterpret_cast<const __nv_bfloat16 *>(gw);
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    stage[r * 33 + e] = __uint_as_float(o[e]) * inv_l * __bfloat162float(gb[e]);
            }
            __syncwarp();
            const int col = col0 + lane;
            if constexpr (VERIFY) {
                const size_t hs = (size_t)(head + quarter) * a.n_splits + split;
                const size_t row_stride = (size_t)a.n_head * a.n_splits * HD;
#pragma unroll 8
                for (int rr = 0; rr < 32; ++rr)
                    if (rr < n_rows && ok)
                        __stcg(a.part_o + rr * row_stride + hs * HD + col,
                               stage[(quarter * 32 + rr) * 33 + lane]);
            } else {
                const size_t row0 = (size_t)(q0 + quarter * 32) * a.n_head + head;
#pragma unroll 8
                for (int rr = 0; rr < 32; ++rr)
                    if (rr < n_rows && ok)
                        __stcs(a.out + (row0 + (size_t)rr * a.n_head) * HD + col,
                               stage[(quarter * 32 + rr) * 33 + lane]);
            }
            __syncwarp();
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
    if (tid == 0 && flag_s) atomicOr(a.status, DEV_TIMEOUT);
}

cudaError_t init_prefill_kernels() {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                pf::SMEM);
}

cudaError_t launch_prefill(const PrefillArgs &a, const CUtensorMap &q_map,
                           const CUtensorMap &kv_map, const CUtensorMap &gate_map,
                           cudaStream_t st) {
    const int n_qt = (a.t + pf::BM - 1) / pf::BM;
    prefill_kernel<false><<<n_qt * a.n_head, pf::THREADS, pf::SMEM, st>>>(a, q_map, kv_map,
                                                                          gate_map);
    return cudaGetLastError();
}

cudaError_t launch_verify_tc(const PrefillArgs &a, const CUtensorMap &vq_map,
                             const CUtensorMap &kv_map, cudaStream_t st) {
    if (a.t < 1 || a.t > kVerifyQBoxRows || a.n_head != 4 * a.n_kv || a.n_splits < 1 ||
        a.split_tiles < 1 || !a.part_o || !a.part_ml)
        return cudaErrorInvalidValue;
    // the gate map is not read in this form
    prefill_kernel<true><<<a.n_splits * a.n_kv, pf::THREADS, pf::SMEM, st>>>(a, vq_map, kv_map,
                                                                             vq_map);
    return cudaGetLastError();
}

}  // namespace rl
