// The chunk scan of the chunked Gated DeltaNet prefill on the fifth-generation
// tensor cores (tcgen05, tensor memory, TMA), sm_100a.
//
// The chunk-local kernel (dn_chunk.cu) leaves, per (value head, chunk of 64
// tokens): W = T diag(beta gamma) K, Ut = T diag(beta) V, Q' = gamma Q,
// K' = gamma_C/gamma K, P = Q K^T o Mgamma and gamma_C.  The scan walks the
// chunks of a head in order (forward.rs:1906-1950 unrolled over a chunk):
//   U_c = Ut_c - W_c S_{c-1}
//   O_c = Q'_c S_{c-1} + P_c U_c               (the chunk's readouts)
//   S_c = gamma_C S_{c-1} + K'_c^T U_c
// It runs them transposed, so that the 128 state columns j are the MMA's 128
// rows (M = 128) and every product is one tcgen05.mma chain:
//   U^T[j][t]  = sum_i S^T[j][i] W[t][i]          (A = S^T, B = W, both K-major)
//   O^T[j][t]  = sum_i S^T[j][i] Q'[t][i] + sum_s U^T[j][s] P[t][s]
//   S^T[j][i] += sum_t U^T[j][t] K'[t][i]         (B = K', N-major)
// The state stays in the compute threads' registers in f32 for the whole scan
// (S_c = gamma_C S_{c-1} + D with D = K'^T U from tensor memory); its bf16
// copy for the next chunk's products goes through shared memory.
//
// Precision (bf16 operands as pairs x = hi + lo where it matters): W S is one
// hi*hi term (the delta rule's feedback corrects it: U = Ut - W S feeds S
// back), O takes the three terms hi*hi + hi*lo + lo*hi of both products, and
// the state update two, U_hi (K'_hi + K'_lo).  A CPU model of these roundings
// against the token-sequential recurrence gave 4e-3 of the per-head output
// at 4096 tokens against 2.7e-3 for f32 products and 1.25e-2 for bf16 pairs
// in Q K^T (the term the chunk-local kernel now takes at 24 bits).
//
// One CTA per value head, fourteen warps:
//   warps 0-7  the compute warps: warp w owns state column j = 32 (w % 4) +
//              lane (tensor-memory lane j) and half w / 4 of every row it
//              touches: U = Ut - acc into shared memory as a bf16 pair; then
//              S_c = gamma_C S_{c-1} + D in registers, and S_c as a bf16 pair
//              for the next products
//   warps 8-11 the readout: O^T from tensor memory to the output rows, off
//              the chain's path (the readout accumulator has NO buffers)
//   warp 12    TMA producer, one lane per operand (W, Q', P, K', each
//              refilled as soon as the MMAs that read it are done), bulk L2
//              prefetches two chunks ahead, and a lane that waits for each
//              chunk's flag and stages its Ut (f32) and gamma_C in shared
//              memory for the compute warps (no global load on the chain)
//   warp 13    tensor-memory owner and MMA issuer (one lane): U, the first
//              readout product while the compute warps convert U (the tensor
//              pipe is otherwise idle then), the state update, the second
//              readout product
// Every wait is bounded; a wait that gives up flags DEV_TIMEOUT and the roles
// wind down (copies and MMAs in flight are waited for before the tensor
// memory and shared memory are released).
#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tc.cuh"

namespace rl {
namespace sc {
constexpr int S = 128, C = 64;
constexpr int THREADS = 448;
constexpr int READOUT_WARP0 = 8, PRODUCER_WARP = 12, MMA_WARP = 13;
constexpr uint32_t BOX64 = 64 * 128;    // 64 rows x 64 bf16 (128-byte rows, swizzled)
constexpr uint32_t BOX128 = 128 * 128;  // 128 rows x 64 bf16
// shared-memory byte offsets from a 1024-byte aligned base
constexpr uint32_t W_OFF = 0;                     // [i box] 64 t x 64 i, hi only
constexpr uint32_t Q_OFF = W_OFF + 2 * BOX64;     // [hi, lo][i box]
constexpr uint32_t P_OFF = Q_OFF + 4 * BOX64;     // [hi, lo] 64 t x 64 s
constexpr uint32_t K_OFF = P_OFF + 2 * BOX64;     // [hi, lo][i box] 64 t x 64 i
constexpr uint32_t UTS_OFF = K_OFF + 4 * BOX64;   // Ut, f32 64 t x 128 j (plain rows)
constexpr uint32_t ST_OFF = UTS_OFF + 4 * BOX64;  // S^T [hi, lo][i box] 128 j x 64 i
constexpr uint32_t UT_OFF = ST_OFF + 4 * BOX128;  // U^T [hi, lo] 128 j x 64 t
constexpr uint32_t SMEM = UT_OFF + 2 * BOX128 + 1024;
constexpr uint32_t TMEM_COLS = 512, S_COL = 0, U_COL = 128, O_COL = 256;  // O: NO x 64
// O accumulator buffers: the readout warps' output stores slow down beside
// the chunk-local kernel's traffic, and the chain's first readout product
// waits for a free buffer, so they get NO - 1 chain steps of slack
constexpr int NO = 4;
constexpr uint32_t W_BYTES = 2 * BOX64, Q_BYTES = 4 * BOX64, P_BYTES = 2 * BOX64,
                   K_BYTES = 4 * BOX64, UT_BYTES = C * S * 4;
}  // namespace sc

// Byte offset of the 16-byte chunk `c` of row `r` in a 128-byte swizzled box.
__device__ __forceinline__ uint32_t sw(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// 32 f32 values of a row as bf16 (hi) or as the low halves x - bf16(x) (lo),
// into 4 consecutive 16-byte chunks c0.. of row r of a swizzled box.
__device__ __forceinline__ void put32(unsigned char *box, int r, int c0, const float *x, bool lo) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a = x[q * 8 + 2 * e], b = x[q * 8 + 2 * e + 1];
            w[e] = lo ? pack_bf16(a - bf16_hi(a), b - bf16_hi(b)) : pack_bf16(a, b);
        }
        *reinterpret_cast<uint4 *>(box + sw(r, c0 + q)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ void as_f32(const uint32_t (&r)[32], float *x) {
#pragma unroll
    for (int e = 0; e < 32; ++e) x[e] = __uint_as_float(r[e]);
}

__global__ void __launch_bounds__(sc::THREADS, 1)
    dn_scan_tc_kernel(const __grid_constant__ DnChunkArgs a, const __grid_constant__ DnScanMaps m) {
    using namespace sc;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t w_full, w_empty, q_full, q_empty, p_full, p_empty,
        k_full, k_empty, ut_full, ut_empty, s_ready, u_done, u_ready, s_done, o_full[NO], o_empty[NO],
        fin;
    __shared__ float gc_s;  // gamma_C of the chunk whose Ut is staged
    __shared__ uint32_t tmem_base;
    __shared__ int flag_s;
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sbase = smem_u32(smem);
    const int vh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nc = a.nc;
    const size_t blk0 = (size_t)vh * nc;
    float *state = a.ssm_state + (size_t)vh * a.slots * S * S + (size_t)a.live * S * S;
    // beside the chunk-local kernel: chunk c of this head may be read once
    // ready[vh * nc + c] holds this value
    const int ready_value = a.ready ? a.ready_epoch[vh] + 1 : 0;
    auto chunk_ready = [&](int c) {
        if (!a.ready) return true;
        const bool ok = wait_flag_gpu(a.ready + blk0 + c, ready_value, a.status);
        // the tensor copies that follow read what the flag published
        asm volatile("fence.proxy.async.global;" ::: "memory");
        return ok;
    };

    if (tid == 0) {
        for (int b = 0; b < NO; ++b) {
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], 128);
        }
        mbar_init(&k_full, 1);
        mbar_init(&k_empty, 1);
        mbar_init(&ut_full, 1);
        mbar_init(&ut_empty, 8);
        mbar_init(&w_full, 1);
        mbar_init(&w_empty, 1);
        mbar_init(&q_full, 1);
        mbar_init(&q_empty, 1);
        mbar_init(&p_full, 1);
        mbar_init(&p_empty, 1);
        mbar_init(&s_ready, 256);
        mbar_init(&u_done, 1);
        mbar_init(&u_ready, 256);
        mbar_init(&s_done, 1);
        mbar_init(&fin, 1);
        flag_s = 0;
        fence_barrier_init();
    }
    if (warp == MMA_WARP) {
        tc::tmem_alloc(&tmem_base, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;

    if (warp == PRODUCER_WARP) {
        // ---------------- TMA producer: lane 0 W (and, after the chunk-local
        // kernel, the L2 prefetch of the chunk after next), 1 Q', 2 P, 3 K',
        // 4 Ut (a bulk copy) and gamma_C for the compute warps.  Each lane
        // waits only on the barrier that gates its own refill, so none can
        // fall two phases behind one. ----------------
        if (lane < 5) {
            const int role = lane;
            if (role == 0) {
                prefetch_tensormap(&m.w);
            } else if (role == 1) {
                prefetch_tensormap(&m.qh);
                prefetch_tensormap(&m.ql);
            } else if (role == 2) {
                prefetch_tensormap(&m.ph);
                prefetch_tensormap(&m.pl);
            } else if (role == 3) {
                prefetch_tensormap(&m.kh);
                prefetch_tensormap(&m.kl);
            }
            int c = 0;
            for (; c < nc; ++c) {
                const int row = (int)(blk0 + c) * C;
                if (!chunk_ready(c)) break;
                if (role == 0) {
                    if (c >= 1 && !mbar_wait(&w_empty, (c - 1) & 1, a.status)) break;
                    mbar_arrive_expect_tx(&w_full, W_BYTES);
                    for (int x = 0; x < 2; ++x)
                        tma_load_2d(smem + W_OFF + x * BOX64, &m.w, 64 * x, row, &w_full);
                    // after the chunk-local kernel the chunk after next into L2,
                    // paced by this chunk's W (beside it the chunks are fresh
                    // in L2 when their flags go up)
                    const int cn = c + 2;
                    if (!a.ready && cn < nc) {
                        const size_t bo = (blk0 + cn) * C;
                        prefetch_l2_bulk(a.w + bo * S, C * S * 2);
                        prefetch_l2_bulk(a.qp + bo * S, C * S * 2);
                        prefetch_l2_bulk(a.qp_lo + bo * S, C * S * 2);
                        prefetch_l2_bulk(a.kp + bo * S, C * S * 2);
                        prefetch_l2_bulk(a.kp_lo + bo * S, C * S * 2);
                        prefetch_l2_bulk(a.p + bo * C, C * C * 2);
                        prefetch_l2_bulk(a.p_lo + bo * C, C * C * 2);
                        prefetch_l2_bulk(a.ut + bo * S, C * S * 4);
                    }
                } else if (role == 1) {
                    if (c >= 1 && !mbar_wait(&q_empty, (c - 1) & 1, a.status)) break;
                    mbar_arrive_expect_tx(&q_full, Q_BYTES);
                    for (int x = 0; x < 2; ++x) {
                        tma_load_2d(smem + Q_OFF + x * BOX64, &m.qh, 64 * x, row, &q_full);
                        tma_load_2d(smem + Q_OFF + (2 + x) * BOX64, &m.ql, 64 * x, row, &q_full);
                    }
                } else if (role == 2) {
                    if (c >= 1 && !mbar_wait(&p_empty, (c - 1) & 1, a.status)) break;
                    mbar_arrive_expect_tx(&p_full, P_BYTES);
                    tma_load_2d(smem + P_OFF, &m.ph, 0, row, &p_full);
                    tma_load_2d(smem + P_OFF + BOX64, &m.pl, 0, row, &p_full);
                } else if (role == 3) {
                    // one buffer: the next K' has a whole chain step to land
                    if (c >= 1 && !mbar_wait(&k_empty, (c - 1) & 1, a.status)) break;
                    mbar_arrive_expect_tx(&k_full, K_BYTES);
                    unsigned char *kd = smem + K_OFF;
                    for (int x = 0; x < 2; ++x) {
                        tma_load_2d(kd + x * BOX64, &m.kh, 64 * x, row, &k_full);
                        tma_load_2d(kd + (2 + x) * BOX64, &m.kl, 64 * x, row, &k_full);
                    }
                } else {
                    // the compute warps read this chunk's Ut and gamma_C from
                    // shared memory once they have converted the previous U
                    if (c >= 1 && !mbar_wait(&ut_empty, (c - 1) & 1, a.status)) break;
                    gc_s = a.gc[blk0 + c];
                    mbar_arrive_expect_tx(&ut_full, UT_BYTES);
                    bulk_g2s(smem + UTS_OFF, a.ut + (blk0 + c) * C * S, UT_BYTES, &ut_full);
                }
            }
            if (c < nc) flag_s = 1;
            // every copy this lane started lands before the shared memory is
            // released (bounded: a consumer that gave up leaves a buffer full)
            const int last = min(c, nc - 1);
            if (last >= 0) {
                if (role == 0) mbar_wait(&w_full, last & 1, a.status);
                if (role == 1) mbar_wait(&q_full, last & 1, a.status);
                if (role == 2) mbar_wait(&p_full, last & 1, a.status);
                if (role == 3) mbar_wait(&k_full, last & 1, a.status);
                if (role == 4) mbar_wait(&ut_full, last & 1, a.status);
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issuer: U; the first readout while U is
        // converted; the state update; the second readout ----------------
        if (lane == 0) {
            constexpr uint32_t id_n64 = tc::idesc_bf16(128, 64, false);
            constexpr uint32_t id_s = tc::idesc_bf16(128, 128, true);
            // descriptors of the operands' first 16-wide step; a step is +32 B
            // (+2 in the descriptor) inside a box, a box +BOX64 or +BOX128
            const uint64_t st_hi = tc::smem_desc(sbase + ST_OFF, 16, 1024);
            const uint64_t st_lo = tc::smem_desc(sbase + ST_OFF + 2 * BOX128, 16, 1024);
            const uint64_t ut_hi = tc::smem_desc(sbase + UT_OFF, 16, 1024);
            const uint64_t ut_lo = tc::smem_desc(sbase + UT_OFF + BOX128, 16, 1024);
            const uint64_t w_hi = tc::smem_desc(sbase + W_OFF, 16, 1024);
            const uint64_t q_hi = tc::smem_desc(sbase + Q_OFF, 16, 1024);
            const uint64_t q_lo = tc::smem_desc(sbase + Q_OFF + 2 * BOX64, 16, 1024);
            const uint64_t p_hi = tc::smem_desc(sbase + P_OFF, 16, 1024);
            const uint64_t p_lo = tc::smem_desc(sbase + P_OFF + BOX64, 16, 1024);
            // K' is N-major: a 16-row step is +2 KiB; its two 64-column boxes
            // are BOX64 apart (the leading byte offset)
            const uint64_t k_d[2] = {tc::smem_desc(sbase + K_OFF, BOX64, 1024),
                                     tc::smem_desc(sbase + K_OFF + 2 * BOX64, BOX64, 1024)};
            auto kstep = [](int kk, uint32_t box) -> uint64_t {
                return (uint64_t)(((kk >> 2) * box + (kk & 3) * 32) >> 4);
            };
            bool ok = true;
            for (int c = 0; c < nc && ok; ++c) {
                const int b = c % NO;
                const uint32_t o_acc = tmem + O_COL + b * 64;
                // U^T = S^T_hi W_hi (K = 128: two boxes of four 16-wide steps)
                ok = mbar_wait(&s_ready, c & 1, a.status) && mbar_wait(&w_full, c & 1, a.status);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    tc::mma_ss(tmem + U_COL, st_hi + kstep(kk, BOX128), w_hi + kstep(kk, BOX64),
                               id_n64, kk > 0);
                tc::commit(&u_done);
                tc::commit(&w_empty);
                // O^T = S^T Q'^T (three terms), in the tensor pipe's idle time
                // while the compute warps convert U
                ok = (c < NO || mbar_wait(&o_empty[b], ((c / NO) - 1) & 1, a.status)) &&
                     mbar_wait(&q_full, c & 1, a.status);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int term = 0; term < 3; ++term) {
                    const uint64_t sa = term == 2 ? st_lo : st_hi;
                    const uint64_t qb = term == 1 ? q_lo : q_hi;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        tc::mma_ss(o_acc, sa + kstep(kk, BOX128), qb + kstep(kk, BOX64), id_n64,
                                   term > 0 || kk > 0);
                }
                tc::commit(&q_empty);
                // the state update's product as soon as U is in shared memory:
                // D = U^T_hi (K'_hi + K'_lo) (the compute warps add gamma_C S);
                // its completion also covers everything above, so S^T's
                // shared copy is free then
                ok = mbar_wait(&u_ready, c & 1, a.status) &&
                     mbar_wait(&k_full, c & 1, a.status);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int term = 0; term < 2; ++term)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc::mma_ss(tmem + S_COL, ut_hi + kk * 2, k_d[term] + kk * 128, id_s,
                                   term > 0 || kk > 0);
                tc::commit(&k_empty);
                tc::commit(&s_done);
                // O^T += U^T P^T, three terms
                ok = mbar_wait(&p_full, c & 1, a.status);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int term = 0; term < 3; ++term) {
                    const uint64_t ua = term == 2 ? ut_lo : ut_hi;
                    const uint64_t pb = term == 1 ? p_lo : p_hi;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc::mma_ss(o_acc, ua + kk * 2, pb + kk * 2, id_n64, true);
                }
                tc::commit(&p_empty);
                tc::commit(&o_full[b]);
            }
            if (!ok) flag_s = 1;
            // every MMA issued is complete before the tensor memory is freed
            tc::commit(&fin);
            mbar_wait(&fin, 0, a.status);
        }
    } else if (warp < READOUT_WARP0) {
        // ---------------- the compute warps: warp w owns state column
        // j = 32 (w % 4) + lane (tensor-memory lane j) and the half w / 4 of
        // each row it converts or reads out ----------------
        const int q4 = warp & 3, hf = warp >> 2, j = q4 * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
        unsigned char *st_hi = smem + ST_OFF + hf * BOX128, *st_lo = st_hi + 2 * BOX128;
        unsigned char *ut_hi = smem + UT_OFF, *ut_lo = smem + UT_OFF + BOX128;
        bool ok = true;
        // the state in registers, f32: this thread's 64 values S[i][j] of its
        // half; S_{-1} from the slot, its bf16 pair for the first products
        float sv[64];
#pragma unroll
        for (int e = 0; e < 64; ++e) sv[e] = state[(size_t)(hf * 64 + e) * S + j];
        put32(st_hi, j, 0, sv, false);
        put32(st_lo, j, 0, sv, true);
        put32(st_hi, j, 4, sv + 32, false);
        put32(st_lo, j, 4, sv + 32, true);
        fence_proxy_async_smem();
        tc::fence_before_sync();
        mbar_arrive(&s_ready);
        const float *uts = reinterpret_cast<const float *>(smem + UTS_OFF) + (hf * 32) * S + j;
        for (int c = 0; c < nc && ok; ++c) {
            // ---- U = Ut - S W for this warp's 32 tokens, into shared memory
            // as a bf16 pair (Ut's column j, staged by the producer, is read
            // while the MMAs run)
            if (!(ok = mbar_wait(&ut_full, c & 1, a.status))) break;
            float x[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) x[e] = uts[e * S];
            const float gc = gc_s;
            __syncwarp();
            if (lane == 0) mbar_arrive(&ut_empty);
            ok = mbar_wait(&u_done, c & 1, a.status);
            if (!ok) break;
            tc::fence_after_sync();
            {
                uint32_t r[32];
                tc::ld32(tmem + lane_addr + U_COL + hf * 32, r);
                tc::wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) x[e] -= __uint_as_float(r[e]);
                put32(ut_hi, j, hf * 4, x, false);
                put32(ut_lo, j, hf * 4, x, true);
            }
            fence_proxy_async_smem();
            tc::fence_before_sync();
            mbar_arrive(&u_ready);
            // ---- S_c = gamma_C S_{c-1} + D, D = K'^T U from tensor memory; its
            // pair for the next chunk, or the state after the last chunk
            ok = mbar_wait(&s_done, c & 1, a.status);
            if (!ok) break;
            tc::fence_after_sync();
            {
                uint32_t r0[32], r1[32];
                tc::ld32(tmem + lane_addr + S_COL + hf * 64, r0);
                tc::ld32(tmem + lane_addr + S_COL + hf * 64 + 32, r1);
                tc::wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    sv[e] = fmaf(gc, sv[e], __uint_as_float(r0[e]));
                    sv[32 + e] = fmaf(gc, sv[32 + e], __uint_as_float(r1[e]));
                }
            }
            tc::fence_before_sync();  // D is read: the next update may overwrite it
            if (c + 1 < nc) {
                put32(st_hi, j, 0, sv, false);
                put32(st_lo, j, 0, sv, true);
                put32(st_hi, j, 4, sv + 32, false);
                put32(st_lo, j, 4, sv + 32, true);
                fence_proxy_async_smem();
                mbar_arrive(&s_ready);
            } else {
#pragma unroll
                for (int e = 0; e < 64; ++e) state[(size_t)(hf * 64 + e) * S + j] = sv[e];
            }
        }
        if (!ok) flag_s = 1;
    } else {
        // ---------------- the readout warps: O^T rows to the output, a
        // chunk behind the chain; warp 8 + q owns state columns 32q .. ----------------
        const int q4 = warp - READOUT_WARP0, j = q4 * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
        const float scale = 1.0f / sqrtf((float)S);
        for (int c = 0; c < nc; ++c) {
            const int b = c % NO;
            if (!mbar_wait(&o_full[b], (c / NO) & 1, a.status)) {
                flag_s = 1;
                break;
            }
            tc::fence_after_sync();
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                uint32_t r[32];
                tc::ld32(tmem + lane_addr + O_COL + b * 64 + h * 32, r);
                tc::wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int tok = c * C + h * 32 + e;
                    if (tok < a.t)
                        a.opre[((size_t)tok * a.n_v + vh) * S + j] = __uint_as_float(r[e]) * scale;
                }
            }
            tc::fence_before_sync();
            mbar_arrive(&o_empty[b]);
            if (a.out_ready) {
                // this warp's rows of the chunk are stored: each of the four
                // readout warps adds 1 with release semantics (cumulative over
                // the lanes' stores, which the warp barrier orders first)
                __syncwarp();
                if (lane == 0) red_release_add_gpu(a.out_ready + (size_t)vh * a.nc + c, 1);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0 && flag_s) atomicOr(a.status, DEV_TIMEOUT);
    // every chunk of this call is consumed: the next call's flags take the
    // next value
    if (tid == 0 && a.ready) a.ready_epoch[vh] = ready_value;
    if (warp == MMA_WARP) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

cudaError_t init_dn_scan_tc_kernel() {
    return cudaFuncSetAttribute(dn_scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sc::SMEM);
}

cudaError_t launch_dn_scan_tc(const DnChunkArgs &a, const DnScanMaps &m, cudaStream_t st) {
    dn_scan_tc_kernel<<<a.n_v, sc::THREADS, sc::SMEM, st>>>(a, m);
    return cudaGetLastError();
}

}  // namespace rl
