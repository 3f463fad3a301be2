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
//               S_j = Q K_j^T for a tile of 128 keys (two halves of M 128,
//               N 64, K 256 from two ring stages: 32 MMAs) into one of two
//               S buffers, then O += P_{j-1} V_{j-1} (M 128, N 256, K 128: 8
//               MMAs) with P read from tensor memory, so the next tile's
//               Q K^T runs while the softmax works on this one
//   warps 2-9   softmax and epilogue, two threads per query row (each half
//               of the tile's 128 keys and of O): S from tensor memory, causal
//               mask on the diagonal tiles, the row max exchanged through
//               shared memory, online softmax in log2 units with a lazy
//               rescale (O is corrected only when a row's max grows by more
//               than 2^12), P written back as bf16 over the S buffer; at the
//               end O / l times the sigmoid output gate (staged in bf16 by
//               the prologue, loaded by TMA over the query tile once the last
//               Q K^T is done), to global memory in whole 128-byte rows
// Tensor memory (512 columns): O in columns 0-255, S buffers of 128 columns
// at 256 and 384; P_j aliases the first 64 columns of its S buffer.  (The
// verify form keeps 64-key tiles: S buffers at 256 and 320, Q at 384.)  MMAs of one thread run
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
// verify form: the queries live in tensor memory, so the ring takes a third
// K/V stage instead
constexpr int QSTAGE = 3 * STAGE;               // verify: 4 x 8 query rows of 512 B
constexpr int SMEM_VERIFY = QSTAGE + 32 * 512 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 0, S_COL = 256;
constexpr uint32_t Q_COL = 384;  // verify: Q, bf16 pairs, 128 columns
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 12.0f;  // P up to 2^12: no range issue in bf16 or f32
}  // namespace pf

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// A 16-byte global load issued where it stands: volatile asm keeps a batch of
// them in program order ahead of the code that consumes them.
__device__ __forceinline__ float4 ld_nc_f4(const float *p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
// Shared -> global bulk copy (16-byte aligned addresses, size a multiple of
// 16) in the calling thread's bulk group.
__device__ __forceinline__ void bulk_store(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_and_wait() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
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
    // ring of NST K/V stages of BN keys (verify: 3, the queries sit in tensor
    // memory); the softmax works on tiles of KT keys, RT ring stages each
    constexpr int NST = VERIFY ? 3 : 2;
    constexpr int KT = VERIFY ? BN : 2 * BN, RT = KT / BN, HALF = KT / 2;
    constexpr int RING = VERIFY ? 0 : Q_BYTES;  // byte offset of the ring
    __shared__ __align__(8) uint64_t q_full, k_full[NST], v_full[NST], k_empty[NST],
        v_empty[NST], s_full[2], p_full[2], o_ready, o_final, g_full, kv_app, q_iss;
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
        n_kt = (a.pos + q_last) / KT + 1;           // key tiles the tile needs
    }
    const uint32_t sbase = smem_u32(smem);

    if (tid == 0) {
        // verify: the eight softmax warps write the queries and arrive
        mbar_init(&q_full, VERIFY ? 8 : 1);
        for (int s = 0; s < NST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 8);
        }
        mbar_init(&o_ready, 1);
        mbar_init(&o_final, 1);
        mbar_init(&g_full, 1);
        mbar_init(&kv_app, 8);
        mbar_init(&q_iss, 8);
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
    // both forms are launched as programmatic dependents, so the set-up
    // above overlaps the grid ahead (prefill: the prologue, whose blocks let
    // it launch at their start); nothing is read before that grid completes
    grid_dep_wait();
    // verify: this CTA's key range holds positions of the appended rows
    const bool appends = VERIFY && (j0 + n_kt) * KT > a.pos;

    if (warp == 0 || warp == 10) {
        // ---------------- TMA producers ----------------
        // warp 0: the query tile, then K tiles (a slot frees when its Q K^T is
        // done); warp 10: V tiles (a slot frees when its P V is done).  Two
        // warps, so K runs ahead of V by as much as the slots allow.
        if (lane == 0) {
            const bool is_k = warp == 0;
            prefetch_tensormap(&kv_map);
            if (is_k && !VERIFY) {
                prefetch_tensormap(&q_map);
                mbar_arrive_expect_tx(&q_full, Q_BYTES);
                for (int b = 0; b < 4; ++b)
                    tma_load_3d(smem + b * Q_BOX, &q_map, b * 64, head, q0, &q_full);
            }
            const int row0 = (is_k ? a.k_row0 : a.v_row0) + kh * a.context;
            uint64_t *full = is_k ? k_full : v_full, *empty = is_k ? k_empty : v_empty;
            int issued = 0;
            bool appended_visible = !appends;
            // verify: the query loads go out ahead of the tile stream (they
            // would queue behind every CTA's first burst of copies)
            if (VERIFY && !mbar_wait(&q_iss, 0, a.status)) flag_s = 1;
            const int n_rt = n_kt * RT;  // ring stages the CTA streams
            for (int u = 0; u < n_rt; ++u) {
                const int s = u % NST;
                if (u >= NST && !mbar_wait(&empty[s], (u / NST - 1) & 1, a.status)) {
                    flag_s = 1;
                    break;
                }
                if (!appended_visible && (j0 * RT + u + 1) * BN > a.pos) {
                    // this tile holds appended rows: the softmax warps have
                    // written them to the cache
                    if (!mbar_wait(&kv_app, 0, a.status)) {
                        flag_s = 1;
                        break;
                    }
                    appended_visible = true;
                }
                // K: box b of stage s at b * NST + s (the stages of a box are
                // adjacent rows); V: stage s's four boxes together
                mbar_arrive_expect_tx(&full[s], KV_HALF);
                for (int b = 0; b < 4; ++b) {
                    unsigned char *dst = is_k ? smem + RING + (b * NST + s) * KV_BOX
                                              : smem + RING + NST * KV_HALF + s * KV_HALF +
                                                    b * KV_BOX;
                    tma_load_2d(dst, &kv_map, b * 64, row0 + (j0 * RT + u) * BN, &full[s]);
                }
                issued = u + 1;
            }
            if (!VERIFY && is_k && issued == n_rt) {
                // the last Q K^T done, the query tile is free: the output gate
                // (sigmoid, bf16, staged by the prologue) takes its place
                const int ul = n_rt - 1;
                if (mbar_wait(&k_empty[ul % NST], (ul / NST) & 1, a.status)) {
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
            if (is_k && !VERIFY) mbar_wait(&q_full, 0, a.status);
            for (int u = max(0, issued - NST); u < issued; ++u)
                mbar_wait(&full[u % NST], (u / NST) & 1, a.status);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t id_qk = tc::idesc_bf16(BM, RT == NST ? KT : BN, false);
            constexpr uint32_t id_pv = tc::idesc_bf16(BM, HD, true);
            bool ok = mbar_wait(&q_full, 0, a.status);
            tc::fence_after_sync();
            for (int j = 0; ok && j <= n_kt; ++j) {
                if (j < n_kt) {
                    const int sb = j & 1;  // S buffer
                    for (int r = 0; r < RT; ++r) {
                        const int u = j * RT + r;
                        if (!mbar_wait(&k_full[u % NST], (u / NST) & 1, a.status)) ok = false;
                    }
                    if (!ok) break;
                    tc::fence_after_sync();
                    // a tile spanning every stage (RT == NST) is one operand of
                    // KT rows: its stages are adjacent within each box
                    constexpr int NQ = RT == NST ? 1 : RT;  // Q K^T issues per tile
#pragma unroll
                    for (int r = 0; r < NQ; ++r) {
                        // keys r*BN.. of the tile from their ring stage, into
                        // columns r*BN.. of the S buffer
                        const int s = RT == NST ? 0 : (j * RT + r) % NST;
                        const uint32_t kst = sbase + RING + s * KV_BOX;
                        const uint32_t d = tmem + S_COL + sb * KT + r * BN;
#pragma unroll
                        for (int kk = 0; kk < HD / 16; ++kk) {
                            const uint32_t off = (kk & 3) * 32;  // 16 dims inside a 64-dim box
                            const uint64_t db = tc::smem_desc(
                                kst + (kk >> 2) * NST * KV_BOX + off, 16, 1024);
                            if constexpr (VERIFY) {
                                // A = Q from tensor memory: 16 dims are 8 columns
                                tc::mma_ts(d, tmem + Q_COL + kk * 8, db, id_qk, kk > 0);
                            } else {
                                const uint64_t da =
                                    tc::smem_desc(sbase + (kk >> 2) * Q_BOX + off, 16, 1024);
                                tc::mma_ss(d, da, db, id_qk, kk > 0);
                            }
                        }
                    }
                    tc::commit(&s_full[sb]);
#pragma unroll
                    for (int r = 0; r < RT; ++r) tc::commit(&k_empty[(j * RT + r) % NST]);
                }
                if (j >= 1) {
                    const int jj = j - 1, sb = jj & 1;
                    if (!mbar_wait(&p_full[sb], (jj >> 1) & 1, a.status)) { ok = false; break; }
                    for (int r = 0; r < RT; ++r) {
                        const int u = jj * RT + r;
                        if (!mbar_wait(&v_full[u % NST], (u / NST) & 1, a.status)) ok = false;
                    }
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t p = tmem + S_COL + sb * KT;
#pragma unroll
                    for (int kk = 0; kk < KT / 16; ++kk) {
                        // 16 keys: ring stage of the tile's part kk / (BN / 16)
                        const int s = (jj * RT + kk / (BN / 16)) % NST;
                        const uint32_t vst = sbase + RING + NST * KV_HALF + s * KV_HALF;
                        const uint64_t db =
                            tc::smem_desc(vst + (kk % (BN / 16)) * 16 * 128, KV_BOX, 1024);
                        tc::mma_ts(tmem + O_COL, p + kk * 8, db, id_pv, jj > 0 || kk > 0);
                    }
#pragma unroll
                    for (int r = 0; r < RT; ++r) tc::commit(&v_empty[(jj * RT + r) % NST]);
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
        const int first_masked = (a.pos + q0) / KT;  // earliest tile a row of the CTA masks
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        if constexpr (VERIFY) {
            // ---- the query rows, straight from the raw f32 input: per-head
            // RMSNorm (f32 squares summed in f64, forward.rs:1697-1711) and
            // RoPE on the first 64 dims with the context's angle table
            // (:1851-1862), as bf16 pairs into tensor memory.  The 256
            // softmax threads each take 32 dims of one (head, row) of the
            // group's 4 heads x 8 rows, with all their loads in flight at
            // once (the eight threads of a row meet by shuffles: the sum of
            // squares, and dims d, d + 32 for the rotation), park the result
            // in shared memory, and each row's owner moves its 64 columns to
            // tensor memory; rows past t are zeros.
            uint32_t *qstage = reinterpret_cast<uint32_t *>(smem + QSTAGE);
            // lane l of a row's eight threads holds dims 4l + 32j + e (j < 8,
            // e < 4): each load instruction reads whole 128-byte segments,
            // and the rotation pairs (d, d + 32) sit in one thread
            const int ts = tid - 64, l8 = ts & 7, rv = ts >> 3;  // lane in row, row slot
            const int g = rv >> 3;                                  // head in the group
            {
                const int i = rv & 7;
                const bool real = i < a.t;
                const float *src =
                    a.qg + ((size_t)(real ? i : 0) * a.n_head + head + g) * 2 * HD + 4 * l8;
                const float *wq = a.q_norm + 4 * l8;
                const int pr = real ? a.pos + i : a.pos;
                float x[32], w[32];
                // every load of the phase in one batch (rows past t read row
                // 0 and are zeroed after)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 xv = ld_nc_f4(src + 32 * j), wv = ld_nc_f4(wq + 32 * j);
                    x[4 * j] = xv.x, x[4 * j + 1] = xv.y, x[4 * j + 2] = xv.z, x[4 * j + 3] = xv.w;
                    w[4 * j] = wv.x, w[4 * j + 1] = wv.y, w[4 * j + 2] = wv.z, w[4 * j + 3] = wv.w;
                }
                const float4 cv = ld_nc_f4(a.rope_cs + (size_t)pr * 32 + 4 * l8);
                const float4 sv = ld_nc_f4(a.rope_sn + (size_t)pr * 32 + 4 * l8);
                // issued, not yet arrived: the tile stream may start
                __syncwarp();
                if (lane == 0)
                    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(
                                     smem_u32(&q_iss))
                                 : "memory");
                if (!real) {
#pragma unroll
                    for (int k = 0; k < 32; ++k) x[k] = 0.0f;
                }
                double sq = 0.0;
#pragma unroll
                for (int k = 0; k < 32; ++k) sq += (double)__fmul_rn(x[k], x[k]);
                sq += __shfl_xor_sync(0xffffffffu, sq, 1);
                sq += __shfl_xor_sync(0xffffffffu, sq, 2);
                sq += __shfl_xor_sync(0xffffffffu, sq, 4);
                const float qs = rms_scale_from_sum(sq, HD, a.eps);
#pragma unroll
                for (int k = 0; k < 32; ++k) x[k] = __fmul_rn(__fmul_rn(x[k], qs), w[k]);
                // dims 4l + e (x[e]) rotate with 4l + 32 + e (x[4 + e])
                const float c4[4] = {cv.x, cv.y, cv.z, cv.w}, s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float lo = x[e], hi = x[4 + e];
                    x[e] = __fsub_rn(__fmul_rn(lo, c4[e]), __fmul_rn(hi, s4[e]));
                    x[4 + e] = __fadd_rn(__fmul_rn(lo, s4[e]), __fmul_rn(hi, c4[e]));
                }
                // bf16 pairs: dims 4l + 32j + {0,1}, {2,3} are the row's
                // columns 16j + 2l, 16j + 2l + 1
                uint32_t *dst = qstage + rv * 128 + 2 * l8;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    __nv_bfloat162 b0 = __floats2bfloat162_rn(x[4 * j], x[4 * j + 1]);
                    __nv_bfloat162 b1 = __floats2bfloat162_rn(x[4 * j + 2], x[4 * j + 3]);
                    *reinterpret_cast<uint2 *>(dst + 16 * j) =
                        make_uint2(*reinterpret_cast<uint32_t *>(&b0),
                                   *reinterpret_cast<uint32_t *>(&b1));
                }
            }
            named_sync(1, 256);
            // the owner of tile row (head quarter, draft row lane) moves it
            const uint32_t qcol = tmem + lane_off + Q_COL + 64 * h;
            const uint32_t *row = qstage + (quarter * 8 + (lane & 7)) * 128 + 64 * h;
#pragma unroll
            for (int half32 = 0; half32 < 2; ++half32) {
                uint32_t qreg[32];
#pragma unroll
                for (int k = 0; k < 32; k += 4) {
                    const uint4 u = lane < a.t
                                        ? *reinterpret_cast<const uint4 *>(row + 32 * half32 + k)
                                        : make_uint4(0u, 0u, 0u, 0u);
                    qreg[k] = u.x, qreg[k + 1] = u.y, qreg[k + 2] = u.z, qreg[k + 3] = u.w;
                }
                tc::st32(qcol + 32 * half32, qreg);
            }
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_full);
            if (appends) {
                // ---- the rows' keys and values (forward.rs:1262-1292): one
                // warp per appended row in this CTA's key range, 8 dims a
                // lane; the key gets the RMSNorm and RoPE of the queries,
                // both go to the cache in bf16
                const int i = warp - 2, p = a.pos + i;
                if (i < a.t && p >= j0 * BN && p < (j0 + n_kt) * BN) {
                    const float *kr = a.k_in + ((size_t)i * a.n_kv + kh) * HD + lane * 8;
                    const float *vr = a.v_in + ((size_t)i * a.n_kv + kh) * HD + lane * 8;
                    const float4 k0 = ld_nc_f4(kr), k1 = ld_nc_f4(kr + 4);
                    const float4 v0 = ld_nc_f4(vr), v1 = ld_nc_f4(vr + 4);
                    const float4 w0 = ld_nc_f4(a.k_norm + lane * 8), w1 = ld_nc_f4(a.k_norm + lane * 8 + 4);
                    const int pr = (lane * 8) & 31;  // RoPE pair index of the first dim (lanes 0-7)
                    const float *cs = a.rope_cs + (size_t)p * 32 + pr, *sn = a.rope_sn + (size_t)p * 32 + pr;
                    const float4 c0 = ld_nc_f4(cs), c1 = ld_nc_f4(cs + 4);
                    const float4 s0 = ld_nc_f4(sn), s1 = ld_nc_f4(sn + 4);
                    const float kx[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
                    const float wx[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    const float cx[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                    const float sx[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                    double sq = 0.0;
#pragma unroll
                    for (int e = 0; e < 8; ++e) sq += (double)__fmul_rn(kx[e], kx[e]);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                    const float ks = rms_scale_from_sum(sq, HD, a.eps);
                    float y[8], rk[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = __fmul_rn(__fmul_rn(kx[e], ks), wx[e]);
                    // dims d < 32 (lanes 0-3) rotate with d + 32 (lanes 4-7)
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float up = __shfl_down_sync(0xffffffffu, y[e], 4);
                        const float dn = __shfl_up_sync(0xffffffffu, y[e], 4);
                        rk[e] = y[e];
                        if (lane < 4)
                            rk[e] = __fsub_rn(__fmul_rn(y[e], cx[e]), __fmul_rn(up, sx[e]));
                        else if (lane < 8)
                            rk[e] = __fadd_rn(__fmul_rn(dn, sx[e]), __fmul_rn(y[e], cx[e]));
                    }
                    const float vx[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                    uint4 ku, vu;
                    uint32_t *kp = &ku.x, *vp = &vu.x;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        __nv_bfloat162 kb = __floats2bfloat162_rn(rk[2 * e], rk[2 * e + 1]);
                        __nv_bfloat162 vb = __floats2bfloat162_rn(vx[2 * e], vx[2 * e + 1]);
                        kp[e] = *reinterpret_cast<uint32_t *>(&kb);
                        vp[e] = *reinterpret_cast<uint32_t *>(&vb);
                    }
                    const size_t row = ((size_t)kh * a.context + p) * HD + lane * 8;
                    *reinterpret_cast<uint4 *>(a.k_cache + row) = ku;
                    *reinterpret_cast<uint4 *>(a.v_cache + row) = vu;
                    // the tensor-copy loads of this CTA read the rows next
                    __threadfence();
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&kv_app);
            }
        }
        for (int j = 0; j < n_kt; ++j) {
            const int s = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[s], (j >> 1) & 1, a.status))) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t sc = tmem + lane_off + S_COL + s * KT;
            // this thread's HALF keys of the tile, in chunks of 32
            uint32_t u[RT][32];
#pragma unroll
            for (int q = 0; q < RT; ++q) tc::ld32(sc + HALF * h + 32 * q, u[q]);
            tc::wait_ld();
            const int kv0 = (j0 + j) * KT + HALF * h;
            if (j0 + j >= first_masked) {
#pragma unroll
                for (int q = 0; q < RT; ++q)
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        if (kv0 + 32 * q + c > qa) u[q][c] = __float_as_uint(-INFINITY);
            }
            float mx0 = __uint_as_float(u[0][0]), mx1 = __uint_as_float(u[0][1]);
#pragma unroll
            for (int q = 0; q < RT; ++q)
#pragma unroll
                for (int c = (q == 0 ? 2 : 0); c < 32; c += 2) {
                    mx0 = fmaxf(mx0, __uint_as_float(u[q][c]));
                    mx1 = fmaxf(mx1, __uint_as_float(u[q][c + 1]));
                }
            // the row's max over both halves (scores scale by a positive
            // constant): post this half's, then compute P optimistically with
            // the running max while the partner's arrives; only a row whose
            // max grows past the lazy threshold (rare) redoes the exponentials
            red_m[j & 1][h][r] = fmaxf(mx0, mx1);
            mbar_arrive(&mx_bar[j & 1]);
            uint32_t pk[RT][16];
            float ps0 = 0.0f, ps1 = 0.0f;
            auto exps = [&](float m) {
                ps0 = 0.0f;
                ps1 = 0.0f;
                // a row with every key so far masked (a verify split past
                // the row) has m = -inf: its P is 0, not NaN
                const float neg_m = m == -INFINITY ? 0.0f : -m;
#pragma unroll
                for (int q = 0; q < RT; ++q)
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const float p0 =
                            ex2_approx(fmaf(__uint_as_float(u[q][2 * c]), scale, neg_m));
                        const float p1 =
                            ex2_approx(fmaf(__uint_as_float(u[q][2 * c + 1]), scale, neg_m));
                        ps0 += p0;
                        ps1 += p1;
                        __nv_bfloat162 hh = __floats2bfloat162_rn(p0, p1);
                        pk[q][c] = *reinterpret_cast<uint32_t *>(&hh);
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
            // P (bf16 pairs) over the first KT / 2 columns of the S buffer
#pragma unroll
            for (int q = 0; q < RT; ++q) tc::st16(sc + (HALF / 2) * h + 16 * q, pk[q]);
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
        const uint32_t oc = tmem + lane_off + O_COL + 128 * h;
        if constexpr (VERIFY) {
            // O as it stands (the merge normalises and gates): the real rows
            // park in the idle ring as [head][row][260 floats] (rows padded
            // off one bank), then one thread sends each 1 KiB row to its
            // partial slot with a bulk copy
            constexpr int OSTRIDE = 260;
            float *ost = reinterpret_cast<float *>(smem + RING);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tc::ld32(oc + c * 32, o);
                tc::wait_ld();
                if (lane < a.t) {
                    float *dst = ost + (quarter * 8 + lane) * OSTRIDE + 128 * h + 32 * c;
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4 *>(dst + e) =
                            make_float4(__uint_as_float(o[e]), __uint_as_float(o[e + 1]),
                                        __uint_as_float(o[e + 2]), __uint_as_float(o[e + 3]));
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            named_sync(1, 256);
            if (tid == 64 && ok) {
                for (int g = 0; g < 4; ++g)
                    for (int i = 0; i < a.t; ++i)
                        bulk_store(a.part_o +
                                       (((size_t)i * a.n_head + head + g) * a.n_splits + split) * HD,
                                   ost + (g * 8 + i) * OSTRIDE, HD * 4);
                bulk_commit_and_wait();
            }
        } else {
            // O / l times the gate goes through shared memory (the K/V ring,
            // idle now) so that the output stores are whole 128-byte rows per
            // warp: per 32-column chunk, each thread parks its row's values,
            // then each warp walks its 32 rows with lane = column
            float *stage = reinterpret_cast<float *>(smem + RING) + h * (BM * 33);
            const int n_rows = max(0, min(32, a.t - (q0 + quarter * 32)));  // valid rows
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tc::ld32(oc + c * 32, o);
                tc::wait_ld();
                const int col0 = 128 * h + 32 * c;
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
                __syncwarp();
                const int col = col0 + lane;
                const size_t row0 = (size_t)(q0 + quarter * 32) * a.n_head + head;
#pragma unroll 8
                for (int rr = 0; rr < 32; ++rr)
                    if (rr < n_rows && ok)
                        __stcs(a.out + (row0 + (size_t)rr * a.n_head) * HD + col,
                               stage[(quarter * 32 + rr) * 33 + lane]);
                __syncwarp();
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    // verify: the partials are written; the split merge may launch
    if constexpr (VERIFY) grid_dep_launch();
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
                                pf::SMEM_VERIFY);
}

cudaError_t launch_prefill(const PrefillArgs &a, const CUtensorMap &q_map,
                           const CUtensorMap &kv_map, const CUtensorMap &gate_map,
                           cudaStream_t st) {
    const int n_qt = (a.t + pf::BM - 1) / pf::BM;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_qt * a.n_head);
    cfg.blockDim = dim3(pf::THREADS);
    cfg.dynamicSmemBytes = pf::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_kernel<false>, a, q_map, kv_map, gate_map);
}

cudaError_t launch_verify_tc(const PrefillArgs &a, const CUtensorMap &kv_map, cudaStream_t st) {
    if (a.t < 1 || a.t > kVerifyRows || a.n_head != 4 * a.n_kv || a.n_splits < 1 ||
        a.split_tiles < 1 || !a.part_o || !a.part_ml || !a.qg || !a.q_norm || !a.rope_cs ||
        !a.rope_sn || !a.k_in || !a.v_in || !a.k_norm || !a.k_cache || !a.v_cache)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits * a.n_kv);
    cfg.blockDim = dim3(pf::THREADS);
    cfg.dynamicSmemBytes = pf::SMEM_VERIFY;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // the query and gate maps are not read in this form
    return cudaLaunchKernelEx(&cfg, prefill_kernel<true>, a, kv_map, kv_map, kv_map);
}

}  // namespace rl
