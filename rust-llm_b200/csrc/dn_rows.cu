// Gated DeltaNet, token-sequential rows kernel for sm_100a: the decode step
// (t = 1), the speculative-verify pass (t rows, one state snapshot per row in
// the ring) and any short batch of rows, with each value head's 128 state
// columns split over four CTAs of a cluster.
//
// Reference: Exec::linear_attn (crates/rust-llm/src/forward.rs:1530-1652),
// delta_net / delta_net_into (:1906-2010), depthwise_conv(_into) (:2018-2059),
// l2_norm_in_place (:1720-1727), softplus / sigmoid / silu (:1730-1743).
//
// The rows run one after the other, as in the reference: decay the state,
// contract it with k, form the delta, add its outer product, contract with q.
// Every row is computed by the same instructions whatever the batch, so a
// batch of rows and the same rows one call at a time give the same outputs
// and states bit for bit (tests/speculate.rs:49-60 asks that of a verify
// pass).
//
// Work split.  The 128 x 128 state of a value head is split by columns over 4
// CTAs (32 columns each), one cluster of 4 * gv CTAs per key head (gv =
// n_v / n_k value heads share a key head), grid (4 * gv, n_k).  A CTA has 8
// compute warps and a store warp; compute warp w owns columns 4w .. 4w+3
// of the CTA's block; lane (rg, cg) = (l & 7, l >> 3) holds column 4w + cg
// at the 16 rows rg + 8e, e = 0..15, in registers.  A column's reductions
// over its 128 rows (S^T k, S^T q) are then 16 products in the lane and three
// butterfly shuffles over the 8 lanes of the column, and the warps run the
// rows' recurrence independently, with no barrier between rows.  The decay
// is taken out of the contraction (g (S^T k) rather than (g S)^T k), so only
// one FMA per state element waits on the shuffles.
//
// State traffic goes through a ring of four 128 x 32 f32 tiles in shared
// memory, laid out with the 128-byte swizzle so that the lanes' column-wise
// writes are free of bank conflicts.  The live slot comes in by coalesced
// 16-byte loads into a tile.  Each row's snapshot n is written into tile
// n % 4; once every compute warp has arrived on that tile's full barrier,
// the tile goes to its ring slot by a TMA tile store and comes back (empty
// barrier) when the copy has read it, two copies later.  The compute warps
// never issue a global store for the state.  Who sends the tiles depends on
// the launch: where rows never write the slot they read (slots > t: the
// verify pass) a ninth warp, the store warp, does it, and the CTAs run one to
// an SM; elsewhere (decode, in-place batches) thread 0 does, one row late,
// and two CTAs may share an SM.  The values are the same either way.
//
// The conv, the gates and the q/k L2 norms come first, for a block of up to
// eight rows at once, and the gated RMSNorm last, warp r of the block taking
// row r; the norm's sum of squares over the head's 128 outputs is pushed into
// the head's four CTAs by asynchronous stores into their shared memory.  The
// cluster's split barrier covers the q/k conv history its CTAs share (each
// reads it and arrives; the one writer waits before it overwrites it).
//
// PDL: as in the single-step kernel, the state and conv history are loaded
// before the grid-dependency wait unless the kernel just ahead is a step of
// the same layer (`early_state`); row inputs are read and every global write
// is made after the wait.
#include "common.cuh"
#include "kernels.h"

namespace rl {
namespace dnr {
constexpr int S = 128;                   // d_state the kernel is built for
constexpr int NCB = 4;                   // column blocks (CTAs) per value head
constexpr int CW = S / NCB;              // 32 state columns per CTA
constexpr int NW = 8;                    // compute warps, 4 state columns each
constexpr int CTHREADS = NW * 32;        // (and a store warp in one form)
constexpr int MAXR = 8;                  // rows per block
constexpr int HIST = 3;                  // conv_kernel - 1
constexpr int RPL = S / 8;               // state rows per lane
constexpr int KP = 20;                   // pitch (floats) of a lane's transposed k / q rows
constexpr int NBUF = 4;                  // snapshot tiles
constexpr int TILE = S * CW * 4;         // one tile: 128 rows x 128 bytes
constexpr int SMEM = NBUF * TILE + 1024; // the tile ring, with room to align
// a launch whose rows never write the slot they read (slots > t) takes
// clusters of one value head's 4 CTAs and asks for this much shared memory,
// so that no SM holds two of its CTAs (ones sharing an SM run at half speed)
constexpr int SMEM_SOLO = 120 * 1024;
}  // namespace dnr

// The warp-wide sums of eight per-lane values v[0..7] at once: a reduce-
// scatter over lane bits 4, 3 and 2 (each step keeps half the values and
// sends the other half), then a plain sum over bits 1 and 0.  Lane l ends with
// the sum for value 4*b4 + 2*b3 + b2 (bk = bit k of l).
__device__ __forceinline__ double warp_sum8_d(const double (&v)[8], int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    double h4[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const double keep = b4 ? v[4 + m] : v[m], send = b4 ? v[m] : v[4 + m];
        h4[m] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    double h2[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const double keep = b3 ? h4[2 + m] : h4[m], send = b3 ? h4[m] : h4[2 + m];
        h2[m] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    double h1 = (b2 ? h2[1] : h2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? h2[0] : h2[1], 4);
    h1 += __shfl_xor_sync(0xffffffffu, h1, 2);
    h1 += __shfl_xor_sync(0xffffffffu, h1, 1);
    return h1;
}

// Sum over the 8 lanes of a column (lane bits 0-2); every one of them gets
// the same bits (each pairwise sum is commutative, the tree is the same).
__device__ __forceinline__ float col_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    return v;
}

// Byte offset of element (row, col) in a 128 x 32 f32 tile written with the
// 128-byte swizzle: 16-byte chunk col / 4 of a row is stored at chunk
// (col / 4) ^ (row % 8).  For lane (rg, cg) of warp w at row rg + 8e, column
// 4w + cg, the 32 lanes of an access hit 32 different banks.
__device__ __forceinline__ uint32_t tile_off(int row, int col) {
    return (uint32_t)(row * 128 + ((((col >> 2) ^ row) & 7) << 4) + ((col & 3) << 2));
}

// SiLU from the hardware exp2 and an approximate divide: within a few f32
// ulps of x / (1 + e^-x), well inside the step's 1e-4 bar
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float4 ld4(const float *p) {
    return *reinterpret_cast<const float4 *>(p);
}

// One CTA block (128 rows x 32 columns) of a state slot from global into a
// swizzled tile, by coalesced 16-byte loads: thread tid moves rows
// (tid >> 3) + 32 j, 16-byte chunk tid & 7 of each.
__device__ __forceinline__ void tile_from_global(uint8_t *tile, const float *src, int tid) {
    using namespace dnr;
    const int c = tid & 7;
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = ld4(src + (size_t)((tid >> 3) + 32 * j) * S + c * 4);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int row = (tid >> 3) + 32 * j;
        *reinterpret_cast<float4 *>(tile + row * 128 + ((c ^ (row & 7)) << 4)) = v[j];
    }
}
// grid (NCB * gv, n_k), blockIdx.x = grp * NCB + cb; value head vh = kh +
// grp * n_k, so that vh % n_k == kh as in forward.rs:1602-1609.  Clusters
// are (NCB * gv) CTAs (a key head, whose CTAs share the q/k history) or, when
// no row writes the slot the rows read, NCB CTAs (a value head).
// MB: rows per block, 1 for a single row (the decode step) or MAXR; a row's
// arithmetic is the same in both (the sums of squares take the same tree),
// so they agree bit for bit.  SW: a store warp sends the snapshot tiles (else
// thread 0 does).
// `map` covers every layer's state as rows of 128 f32 (box 128 rows x 32
// columns, 128-byte swizzle); head vh, slot s of this layer starts at row
// a.ssm_row0 + (vh * slots + s) * 128.
template <int MB, bool SW>
__global__ void __maxnreg__(112)
    dn_rows_kernel(const LinArgs a, const __grid_constant__ CUtensorMap map) {
    using namespace dnr;
    extern __shared__ uint8_t dsm[];
    uint8_t *tiles = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(dsm) + 1023) & ~static_cast<uintptr_t>(1023));
    __shared__ __align__(16) float kt_s[MB][8 * KP], qt_s[MB][8 * KP];  // k, q transposed
    __shared__ float v_s[MB][CW], o_s[MB][CW];
    __shared__ float g_s[MB], beta_s[MB];
    __shared__ double nred[MB][NW];       // q/k sums of squares by warp
    __shared__ double osum[2][NCB][MB];   // output sums of squares by block parity, column block
    __shared__ __align__(8) uint64_t full[NBUF], empty[NBUF], xbar[2];

    const int n_k = a.n_k, n_v = a.n_v, slots = a.slots, t = a.t, live = a.live;
    const int cb = blockIdx.x % NCB, grp = blockIdx.x / NCB, kh = blockIdx.y;
    const int vh = kh + grp * n_k;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool store_warp = SW && warp == NW;
    const int rg = lane & 7, cg = lane >> 3;
    const int col = warp * 4 + cg;  // this lane's state column within the CTA's block
    const int key_dim = n_k * S, d_inner = n_v * S, conv_dim = 2 * key_dim + d_inner;
    const int nst = slots > 1 ? t : 1;  // snapshots stored
    // row r's history goes to slot (live + r + 1) % slots unless a later row
    // of the call goes there too (t > slots, or slots == 1): the v history of
    // different rows is written by different warps, so only the last writes
    auto last_in_slot = [&](int r) { return r + slots >= t; };
    const float scale = 1.0f / sqrtf((float)S);
    const float shrink = 1.0f / sqrtf((float)S);
    const float l2_eps = a.eps / (float)S;
    const float *head = a.ssm_state + (size_t)vh * slots * S * S + cb * CW;  // slot 0, this block
    const int row0 = a.ssm_row0 + vh * slots * S;  // map row of this head's slot 0
    // snapshot m to its slot once every compute warp has written it; the
    // tile of snapshot m - 2 goes back once its copy has read it
    auto send = [&](int m) {
        const int b = m % NBUF;
        if (!mbar_wait(&full[b], (m / NBUF) & 1, a.status)) return false;
        const int slot = slots > 1 ? (live + m + 1) % slots : live;
        tma_store_2d(&map, cb * CW, row0 + slot * S, tiles + b * TILE);
        bulk_commit();
        if (m >= 2) {
            bulk_wait_read<2>();
            mbar_arrive(&empty[(m - 2) % NBUF]);
        }
        return true;
    };
    uint32_t crank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    const int rank0 = (int)crank - cb;  // cluster rank of this head's column block 0

    if (tid == 0) {
#pragma unroll
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&full[b], NW);
            mbar_init(&empty[b], 1);
        }
        mbar_init(&xbar[0], 1);
        mbar_init(&xbar[1], 1);
        fence_barrier_init();  // before the cluster barrier lets a peer store into xbar
    }
    __syncthreads();

    // conv channels: one q (tid < 128) or k channel of key head kh per
    // thread, over the block's rows; and v channel `lane` of this CTA's
    // column block for row `warp` of the block
    const int ch = tid < S ? kh * S + tid : key_dim + kh * S + (tid - S);
    const int vch = 2 * key_dim + vh * S + cb * CW + lane;
    const bool writes_qk = blockIdx.x == 0;  // the one writer of the shared q/k history
    float w[4], wv[4];
    {
        const float4 x = ld4(a.conv1d + (size_t)ch * 4), y = ld4(a.conv1d + (size_t)vch * 4);
        w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w;
        wv[0] = y.x, wv[1] = y.y, wv[2] = y.z, wv[3] = y.w;
    }
    const float dt_bias = a.dt_bias[vh], ssm_a = a.ssm_a[vh];
    const float wn = a.norm[cb * CW + lane];  // the norm weight of this lane's output column

    float h[HIST], hv[HIST];
    const float *hist_live = a.conv_state + (size_t)live * conv_dim * HIST;
    auto load_state = [&]() {
        if (!store_warp) {
            tile_from_global(tiles + (NBUF - 1) * TILE, head + (size_t)live * S * S, tid);
#pragma unroll
            for (int e = 0; e < HIST; ++e) {
                h[e] = hist_live[(size_t)ch * HIST + e];
                hv[e] = hist_live[(size_t)vch * HIST + e];
            }
        }
        cluster_arrive_release();  // this CTA has read the history it shares
    };
    if (a.early_state) load_state();
    grid_dep_wait();
    grid_dep_launch();
    if (!a.early_state) load_state();
    // every CTA of the cluster has read the q/k history: it may be written
    cluster_wait_acquire();

    if (store_warp) {
        if (lane == 0) {
            for (int m = 0; m < nst; ++m)
                if (!send(m)) break;
            bulk_wait_all();  // the copies are done before the tiles go away
        }
        return;
    }
    named_sync(1, CTHREADS);  // the live state is in the last tile
    float st[RPL];
#pragma unroll
    for (int e = 0; e < RPL; ++e)
        st[e] = *reinterpret_cast<const float *>(tiles + (NBUF - 1) * TILE + tile_off(rg + 8 * e, col));

    int n = 0;  // snapshots written so far
    for (int blk = 0, par = 0; blk < t; blk += MB, par ^= 1) {
        const int nb = min(MB, t - blk);
        // ---- the block's inputs, issued together (rows past the block's end
        // load its last row again, unused, so that the loads are unconditional)
        float x[MB];
#pragma unroll
        for (int r = 0; r < MB; ++r) x[r] = a.qkv[(size_t)(blk + min(r, nb - 1)) * conv_dim + ch];
        const bool row_w = warp < nb;  // warp r takes row r of the block's v conv and output
        const int gr = blk + min(warp, nb - 1);
        float xt[4];  // the v channel's conv taps for row gr: rows gr-3 .. gr
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rr = gr - 3 + j;
            xt[j] = rr >= 0 ? a.qkv[(size_t)rr * conv_dim + vch]
                            : rr == -3 ? hv[0] : rr == -2 ? hv[1] : hv[2];
        }
        const float zz = a.z[(size_t)gr * d_inner + (size_t)vh * S + cb * CW + lane];
        // ---- gates (forward.rs:1530-1546), by the last warp
        if (warp == NW - 1 && lane < nb) {
            const size_t gi = (size_t)(blk + lane) * n_v + vh;
            // hardware exp2 / log2 forms: softplus to ~1e-7 absolute (the
            // decay it scales enters g = e^decay, so absolute error is what
            // counts), well inside the step's 1e-4 bar
            const float x = __fadd_rn(a.alpha[gi], dt_bias);
            const float sp = x > 20.0f ? x : __logf(1.0f + __expf(x));
            const float decay = __fmul_rn(sp, ssm_a);
            g_s[lane] = __expf(decay);
            beta_s[lane] = __fdividef(1.0f, 1.0f + __expf(-a.beta[gi]));
        }
        // ---- conv (forward.rs:2018-2059: x*w[3] first, then the history
        // taps in order), SiLU, and the history each row leaves in its slot
        float c[MB];
#pragma unroll
        for (int r = 0; r < MB; ++r) {
            c[r] = 0.0f;
            if (r < nb) {
                float y = __fmul_rn(x[r], w[3]);
#pragma unroll
                for (int e = 0; e < HIST; ++e) y = __fadd_rn(y, __fmul_rn(h[e], w[e]));
                c[r] = silu_fast(y);
                h[0] = h[1], h[1] = h[2], h[2] = x[r];
                if (writes_qk && last_in_slot(blk + r)) {
                    float *hs = a.conv_state + (size_t)((live + blk + r + 1) % slots) * conv_dim * HIST +
                                (size_t)ch * HIST;
#pragma unroll
                    for (int e = 0; e < HIST; ++e) hs[e] = h[e];
                }
            }
        }
        float cv = 0.0f;
        if (row_w) {
            float y = __fmul_rn(xt[3], wv[3]);
#pragma unroll
            for (int e = 0; e < HIST; ++e) y = __fadd_rn(y, __fmul_rn(xt[e], wv[e]));
            cv = silu_fast(y);
            if (last_in_slot(gr)) {
                float *hs = a.conv_state + (size_t)((live + gr + 1) % slots) * conv_dim * HIST +
                            (size_t)vch * HIST;
#pragma unroll
                for (int e = 0; e < HIST; ++e) hs[e] = xt[e + 1];
            }
        }
        // ---- q/k L2 norm (forward.rs:1577-1584, :1720-1727): warps 0-3 hold
        // q, warps 4-7 hold k
        float my;  // the scale of row (lane >> 2) & 7 of this lane's group
        {
            double sq[MB];
#pragma unroll
            for (int r = 0; r < MB; ++r) sq[r] = (double)__fmul_rn(c[r], c[r]);
            if constexpr (MB == MAXR) {
                // lane l ends with the warp's sum for row (l >> 2) & 7
                const double s8 = warp_sum8_d(sq, lane);
                if ((lane & 3) == 0) nred[lane >> 2][warp] = s8;
            } else {
                const double s1 = warp_sum_d(sq[0]);  // the same tree for row 0
                if (lane == 0) nred[0][warp] = s1;
            }
            if (row_w) v_s[warp][lane] = cv;
            named_sync(1, CTHREADS);
            const int w0 = warp < 4 ? 0 : 4, rr = MB == MAXR ? (lane >> 2) & 7 : 0;
            my = 1.0f;
            if (rr < nb) {
                double sum = -0.0;
#pragma unroll
                for (int q = 0; q < 4; ++q) sum += nred[rr][w0 + q];
                my = rms_scale_fast(sum, S, l2_eps);  // both norms sit on the critical path
            }
        }
        {
            const int i = tid & (S - 1);  // the channel within q or k
            float *dst = (tid < S ? &qt_s[0][0] : &kt_s[0][0]) + (i & 7) * KP + (i >> 3);
#pragma unroll
            for (int r = 0; r < MB; ++r) {
                const float sc = MB == MAXR ? __shfl_sync(0xffffffffu, my, 4 * r) : my;
                if (r < nb) dst[r * 8 * KP] = __fmul_rn(__fmul_rn(c[r], sc), shrink);
            }
        }
        named_sync(1, CTHREADS);
        // ---- the rows, one after the other (forward.rs:1964-2010), each warp
        // on its own four columns: contract with k, decay, delta, add its
        // outer product, contract with q; snapshot n goes into tile n % 4 and
        // is sent while the next row runs
#pragma unroll 1
        for (int r = 0; r < nb; ++r) {
            float kk[RPL], qq[RPL];
#pragma unroll
            for (int m = 0; m < RPL / 4; ++m) {
                const float4 k4 = ld4(&kt_s[r][rg * KP + 4 * m]);
                const float4 q4 = ld4(&qt_s[r][rg * KP + 4 * m]);
                kk[4 * m] = k4.x, kk[4 * m + 1] = k4.y, kk[4 * m + 2] = k4.z, kk[4 * m + 3] = k4.w;
                qq[4 * m] = q4.x, qq[4 * m + 1] = q4.y, qq[4 * m + 2] = q4.z, qq[4 * m + 3] = q4.w;
            }
            const float g = g_s[r], be = beta_s[r], vj = v_s[r][col];
            float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
            for (int e = 0; e < RPL; e += 2) {
                p0 = fmaf(st[e], kk[e], p0);
                p1 = fmaf(st[e + 1], kk[e + 1], p1);
            }
#pragma unroll
            for (int e = 0; e < RPL; ++e) st[e] = __fmul_rn(st[e], g);
            const float sk = __fmul_rn(g, col_sum(p0 + p1));
            const float d = __fmul_rn(__fsub_rn(vj, sk), be);
            float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
            for (int e = 0; e < RPL; e += 2) {
                st[e] = fmaf(d, kk[e], st[e]);
                st[e + 1] = fmaf(d, kk[e + 1], st[e + 1]);
                o0 = fmaf(st[e], qq[e], o0);
                o1 = fmaf(st[e + 1], qq[e + 1], o1);
            }
            const float o = col_sum(o0 + o1);
            if (rg == 0) o_s[r][col] = o;
            if (slots > 1 || blk + r == t - 1) {
                const int b = n % NBUF;
                // the tile's previous snapshot (n - 4) has been read by its copy
                if (n >= NBUF) mbar_wait(&empty[b], (n / NBUF - 1) & 1, a.status);
                uint8_t *tile = tiles + b * TILE;
#pragma unroll
                for (int e = 0; e < RPL; ++e)
                    *reinterpret_cast<float *>(tile + tile_off(rg + 8 * e, col)) = st[e];
                fence_proxy_async_smem();  // the tile copy reads these writes
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[b]);
                if (!SW && tid == 0 && n >= 1) send(n - 1);
                ++n;
            }
        }
        if (tid == 0) mbar_arrive_expect_tx(&xbar[par], (uint32_t)(nb * NCB * sizeof(double)));
        named_sync(1, CTHREADS);
        // the last snapshot, complete in its tile after the barrier above,
        // goes out while the norm exchange runs
        if (!SW && blk + MB >= t && tid == 0) send(nst - 1);
        // ---- gated RMSNorm (forward.rs:1642-1652): warp r takes row r at the
        // CTA's 32 columns; its sum of squares goes to the head's four CTAs
        // by asynchronous stores that complete on each one's barrier
        if (row_w) {
            const float o = __fmul_rn(o_s[warp][lane], scale);
            const double ss = warp_sum_d((double)__fmul_rn(o, o));
            if (lane < NCB)
                st_async_cluster_f64(&osum[par][cb][warp], &xbar[par], rank0 + lane, ss);
            mbar_wait(&xbar[par], (blk / MB >> 1) & 1, a.status);
            double sum = -0.0;
#pragma unroll
            for (int q = 0; q < NCB; ++q) sum += osum[par][q][warp];
            const float sc = rms_scale_fast(sum, S, a.eps);
            a.out[(size_t)(blk + warp) * d_inner + (size_t)vh * S + cb * CW + lane] =
                __fmul_rn(__fmul_rn(__fmul_rn(o, sc), wn), silu_fast(zz));
        }
    }
    if (!SW && tid == 0) bulk_wait_all();  // the copies are done before the tiles go away
}

cudaError_t init_dn_rows_kernel() {
    const void *k[4] = {(const void *)dn_rows_kernel<1, false>,
                        (const void *)dn_rows_kernel<dnr::MAXR, false>,
                        (const void *)dn_rows_kernel<1, true>,
                        (const void *)dn_rows_kernel<dnr::MAXR, true>};
    for (const void *f : k) {
        const cudaError_t e =
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, dnr::SMEM_SOLO);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// The rows kernel's shape limits: d_state 128, conv kernel 4, and a key
// head's value heads times four column blocks in one portable cluster.
bool dn_rows_fits(const LinArgs &a) {
    return a.s == dnr::S && a.kernel == dnr::HIST + 1 && a.t >= 1 && a.n_k > 0 &&
           a.n_v % a.n_k == 0 && dnr::NCB * (a.n_v / a.n_k) <= 8;
}

cudaError_t launch_dn_rows(const LinArgs &a, const CUtensorMap &map, cudaStream_t st) {
    const int gv = a.n_v / a.n_k;
    // rows that never write the live slot leave the shared q/k history alone
    const bool solo = a.slots > a.t;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dnr::NCB * gv, a.n_k);
    cfg.blockDim = dim3(dnr::CTHREADS + (solo ? 32 : 0));
    cfg.dynamicSmemBytes = solo ? dnr::SMEM_SOLO : dnr::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = solo ? dnr::NCB : dnr::NCB * gv;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (solo)
        return a.t == 1 ? cudaLaunchKernelEx(&cfg, dn_rows_kernel<1, true>, a, map)
                        : cudaLaunchKernelEx(&cfg, dn_rows_kernel<dnr::MAXR, true>, a, map);
    return a.t == 1 ? cudaLaunchKernelEx(&cfg, dn_rows_kernel<1, false>, a, map)
                    : cudaLaunchKernelEx(&cfg, dn_rows_kernel<dnr::MAXR, false>, a, map);
}

}  // namespace rl
