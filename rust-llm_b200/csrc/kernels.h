// Internal launch interface between the C ABI (rlcuda.cu) and the kernels.
// Every pointer here is device memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace rl {

// One call of the full-attention path: t rows at positions pos..pos+t-1 of
// one layer's cache.
struct FullArgs {
    const float *qg;       // [t][n_head][2*hd]  query | gate
    const float *k, *v;    // [t][n_kv][hd]
    const float *q_norm, *k_norm;  // [hd]
    const float *rope_cs, *rope_sn;  // [context][n_rot/2] cos, sin of the RoPE angles
    void *k_cache, *v_cache;       // [n_kv][context][hd], f32 or bf16
    float *q_f32;                  // [t][n_head][hd] normalised, rotated queries, or null
    __nv_bfloat16 *q_bf16;         // same in bf16, or null when not needed
    __nv_bfloat16 *gate_bf16;      // [t][n_head][hd] sigmoid of the gate in bf16, or null
    int t, pos, n_head, n_kv, hd, context, n_rot;
    float theta_scale, eps;
    bool kv_bf16;
    // append the rows' keys and values only (the queries are normalised
    // inside the tensor-core verify kernel)
    bool kv_only;
};

// One sequence of a batched bf16 decode (rl_batch_*): its context's cache of
// one layer, seen through its own tensor map (kept in global memory).
struct BatchRow {
    const CUtensorMap *map;        // 64-byte aligned, in device memory
    void *k_cache, *v_cache;       // this layer's [n_kv][context][hd] bf16
    const float *q_norm, *k_norm;  // this layer's norm weights
    const float *rope_cs, *rope_sn;
    int context, k_row0, v_row0;   // tensor-map rows as in DecodeArgs
};

// One launch of the split-KV decode kernel (decode_attn.cu).
struct DecodeArgs {
    const float *qg;              // [t][n_head][2*hd] raw query | gate
    const float *k_in, *v_in;     // [t][n_kv][hd] raw (fused path: appended here)
    const float *q_f32;           // [t][n_head][hd] normalised queries (unfused path)
    const float *q_norm, *k_norm;
    const float *rope_cs, *rope_sn;  // [context][n_rot/2] cos, sin of the RoPE angles
    void *k_cache_v, *v_cache_v;  // [n_kv][context][hd]
    float *part_o, *part_ml;      // cross-cluster partials
    int *counters;                // [rows][n_kv][8] arrival counters, zero between launches
    float *out;                   // [t][n_head*hd]
    int *status;
    int pos, t, context, n_head, n_kv, chunk, n_splits, csize, n_rot;
    float theta_scale, eps;
    bool kv_bf16, fused;
    // tensor-map rows of this layer's K and V caches (bf16 tensor-core
    // kernel): row of (KV head kh, position p) = k_row0 + kh * context + p
    int k_row0, v_row0;
    // bf16 walk: the producer may stream the cache before the previous
    // grid completes (nothing since the last decode wrote the cache)
    bool early_kv;
    // bf16 walk: tiles streamed before the consumers hold their inputs
    int early_tiles;
    // the cache holds sequence positions shard_lo .. shard_lo + context - 1
    // (0 unless the sequence is split across GPUs)
    int shard_lo;
    // non-null: the merge writes this shard's partial [t*n_head][hd + 2]
    // (unnormalised output, max in log2 units, sum) instead of the output
    float *part_out;
    // non-null (a split sequence, peer exchange): each merge CTA (head, 64-dim
    // slice) writes its slice of this GPU's partial into slot (epoch & 1,
    // xrank) of every GPU's exchange buffer, each value beside the epoch, its
    // own count of steps (xepochs, one word per CTA)
    float *const *xpeers;  // [xworld] exchange buffers, as addressed from this GPU
    int xrank, xworld;
    unsigned *xepochs;     // [rows_heads * 4] steps published, per merge CTA
    // non-null (bf16 walk, one row per sequence): row r is sequence r, at
    // position batch_pos[r] of its own context, described by rows[r]
    const BatchRow *rows;
    const int *batch_pos;
    // non-null: the bf16 walk records its span on the global timer into
    // this launch's slot, {first CTA start, CTAs done, sum of spans, launches}
    unsigned long long *span;
};
cudaError_t init_decode_kernels();
cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t st);
int decode_positions_per_tile(bool kv_bf16);
int decode_max_active_clusters(bool kv_bf16, bool fused, int csize);
// bf16 caches: the same step with K/V tiles staged by TMA tensor copies and
// both dot products on mma.sync (decode_mma.cu).  `kv_map` covers the
// whole KV allocation as rows of head_dim bf16, in boxes of 64 x 64.
// The walk writes one partial per (row, query head, split) into part_o
// [t][n_head][n_splits][hd] and part_ml [t][n_head][n_splits][2];
// launch_decode_combine merges them and applies the output gate.
cudaError_t init_decode_mma_kernels();
cudaError_t launch_decode_mma(const DecodeArgs &a, const CUtensorMap &kv_map, cudaStream_t st);
cudaError_t launch_decode_combine(const DecodeArgs &a, cudaStream_t st);
// The exchange buffer of one GPU for a split sequence: [2 slots][world]
// [rows_heads][hd + 2] 64-bit words, each an f32 value (low half: the
// unnormalised output, then the max in log2 units and the sum) beside the
// epoch of the step that stored it (high half).  Slot = epoch & 1.
__host__ __device__ inline size_t xbuf_bytes(int world, int rows_heads, int hd) {
    return (size_t)2 * world * rows_heads * (hd + 2) * sizeof(unsigned long long);
}
// Waits (bounded, limit_ns) until every GPU's values of a head in this GPU's
// exchange buffer carry the step's epoch (epochs: [rows_heads] steps merged,
// per CTA), then merges them and applies the gate: out [rows_heads][hd].
// Launched as a programmatic dependent.
cudaError_t launch_peer_merge(const unsigned long long *xbuf, int world, int rows_heads,
                              const float *qg, float *out, int *status, unsigned *epochs,
                              unsigned long long limit_ns, cudaStream_t st);
// parts [n_parts][rows_heads][hd + 2] -> out [rows_heads][hd], gated
cudaError_t launch_merge_parts(const float *parts, int n_parts, int rows_heads, const float *qg,
                               float *out, cudaStream_t st);
constexpr int kDecodeBoxRows = 64, kDecodeBoxCols = 64;
int decode_mma_max_active_ctas(bool fused);  // resident walk CTAs per SM
int decode_mma_positions_per_tile();

// One call of the tcgen05 causal prefill (prefill.cu): t rows at positions
// pos..pos+t-1 whose queries the prologue staged in bf16 (q_map: [t][n_head]
// [hd] in boxes of 128 rows x 64 dims) and whose keys and values it appended
// to the bf16 cache (kv_map, as for the decode walk).
struct PrefillArgs {
    float *out;       // [t][n_head*hd]
    int *status;
    int t, pos, n_head, n_kv, context, k_row0, v_row0;
    // verify form only: partials [t][n_head][n_splits][hd] and
    // [t][n_head][n_splits][2] (max in log2 units, sum); split s walks key
    // tiles s * split_tiles .. (s + 1) * split_tiles - 1
    float *part_o, *part_ml;
    int n_splits, split_tiles;
    // verify form only: the raw rows (query | gate), the query norm weight,
    // the RoPE table and eps; the kernel normalises and rotates the queries
    // itself (n_rot 64)
    const float *qg, *q_norm, *rope_cs, *rope_sn;
    float eps;
    // verify form only: the rows' raw keys and values [t][n_kv][hd], the key
    // norm weight and this layer's bf16 caches [n_kv][context][hd]; the CTA
    // whose key range holds a new position appends that row itself
    const float *k_in, *v_in, *k_norm;
    __nv_bfloat16 *k_cache, *v_cache;
};
cudaError_t init_prefill_kernels();
// gate_map: the prologue's bf16 sigmoid(gate) staging, laid out and boxed as
// q_map
cudaError_t launch_prefill(const PrefillArgs &a, const CUtensorMap &q_map,
                           const CUtensorMap &kv_map, const CUtensorMap &gate_map,
                           cudaStream_t st);
constexpr int kPrefillQBoxRows = 128;
// Multi-row verify (1..8 rows, 4 query heads per KV head, n_rot 64) on the
// same tensor-core tiles: one CTA per (key split, KV head), its 128 tile rows
// the group's 4 heads x 32 rows (rows 8..31 of each head padding).  The
// kernel appends the rows' keys and values and normalises the queries
// itself; launch_decode_combine merges the partials.
cudaError_t launch_verify_tc(const PrefillArgs &a, const CUtensorMap &kv_map, cudaStream_t st);
constexpr int kVerifyRows = 8;

cudaError_t init_full_attn_kernels();
// cos/sin of every position's RoPE angles, [context][n_rot/2] each
cudaError_t launch_rope_table(float *cs, float *sn, int context, int n_rot, float theta_scale,
                              cudaStream_t st);
cudaError_t launch_full_prologue(const FullArgs &a, cudaStream_t st);

// One call of the Gated DeltaNet path: t sequential rows over ring slots
// (live+i)%slots -> (live+i+1)%slots of one layer.
struct LinArgs {
    const float *qkv;     // [t][conv_dim]
    const float *z;       // [t][n_v*s]
    const float *alpha;   // [t][n_v] raw
    const float *beta;    // [t][n_v] raw
    float *conv_state;    // [slots][conv_dim][kernel-1]
    float *ssm_state;     // [n_v][slots][s][s]
    const float *conv1d;  // [conv_dim][kernel]
    const float *ssm_a, *dt_bias;  // [n_v]
    const float *norm;    // [s]
    float *out;           // [t][n_v*s]
    int *status;
    int t, slots, live, s, n_k, n_v, kernel;
    float eps;
    // the state and conv history may be read before the grid-dependency
    // wait: the kernel just ahead on the stream is not a step of this layer
    bool early_state;
    // the rows kernel's state map row of this layer's head 0, slot 0
    int ssm_row0;
};

cudaError_t init_dn_kernels();
cudaError_t launch_dn_step(const LinArgs &a, cudaStream_t st);
int dn_max_group();
// The same rows, up to eight, through the closed-form rows kernel
// (dn_rows.cu), whose shape limits dn_rows_fits states.
// `map`: every layer's state as rows of d_state f32, boxes of 128 rows x 32
// columns with the 128-byte swizzle (encode_f32_2d).
bool dn_rows_fits(const LinArgs &a);
cudaError_t init_dn_rows_kernel();
cudaError_t launch_dn_rows(const LinArgs &a, const CUtensorMap &map, cudaStream_t st);

// One chunked Gated DeltaNet prefill (dn_chunk.cu): t rows of one layer
// updating ring slot `live` in place (slots == 1), in chunks of 64 tokens.
struct DnChunkArgs {
    const float *qkv, *z, *alpha, *beta;  // [t][conv_dim], [t][n_v*s], [t][n_v] x2
    float *conv_state;                    // [conv_dim][kernel-1] of slot `live`
    float *ssm_state;                     // [n_v][slots][s][s]
    const float *conv1d, *ssm_a, *dt_bias, *norm;
    float *out;                           // [t][n_v*s]
    // scratch, sized for max_batch rows
    __nv_bfloat16 *qn, *kn, *vn;          // [t][n_k][s], [t][n_k][s], [t][n_v][s]
    __nv_bfloat16 *qn_lo, *kn_lo, *vn_lo;  // low halves: every operand is a bf16 pair
    __nv_bfloat16 *qn_l2, *kn_l2;         // third terms of q and k (Q K^T needs 24 bits)
    float *lg, *bt;                       // [t][n_v] log decay, beta
    __nv_bfloat16 *w, *qp, *kp, *p;       // [n_v][nc][64][s] (p: [n_v][nc][64][64])
    __nv_bfloat16 *w_lo, *qp_lo, *kp_lo, *p_lo;  // their low halves
    float *ut, *gc;                       // [n_v][nc][64][s], [n_v][nc]
    float *opre;                          // [t][n_v][s] readout before the gated norm
    int *status;
    int t, nc, n_k, n_v, live, slots;
    float eps;
    bool w_lo_out;  // write W's low half (the mma.sync scan reads it)
    // overlapped chunk-local and tcgen05 scan (null: one after the other):
    // the chunk-local CTA of (value head, chunk) stores ready[head * nc +
    // chunk] = ready_epoch[head] + 1 once its outputs are written; the scan
    // waits for that value and, done, advances ready_epoch[head]
    int *ready, *ready_epoch;
    // CTAs of the tcgen05 chunk-local kernel, one per SM it gets (0: one per
    // item), and the item counter they claim from (zeroed by the prep kernel;
    // null: a CTA takes every gridDim.x-th item)
    int local_ctas;
    int *local_next;
    // out_ready[head * nc + chunk]: zeroed by the prep kernel; each of the
    // tcgen05 scan's four readout warps adds 1 once its pre-norm rows of the
    // chunk are stored; the output kernel waits for 4 (null: it runs after
    // the scan)
    int *out_ready;
};
// The prep kernel's q and k planes (hi, lo, third term) as [t][n_k][128]
// bf16 with t the call's rows, boxes of 64 channels x 1 head x 64 tokens, the
// 128-byte swizzle: the chunk-local kernel's tcgen05 form loads them by TMA.
struct DnPlaneMaps {
    CUtensorMap q[3], k[3];
};
// The second stream and events of an overlapped chunked prefill.
struct DnOverlap {
    cudaStream_t scan_stream;
    cudaEvent_t fork, join;
};
cudaError_t init_dn_chunk_kernels();
// The chunk scan on tcgen05 (dn_scan_tc.cu) reads the chunk-local kernel's
// outputs through these tensor maps: W (hi), Q' and K' (hi, lo) as
// [n_v * nc * 64][128] bf16 and P (hi, lo) as [n_v * nc * 64][64] bf16, all in
// boxes of 64 rows x 64 columns with the 128-byte swizzle.
struct DnScanMaps {
    CUtensorMap w, qh, ql, kh, kl, ph, pl;
};
cudaError_t init_dn_scan_tc_kernel();
cudaError_t launch_dn_scan_tc(const DnChunkArgs &a, const DnScanMaps &m, cudaStream_t st);
// The whole chunked prefill of one call; `scan_maps` non-null selects the
// tcgen05 chunk scan, null the mma.sync one.  With `overlap` (and the tcgen05
// scan, and a.ready set) the scan runs on overlap->scan_stream beside the
// chunk-local kernel, forked after the prep kernel and joined before the
// output kernel.  With `planes` the chunk-local kernel takes K K^T and
// Q K^T on tcgen05 (its tcgen05 form), else on mma.sync.
cudaError_t launch_dn_chunk(const DnChunkArgs &a, const DnScanMaps *scan_maps, cudaStream_t st,
                            const DnOverlap *overlap = nullptr,
                            const DnPlaneMaps *planes = nullptr);

// KV cache fill from f32 (host-visible test and bench helper): positions
// [p0, p0+n) of every KV head, src [2][n_kv][n][hd] f32 on the device.
cudaError_t launch_kv_fill(void *k_cache, void *v_cache, const float *src, int n_kv,
                           int context, int hd, int p0, int n, bool kv_bf16, cudaStream_t st);
cudaError_t launch_kv_read(const void *k_cache, const void *v_cache, float *dst, int n_kv,
                           int context, int hd, int p0, int n, bool kv_bf16, cudaStream_t st);

// Projections (proj.cu): t rows of k activations quantized to int8 per
// 256-value super-block (d [t][nb], qs [t][nb][256], bs [t][nb][16]), then
// out [t][rows] = W . x for a weight of GGML type 12 (Q4_K), 14 (Q6_K) or
// 8 (Q8_0) stored as rows of proj_row_bytes(type, k) bytes.
size_t proj_row_bytes(int ggml_type, int k);
cudaError_t launch_q8k_quantize(const float *x, int t, int k, float *d, int8_t *qs, int16_t *bs,
                                cudaStream_t st);
// A group of up to 8 weights dotted with the same activations, one launch.
constexpr int kMatvecGroupMax = 8;
struct MatvecGroup {
    int n;
    int type[kMatvecGroupMax], rows[kMatvecGroupMax];
    size_t stride[kMatvecGroupMax];
    const void *w[kMatvecGroupMax];
    float *out[kMatvecGroupMax];
    // set by the one-launch kernel's launcher: rows per warp of each part and
    // the first warp of each part (wfirst[n] = the warps in all)
    int rpw[kMatvecGroupMax], wfirst[kMatvecGroupMax + 1];
};
// A weight row is staged in shared memory: at most this many bytes (k up to
// 16384 for Q8_0, the largest row of the reference's tests).
constexpr int kMatvecRowSmemMax = 17456;
cudaError_t init_matvec_kernel();
// Exec::matmul_group in one launch (quantization of x [t][k] included), when
// its shared memory fits: the quantized rows plus two staged weight rows per
// warp.
constexpr int kMatmulSmemMax = 200 * 1024;
size_t matmul_group_smem(int t, int k, size_t stride_max);
cudaError_t launch_matmul_group(const MatvecGroup &g, const float *x, int t, int k,
                                cudaStream_t st);
cudaError_t launch_matvec_group(const MatvecGroup &g, int k, const float *d, const int8_t *qs,
                                const int16_t *bs, int t, cudaStream_t st);

// Sets the calling thread's message for rl_last_error(NULL).
void set_thread_error(const char *msg);

}  // namespace rl
