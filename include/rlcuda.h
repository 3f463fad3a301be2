/*
 * rlcuda.h — C ABI of the B200 (sm_100a) attention path for the rust-llm
 * Qwen3.5 hybrid runner.
 *
 * The library replaces the hot span of the reference's two attention
 * methods and the caches they run on:
 *   Exec::full_attn    crates/rust-llm/src/forward.rs:1220-1344 (span 1259-1340)
 *   Exec::linear_attn  crates/rust-llm/src/forward.rs:1484-1663 (span 1530-1652)
 *   Caches             crates/rust-llm/src/forward.rs:236-254, sized at :468-474
 *   Runner::{reset, verify, accept, pos}  forward.rs:558-577, :641-650, :675-688, :553-555
 * The projections on either side (forward.rs:1250, :1342, :1517, :1656) stay
 * with the caller: a call takes the projection outputs and returns the
 * `heads` buffer the output projection reads.
 *
 * Conventions
 *   - Every function returns an rl_status (0 = ok, negative = error) unless
 *     its comment says otherwise; rl_last_error() describes the last failure
 *     on that context (or, for a NULL context, on the calling thread).
 *   - A context is not thread-safe, like `&mut Runner`: one caller at a time.
 *   - Device memory is owned by the context and freed by rl_ctx_destroy.
 *   - Entry points named *_host take host pointers and return once the
 *     result is in host memory.  The others take device pointers, are
 *     enqueued on the context's stream and return immediately; rl_sync()
 *     waits and reports any error a kernel flagged on the device.
 *   - Arrays are f32, row-major, token-major, laid out as the reference's
 *     buffers are (forward.rs:256-320).
 */
#ifndef RLCUDA_H
#define RLCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    RL_OK = 0,
    RL_EINVAL = -1,       /* bad argument: the reference's contract panics, forward.rs:811-820, :642-647, :676-681 */
    RL_ECONTEXT = -2,     /* the batch does not fit the remaining context (forward.rs:815-820) */
    RL_ECUDA = -3,        /* a CUDA runtime error */
    RL_ENCCL = -4,        /* an NCCL error */
    RL_ETIMEOUT = -5,     /* a bounded device-side wait gave up */
    RL_EUNSUPPORTED = -6, /* a shape the kernels are not built for */
    RL_ENOMEM = -7        /* device allocation failed */
} rl_status;

typedef enum { RL_KV_F32 = 0, RL_KV_BF16 = 1 } rl_kv_dtype;

typedef struct rl_ctx rl_ctx;

/* Shapes and sizes.  The model fields mirror Config (crates/rust-llm/src/
 * model.rs:41-66); context and slots mirror Runner::with_speculation's
 * `context` and `draft + 1` (forward.rs:445-491). */
typedef struct {
    int32_t n_full;      /* full-attention layers (KV caches) */
    int32_t n_linear;    /* DeltaNet layers (conv + recurrent state rings) */
    int32_t n_head;      /* 16 */
    int32_t n_head_kv;   /* 4 */
    int32_t head_dim;    /* 256 */
    int32_t n_rot;       /* 64 */
    float rope_theta;    /* 1e7 */
    float rms_eps;       /* 1e-6 */
    int32_t d_state;     /* 128 */
    int32_t n_k_heads;   /* 16 */
    int32_t n_v_heads;   /* 32 */
    int32_t conv_kernel; /* 4 */
    int32_t context;     /* positions per KV cache */
    int32_t slots;       /* ring slots of the DeltaNet state: draft + 1 */
    int32_t kv_dtype;    /* rl_kv_dtype */
    int32_t max_batch;   /* most rows one call may carry (sizes the scratch) */
} rl_config;

/* Allocates the caches and scratch on `device` and zeroes them
 * (Runner::with_speculation, forward.rs:445-491). */
int rl_ctx_create(int device, const rl_config *cfg, rl_ctx **out);
/* Frees everything the context owns.  NULL is a no-op. */
void rl_ctx_destroy(rl_ctx *ctx);
/* The last error on `ctx`, or on the calling thread if ctx is NULL.  Never NULL. */
const char *rl_last_error(const rl_ctx *ctx);

/* Enqueue on `stream` (a cudaStream_t) instead of the context's own stream. */
int rl_set_stream(rl_ctx *ctx, void *stream);
void *rl_get_stream(const rl_ctx *ctx);

/* Zeroes the KV, conv and recurrent state and sets pos = live = 0
 * (Runner::reset, forward.rs:558-577). */
int rl_reset(rl_ctx *ctx);

/* Per-layer weights, copied once from host memory.
 * full:   q_norm, k_norm [head_dim] (FullBlock, model.rs:187-198)
 * linear: conv1d [conv_dim][conv_kernel], ssm_a [n_v] (already -exp(A_log)),
 *         dt_bias [n_v], norm [d_state] (LinearBlock, model.rs:200-216) */
int rl_set_weights_full(rl_ctx *ctx, int layer, const float *q_norm, const float *k_norm);
int rl_set_weights_linear(rl_ctx *ctx, int layer, const float *conv1d, const float *ssm_a,
                          const float *dt_bias, const float *norm);

/*
 * Full attention for t rows at positions pos..pos+t-1 of full layer `layer`
 * (Exec::full_attn's span forward.rs:1259-1340, called from Runner::run at
 * forward.rs:850-855 with caches.pos): per-head q/k RMSNorm and RoPE, KV
 * append, causal attention of row i over pos+i+1 positions, sigmoid output
 * gate, transpose.
 *   qg  [t][n_head][2*head_dim]  query | gate per head (the attn_q output)
 *   k,v [t][n_head_kv][head_dim]
 *   out [t][n_head*head_dim]     the `heads` buffer attn_output reads
 * t = 1 runs split-KV flash decoding; larger t runs the same split-KV walk
 * per row, or the tcgen05 prefill kernel from RL_OPT_PREFILL_ROWS rows on.
 */
int rl_full_attn(rl_ctx *ctx, int layer, int pos, int t, const float *qg, const float *k,
                 const float *v, float *out);
int rl_full_attn_host(rl_ctx *ctx, int layer, int pos, int t, const float *qg, const float *k,
                      const float *v, float *out);

/*
 * Gated DeltaNet for t sequential rows of linear layer `layer`
 * (Exec::linear_attn's span forward.rs:1530-1652, called at forward.rs:856-864
 * with caches.live): row i reads ring slot (live+i)%slots and writes
 * (live+i+1)%slots; with slots == 1 the state is updated in place.
 *   qkv   [t][conv_dim]    conv_dim = 2*n_k*d_state + n_v*d_state
 *   z     [t][n_v*d_state] output-gate logits
 *   alpha [t][n_v]         raw, before softplus(alpha + dt_bias)*ssm_a
 *   beta  [t][n_v]         raw, before the sigmoid
 *   out   [t][n_v*d_state]
 */
int rl_linear_attn(rl_ctx *ctx, int layer, int live, int t, const float *qkv, const float *z,
                   const float *alpha, const float *beta, float *out);
int rl_linear_attn_host(rl_ctx *ctx, int layer, int live, int t, const float *qkv,
                        const float *z, const float *alpha, const float *beta, float *out);

/*
 * A sequence split across GPUs (long-context decode).  Each GPU's context
 * holds positions lo .. lo + context - 1 of a sequence of seq_context
 * positions (rl_set_shard; bf16 caches).  For one decode row at sequence
 * position pos, rl_full_attn_partial walks this GPU's positions <= pos
 * (appending the new key and value only on the GPU whose shard holds pos)
 * and writes the shard's partial [n_head][head_dim + 2]: the unnormalised
 * output, the running max (log2 units) and the sum of weights.  Once the
 * callers have gathered every GPU's partial into parts [n_parts][n_head]
 * [head_dim + 2] (an all-gather over NCCL), rl_merge_partials merges them
 * with the log-sum-exp rule and applies the sigmoid output gate, giving the
 * `heads` row rl_full_attn would have given (forward.rs:1259-1340).  All
 * pointers are device pointers.  A sharded context refuses rl_full_attn.
 */
int rl_set_shard(rl_ctx *ctx, int lo, int seq_context);
/*
 * The same decode row with the exchange over peer memory instead of NCCL:
 * every GPU's merge pushes its partial into a slot of every GPU's exchange
 * buffer (NVLink stores) and then raises its flag there; each GPU's merge
 * kernel waits (bounded) for all flags of the step and merges from its own
 * memory.  Set-up, once per context: rl_exchange_init(rank, world) allocates
 * this GPU's buffer and writes its CUDA IPC handle (RL_IPC_HANDLE_BYTES);
 * the callers exchange the handles (any host channel, in rank order) and
 * call rl_exchange_connect with all of them.  rl_exchange_connect_ptrs
 * takes device pointers instead (contexts of one process, e.g. shards
 * emulated on one GPU: publish on every shard before merging on any).  Each
 * step every GPU calls rl_split_publish then rl_split_merge (or
 * rl_full_attn_split, both); all GPUs take the same steps.
 */
#define RL_IPC_HANDLE_BYTES 64
#define RL_EXCHANGE_MAX_GPUS 8
int rl_exchange_init(rl_ctx *ctx, int rank, int world, void *handle_out);
int rl_exchange_connect(rl_ctx *ctx, const void *handles);
int rl_exchange_connect_ptrs(rl_ctx *ctx, const uint64_t *bufs);
uint64_t rl_exchange_buffer(const rl_ctx *ctx);
int rl_split_publish(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                     const float *v);
int rl_split_merge(rl_ctx *ctx, const float *qg, float *out);
int rl_full_attn_split(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                       const float *v, float *out);
int rl_full_attn_partial(rl_ctx *ctx, int layer, int pos, const float *qg, const float *k,
                         const float *v, float *partial);
int rl_merge_partials(rl_ctx *ctx, int n_parts, const float *parts, const float *qg,
                      float *out);

/* Commits `rows` >= 1 rows of the batch that just ran: pos += rows,
 * live = (live + rows) % slots (Runner::accept, forward.rs:675-688). */
int rl_accept(rl_ctx *ctx, int rows);
/* Position of the next token (Runner::pos, forward.rs:553-555); -1 on NULL. */
int rl_pos(const rl_ctx *ctx);
/* Ring slot holding the committed state (Caches::live); -1 on NULL. */
int rl_live(const rl_ctx *ctx);

/* Waits for the context's stream; returns RL_ETIMEOUT / RL_EINVAL when a
 * kernel flagged a bounded wait that gave up or a bad argument on the device. */
int rl_sync(rl_ctx *ctx);

/*
 * Batched decode over many sequences on one GPU (no counterpart in the
 * reference, whose Runner holds one sequence).  rl_batch_create takes n
 * contexts (bf16 caches, same shapes, same device; each its own sequence);
 * rl_batch_full_attn runs one decode row per sequence of a full layer in one
 * walk launch: row i is sequence i at position pos[i] (a device array), with
 * qg [n][n_head][2*hd], k, v [n][n_kv][hd] and out [n][n_head*hd] device
 * arrays.  Each row appends its key and value to its own context, exactly
 * as rl_full_attn(ctxs[i], layer, pos[i], 1, ...) would, and gives the same
 * row.  The batch runs on ctxs[0]'s stream; a batch must not outlive its
 * contexts.
 */
typedef struct rl_batch rl_batch;
int rl_batch_create(rl_ctx *const *ctxs, int n, rl_batch **out);
int rl_batch_full_attn(rl_batch *b, int layer, const int *pos, const float *qg, const float *k,
                       const float *v, float *out);
void rl_batch_destroy(rl_batch *b);

/* Tuning and dispatch knobs (rl_set_option). */
typedef enum {
    RL_OPT_SPLITS = 0,        /* force the KV splits of the decode walk (0: automatic) */
    RL_OPT_PREFILL_ROWS = 1,  /* rows from which full attention takes the tensor-core
                                 prefill kernel (needs a bf16 cache); 0 disables */
    RL_OPT_CHUNK_ROWS = 2,    /* rows from which a DeltaNet call with slots == 1 takes
                                 the chunked tensor-core kernel; 0 disables */
    RL_OPT_CLUSTER = 3,       /* force the cluster size (1, 2, 4, 8) of the f32 decode
                                 walk's splits (0: automatic) */
    RL_OPT_EARLY_TILES = 4,   /* bf16 decode: 64-position tiles a walk CTA streams before
                                 its inputs are loaded (1..3, default 2) */
    RL_OPT_VERIFY_TC = 5,     /* 1 (default): 2..8 rows over a bf16 cache take the
                                 tensor-core verify kernel (bf16 P, the prefill
                                 tolerance); 0: the exact split-KV walk */
    RL_OPT_DN_ROWS = 6,       /* 1 (default): DeltaNet calls outside the chunked prefill
                                 take the rows kernel, each head's state columns split
                                 over a cluster of four CTAs; 0: the one-CTA-per-head
                                 step kernel.  Both run the rows in order and give a
                                 batch the bits of its rows one call at a time. */
    RL_OPT_WAIT_LIMIT_US = 7, /* how long rl_split_merge's kernel waits for the other
                                 GPUs' flags before it gives up, in microseconds
                                 (0, the default: one second).  A wait that gives up
                                 makes the next rl_sync return RL_ETIMEOUT; the
                                 context stays usable. */
    RL_OPT_WALK_SPANS = 8,    /* 1: every bf16 decode walk records its span on the
                                 global timer (RL_PROF_WALK_SPAN); 0 (default): off.
                                 Costs two atomics per CTA. */
    RL_OPT_DN_SCAN_TC = 9,    /* 1 (default): the chunked DeltaNet prefill walks its
                                 chunks with the tcgen05 scan (one CTA per value head,
                                 the state in tensor memory); 0: the mma.sync scan */
    RL_OPT_DN_OVERLAP = 10,   /* 1 (default): the tcgen05 chunk scan runs on a second,
                                 high-priority stream beside the chunk-local kernel,
                                 taking each chunk as its ready flag goes up (forked
                                 from and joined back into the context's stream, so a
                                 CUDA-graph capture of that stream takes both); 0: one
                                 after the other (for a profiler that serialises
                                 kernels, under which the overlapped scan waits in vain
                                 and gives up) */
    RL_OPT_DN_LOCAL_TC = 11   /* 1 (default): the chunked prefill's chunk-local kernel
                                 takes K K^T and Q K^T on tcgen05 (q and k by TMA, one
                                 M = 128 product of [K; Q] against K); 0: on mma.sync */
} rl_option;
int rl_set_option(rl_ctx *ctx, int option, int64_t value);
int64_t rl_get_option(const rl_ctx *ctx, int option);

/* ---- state access (tests, checkpoints, benchmark set-up) --------------
 * `where`: 0 = host pointer, 1 = device pointer.  f32 in the reference's
 * layouts (forward.rs:236-254):
 *   KV   [2][n_head_kv][n][head_dim] for positions p0..p0+n-1 of `layer`
 *   conv [slots][conv_dim][conv_kernel-1] of linear layer `layer`
 *   ssm  [n_v][slots][d_state][d_state]   of linear layer `layer`  */
int rl_write_kv(rl_ctx *ctx, int layer, int p0, int n, const float *src, int where);
int rl_read_kv(rl_ctx *ctx, int layer, int p0, int n, float *dst, int where);
int rl_write_conv(rl_ctx *ctx, int layer, const float *src, int where);
int rl_read_conv(rl_ctx *ctx, int layer, float *dst, int where);
int rl_write_ssm(rl_ctx *ctx, int layer, const float *src, int where);
int rl_read_ssm(rl_ctx *ctx, int layer, float *dst, int where);

/* ---- per-kernel timing (the device side of the reference's Profile,
 * forward.rs:102-233) --------------------------------------------------
 * Launch counts are always kept.  With timing on, every launch of a kernel
 * is bracketed by CUDA events on the context's stream; rl_profile_read
 * waits for the stream and returns the summed event time of the launches
 * recorded since the last rl_profile_reset.  Do not enable it while the
 * stream is being captured into a CUDA graph. */
typedef enum {
    RL_PROF_PROLOGUE = 0, /* q/k norm + RoPE + KV append */
    RL_PROF_DECODE = 1,   /* split-KV attention walk */
    RL_PROF_MERGE = 2,    /* split merge + output gate */
    RL_PROF_DN_STEP = 3,  /* DeltaNet token-sequential step */
    RL_PROF_PREFILL = 4,  /* tensor-core causal prefill attention */
    RL_PROF_DN_CHUNK = 5, /* DeltaNet chunked prefill */
    RL_PROF_VERIFY = 6,   /* tensor-core multi-row verify attention */
    RL_PROF_WALK_SPAN = 7, /* bf16 decode walk, timed on the GPU's global timer from
                              its first CTA's start to its last CTA's end, inside
                              whatever stream or graph it runs in (no events, so
                              programmatic launch overlap is kept); needs
                              RL_OPT_WALK_SPANS = 1 */
    RL_PROF_KERNELS = 8
} rl_prof_kernel;
int rl_profile_enable(rl_ctx *ctx, int on);
int rl_profile_read(rl_ctx *ctx, int kernel, double *total_ms, int64_t *launches);
int rl_profile_reset(rl_ctx *ctx);

/* ---- projections -------------------------------------------------------
 * The matmuls either side of the attention spans (forward.rs:1250, :1342,
 * :1517, :1656 through Exec::matmul_group, :1157-1180), on the device, in the
 * reference's arithmetic: rl_act_quantize is Activations::quantize_batch
 * (crates/llm-core/src/quant.rs:337-372): t rows of k f32 activations
 * (device, [t][k]) to int8 per 256-value super-block; rl_matvec is one weight
 * of the group (Pool::matvec_group, pool.rs:289-342, with the scalar dots of
 * crates/llm-core/src/kernels/mod.rs:245-320): out [t][rows] (device) = W . x
 * for W (device) of GGML type 12 Q4_K, 14 Q6_K or 8 Q8_0, rows of k values in
 * the GGUF block layout, against the activations the last rl_act_quantize
 * left.  Each output is the scalar tier's bit for bit.  rl_act_quantize
 * allocates once, when a batch needs more scratch than any before it (call it
 * at the largest size before capturing a graph). */
int rl_act_quantize(rl_ctx *ctx, const float *x, int t, int k);
int rl_matvec(rl_ctx *ctx, int ggml_type, const void *w, int rows, float *out);
/* The whole group of Exec::matmul_group in one launch: n (1..8) weights that
 * share the activations, e.g. a layer's qg, k and v (forward.rs:1250). */
int rl_matvec_group(rl_ctx *ctx, int n, const int *types, const void *const *ws, const int *rows,
                    float *const *outs);
/* Exec::matmul_group itself (forward.rs:1157-1180): x [t][k] (device)
 * quantized and dotted with the group's n weights in one launch, the same
 * bits as rl_act_quantize followed by rl_matvec_group (which it falls back to
 * when the batch's quantized rows do not fit a CTA's shared memory). */
int rl_matmul_group(rl_ctx *ctx, const float *x, int t, int k, int n, const int *types,
                    const void *const *ws, const int *rows, float *const *outs);

/* ---- full attention without allocation ---------------------------------
 * No counterpart in the reference: its runner owns all of its memory, so it
 * never needed one.  Some callers of this library cannot allocate device
 * memory or hold an rl_ctx: a serving loop that plans every byte up front and
 * must not allocate once tokens are flowing (the reference runner's own
 * "the pass allocates nothing" rule), or a plug-in living inside another
 * framework's memory budget.  This entry point allocates nothing.  The
 * caller passes its own KV cache for one layer (k_cache, v_cache:
 * [n_head_kv][context][head_dim] of cfg->kv_dtype), the layer's q_norm and
 * k_norm ([head_dim], device), the inputs and the output, all device
 * pointers with the layouts of rl_full_attn; only cfg's full-attention
 * fields (n_head, n_head_kv, head_dim, n_rot, rope_theta, rms_eps, context,
 * kv_dtype) are read.  The work is enqueued on `stream` of the current
 * device; the call returns without waiting.
 *
 * Scratch lives in one static device array of RL_NOALLOC_SCRATCH_BYTES per
 * GPU that loads the library, held until the process exits.  A call whose
 * scratch would not fit (many rows at long context) is refused with
 * RL_EINVAL.  Every call shares that array and it keeps the last call's
 * contents (the call clears what must start at zero itself), so calls whose
 * work overlaps on the GPU (other streams, other host threads) race: run them
 * one after another.  The first call on a device, with that device current,
 * resolves the array's device address and the kernels' launch limits; make
 * that first call before any stream capture.  The return code covers
 * argument and launch errors; every pointer must be 16-byte aligned and
 * n_rot a multiple of 16, or the call returns RL_EINVAL before it enqueues
 * anything.  A device-side wait that gives up (about a second) leaves `out`
 * unwritten and sets a sticky status word in the array's last 256 bytes,
 * which rl_noalloc_status reads. */
#define RL_NOALLOC_SCRATCH_BYTES (4u << 20)
int rl_full_attn_noalloc(const rl_config *cfg, void *stream, void *k_cache, void *v_cache,
                         const float *q_norm, const float *k_norm, int pos, int t,
                         const float *qg, const float *k, const float *v, float *out);
/* The device-side status of the rl_full_attn_noalloc calls enqueued on the
 * current device since the last read: waits for `stream`, then returns
 * RL_OK, RL_ETIMEOUT (a kernel's bounded wait gave up, so some `out` is not
 * valid) or RL_EINVAL (a kernel flagged a bad argument), and clears the
 * word.  Allocates nothing.  No counterpart in the reference: it is the
 * no-alloc path's stand-in for the status an rl_ctx keeps (rl_sync). */
int rl_noalloc_status(void *stream);

/* Library version string; never NULL. */
const char *rl_version(void);

#ifdef __cplusplus
}
#endif
#endif /* RLCUDA_H */
