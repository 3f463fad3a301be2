/*
 * CPU oracle for the rust-llm attention path.  TEST INFRASTRUCTURE ONLY.
 *
 * A C++ restatement of the attention functions of the reference's
 * crates/rust-llm/src/forward.rs (gated GQA full attention and the Gated
 * DeltaNet), written to be bit-faithful to the Rust build:
 *   - f32 iterator sums are strictly sequential and start from -0.0, as
 *     Rust's `impl Sum for f32/f64` does;
 *   - f64 accumulation exactly where the reference uses it (softmax sum,
 *     RMS sum of squares);
 *   - no FMA contraction (the library is compiled with -ffp-contract=off,
 *     because rustc never fuses a multiply and an add);
 *   - exp / ln_1p / powf / sin / cos are glibc's expf, log1pf, powf, sinf,
 *     cosf, which is what Rust's std calls on Linux.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker or the timed CPU baseline; the CUDA
 * library never links or calls it.
 *
 * Parity pinning: the reference ships no golden attention or DeltaNet output
 * vectors.  The restatement is pinned by the reference's own known-answer and
 * relation tests (forward.rs:2159-2561), replayed in tests/test_oracle_kats.py
 * with the same xorshift64* case generator (forward.rs:2288-2298).
 */
#ifndef RL_ORACLE_H
#define RL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Shapes, mirroring the fields of Config (crates/rust-llm/src/model.rs:41-66)
 * that the attention path reads. */
typedef struct {
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
    int32_t context;     /* positions the KV cache holds */
    int32_t kv_bf16;     /* 1: keys/values appended to the cache are rounded to
                            bf16 first, as a bf16 device cache stores them */
} orc_config;

/* ---- seeded input generator (SplitMix64-seeded xoshiro256**) ---------- */
void orc_rng_seed(uint64_t state[4], uint64_t seed);
uint64_t orc_rng_next(uint64_t state[4]);
/* N(mu, sigma) by Box-Muller in f64, both outputs of a pair used, cast to f32. */
void orc_fill_normal(uint64_t state[4], float *out, size_t n, double mu, double sigma);
/* U[a, b) from 24-bit uniforms. */
void orc_fill_uniform(uint64_t state[4], float *out, size_t n, float a, float b);
/* The reference tests' xorshift64* noise in [-1, 1) (forward.rs:2288-2298). */
void orc_noise(uint64_t *x, float *out, size_t n);
/* Round-to-nearest-even f32 -> bf16 -> f32, elementwise, in place. */
void orc_round_bf16(float *x, size_t n);

/* ---- primitives (forward.rs:1683-1748, 1783-1862, 1906-2076) ---------- */
float orc_rms_scale(const float *x, size_t n, float eps);
void orc_rms_norm(const float *x, const float *w, size_t n, float eps, float *out);
void orc_rms_norm_in_place(float *x, const float *w, size_t n, float eps);
void orc_l2_norm_in_place(float *x, size_t n, float eps);
float orc_silu(float x);
float orc_sigmoid(float x);
float orc_softplus(float x);
float orc_dot(const float *a, const float *b, size_t n);
void orc_rope(float *x, size_t pos, size_t n_rot, float theta_base);
void orc_softmax(float *x, size_t n);
/* the tests' naive one-query attention (forward.rs:2091-2104) */
void orc_attend(const float *q, const float *k, const float *v, size_t n_kv, size_t hd,
                float scale, float *out);
/* the product's tiled batch attention (forward.rs:1783-1826) */
void orc_attend_batch(const float *q, size_t q_stride, const float *k, const float *v,
                      size_t t, size_t pos, size_t hd, float scale, size_t row,
                      float *scores, float *out);
void orc_delta_net(float *state, const float *q, const float *k, const float *v, float g,
                   float beta, float scale, float *out, size_t s);
void orc_delta_net_into(const float *prev, float *next, const float *q, const float *k,
                        const float *v, float g, float beta, float scale, float *out,
                        size_t s);
/* the tests' one-component-at-a-time recurrence on the transposed [j][i]
 * state (forward.rs:2116-2141) */
void orc_delta_net_scalar(float *state, const float *q, const float *k, const float *v,
                          float g, float beta, float scale, float *out, size_t s);
void orc_depthwise_conv(const float *x, const float *w, size_t kernel, float *state,
                        float *out, size_t channels);
void orc_depthwise_conv_into(const float *x, const float *w, size_t kernel,
                             const float *prev, float *next, float *out, size_t channels);

/* ---- the two hot spans ------------------------------------------------ */
/*
 * Exec::full_attn without its projections (forward.rs:1259-1340): per-row
 * q/k RMSNorm and RoPE (qg and k are normalised in place, as the reference
 * does to its buffers), KV append at pos..pos+t, causal attention of every
 * head over pos+i+1 positions, sigmoid gate and transpose.
 *   qg  [t][n_head][2*head_dim]    (query | gate per head)
 *   k,v [t][n_head_kv][head_dim]
 *   kv  [2][n_head_kv][context][head_dim]  (this layer's cache)
 *   out [t][n_head*head_dim]
 * `threads` workers share the heads, one head per claimed chunk, as
 * Pool::chunks does (pool.rs:351-390).
 */
void orc_full_attn(const orc_config *c, size_t pos, size_t t, float *qg, float *k,
                   const float *v, float *kv, const float *q_norm, const float *k_norm,
                   float *out, int threads);

/*
 * Exec::linear_attn without its projections (forward.rs:1530-1652): decay and
 * beta gates, depthwise conv over the ring, SiLU, q/k L2 norm, the delta rule
 * per value head over ring slots (live+i)%slots -> (live+i+1)%slots, gated
 * RMSNorm.
 *   qkv   [t][conv_dim]   conv_dim = 2*n_k*d_state + n_v*d_state
 *   z     [t][n_v*d_state]
 *   alpha [t][n_v]  raw (before softplus), beta [t][n_v] raw (before sigmoid)
 *   conv_state [slots][conv_dim][conv_kernel-1]
 *   ssm_state  [n_v][slots][d_state][d_state]
 *   conv1d [conv_dim][conv_kernel], ssm_a [n_v] (= -exp(A_log)),
 *   dt_bias [n_v], norm [d_state]
 *   out [t][n_v*d_state]
 */
void orc_linear_attn(const orc_config *c, size_t slots, size_t live, size_t t,
                     const float *qkv, const float *z, const float *alpha,
                     const float *beta, float *conv_state, float *ssm_state,
                     const float *conv1d, const float *ssm_a, const float *dt_bias,
                     const float *norm, float *out, int threads);

/* ---- projections (crates/llm-core/src/quant.rs, kernels/mod.rs) -------- */
/* GGML type ids: 8 Q8_0, 12 Q4_K, 14 Q6_K (quant.rs:36-70). */
float orc_f16_to_f32(uint16_t h);
/* n raw outputs of the reference kernel tests' xorshift64* generator. */
void orc_xorshift_stream(uint64_t *state, uint64_t *out, size_t n);
/* Activations::quantize_batch: t rows of k f32 -> per 256-value super-block
 * d [t][nb], qs [t][nb][256] (tail zero), bsums [t][nb][16]. */
void orc_q8k_quantize(const float *x, size_t k, size_t t, float *d, int8_t *qs, int16_t *bsums);
/* The scalar tier's dot of one weight row with one quantized activation row. */
float orc_dot_q4k(const uint8_t *w, const float *ad, const int8_t *aq, const int16_t *absums,
                  size_t nb);
float orc_dot_q6k(const uint8_t *w, const float *ad, const int8_t *aq, size_t nb);
float orc_dot_q80(const uint8_t *w, const float *ad, const int8_t *aq, size_t k);
size_t orc_row_bytes(int type, size_t k);
/* out [t][rows] = W [rows][k] (type) . x [t][k], activations quantized first. */
int orc_matvec(int type, const uint8_t *w, size_t rows, size_t k, const float *x, size_t t,
               float *out, int threads);

#ifdef __cplusplus
}
#endif
#endif
