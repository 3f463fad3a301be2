// CPU oracle for the rust-llm attention path.  TEST INFRASTRUCTURE ONLY: the
// checker the CUDA library is compared against, and the timed CPU baseline.
// Nothing in the product links or calls it.
//
// Every function restates one function of the reference's
// crates/rust-llm/src/forward.rs, cited beside it, in the same arithmetic:
// sequential f32 sums from -0.0, f64 where the reference accumulates in f64,
// glibc libm, and no FMA contraction (built with -ffp-contract=off).
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ----------------------------------------------------------------------------
// A persistent worker pool handing out one chunk index at a time from an
// atomic counter, as Pool::chunks does (crates/rust-llm/src/pool.rs:351-390):
// the submitting thread works too, and the call returns once every chunk ran.
class Pool {
  public:
    explicit Pool(int threads) {
        for (int i = 1; i < threads; ++i) workers_.emplace_back([this] { loop(); });
    }
    void run(size_t chunks, const std::function<void(size_t)> &fn) {
        if (workers_.empty() || chunks <= 1) {
            for (size_t i = 0; i < chunks; ++i) fn(i);
            return;
        }
        {
            std::lock_guard<std::mutex> lk(m_);
            fn_ = &fn;
            total_ = chunks;
            next_.store(0);
            pending_ = workers_.size();
            ++generation_;
        }
        cv_.notify_all();
        work();
        std::unique_lock<std::mutex> lk(m_);
        done_.wait(lk, [&] { return pending_ == 0; });
        fn_ = nullptr;
    }

  private:
    void work() {
        size_t i;
        while ((i = next_.fetch_add(1)) < total_) (*fn_)(i);
    }
    void loop() {
        size_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(m_);
            cv_.wait(lk, [&] { return generation_ != seen; });
            seen = generation_;
            lk.unlock();
            work();
            lk.lock();
            if (--pending_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_, done_;
    const std::function<void(size_t)> *fn_ = nullptr;
    size_t total_ = 0;
    std::atomic<size_t> next_{0};
    size_t pending_ = 0;
    size_t generation_ = 0;
};

// One pool per thread count, created on first use and kept for the life of
// the process (its workers park on a condition variable between calls).
Pool &pool_for(int threads) {
    static std::mutex m;
    static std::map<int, Pool *> pools;
    std::lock_guard<std::mutex> lk(m);
    if (threads < 1) threads = 1;
    auto it = pools.find(threads);
    if (it != pools.end()) return *it->second;
    Pool *p = new Pool(threads);  // never destroyed: workers live until exit
    pools[threads] = p;
    return *p;
}

inline float round_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return x;  // NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// TILE of forward.rs:1756: positions a tile of the KV walk covers.
constexpr size_t TILE = 128;
// J_BLOCK of forward.rs:1887: output components the recurrence takes at a time.
constexpr size_t J_BLOCK = 64;

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Seeded inputs.  SplitMix64 (Steele, Lea, Flood 2014) expands the seed into
// the 256-bit state of xoshiro256** (Blackman and Vigna 2018).
void orc_rng_seed(uint64_t s[4], uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; ++i) {
        uint64_t z = (x += 0x9e3779b97f4a7c15ull);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        s[i] = z ^ (z >> 31);
    }
}

static inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t orc_rng_next(uint64_t s[4]) {
    const uint64_t result = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
}

void orc_fill_normal(uint64_t s[4], float *out, size_t n, double mu, double sigma) {
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        // u1 in (0, 1] so the log is finite; u2 in [0, 1).
        double u1 = (double)((orc_rng_next(s) >> 11) + 1) * 0x1.0p-53;
        double u2 = (double)(orc_rng_next(s) >> 11) * 0x1.0p-53;
        double r = std::sqrt(-2.0 * std::log(u1));
        out[i] = (float)(mu + sigma * r * std::cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)(mu + sigma * r * std::sin(two_pi * u2));
    }
}

void orc_fill_uniform(uint64_t s[4], float *out, size_t n, float a, float b) {
    for (size_t i = 0; i < n; ++i) {
        double u = (double)(orc_rng_next(s) >> 40) * 0x1.0p-24;
        out[i] = (float)((double)a + ((double)b - (double)a) * u);
    }
}

// forward.rs:2288-2298 (the tests' `noise`): xorshift64*, 23 bits onto [-1, 1).
void orc_noise(uint64_t *state, float *out, size_t n) {
    uint64_t x = *state;
    for (size_t i = 0; i < n; ++i) {
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        out[i] = ((float)((x * 0x2545f4914f6cdd1dull) >> 41) / 4194304.0f) - 1.0f;
    }
    *state = x;
}

void orc_round_bf16(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = round_bf16(x[i]);
}

// ---------------------------------------------------------------------------
// forward.rs:1697-1711 `rms_scale`: squares in f32, summed in f64, the mean
// rounded to f32 before eps is added, an f32 root and an f32 reciprocal.
float orc_rms_scale(const float *x, size_t n, float eps) {
    double sum = -0.0;
    for (size_t i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    float mean = (float)(sum / (double)n);
    return 1.0f / std::sqrt(mean + eps);
}

// forward.rs:1683-1688 `rms_norm`: out = (x * scale) * w.
void orc_rms_norm(const float *x, const float *w, size_t n, float eps, float *out) {
    float scale = orc_rms_scale(x, n, eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

// forward.rs:1690-1695 `rms_norm_in_place`.
void orc_rms_norm_in_place(float *x, const float *w, size_t n, float eps) {
    float scale = orc_rms_scale(x, n, eps);
    for (size_t i = 0; i < n; ++i) x[i] = x[i] * scale * w[i];
}

// forward.rs:1720-1727 `l2_norm_in_place`: rms_scale with eps/n, then a
// separate 1/sqrt(n), applied one after the other.
void orc_l2_norm_in_place(float *x, size_t n, float eps) {
    float nf = (float)n;
    float scale = orc_rms_scale(x, n, eps / nf);
    float shrink = 1.0f / std::sqrt(nf);
    for (size_t i = 0; i < n; ++i) x[i] = (x[i] * scale) * shrink;
}

// forward.rs:1730-1743.
float orc_silu(float x) { return x / (1.0f + std::exp(-x)); }
float orc_sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }
float orc_softplus(float x) { return x > 20.0f ? x : std::log1p(std::exp(x)); }

// forward.rs:1746 `dot`: a sequential f32 sum.
float orc_dot(const float *a, const float *b, size_t n) {
    float s = -0.0f;
    for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

// forward.rs:1851-1862 `rope`: pairs (i, i + n_rot/2) for i < n_rot/2, the
// angle advanced by repeated f32 multiplication.
void orc_rope(float *x, size_t pos, size_t n_rot, float theta_base) {
    size_t half = n_rot / 2;
    float theta_scale = std::pow(theta_base, -2.0f / (float)n_rot);
    float theta = (float)pos;
    for (size_t i = 0; i < half; ++i) {
        float c = std::cos(theta), s = std::sin(theta);
        float x0 = x[i], x1 = x[i + half];
        x[i] = x0 * c - x1 * s;
        x[i + half] = x0 * s + x1 * c;
        theta *= theta_scale;
    }
}

// forward.rs:1831-1842 `softmax`: f32 exp, f64 sum from 0.0, the reciprocal
// rounded to f32 before it is applied.
void orc_softmax(float *x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, x[i]);
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) {
        x[i] = std::exp(x[i] - mx);
        sum += (double)x[i];
    }
    float inv = (float)(1.0 / sum);
    for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

// forward.rs:2091-2104 (tests): one query, one score row, one softmax, one
// pass over the values.
void orc_attend(const float *q, const float *k, const float *v, size_t n_kv, size_t hd,
                float scale, float *out) {
    std::vector<float> scores(n_kv);
    for (size_t p = 0; p < n_kv; ++p) scores[p] = orc_dot(q, k + p * hd, hd) * scale;
    orc_softmax(scores.data(), n_kv);
    for (size_t d = 0; d < hd; ++d) out[d] = 0.0f;
    for (size_t p = 0; p < n_kv; ++p) {
        float w = scores[p];
        const float *vp = v + p * hd;
        for (size_t d = 0; d < hd; ++d) out[d] += w * vp[d];
    }
}

// forward.rs:1783-1826 `attend_batch`: the tiled walk with materialised score
// rows; query i attends over pos+i+1 positions.
void orc_attend_batch(const float *q, size_t q_stride, const float *k, const float *v,
                      size_t t, size_t pos, size_t hd, float scale, size_t row,
                      float *scores, float *out) {
    size_t n_kv = pos + t;
    for (size_t base = 0; base < n_kv; base += TILE) {
        size_t tile = std::min(base + TILE, n_kv);
        for (size_t i = 0; i < t; ++i) {
            size_t upto = std::min(tile, pos + i + 1);
            const float *qi = q + i * q_stride;
            for (size_t p = base; p < upto; ++p)
                scores[i * row + p] = orc_dot(qi, k + p * hd, hd) * scale;
        }
    }
    for (size_t i = 0; i < t; ++i) orc_softmax(scores + i * row, pos + i + 1);
    for (size_t e = 0; e < t * hd; ++e) out[e] = 0.0f;
    for (size_t base = 0; base < n_kv; base += TILE) {
        size_t tile = std::min(base + TILE, n_kv);
        for (size_t i = 0; i < t; ++i) {
            size_t upto = std::min(tile, pos + i + 1);
            float *o = out + i * hd;
            for (size_t p = base; p < upto; ++p) {
                float w = scores[i * row + p];
                const float *vp = v + p * hd;
                for (size_t d = 0; d < hd; ++d) o[d] += w * vp[d];
            }
        }
    }
}

// forward.rs:1906-1950 `delta_net`: blocked over output components j, each
// j's two reductions over i serial and ascending.
void orc_delta_net(float *state, const float *q, const float *k, const float *v, float g,
                   float beta, float scale, float *out, size_t s) {
    float sk[J_BLOCK], d[J_BLOCK], o[J_BLOCK];
    for (size_t j0 = 0; j0 < s; j0 += J_BLOCK) {
        size_t w = std::min(J_BLOCK, s - j0);
        for (size_t j = 0; j < w; ++j) sk[j] = 0.0f, o[j] = 0.0f;
        for (size_t i = 0; i < s; ++i) {
            float ki = k[i];
            float *r = state + i * s + j0;
            for (size_t j = 0; j < w; ++j) {
                r[j] *= g;
                sk[j] += r[j] * ki;
            }
        }
        for (size_t j = 0; j < w; ++j) d[j] = (v[j0 + j] - sk[j]) * beta;
        for (size_t i = 0; i < s; ++i) {
            float ki = k[i], qi = q[i];
            float *r = state + i * s + j0;
            for (size_t j = 0; j < w; ++j) {
                r[j] += d[j] * ki;
                o[j] += r[j] * qi;
            }
        }
        for (size_t j = 0; j < w; ++j) out[j0 + j] = o[j] * scale;
    }
}

// forward.rs:1964-2010 `delta_net_into`: the same arithmetic reading prev and
// writing next.
void orc_delta_net_into(const float *prev, float *next, const float *q, const float *k,
                        const float *v, float g, float beta, float scale, float *out,
                        size_t s) {
    float sk[J_BLOCK], d[J_BLOCK], o[J_BLOCK];
    for (size_t j0 = 0; j0 < s; j0 += J_BLOCK) {
        size_t w = std::min(J_BLOCK, s - j0);
        for (size_t j = 0; j < w; ++j) sk[j] = 0.0f, o[j] = 0.0f;
        for (size_t i = 0; i < s; ++i) {
            float ki = k[i];
            const float *p = prev + i * s + j0;
            float *r = next + i * s + j0;
            for (size_t j = 0; j < w; ++j) {
                r[j] = p[j] * g;
                sk[j] += r[j] * ki;
            }
        }
        for (size_t j = 0; j < w; ++j) d[j] = (v[j0 + j] - sk[j]) * beta;
        for (size_t i = 0; i < s; ++i) {
            float ki = k[i], qi = q[i];
            float *r = next + i * s + j0;
            for (size_t j = 0; j < w; ++j) {
                r[j] += d[j] * ki;
                o[j] += r[j] * qi;
            }
        }
        for (size_t j = 0; j < w; ++j) out[j0 + j] = o[j] * scale;
    }
}

// forward.rs:2116-2141 (tests) `delta_net_scalar`, on the [j][i] layout.
void orc_delta_net_scalar(float *state, const float *q, const float *k, const float *v,
                          float g, float beta, float scale, float *out, size_t s) {
    for (size_t j = 0; j < s; ++j) {
        float *srow = state + j * s;
        float sk = 0.0f;
        for (size_t i = 0; i < s; ++i) {
            srow[i] *= g;
            sk += srow[i] * k[i];
        }
        float d = (v[j] - sk) * beta;
        float o = 0.0f;
        for (size_t i = 0; i < s; ++i) {
            srow[i] += d * k[i];
            o += srow[i] * q[i];
        }
        out[j] = o * scale;
    }
}

// forward.rs:2018-2031 `depthwise_conv`: out = x*w[hist] + sum_j h[j]*w[j];
// the history rotates left and takes the new sample last.
void orc_depthwise_conv(const float *x, const float *w, size_t kernel, float *state,
                        float *out, size_t channels) {
    size_t hist = kernel - 1;
    for (size_t c = 0; c < channels; ++c) {
        const float *taps = w + c * kernel;
        float *h = state + c * hist;
        float sum = x[c] * taps[hist];
        for (size_t j = 0; j < hist; ++j) sum += h[j] * taps[j];
        out[c] = sum;
        for (size_t j = 0; j + 1 < hist; ++j) h[j] = h[j + 1];
        h[hist - 1] = x[c];
    }
}

// forward.rs:2038-2059 `depthwise_conv_into`.
void orc_depthwise_conv_into(const float *x, const float *w, size_t kernel,
                             const float *prev, float *next, float *out, size_t channels) {
    size_t hist = kernel - 1;
    for (size_t c = 0; c < channels; ++c) {
        const float *taps = w + c * kernel;
        const float *h = prev + c * hist;
        float sum = x[c] * taps[hist];
        for (size_t j = 0; j < hist; ++j) sum += h[j] * taps[j];
        out[c] = sum;
        float *to = next + c * hist;
        for (size_t j = 0; j + 1 < hist; ++j) to[j] = h[j + 1];
        to[hist - 1] = x[c];
    }
}

// ---------------------------------------------------------------------------
// forward.rs:1259-1340, the hot span of Exec::full_attn.
void orc_full_attn(const orc_config *c, size_t pos, size_t t, float *qg, float *k,
                   const float *v, float *kv, const float *q_norm, const float *k_norm,
                   float *out, int threads) {
    const size_t hd = c->head_dim, n_head = c->n_head, n_kv = c->n_head_kv;
    const size_t group = n_head / n_kv, context = c->context;
    const size_t qg_dim = 2 * hd * n_head, kv_dim = hd * n_kv, attn_dim = hd * n_head;
    // q/k norm and rope per row (forward.rs:1261-1277)
    for (size_t i = 0; i < t; ++i) {
        size_t p = pos + i;
        for (size_t h = 0; h < n_head; ++h) {
            float *q = qg + i * qg_dim + h * 2 * hd;
            orc_rms_norm_in_place(q, q_norm, hd, c->rms_eps);
            orc_rope(q, p, c->n_rot, c->rope_theta);
        }
        for (size_t h = 0; h < n_kv; ++h) {
            float *kk = k + i * kv_dim + h * hd;
            orc_rms_norm_in_place(kk, k_norm, hd, c->rms_eps);
            orc_rope(kk, p, c->n_rot, c->rope_theta);
        }
    }
    // append (forward.rs:1281-1292)
    float *k_cache = kv, *v_cache = kv + n_kv * context * hd;
    for (size_t i = 0; i < t; ++i)
        for (size_t h = 0; h < n_kv; ++h) {
            size_t to = (h * context + pos + i) * hd, from = i * kv_dim + h * hd;
            for (size_t d = 0; d < hd; ++d) {
                float kd = k[from + d], vd = v[from + d];
                if (c->kv_bf16) kd = round_bf16(kd), vd = round_bf16(vd);
                k_cache[to + d] = kd;
                v_cache[to + d] = vd;
            }
        }
    // attention, one head per chunk (forward.rs:1294-1322)
    const float scale = 1.0f / std::sqrt((float)hd);
    std::vector<float> head_major(n_head * t * hd);
    std::vector<float> scores(n_head * t * context);
    pool_for(threads).run(n_head, [&](size_t h) {
        size_t kh = h / group;
        orc_attend_batch(qg + h * 2 * hd, qg_dim, k_cache + kh * context * hd,
                         v_cache + kh * context * hd, t, pos, hd, scale, context,
                         scores.data() + h * t * context, head_major.data() + h * t * hd);
    });
    // sigmoid gate and transpose (forward.rs:1327-1340)
    for (size_t i = 0; i < t; ++i)
        for (size_t h = 0; h < n_head; ++h) {
            const float *gate = qg + i * qg_dim + h * 2 * hd + hd;
            const float *from = head_major.data() + (h * t + i) * hd;
            float *into = out + i * attn_dim + h * hd;
            for (size_t d = 0; d < hd; ++d) into[d] = from[d] * orc_sigmoid(gate[d]);
        }
}

// forward.rs:1530-1652, the hot span of Exec::linear_attn.
void orc_linear_attn(const orc_config *c, size_t slots, size_t live, size_t t,
                     const float *qkv, const float *z, const float *alpha,
                     const float *beta_raw, float *conv_state, float *ssm_state,
                     const float *conv1d, const float *ssm_a, const float *dt_bias,
                     const float *norm, float *out, int threads) {
    const size_t s = c->d_state, n_kh = c->n_k_heads, n_vh = c->n_v_heads;
    const size_t key_dim = s * n_kh, d_inner = s * n_vh, conv_dim = 2 * key_dim + d_inner;
    const size_t kernel = c->conv_kernel, conv_span = conv_dim * (kernel - 1);
    // gates (forward.rs:1530-1546)
    std::vector<float> decay(t * n_vh), beta(t * n_vh);
    for (size_t i = 0; i < t; ++i)
        for (size_t h = 0; h < n_vh; ++h) {
            decay[i * n_vh + h] = orc_softplus(alpha[i * n_vh + h] + dt_bias[h]) * ssm_a[h];
            beta[i * n_vh + h] = orc_sigmoid(beta_raw[i * n_vh + h]);
        }
    // convolution over the ring, row by row (forward.rs:1548-1567)
    std::vector<float> conv(t * conv_dim);
    for (size_t i = 0; i < t; ++i) {
        size_t from = (live + i) % slots, to = (live + i + 1) % slots;
        if (from == to)
            orc_depthwise_conv(qkv + i * conv_dim, conv1d, kernel,
                               conv_state + from * conv_span, conv.data() + i * conv_dim,
                               conv_dim);
        else
            orc_depthwise_conv_into(qkv + i * conv_dim, conv1d, kernel,
                                    conv_state + from * conv_span,
                                    conv_state + to * conv_span, conv.data() + i * conv_dim,
                                    conv_dim);
    }
    for (auto &x : conv) x = orc_silu(x);  // forward.rs:1569
    // q/k L2 norm (forward.rs:1577-1584)
    for (size_t i = 0; i < t; ++i)
        for (size_t h = 0; h < 2 * n_kh; ++h)
            orc_l2_norm_in_place(conv.data() + i * conv_dim + h * s, s, c->rms_eps);
    // recurrence, one value head per chunk (forward.rs:1586-1631)
    const float scale = 1.0f / std::sqrt((float)s);
    std::vector<float> head_major(n_vh * t * s);
    pool_for(threads).run(n_vh, [&](size_t vh) {
        size_t kh = vh % n_kh;
        float *ring = ssm_state + vh * slots * s * s;
        for (size_t i = 0; i < t; ++i) {
            const float *row = conv.data() + i * conv_dim;
            const float *q = row + kh * s;
            const float *kk = row + key_dim + kh * s;
            const float *vv = row + 2 * key_dim + vh * s;
            float g = std::exp(decay[i * n_vh + vh]);
            float b = beta[i * n_vh + vh];
            float *o = head_major.data() + (vh * t + i) * s;
            size_t from = (live + i) % slots, to = (live + i + 1) % slots;
            if (from == to)
                orc_delta_net(ring + from * s * s, q, kk, vv, g, b, scale, o, s);
            else
                orc_delta_net_into(ring + from * s * s, ring + to * s * s, q, kk, vv, g, b,
                                   scale, o, s);
        }
    });
    // gated norm (forward.rs:1642-1652)
    for (size_t i = 0; i < t; ++i)
        for (size_t h = 0; h < n_vh; ++h) {
            float *head = out + i * d_inner + h * s;
            orc_rms_norm(head_major.data() + (h * t + i) * s, norm, s, c->rms_eps, head);
            const float *zz = z + i * d_inner + h * s;
            for (size_t j = 0; j < s; ++j) head[j] *= orc_silu(zz[j]);
        }
}

// ---- projections: int8 activations against k-quant weight rows ----------
// crates/llm-core/src/quant.rs (read_f16 :120-122, q4k_scale_min :215-226,
// Activations::quantize_batch :337-372) and the scalar tier of
// crates/llm-core/src/kernels/mod.rs (matvec_row :218-243, q4k_dot_scalar
// :245-271, q6k_dot_scalar :273-301, q80_dot_scalar :303-320).

// The reference kernel tests' xorshift64* stream (crates/llm-core/tests/
// kernels.rs:48-61), n raw outputs; *state is the generator's state.
void orc_xorshift_stream(uint64_t *state, uint64_t *out, size_t n) {
    uint64_t x = *state;
    for (size_t i = 0; i < n; ++i) {
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        out[i] = x * 0x2545F4914F6CDD1Dull;
    }
    *state = x;
}

// half::f16::to_f32: IEEE binary16 to binary32, exact (subnormals included).
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            // subnormal: m * 2^-24, exact in f32
            float f = (float)m * 0x1p-24f;
            std::memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float out;
    std::memcpy(&out, &bits, 4);
    return out;
}

static float rd16(const uint8_t *b, size_t off) {
    return orc_f16_to_f32((uint16_t)(b[off] | (b[off + 1] << 8)));
}

static void scale_min_k4(size_t j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

void orc_q8k_quantize(const float *x, size_t k, size_t t, float *d, int8_t *qs, int16_t *bsums) {
    const size_t nb = (k + 255) / 256;
    for (size_t r = 0; r < t; ++r) {
        for (size_t b = 0; b < nb; ++b) {
            const float *chunk = x + r * k + b * 256;
            const size_t n = std::min<size_t>(256, k - b * 256);
            float amax = 0.0f;  // fold(0.0, |m, v| m.max(v.abs()))
            for (size_t i = 0; i < n; ++i) amax = std::fmax(amax, std::fabs(chunk[i]));
            const size_t blk = r * nb + b;
            d[blk] = amax / 127.0f;
            const float id = amax > 0.0f ? 127.0f / amax : 0.0f;
            int8_t *q = qs + blk * 256;
            for (size_t i = 0; i < 256; ++i) q[i] = 0;
            for (size_t i = 0; i < n; ++i) {
                float v = std::round(chunk[i] * id);  // round half away from zero
                v = std::fmin(std::fmax(v, -127.0f), 127.0f);
                q[i] = (int8_t)v;
            }
            for (size_t g = 0; g < 16; ++g) {
                int s16 = 0;
                for (size_t i = 0; i < 16; ++i) s16 += q[g * 16 + i];
                bsums[blk * 16 + g] = (int16_t)s16;
            }
        }
    }
}

float orc_dot_q4k(const uint8_t *w, const float *ad, const int8_t *aq, const int16_t *absums,
                  size_t nb) {
    float sum = 0.0f;
    for (size_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = w + ib * 144;
        const float d = rd16(b, 0), dmin = rd16(b, 2);
        const uint8_t *scales = b + 4, *qs = b + 16;
        const int8_t *qa_blk = aq + ib * 256;
        const int16_t *bs = absums + ib * 16;
        int32_t isum = 0, imin = 0;
        for (size_t j = 0; j < 8; ++j) {
            uint8_t sc, m;
            scale_min_k4(j, scales, &sc, &m);
            const uint8_t *qw = qs + (j / 2) * 32;
            const int8_t *qa = qa_blk + j * 32;
            const int shift = j % 2 == 0 ? 0 : 4;
            int32_t dot = 0;
            for (size_t l = 0; l < 32; ++l) dot += (int32_t)((qw[l] >> shift) & 0xF) * qa[l];
            isum += (int32_t)sc * dot;
            imin += (int32_t)m * ((int32_t)bs[j * 2] + (int32_t)bs[j * 2 + 1]);
        }
        sum += ad[ib] * (d * (float)isum - dmin * (float)imin);
    }
    return sum;
}

float orc_dot_q6k(const uint8_t *w, const float *ad, const int8_t *aq, size_t nb) {
    float sum = 0.0f;
    for (size_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = w + ib * 210;
        const uint8_t *ql = b, *qh = b + 128, *sc = b + 192;
        const float d = rd16(b, 208);
        const int8_t *qa = aq + ib * 256;
        int32_t isum = 0;
        for (size_t h = 0; h < 2; ++h) {
            const uint8_t *ql_h = ql + h * 64, *qh_h = qh + h * 32;
            for (size_t g = 0; g < 4; ++g) {
                for (size_t l = 0; l < 32; ++l) {
                    uint8_t low;
                    switch (g) {
                    case 0: low = ql_h[l] & 0xF; break;
                    case 1: low = ql_h[32 + l] & 0xF; break;
                    case 2: low = ql_h[l] >> 4; break;
                    default: low = ql_h[32 + l] >> 4; break;
                    }
                    const int32_t q = (int32_t)(low | (((qh_h[l] >> (2 * g)) & 3) << 4)) - 32;
                    const int32_t s = (int8_t)sc[h * 8 + 2 * g + l / 16];
                    isum += s * q * qa[h * 128 + g * 32 + l];
                }
            }
        }
        sum += ad[ib] * d * (float)isum;
    }
    return sum;
}

float orc_dot_q80(const uint8_t *w, const float *ad, const int8_t *aq, size_t k) {
    float sum = 0.0f;
    for (size_t ib = 0; ib < (k + 31) / 32; ++ib) {
        const uint8_t *b = w + ib * 34;
        const float dw = rd16(b, 0);
        const size_t blk = ib / 8;
        const int8_t *qa = aq + blk * 256 + (ib % 8) * 32;
        int32_t dot = 0;
        for (size_t l = 0; l < 32; ++l) dot += (int32_t)(int8_t)b[2 + l] * qa[l];
        sum += dw * ad[blk] * (float)dot;
    }
    return sum;
}

// Bytes of one weight row of k values (GgmlType::bytes_for, quant.rs).
size_t orc_row_bytes(int type, size_t k) {
    switch (type) {
    case 12: return (k + 255) / 256 * 144;  // Q4_K
    case 14: return (k + 255) / 256 * 210;  // Q6_K
    case 8: return (k + 31) / 32 * 34;      // Q8_0
    default: return 0;
    }
}

// Exec::matmul_group's per-weight product (forward.rs:1157-1180 through
// Pool::matvec_group, pool.rs:289-342): the rows quantized once, then
// out[tt][r] = row r . row tt of the activations, token-major.
int orc_matvec(int type, const uint8_t *w, size_t rows, size_t k, const float *x, size_t t,
               float *out, int threads) {
    const size_t stride = orc_row_bytes(type, k);
    if (!stride) return -1;
    const size_t nb = (k + 255) / 256;
    std::vector<float> d(t * nb);
    std::vector<int8_t> qs(t * nb * 256);
    std::vector<int16_t> bs(t * nb * 16);
    orc_q8k_quantize(x, k, t, d.data(), qs.data(), bs.data());
    const size_t chunk = 256;
    pool_for(threads).run((rows + chunk - 1) / chunk, [&](size_t c) {
        for (size_t r = c * chunk; r < std::min(rows, (c + 1) * chunk); ++r) {
            const uint8_t *row = w + r * stride;
            for (size_t tt = 0; tt < t; ++tt) {
                const float *ad = d.data() + tt * nb;
                const int8_t *aq = qs.data() + tt * nb * 256;
                float v;
                if (type == 12) v = orc_dot_q4k(row, ad, aq, bs.data() + tt * nb * 16, nb);
                else if (type == 14) v = orc_dot_q6k(row, ad, aq, nb);
                else v = orc_dot_q80(row, ad, aq, k);
                out[tt * rows + r] = v;
            }
        }
    });
    return 0;
}

}  // extern "C"
