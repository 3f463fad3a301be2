"""ctypes bindings for the CPU oracle (liboracle.so).  TEST INFRASTRUCTURE ONLY.

The oracle is a C++ restatement of the reference's attention path
(crates/rust-llm/src/forward.rs).  Only tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` import this module, as the checker or the
timed CPU baseline; the CUDA library neither links nor calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_sz = ctypes.c_size_t


class Config(ctypes.Structure):
    """orc_config: the Config fields (model.rs:41-66) the attention path reads."""

    _fields_ = [
        ("n_head", ctypes.c_int32),
        ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_rot", ctypes.c_int32),
        ("rope_theta", ctypes.c_float),
        ("rms_eps", ctypes.c_float),
        ("d_state", ctypes.c_int32),
        ("n_k_heads", ctypes.c_int32),
        ("n_v_heads", ctypes.c_int32),
        ("conv_kernel", ctypes.c_int32),
        ("context", ctypes.c_int32),
        ("kv_bf16", ctypes.c_int32),
    ]


def qwen35_config(context: int, kv_bf16: bool = False) -> Config:
    """The Qwen3.5-4B attention shapes (docs/models.md:100-105)."""
    return Config(16, 4, 256, 64, 1e7, 1e-6, 128, 16, 32, 4, context, int(kv_bf16))


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_rng_seed.argtypes = [_u64p, ctypes.c_uint64]
        L.orc_rng_next.argtypes = [_u64p]
        L.orc_rng_next.restype = ctypes.c_uint64
        L.orc_fill_normal.argtypes = [_u64p, _f32p, _sz, ctypes.c_double, ctypes.c_double]
        L.orc_fill_uniform.argtypes = [_u64p, _f32p, _sz, ctypes.c_float, ctypes.c_float]
        L.orc_noise.argtypes = [_u64p, _f32p, _sz]
        L.orc_round_bf16.argtypes = [_f32p, _sz]
        L.orc_rms_scale.argtypes = [_f32p, _sz, ctypes.c_float]
        L.orc_rms_scale.restype = ctypes.c_float
        L.orc_rms_norm.argtypes = [_f32p, _f32p, _sz, ctypes.c_float, _f32p]
        L.orc_rms_norm_in_place.argtypes = [_f32p, _f32p, _sz, ctypes.c_float]
        L.orc_l2_norm_in_place.argtypes = [_f32p, _sz, ctypes.c_float]
        for name in ("orc_silu", "orc_sigmoid", "orc_softplus"):
            getattr(L, name).argtypes = [ctypes.c_float]
            getattr(L, name).restype = ctypes.c_float
        L.orc_dot.argtypes = [_f32p, _f32p, _sz]
        L.orc_dot.restype = ctypes.c_float
        L.orc_rope.argtypes = [_f32p, _sz, _sz, ctypes.c_float]
        L.orc_softmax.argtypes = [_f32p, _sz]
        L.orc_attend.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, ctypes.c_float, _f32p]
        L.orc_attend_batch.argtypes = [_f32p, _sz, _f32p, _f32p, _sz, _sz, _sz,
                                       ctypes.c_float, _sz, _f32p, _f32p]
        L.orc_delta_net.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float, _f32p, _sz]
        L.orc_delta_net_into.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
                                         ctypes.c_float, ctypes.c_float, _f32p, _sz]
        L.orc_delta_net_scalar.argtypes = L.orc_delta_net.argtypes
        L.orc_depthwise_conv.argtypes = [_f32p, _f32p, _sz, _f32p, _f32p, _sz]
        L.orc_depthwise_conv_into.argtypes = [_f32p, _f32p, _sz, _f32p, _f32p, _f32p, _sz]
        L.orc_full_attn.argtypes = [ctypes.POINTER(Config), _sz, _sz, _f32p, _f32p, _f32p,
                                    _f32p, _f32p, _f32p, _f32p, ctypes.c_int]
        L.orc_linear_attn.argtypes = [ctypes.POINTER(Config), _sz, _sz, _sz, _f32p, _f32p,
                                      _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                      _f32p, _f32p, ctypes.c_int]
        _i8p = ctypes.POINTER(ctypes.c_int8)
        _i16p = ctypes.POINTER(ctypes.c_int16)
        _u8p = ctypes.POINTER(ctypes.c_uint8)
        L.orc_xorshift_stream.argtypes = [_u64p, _u64p, _sz]
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_q8k_quantize.argtypes = [_f32p, _sz, _sz, _f32p, _i8p, _i16p]
        L.orc_dot_q4k.argtypes = [_u8p, _f32p, _i8p, _i16p, _sz]
        L.orc_dot_q4k.restype = ctypes.c_float
        L.orc_dot_q6k.argtypes = [_u8p, _f32p, _i8p, _sz]
        L.orc_dot_q6k.restype = ctypes.c_float
        L.orc_dot_q80.argtypes = [_u8p, _f32p, _i8p, _sz]
        L.orc_dot_q80.restype = ctypes.c_float
        L.orc_row_bytes.argtypes = [ctypes.c_int, _sz]
        L.orc_row_bytes.restype = _sz
        L.orc_matvec.argtypes = [ctypes.c_int, _u8p, _sz, _sz, _f32p, _sz, _f32p, ctypes.c_int]
        L.orc_matvec.restype = ctypes.c_int
        _lib = L
    return _lib


def P(a: np.ndarray):
    """Pointer to a C-contiguous float32 array."""
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


# ---------------------------------------------------------------------------
# Seeded inputs


class Rng:
    """SplitMix64-seeded xoshiro256**; the draw order is the caller's order."""

    def __init__(self, seed: int):
        self.state = np.zeros(4, dtype=np.uint64)
        lib().orc_rng_seed(self.state.ctypes.data_as(_u64p), seed)

    def normal(self, shape, mu=0.0, sigma=1.0) -> np.ndarray:
        out = np.empty(shape, dtype=np.float32)
        lib().orc_fill_normal(self.state.ctypes.data_as(_u64p), P(out), out.size, mu, sigma)
        return out

    def uniform(self, shape, a, b) -> np.ndarray:
        out = np.empty(shape, dtype=np.float32)
        lib().orc_fill_uniform(self.state.ctypes.data_as(_u64p), P(out), out.size, a, b)
        return out


class Noise:
    """The reference tests' xorshift64* generator (forward.rs:2288-2298)."""

    def __init__(self, seed: int):
        self.x = np.array([seed | 1], dtype=np.uint64)

    def __call__(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().orc_noise(self.x.ctypes.data_as(_u64p), P(out), n)
        return out


def round_bf16(a: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(a, dtype=np.float32).copy()
    lib().orc_round_bf16(P(out), out.size)
    return out


# ---------------------------------------------------------------------------
# Primitives


def rms_scale(x, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    return lib().orc_rms_scale(P(x), x.size, eps)


def l2_norm(x, eps):
    x = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_l2_norm_in_place(P(x), x.size, eps)
    return x


def rope(x, pos, n_rot, theta):
    x = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().orc_rope(P(x), pos, n_rot, theta)
    return x


def softplus(x):
    return lib().orc_softplus(x)


def sigmoid(x):
    return lib().orc_sigmoid(x)


def silu(x):
    return lib().orc_silu(x)


def attend(q, k, v, n_kv, hd, scale):
    out = np.empty(hd, dtype=np.float32)
    lib().orc_attend(P(q), P(k), P(v), n_kv, hd, scale, P(out))
    return out


def attend_batch(q, q_stride, k, v, t, pos, hd, scale, row):
    scores = np.zeros(t * row, dtype=np.float32)
    out = np.empty(t * hd, dtype=np.float32)
    lib().orc_attend_batch(P(q), q_stride, P(k), P(v), t, pos, hd, scale, row, P(scores),
                           P(out))
    return out


def delta_net(state, q, k, v, g, beta, scale):
    s = q.size
    out = np.empty(s, dtype=np.float32)
    lib().orc_delta_net(P(state), P(q), P(k), P(v), g, beta, scale, P(out), s)
    return out


def delta_net_into(prev, nxt, q, k, v, g, beta, scale):
    s = q.size
    out = np.empty(s, dtype=np.float32)
    lib().orc_delta_net_into(P(prev), P(nxt), P(q), P(k), P(v), g, beta, scale, P(out), s)
    return out


def delta_net_scalar(state, q, k, v, g, beta, scale):
    s = q.size
    out = np.empty(s, dtype=np.float32)
    lib().orc_delta_net_scalar(P(state), P(q), P(k), P(v), g, beta, scale, P(out), s)
    return out


def depthwise_conv(x, w, kernel, state):
    out = np.empty(x.size, dtype=np.float32)
    lib().orc_depthwise_conv(P(x), P(w), kernel, P(state), P(out), x.size)
    return out


def depthwise_conv_into(x, w, kernel, prev, nxt):
    out = np.empty(x.size, dtype=np.float32)
    lib().orc_depthwise_conv_into(P(x), P(w), kernel, P(prev), P(nxt), P(out), x.size)
    return out


# ---------------------------------------------------------------------------
# The hot spans


def full_attn(cfg: Config, pos, qg, k, v, kv, q_norm, k_norm, threads=1):
    """forward.rs:1259-1340.  qg/k are copied (the reference normalises its own
    buffers in place); kv, this layer's [2][n_kv][context][hd] cache, is
    updated in place.  Returns out [t][n_head*hd]."""
    t = qg.shape[0]
    qg = np.ascontiguousarray(qg, dtype=np.float32).copy()
    k = np.ascontiguousarray(k, dtype=np.float32).copy()
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty((t, cfg.n_head * cfg.head_dim), dtype=np.float32)
    lib().orc_full_attn(ctypes.byref(cfg), pos, t, P(qg), P(k), P(v), P(kv), P(q_norm),
                        P(k_norm), P(out), threads)
    return out


def linear_attn(cfg: Config, slots, live, qkv, z, alpha, beta, conv_state, ssm_state,
                conv1d, ssm_a, dt_bias, norm, threads=1):
    """forward.rs:1530-1652.  conv_state [slots][conv_dim][k-1] and ssm_state
    [n_v][slots][s][s] are updated in place.  Returns out [t][n_v*s]."""
    t = qkv.shape[0]
    out = np.empty((t, cfg.n_v_heads * cfg.d_state), dtype=np.float32)
    args = [np.ascontiguousarray(a, dtype=np.float32) for a in (qkv, z, alpha, beta)]
    lib().orc_linear_attn(ctypes.byref(cfg), slots, live, t, *(P(a) for a in args),
                          P(conv_state), P(ssm_state), P(conv1d), P(ssm_a), P(dt_bias),
                          P(norm), P(out), threads)
    return out


# ---------------------------------------------------------------------------
# Projections: int8 activations against k-quant weight rows
# (crates/llm-core/src/quant.rs, kernels/mod.rs)

Q8_0, Q4_K, Q6_K = 8, 12, 14


def row_bytes(ggml_type: int, k: int) -> int:
    return int(lib().orc_row_bytes(ggml_type, k))


def q8k_quantize(x: np.ndarray, k: int):
    """Activations::quantize_batch (quant.rs:337-372): x [t][k] -> (d [t][nb],
    qs [t][nb][256] int8, bsums [t][nb][16] int16)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    t, nb = x.shape[0], (k + 255) // 256
    d = np.empty((t, nb), np.float32)
    qs = np.empty((t, nb, 256), np.int8)
    bs = np.empty((t, nb, 16), np.int16)
    lib().orc_q8k_quantize(P(x), k, t, P(d), qs.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                           bs.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)))
    return d, qs, bs


def matvec(ggml_type: int, w: np.ndarray, rows: int, k: int, x: np.ndarray, threads=1):
    """The scalar tier's out [t][rows] = W . x with x quantized first
    (Exec::matmul_group, forward.rs:1157-1180; kernels/mod.rs:218-320)."""
    w = np.ascontiguousarray(w, np.uint8)
    assert w.size >= rows * row_bytes(ggml_type, k)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    out = np.empty((x.shape[0], rows), np.float32)
    code = lib().orc_matvec(ggml_type, w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), rows, k,
                            P(x), x.shape[0], P(out), threads)
    assert code == 0, ggml_type
    return out


def xorshift_stream(state: np.ndarray, n: int) -> np.ndarray:
    """n raw xorshift64* outputs; `state` (a 1-element uint64 array) advances."""
    out = np.empty(n, np.uint64)
    lib().orc_xorshift_stream(state.ctypes.data_as(_u64p), out.ctypes.data_as(_u64p), n)
    return out
