"""Seeded inputs for the parity tests, and the parity metric.

Every case is drawn from the oracle's SplitMix64-seeded xoshiro256**
generator (oracle/oracle.cpp) in the order the functions below list, so the
GPU and the oracle always see the same values.  Distributions follow the
configs of the build's BASELINE: N(0,1) q/k/v/gate/cache for full attention;
for the DeltaNet qkv N(0,1), conv weights and history N(0,0.5),
A_log ~ U(ln 1, ln 16), a ~ N(0,1), dt_bias ~ N(0,0.1), b ~ N(0,1),
state N(0,0.1), z N(0,1).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np

import oracle as orc

N_HEAD, N_KV, HD = 16, 4, 256
# the oracle shares heads over every host core, as Pool::chunks does
THREADS = max(1, min(64, os.cpu_count() or 1))
S, N_K, N_V, KERNEL = 128, 16, 32, 4
CONV_DIM = 2 * N_K * S + N_V * S


def rel_err_per_head(got: np.ndarray, want: np.ndarray, width: int) -> float:
    """max over heads of ||got - want||_inf / ||want||_inf, heads of `width`."""
    g = got.reshape(-1, width).astype(np.float64)
    w = want.reshape(-1, width).astype(np.float64)
    num = np.abs(g - w).max(axis=1)
    den = np.maximum(np.abs(w).max(axis=1), 1e-30)
    return float((num / den).max())


def cosine_per_head(got, want, width) -> float:
    g = got.reshape(-1, width).astype(np.float64)
    w = want.reshape(-1, width).astype(np.float64)
    c = (g * w).sum(1) / np.maximum(np.linalg.norm(g, axis=1) * np.linalg.norm(w, axis=1), 1e-30)
    return float(c.min())


@dataclass
class FullCase:
    pos: int
    qg: np.ndarray   # [t][16][512]
    k: np.ndarray    # [t][4][256]
    v: np.ndarray    # [t][4][256]
    cache: np.ndarray  # [2][4][pos][256]  positions 0..pos-1
    q_norm: np.ndarray
    k_norm: np.ndarray


def full_case(seed: int, pos: int, t: int, kv_bf16: bool = False, unit_norms: bool = True):
    """Draw order: qg, k, v, cached K, cached V, then (if not unit) q_norm, k_norm."""
    r = orc.Rng(seed)
    qg = r.normal((t, N_HEAD, 2 * HD))
    k = r.normal((t, N_KV, HD))
    v = r.normal((t, N_KV, HD))
    kc = r.normal((N_KV, pos, HD))
    vc = r.normal((N_KV, pos, HD))
    cache = np.stack([kc, vc])
    if kv_bf16:
        cache = orc.round_bf16(cache).reshape(cache.shape)
    if unit_norms:
        qn = np.ones(HD, np.float32)
        kn = np.ones(HD, np.float32)
    else:
        qn = r.normal(HD, 1.0, 0.2)
        kn = r.normal(HD, 1.0, 0.2)
    return FullCase(pos, qg, k, v, cache, qn, kn)


def oracle_full(case: FullCase, context: int, kv_bf16=False, threads=THREADS):
    """Runs the oracle on a fresh [2][4][context][256] cache holding the case's
    positions; returns (out [t][4096], cache after the append)."""
    cfg = orc.qwen35_config(context, kv_bf16)
    kv = np.zeros((2, N_KV, context, HD), np.float32)
    kv[:, :, :case.pos] = case.cache
    t = case.qg.shape[0]
    out = orc.full_attn(cfg, case.pos, case.qg.reshape(t, -1), case.k.reshape(t, -1),
                        case.v.reshape(t, -1), kv, case.q_norm, case.k_norm, threads)
    return out, kv


@dataclass
class LinWeights:
    conv1d: np.ndarray   # [conv_dim][4]
    ssm_a: np.ndarray    # [32]
    dt_bias: np.ndarray  # [32]
    norm: np.ndarray     # [128]


@dataclass
class LinRows:
    qkv: np.ndarray      # [t][conv_dim]
    z: np.ndarray        # [t][4096]
    alpha: np.ndarray    # [t][32]
    beta: np.ndarray     # [t][32]


def lin_weights(r: orc.Rng, unit_norm=True) -> LinWeights:
    """Draw order: conv1d N(0,.5), A_log U(ln1,ln16) -> ssm_a = -exp, dt_bias N(0,.1)."""
    conv1d = r.normal((CONV_DIM, KERNEL), 0.0, 0.5)
    a_log = r.uniform(N_V, math.log(1.0), math.log(16.0))
    ssm_a = (-np.exp(a_log.astype(np.float64))).astype(np.float32)
    dt_bias = r.normal(N_V, 0.0, 0.1)
    norm = np.ones(S, np.float32) if unit_norm else r.normal(S, 1.0, 0.2)
    return LinWeights(conv1d, ssm_a, dt_bias, norm)


def lin_rows(r: orc.Rng, t: int) -> LinRows:
    """Draw order per call: qkv N(0,1), a N(0,1), b N(0,1), z N(0,1)."""
    qkv = r.normal((t, CONV_DIM))
    alpha = r.normal((t, N_V))
    beta = r.normal((t, N_V))
    z = r.normal((t, N_V * S))
    return LinRows(qkv, z, alpha, beta)


def lin_state(r: orc.Rng, slots: int, live: int = 0):
    """conv history N(0,.5) [slots][conv_dim][3] and state N(0,.1)
    [32][slots][128][128]; only slot `live` is drawn, the rest are zero."""
    conv = np.zeros((slots, CONV_DIM, KERNEL - 1), np.float32)
    ssm = np.zeros((N_V, slots, S, S), np.float32)
    conv[live] = r.normal((CONV_DIM, KERNEL - 1), 0.0, 0.5)
    ssm[:, live] = r.normal((N_V, S, S), 0.0, 0.1)
    return conv, ssm


def oracle_linear(w: LinWeights, rows: LinRows, conv, ssm, slots, live, threads=THREADS):
    cfg = orc.qwen35_config(16)
    return orc.linear_attn(cfg, slots, live, rows.qkv, rows.z, rows.alpha, rows.beta, conv, ssm,
                           w.conv1d, w.ssm_a, w.dt_bias, w.norm, threads)
