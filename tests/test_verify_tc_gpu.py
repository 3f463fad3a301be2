"""Parity of the tensor-core verify kernel (2..8 rows over a bf16 cache,
the four query heads of a KV head packed into one tile, the key sequence
split over the GPU's SMs) with the oracle's restatement of Exec::full_attn
over a batch of rows (forward.rs:1259-1340, attend_batch :1783-1826).

Probabilities enter the P V product in bf16, as in the prefill kernel, so
the bar is the north star's tensor-core bar: per head max-abs-diff /
max-abs-ref <= 1e-2 and cosine >= 0.9999 against the oracle on the same
bf16-rounded cache.  RL_OPT_VERIFY_TC = 0 keeps the exact split-KV walk
(tested at 1e-4 in test_full_attn_gpu.py).
"""
import numpy as np
import pytest

import cases
import rlcuda

REL_TOL = 1e-2
COS_MIN = 0.9999
pytestmark = pytest.mark.gpu


def run_verify(case, context, max_batch, splits=0, layer=0, n_full=1):
    cfg = rlcuda.qwen35_config(n_full=n_full, n_linear=0, context=context,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=max_batch)
    with rlcuda.Context(cfg) as ctx:
        assert ctx.get_option(rlcuda.RL_OPT_VERIFY_TC) == 1
        if splits:
            ctx.set_option(rlcuda.RL_OPT_SPLITS, splits)
        if case.pos:
            ctx.write_kv(layer, 0, case.cache)
        ctx.set_weights_full(layer, case.q_norm, case.k_norm)
        t = case.qg.shape[0]
        ctx.profile_reset()
        got = ctx.full_attn_host(layer, case.pos, case.qg.reshape(t, -1), case.k.reshape(t, -1),
                                 case.v.reshape(t, -1))
        prof = ctx.profile_read()
        kv = ctx.read_kv(layer, case.pos, t)
    return got, kv, prof


def check(got, want):
    assert np.isfinite(got).all()
    err = cases.rel_err_per_head(got, want, cases.HD)
    cos = cases.cosine_per_head(got, want, cases.HD)
    assert err <= REL_TOL and cos >= COS_MIN, (err, cos)


@pytest.mark.parametrize("pos,t", [(0, 2), (0, 8), (5, 3), (63, 5), (100, 2), (4096, 8),
                                   (16380, 8), (3000, 7), (127, 8), (8191, 6)])
def test_verify_rows_match_the_oracle(pos, t):
    """Draft rows straddling key tiles (pos % 64 near 64), a split holding
    only keys past the first rows (16380 + 8), and 2..8 rows."""
    case = cases.full_case(700 + pos + t, pos, t, kv_bf16=True)
    context = pos + t + 3
    want, kv_want = cases.oracle_full(case, context, kv_bf16=True)
    got, kv_got, prof = run_verify(case, context, max(t, 8))
    assert prof["verify"][1] == 1 and prof["decode"][1] == 0, prof
    check(got, want)
    assert cases.rel_err_per_head(kv_got, kv_want[:, :, pos:pos + t], cases.HD) <= 1e-2


def test_config3_shape_16384():
    """BASELINE config 3's attention: k = 8 rows at position 16384."""
    case = cases.full_case(3, 16384, 8, kv_bf16=True)
    want, _ = cases.oracle_full(case, 16392, kv_bf16=True)
    got, _, _ = run_verify(case, 16392, 8)
    check(got, want)


@pytest.mark.parametrize("splits", [1, 2, 7, 40])
def test_forced_split_counts_agree(splits):
    case = cases.full_case(77, 2500, 8, kv_bf16=True)
    want, _ = cases.oracle_full(case, 2508, kv_bf16=True)
    got, _, _ = run_verify(case, 2508, 8, splits=splits)
    check(got, want)


def test_verify_on_a_later_layer_with_norm_weights():
    case = cases.full_case(78, 1500, 8, kv_bf16=True, unit_norms=False)
    want, _ = cases.oracle_full(case, 1600, kv_bf16=True)
    got, _, _ = run_verify(case, 1600, 16, layer=2, n_full=3)
    check(got, want)


def test_verify_then_decode_continues_the_cache():
    """8 draft rows through the verify kernel, then one decode row through
    the walk: the decode reads the rows the verify prologue appended."""
    r_case = cases.full_case(79, 700, 9, kv_bf16=True)
    want, _ = cases.oracle_full(r_case, 720, kv_bf16=True)
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=720, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=8)
    with rlcuda.Context(cfg) as ctx:
        ctx.write_kv(0, 0, r_case.cache)
        qg, k, v = r_case.qg, r_case.k, r_case.v
        first = ctx.full_attn_host(0, 700, qg[:8].reshape(8, -1), k[:8].reshape(8, -1),
                                   v[:8].reshape(8, -1))
        last = ctx.full_attn_host(0, 708, qg[8:].reshape(1, -1), k[8:].reshape(1, -1),
                                  v[8:].reshape(1, -1))
    check(first, want[:8])
    assert cases.rel_err_per_head(last, want[8:], cases.HD) <= 1e-4


def test_walk_is_kept_when_the_option_is_off():
    case = cases.full_case(80, 900, 8, kv_bf16=True)
    want, _ = cases.oracle_full(case, 910, kv_bf16=True)
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=910, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=8)
    with rlcuda.Context(cfg) as ctx:
        ctx.set_option(rlcuda.RL_OPT_VERIFY_TC, 0)
        ctx.write_kv(0, 0, case.cache)
        ctx.set_weights_full(0, case.q_norm, case.k_norm)
        ctx.profile_reset()
        got = ctx.full_attn_host(0, 900, case.qg.reshape(8, -1), case.k.reshape(8, -1),
                                 case.v.reshape(8, -1))
        prof = ctx.profile_read()
    assert prof["verify"][1] == 0 and prof["decode"][1] == 1
    assert cases.rel_err_per_head(got, want, cases.HD) <= 1e-4


@pytest.mark.parametrize("t", [9, 17, 40])
def test_longer_batches_take_the_exact_walk(t):
    """9..63 rows stay on the exact split-KV walk (1e-4)."""
    case = cases.full_case(81 + t, 2000, t, kv_bf16=True)
    want, _ = cases.oracle_full(case, 2000 + t, kv_bf16=True)
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=2000 + t,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=t)
    with rlcuda.Context(cfg) as ctx:
        ctx.write_kv(0, 0, case.cache)
        ctx.set_weights_full(0, case.q_norm, case.k_norm)
        ctx.profile_reset()
        got = ctx.full_attn_host(0, 2000, case.qg.reshape(t, -1), case.k.reshape(t, -1),
                                 case.v.reshape(t, -1))
        prof = ctx.profile_read()
    assert prof["verify"][1] == 0 and prof["decode"][1] == 1
    assert cases.rel_err_per_head(got, want, cases.HD) <= 1e-4
