"""Parity of the tcgen05 causal prefill (bf16 cache) with the oracle's
restatement of Exec::full_attn over a batch of rows (forward.rs:1259-1340,
attend_batch :1783-1826).

The kernel multiplies bf16 queries, keys, probabilities and values with f32
accumulation, so the bar is the north star's for the tensor-core prefill:
per head (one query row of one head) max-abs-diff / max-abs-ref <= 1e-2 and
cosine >= 0.9999 against the oracle run on the same bf16-rounded cache.
"""
import numpy as np
import pytest

import cases
import rlcuda

REL_TOL = 1e-2
COS_MIN = 0.9999
pytestmark = pytest.mark.gpu


def run_prefill(case, context, max_batch):
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=context,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=max_batch)
    with rlcuda.Context(cfg) as ctx:
        assert ctx.get_option(rlcuda.RL_OPT_PREFILL_ROWS) > 0
        if case.pos:
            ctx.write_kv(0, 0, case.cache)
        ctx.set_weights_full(0, case.q_norm, case.k_norm)
        t = case.qg.shape[0]
        ctx.profile_reset()
        got = ctx.full_attn_host(0, case.pos, case.qg.reshape(t, -1), case.k.reshape(t, -1),
                                 case.v.reshape(t, -1))
        launches = ctx.profile_read()["prefill"][1]
        kv = ctx.read_kv(0, 0, case.pos + t)
    return got, kv, launches


@pytest.mark.parametrize("pos,t", [(0, 64), (0, 128), (0, 200), (37, 131), (500, 256),
                                   (0, 1024), (1000, 640), (0, 4096)])
def test_prefill_matches_the_oracle(pos, t):
    """Query tiles of 128 rows and key tiles of 64: ragged last tiles on both
    sides, a prefix already in the cache (pos > 0) and the causal diagonal.
    (0, 4096) is the benchmarked config-2 prefill of a full-attention layer."""
    case = cases.full_case(300 + pos + t, pos, t, kv_bf16=True)
    context = pos + t + 5
    want, kv_want = cases.oracle_full(case, context, kv_bf16=True)
    got, kv_got, launches = run_prefill(case, context, max(t, 16))
    assert launches == 1, "the call did not take the tensor-core prefill kernel"
    assert np.isfinite(got).all()
    err = cases.rel_err_per_head(got, want, cases.HD)
    cos = cases.cosine_per_head(got, want, cases.HD)
    assert err <= REL_TOL and cos >= COS_MIN, (err, cos)
    # the prologue appended the batch's keys and values (bf16) as the oracle did
    assert cases.rel_err_per_head(kv_got[:, :, pos:pos + t], kv_want[:, :, pos:pos + t],
                                  cases.HD) <= 1e-2


def test_prefill_with_norm_weights():
    case = cases.full_case(41, 64, 192, kv_bf16=True, unit_norms=False)
    want, _ = cases.oracle_full(case, 300, kv_bf16=True)
    got, _, launches = run_prefill(case, 300, 192)
    assert launches == 1
    assert cases.rel_err_per_head(got, want, cases.HD) <= REL_TOL
    assert cases.cosine_per_head(got, want, cases.HD) >= COS_MIN


def test_prefill_then_decode_continues_the_cache():
    """A prefill of 256 rows, then one decode row through the walk: the decode
    reads the keys the prefill appended."""
    import oracle as orc
    r_case = cases.full_case(55, 0, 257, kv_bf16=True)
    want, _ = cases.oracle_full(r_case, 300, kv_bf16=True)
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=300, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=256)
    with rlcuda.Context(cfg) as ctx:
        qg, k, v = r_case.qg, r_case.k, r_case.v
        first = ctx.full_attn_host(0, 0, qg[:256].reshape(256, -1), k[:256].reshape(256, -1),
                                   v[:256].reshape(256, -1))
        last = ctx.full_attn_host(0, 256, qg[256:].reshape(1, -1), k[256:].reshape(1, -1),
                                  v[256:].reshape(1, -1))
    got = np.concatenate([first, last])
    assert cases.rel_err_per_head(got[:256], want[:256], cases.HD) <= REL_TOL
    assert cases.rel_err_per_head(got[256:], want[256:], cases.HD) <= 1e-4
    del orc
