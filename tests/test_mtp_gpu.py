"""The multi-token-prediction block's cache, driven the way the reference's
Runner drives it, against the oracle running the same calls.

The MTP block is one more full-attention block with a cache of its own
(`Mtp::kv`, forward.rs:709-779 `catch_up`, :961-1027 `draft_mtp`, :1391-1438
`mtp_block`, whose attention is the trunk's `full_attn`).  On the device it is
a one-layer context.  Its cache sees two kinds of call:
  - a draft step: one row at the next position, whose key and value land in
    the cache although the token may be rejected;
  - a catch-up: the rows the trunk accepted, as one multi-row call at the
    position the block is caught up to, overwriting what the drafts left in
    those positions.
Rows drafted past what was accepted stay in the cache until a later call
overwrites them; a row at position p reads positions 0..p only, so they are
never read.  Every call's output is compared per head at 1e-4 (max-abs-diff
/ max-abs-ref) where the arithmetic is f32 (the f32 cache; the bf16 cache's
single-row walk and multi-row walk), and at 1e-2 with cosine >= 0.9999
where a bf16 batch of 2-8 rows takes the tensor-core verify kernel, the bar
of tests/test_verify_tc_gpu.py; the accepted part of the cache at 1e-6 at
the end.
"""
import numpy as np
import pytest

import cases
import oracle as orc
import rlcuda

pytestmark = pytest.mark.gpu
TOL = 1e-4
TC_TOL, TC_COS = 1e-2, 0.9999
CONTEXT = 320


def rows(seed, t):
    r = orc.Rng(seed)
    return (r.normal((t, cases.N_HEAD * 2 * cases.HD)), r.normal((t, cases.N_KV * cases.HD)),
            r.normal((t, cases.N_KV * cases.HD)))


@pytest.mark.parametrize("kv_dtype,verify_tc", [(rlcuda.RL_KV_F32, 1), (rlcuda.RL_KV_BF16, 0),
                                                 (rlcuda.RL_KV_BF16, 1)],
                         ids=["f32", "bf16", "bf16_verify_tc"])
def test_drafts_and_catch_ups_match_the_oracle(kv_dtype, verify_tc):
    bf16 = kv_dtype == rlcuda.RL_KV_BF16
    r = orc.Rng(91)
    qn = r.normal(cases.HD, 1.0, 0.2)
    kn = r.normal(cases.HD, 1.0, 0.2)
    cfg = orc.qwen35_config(CONTEXT, bf16)
    kv = np.zeros((2, cases.N_KV, CONTEXT, cases.HD), np.float32)
    mcfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=CONTEXT, kv_dtype=kv_dtype,
                                max_batch=16)
    seed = 1000
    worst = 0.0
    with rlcuda.Context(mcfg) as ctx:
        ctx.set_weights_full(0, qn, kn)
        ctx.set_option(rlcuda.RL_OPT_VERIFY_TC, verify_tc)

        def call(pos, t):
            nonlocal seed, worst
            seed += 1
            qg, k, v = rows(seed, t)
            want = orc.full_attn(cfg, pos, qg, k, v, kv, qn, kn, cases.THREADS)
            got = ctx.full_attn_host(0, pos, qg, k, v)
            err = cases.rel_err_per_head(got, want, cases.HD)
            if bf16 and verify_tc and 2 <= t <= 8:
                cos = cases.cosine_per_head(got, want, cases.HD)
                assert err <= TC_TOL and cos >= TC_COS, (pos, t, err, cos)
                return
            worst = max(worst, err)
            assert err <= TOL, (pos, t, err)

        # the prompt: the block catches up over it in one batch
        pos = 0
        call(pos, 9)
        pos += 9
        # rounds of (draft n, accept j, catch up j): (n, j) as a verify pass
        # would leave them, including a draft past the last accepted row and
        # a round that accepts nothing but the trunk's own token
        for n, j in [(3, 3), (4, 1), (2, 2), (5, 3), (1, 1), (6, 4), (3, 2)]:
            for i in range(n):
                call(pos + i, 1)        # draft step i writes row pos + i
            call(pos, j)                # catch-up overwrites rows pos .. pos + j - 1
            pos += j
        # a long catch-up straddling the walk's 64-position tiles
        call(pos, 16)
        pos += 16
        call(pos, 1)
        pos += 1
        got_kv = ctx.read_kv(0, 0, pos)
    assert cases.rel_err_per_head(got_kv, kv[:, :, :pos], cases.HD) <= 1e-6
    assert worst <= TOL
