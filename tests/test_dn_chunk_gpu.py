"""Parity of the chunked Gated DeltaNet prefill (tensor-core chunk products,
f32 state between chunks) with the oracle's token-by-token restatement of
Exec::linear_attn (forward.rs:1530-1652, delta_net :1906-1950).

The chunk products run on bf16 tensor cores (with the state and the
intermediate U carried as bf16 pairs), so the bar is the north star's for the
tensor-core prefill: per head max-abs-diff / max-abs-ref <= 1e-2 and cosine
>= 0.9999, on the outputs and on the state left behind.  The conv history is
copied, never computed, so it must match exactly.
"""
import numpy as np
import pytest

import cases
import oracle as orc
import rlcuda

REL_TOL = 1e-2
COS_MIN = 0.9999
pytestmark = pytest.mark.gpu


def run_chunked(t, seed, unit_norm=True, scan_tc=1, overlap=1, local_tc=1):
    r = orc.Rng(seed)
    rows = cases.lin_rows(r, t)
    w = cases.lin_weights(r, unit_norm=unit_norm)
    conv, ssm = cases.lin_state(r, 1)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, 1, 0)
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=1, context=max(t, 64), slots=1,
                               max_batch=max(t, 64))
    with rlcuda.Context(cfg) as ctx:
        ctx.set_option(rlcuda.RL_OPT_DN_SCAN_TC, scan_tc)
        ctx.set_option(rlcuda.RL_OPT_DN_OVERLAP, overlap)
        ctx.set_option(rlcuda.RL_OPT_DN_LOCAL_TC, local_tc)
        ctx.set_weights_linear(0, w.conv1d, w.ssm_a, w.dt_bias, w.norm)
        ctx.write_conv(0, conv)
        ctx.write_ssm(0, ssm)
        ctx.profile_reset()
        got = ctx.linear_attn_host(0, 0, rows.qkv, rows.z, rows.alpha, rows.beta)
        chunk_launches = ctx.profile_read()["dn_chunk"][1]
        conv_got, ssm_got = ctx.read_conv(0), ctx.read_ssm(0)
    return got, want, conv_got, conv_w, ssm_got, ssm_w, chunk_launches


@pytest.mark.parametrize("scan_tc,overlap,local_tc",
                         [(1, 1, 1), (1, 0, 1), (1, 1, 0), (0, 0, 0)],
                         ids=["tcgen05_scan_overlapped", "tcgen05_scan", "mma_sync_local",
                              "mma_sync_scan"])
@pytest.mark.parametrize("t", [64, 100, 257, 1024, 4096])
def test_chunked_prefill_matches_the_token_sequential_oracle(t, scan_tc, overlap, local_tc):
    """t = 4096 is the benchmarked config-2 DeltaNet layer: the state is
    carried through 64 chunks, where the bf16-pair products' error would
    grow if it were going to.  Both chunk scans: tcgen05 (the default, beside
    the chunk-local kernel or after it) and mma.sync; the chunk-local kernel's
    K K^T and Q K^T on tcgen05 (the default) and on mma.sync."""
    got, want, conv_got, conv_w, ssm_got, ssm_w, n = run_chunked(t, 900 + t, scan_tc=scan_tc,
                                                                 overlap=overlap,
                                                                 local_tc=local_tc)
    assert n == 1, "the call did not take the chunked kernels"
    assert np.isfinite(got).all()
    err = cases.rel_err_per_head(got, want, cases.S)
    cos = cases.cosine_per_head(got, want, cases.S)
    assert err <= REL_TOL and cos >= COS_MIN, (err, cos)
    serr = cases.rel_err_per_head(ssm_got, ssm_w, cases.S * cases.S)
    scos = cases.cosine_per_head(ssm_got, ssm_w, cases.S * cases.S)
    assert serr <= REL_TOL and scos >= COS_MIN, (serr, scos)
    assert np.array_equal(conv_got, conv_w)


def test_consecutive_chunked_calls_over_two_layers():
    """Three chunked calls on one context (layer 0, layer 1, layer 0 again):
    each overlapped scan waits for its own call's chunk flags, whatever the
    calls before it left in them."""
    r = orc.Rng(57)
    rows = cases.lin_rows(r, 384)
    w0, w1 = cases.lin_weights(r), cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 1)
    c0, s0 = conv.copy(), ssm.copy()
    c1, s1 = conv.copy(), ssm.copy()
    half = [slice(0, 192), slice(192, 384)]
    pick = lambda sl: cases.LinRows(rows.qkv[sl], rows.z[sl], rows.alpha[sl], rows.beta[sl])
    want = [cases.oracle_linear(w0, pick(half[0]), c0, s0, 1, 0),
            cases.oracle_linear(w1, pick(half[0]), c1, s1, 1, 0),
            cases.oracle_linear(w0, pick(half[1]), c0, s0, 1, 0)]
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=2, context=256, slots=1, max_batch=192)
    with rlcuda.Context(cfg) as ctx:
        for layer, w in ((0, w0), (1, w1)):
            ctx.set_weights_linear(layer, w.conv1d, w.ssm_a, w.dt_bias, w.norm)
            ctx.write_conv(layer, conv)
            ctx.write_ssm(layer, ssm)
        got = []
        for layer, sl in ((0, half[0]), (1, half[0]), (0, half[1])):
            x = pick(sl)
            got.append(ctx.linear_attn_host(layer, 0, x.qkv, x.z, x.alpha, x.beta))
        ssm0 = ctx.read_ssm(0)
    for g_, w_ in zip(got, want):
        assert cases.rel_err_per_head(g_, w_, cases.S) <= REL_TOL
        assert cases.cosine_per_head(g_, w_, cases.S) >= COS_MIN
    assert cases.cosine_per_head(ssm0, s0, cases.S * cases.S) >= COS_MIN


def test_chunked_prefill_with_norm_weights():
    got, want, _, _, _, _, n = run_chunked(192, 77, unit_norm=False)
    assert n == 1
    assert cases.rel_err_per_head(got, want, cases.S) <= REL_TOL
    assert cases.cosine_per_head(got, want, cases.S) >= COS_MIN


def test_a_decode_step_continues_the_chunked_state():
    """A 128-row chunked prefill, then one step through the decode kernel: the
    step starts from the state and history the prefill left."""
    r = orc.Rng(31)
    rows = cases.lin_rows(r, 129)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 1)
    want = cases.oracle_linear(w, rows, conv.copy(), ssm.copy(), 1, 0)
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=1, context=256, slots=1, max_batch=128)
    with rlcuda.Context(cfg) as ctx:
        ctx.set_weights_linear(0, w.conv1d, w.ssm_a, w.dt_bias, w.norm)
        ctx.write_conv(0, conv)
        ctx.write_ssm(0, ssm)
        a = ctx.linear_attn_host(0, 0, rows.qkv[:128], rows.z[:128], rows.alpha[:128],
                                 rows.beta[:128])
        b = ctx.linear_attn_host(0, 0, rows.qkv[128:], rows.z[128:], rows.alpha[128:],
                                 rows.beta[128:])
    got = np.concatenate([a, b])
    assert cases.rel_err_per_head(got, want, cases.S) <= REL_TOL
    assert cases.cosine_per_head(got[128:], want[128:], cases.S) >= COS_MIN
