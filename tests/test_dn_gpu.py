"""Parity of the Gated DeltaNet step path (C ABI -> sm_100a kernel) with the
oracle's restatement of Exec::linear_attn (forward.rs:1530-1652), plus the
ring relations the reference's tests hold (forward.rs:2207-2268) and its
speculative verify / rollback behaviour (tests/speculate.rs:68-202), at the
attention level.

Tolerance: 1e-4 relative per head (max-abs-diff / max-abs-ref) on the
outputs and on every ring slot of the state, the north star's bar for the
f32 DeltaNet step.  Relations between two device runs of the same kernel
are bit for bit.
"""
import numpy as np
import pytest

import cases
import oracle as orc
import rlcuda

TOL = 1e-4
pytestmark = pytest.mark.gpu
KERNEL = {"rows": 1}


@pytest.fixture(autouse=True, params=[1, 0], ids=["rows_kernel", "step_kernel"])
def dn_kernel(request):
    """Every case runs on both step kernels: the rows kernel (each head's
    columns over a cluster of four CTAs, the default) and the one-CTA-per-head
    kernel (RL_OPT_DN_ROWS = 0)."""
    KERNEL["rows"] = request.param
    yield request.param


def make_ctx(slots=1, max_batch=16, n_linear=1):
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=n_linear, context=4096, slots=slots,
                               max_batch=max_batch)
    ctx = rlcuda.Context(cfg)
    ctx.set_option(rlcuda.RL_OPT_DN_ROWS, KERNEL["rows"])
    assert ctx.get_option(rlcuda.RL_OPT_DN_ROWS) == KERNEL["rows"]
    return ctx


def load(ctx, w, conv, ssm, layer=0):
    ctx.set_weights_linear(layer, w.conv1d, w.ssm_a, w.dt_bias, w.norm)
    ctx.write_conv(layer, conv)
    ctx.write_ssm(layer, ssm)


def run(ctx, rows, live, layer=0):
    return ctx.linear_attn_host(layer, live, rows.qkv, rows.z, rows.alpha, rows.beta)


def check_state(ctx, conv_want, ssm_want, layer=0):
    conv = ctx.read_conv(layer)
    ssm = ctx.read_ssm(layer)
    assert np.array_equal(conv, conv_want)  # the history is copied, never rounded
    assert cases.rel_err_per_head(ssm, ssm_want, cases.S * cases.S) <= TOL


def test_config1_single_step():
    """one decode step, seed 1."""
    r = orc.Rng(1)
    rows = cases.lin_rows(r, 1)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 1)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, 1, 0)
    with make_ctx() as ctx:
        load(ctx, w, conv, ssm)
        got = run(ctx, rows, 0)
        assert cases.rel_err_per_head(got, want, cases.S) <= TOL
        check_state(ctx, conv_w, ssm_w)


@pytest.mark.parametrize("t", [2, 4, 16])
def test_sequential_rows_in_place(t):
    r = orc.Rng(30 + t)
    rows = cases.lin_rows(r, t)
    w = cases.lin_weights(r, unit_norm=False)
    conv, ssm = cases.lin_state(r, 1)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, 1, 0)
    with make_ctx() as ctx:
        load(ctx, w, conv, ssm)
        got = run(ctx, rows, 0)
        assert cases.rel_err_per_head(got, want, cases.S) <= TOL
        check_state(ctx, conv_w, ssm_w)


@pytest.mark.parametrize("slots,live,t", [(9, 0, 8), (9, 5, 8), (9, 3, 9), (4, 2, 7)])
def test_verify_rows_over_the_ring(slots, live, t):
    """BASELINE config 3's DeltaNet side: t sequential rows writing ring
    slots live+1..live+t (mod slots); every snapshot is checked."""
    r = orc.Rng(3 + slots + live + t)
    rows = cases.lin_rows(r, t)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, slots, live)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, slots, live)
    with make_ctx(slots=slots) as ctx:
        load(ctx, w, conv, ssm)
        got = run(ctx, rows, live)
        assert cases.rel_err_per_head(got, want, cases.S) <= TOL
        check_state(ctx, conv_w, ssm_w)


@pytest.mark.parametrize("slots,live,t", [(1, 0, 1), (1, 0, 9), (1, 0, 40), (13, 5, 12),
                                          (41, 7, 40), (5, 4, 11), (3, 2, 3)])
def test_rows_across_blocks_and_ring_wraps(slots, live, t):
    """Row counts on both sides of the rows kernel's blocks of eight (its
    norm exchange runs once per block), batches longer than the ring (later
    rows overwrite the slots of earlier ones, the live slot included), and
    every snapshot checked against the oracle."""
    r = orc.Rng(200 + slots + live + t)
    rows = cases.lin_rows(r, t)
    w = cases.lin_weights(r, unit_norm=False)
    conv, ssm = cases.lin_state(r, slots, live)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, slots, live)
    with make_ctx(slots=slots, max_batch=64) as ctx:
        load(ctx, w, conv, ssm)
        got = run(ctx, rows, live)
        assert cases.rel_err_per_head(got, want, cases.S) <= TOL
        check_state(ctx, conv_w, ssm_w)


def test_a_decay_that_underflows():
    """Gate logits that drive g = exp(softplus(a + dt_bias) * A) to zero in
    f32: the state and its snapshots become the rows' own outer products,
    as in the sequential recurrence."""
    r = orc.Rng(211)
    rows = cases.lin_rows(r, 8)
    rows.alpha[:] += 40.0
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 9)
    conv_w, ssm_w = conv.copy(), ssm.copy()
    want = cases.oracle_linear(w, rows, conv_w, ssm_w, 9, 0)
    with make_ctx(slots=9) as ctx:
        load(ctx, w, conv, ssm)
        got = run(ctx, rows, 0)
        assert cases.rel_err_per_head(got, want, cases.S) <= TOL
        check_state(ctx, conv_w, ssm_w)


def test_ring_slot_equals_in_place_bit_for_bit():
    """forward.rs:2207-2268 on the device: the same rows through a ring of 5
    and in place give the same outputs and the same final state, bit for bit."""
    r = orc.Rng(77)
    rows = cases.lin_rows(r, 4)
    w = cases.lin_weights(r)
    conv1, ssm1 = cases.lin_state(r, 1)
    conv5 = np.zeros((5,) + conv1.shape[1:], np.float32)
    ssm5 = np.zeros((ssm1.shape[0], 5) + ssm1.shape[2:], np.float32)
    conv5[0], ssm5[:, 0] = conv1[0], ssm1[:, 0]
    with make_ctx(1) as a, make_ctx(5) as b:
        load(a, w, conv1, ssm1)
        load(b, w, conv5, ssm5)
        out_a = run(a, rows, 0)
        out_b = run(b, rows, 0)
        assert np.array_equal(out_a, out_b)
        assert np.array_equal(a.read_ssm(0)[:, 0], b.read_ssm(0)[:, 4])
        assert np.array_equal(a.read_conv(0)[0], b.read_conv(0)[4])


@pytest.mark.parametrize("t", [8, 12])
def test_a_batch_equals_its_rows_one_at_a_time_bit_for_bit(t):
    """verify rows == sequential passes (tests/speculate.rs:68-202): one call
    of t rows and t calls of one row leave the same outputs and ring (12
    rows cross the rows kernel's block of eight)."""
    r = orc.Rng(88 + t)
    rows = cases.lin_rows(r, t)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, t + 1)
    with make_ctx(t + 1) as a, make_ctx(t + 1) as b:
        load(a, w, conv, ssm)
        load(b, w, conv, ssm)
        batch = run(a, rows, 0)
        single = []
        for i in range(t):
            one = cases.LinRows(rows.qkv[i:i + 1], rows.z[i:i + 1], rows.alpha[i:i + 1],
                                rows.beta[i:i + 1])
            single.append(run(b, one, i))
        assert np.array_equal(batch, np.concatenate(single))
        assert np.array_equal(a.read_ssm(0), b.read_ssm(0))
        assert np.array_equal(a.read_conv(0), b.read_conv(0))


@pytest.mark.parametrize("keep", [1, 3, 8])
def test_rollback_leaves_no_trace(keep):
    """Verify 8 rows over a ring of 9, accept `keep`, then run 2 more rows:
    the same as a fresh context that only ever saw the first `keep` rows."""
    r = orc.Rng(99)
    rows = cases.lin_rows(r, 8)
    nxt = cases.lin_rows(r, 2)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 9)
    with make_ctx(9) as spec, make_ctx(9) as fresh:
        load(spec, w, conv, ssm)
        load(fresh, w, conv, ssm)
        run(spec, rows, spec.live)
        spec.accept(keep)
        kept = cases.LinRows(rows.qkv[:keep], rows.z[:keep], rows.alpha[:keep],
                             rows.beta[:keep])
        run(fresh, kept, fresh.live)
        fresh.accept(keep)
        assert spec.live == fresh.live == keep % 9
        a = run(spec, nxt, spec.live)
        b = run(fresh, nxt, fresh.live)
        assert np.array_equal(a, b)


def test_two_layers_keep_separate_state():
    r = orc.Rng(5)
    w0, w1 = cases.lin_weights(r), cases.lin_weights(r)
    rows = cases.lin_rows(r, 2)
    c0, s0 = cases.lin_state(r, 1)
    c1, s1 = cases.lin_state(r, 1)
    want0 = cases.oracle_linear(w0, rows, c0.copy(), s0.copy(), 1, 0)
    want1 = cases.oracle_linear(w1, rows, c1.copy(), s1.copy(), 1, 0)
    with make_ctx(n_linear=2) as ctx:
        load(ctx, w0, c0, s0, 0)
        load(ctx, w1, c1, s1, 1)
        assert cases.rel_err_per_head(run(ctx, rows, 0, 1), want1, cases.S) <= TOL
        assert cases.rel_err_per_head(run(ctx, rows, 0, 0), want0, cases.S) <= TOL


def test_reset_zeroes_the_state():
    r = orc.Rng(6)
    w = cases.lin_weights(r)
    conv, ssm = cases.lin_state(r, 3)
    with make_ctx(3) as ctx:
        load(ctx, w, conv, ssm)
        ctx.accept(2)
        ctx.reset()
        assert ctx.pos == 0 and ctx.live == 0
        assert not ctx.read_ssm(0).any() and not ctx.read_conv(0).any()


def test_contract_errors():
    with make_ctx(3, max_batch=4) as ctx:
        rows = cases.lin_rows(orc.Rng(1), 1)
        with pytest.raises(rlcuda.RlError) as e:
            run(ctx, rows, 3)
        assert e.value.code == rlcuda.RL_EINVAL
        with pytest.raises(rlcuda.RlError) as e:
            ctx.linear_attn_host(1, 0, rows.qkv, rows.z, rows.alpha, rows.beta)
        assert e.value.code == rlcuda.RL_EINVAL
