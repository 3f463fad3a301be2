"""The north star's greedy-token check: the attention-only harness
(greedy_harness.py, a 32-layer hybrid toy stack whose projections, residual
and argmax head are shared host code) generates the same tokens with the
sm_100a attention ops as with the oracle's restatement of the reference's
(forward.rs:1259-1340, :1530-1652).  f32 caches, the path the reference
has; the prompt goes in as one batch of rows (the multi-row full-attention
walk and the token-sequential DeltaNet kernel), then one row per step (the
fused decode and the DeltaNet decode step)."""
import pytest

import greedy_harness as gh

pytestmark = pytest.mark.gpu

PROMPT = [17, 200, 3, 99, 54, 128, 7, 250]
N_NEW = 24


@pytest.mark.parametrize("seed", [0, 1])
def test_greedy_tokens_identical(seed):
    stack = gh.ToyStack(seed)
    context = 64
    want = stack.run(gh.OracleBackend(stack, context), PROMPT, N_NEW)
    dev = gh.DeviceBackend(stack, context, max_batch=len(PROMPT))
    try:
        got = stack.run(dev, PROMPT, N_NEW)
    finally:
        dev.close()
    assert got == want, (got, want)
    # a sanity check on the harness itself: the stack does not emit one token
    assert len(set(want)) > 3, want


def test_speculative_verify_and_accept_give_the_sequential_tokens():
    """The speculative side of the greedy check (tests/speculate.rs:49-60 and
    on, forward.rs:641-688): on the device, a verify batch of DRAFT + 1 rows
    over a ring of DRAFT + 1 DeltaNet slots, then accept(k) up to the first
    wrong draft (a rollback of the rest, by pointer), then single rows.  The
    batch's rows predict the oracle's sequential tokens, their logits agree
    with the single passes' to 1e-4, and the tokens after the rollback are
    those of an oracle runner that only ever saw the k rows."""
    import numpy as np
    import test_greedy_harness as th
    stack = gh.ToyStack(5)
    ctx = 64
    rows, want, tails = th.sequential_reference(stack,
                                                lambda s: gh.OracleBackend(stack, ctx, s))
    for what, batch in th.spec_batches(rows):
        dev = gh.DeviceBackend(stack, ctx, max_batch=len(th.SPEC_PROMPT), slots=th.DRAFT + 1)
        try:
            logits, accepted, got = th.speculative_run(stack, dev, batch, rows)
            assert dev.ctx.pos == len(th.SPEC_PROMPT) + accepted + 1 + 4
        finally:
            dev.close()
        for r in range(accepted + 1):
            assert int(np.argmax(logits[r])) == int(np.argmax(want[r])), (what, r)
            err = np.abs(logits[r] - want[r]).max() / np.abs(want[r]).max()
            assert err <= 1e-4, (what, r, err)
        assert got == tails[accepted], (what, got, tails[accepted])
