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
