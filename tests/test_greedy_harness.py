"""The greedy harness on the CPU: the oracle backend is deterministic, the
layer numbering covers 8 full and 24 DeltaNet layers once each, and the
stack's tokens react to its attention (a run whose attention outputs are
zeroed generates different tokens), so the GPU comparison is not vacuous."""
import numpy as np

import greedy_harness as gh

PROMPT = [17, 200, 3, 99]


class ZeroBackend:
    def full(self, layer, pos, qg, k, v):
        return np.zeros((qg.shape[0], gh.N_HEAD * gh.HD), np.float32)

    def linear(self, layer, live, qkv, z, alpha, beta):
        return np.zeros((qkv.shape[0], gh.N_V * gh.S), np.float32)


class CountingBackend(ZeroBackend):
    def __init__(self):
        self.full_layers, self.lin_layers = [], []

    def full(self, layer, pos, qg, k, v):
        self.full_layers.append(layer)
        return super().full(layer, pos, qg, k, v)

    def linear(self, layer, live, qkv, z, alpha, beta):
        self.lin_layers.append(layer)
        return super().linear(layer, live, qkv, z, alpha, beta)


def test_layer_numbering():
    stack = gh.ToyStack(0)
    b = CountingBackend()
    stack.run(b, PROMPT, 1)
    assert b.full_layers == list(range(8))
    assert b.lin_layers == list(range(24))


def test_oracle_run_is_deterministic_and_uses_attention():
    stack = gh.ToyStack(3)
    a = stack.run(gh.OracleBackend(stack, 32), PROMPT, 6)
    b = stack.run(gh.OracleBackend(stack, 32), PROMPT, 6)
    assert a == b
    z = stack.run(ZeroBackend(), PROMPT, 6)
    assert z != a


DRAFT = 4
SPEC_PROMPT = [17, 200, 3, 99, 54, 128, 7, 250]


def spec_batches(rows, vocab=gh.VOCAB):
    """The three batches of the reference's speculative test
    (tests/speculate.rs:49-60 and on): every draft right, every draft wrong,
    and wrong from the middle (row 3)."""
    wrong = [(t + 1) % vocab for t in rows]
    return [("every draft right", list(rows)),
            ("every draft wrong", [rows[0]] + wrong[1:]),
            ("wrong in the middle", [t if i != 3 else wrong[i] for i, t in enumerate(rows)])]


def sequential_reference(stack, make_backend):
    """The one-pass-at-a-time side: the prompt, then DRAFT + 1 single rows;
    the rows, each pass's logits, and per number of committed rows the
    tokens a runner that only ever saw those rows generates next."""
    r = gh.Runner(stack, make_backend(1))
    nxt = int(np.argmax(r.forward_batch(SPEC_PROMPT)))
    rows, want = [], []
    for _ in range(DRAFT + 1):
        rows.append(nxt)
        logits = r.forward_batch([nxt])
        want.append(logits)
        nxt = int(np.argmax(logits))
    tails = []
    for keep in range(1, DRAFT + 2):
        r = gh.Runner(stack, make_backend(1))
        nxt = int(np.argmax(r.forward_batch(SPEC_PROMPT)))
        for row in rows[:keep]:
            assert nxt == row
            nxt = int(np.argmax(r.forward_batch([row])))
        out = [nxt]
        for _ in range(4):
            nxt = int(np.argmax(r.forward_batch([nxt])))
            out.append(nxt)
        tails.append(out)
    return rows, want, tails


def speculative_run(stack, backend, batch, rows):
    """Prompt, one verify batch, accept up to the first wrong draft, then 4
    single rows: (verify logits, accepted count, tokens after the accept)."""
    r = gh.Runner(stack, backend)
    at = int(np.argmax(r.forward_batch(SPEC_PROMPT)))
    assert at == rows[0]
    logits = r.verify(batch)
    accepted = 0
    for a, b in zip(batch[1:], rows[1:]):
        if a != b:
            break
        accepted += 1
    keep = accepted + 1
    r.accept(keep)
    assert r.pos == len(SPEC_PROMPT) + keep and r.live == r.pos % r.slots
    got = [int(np.argmax(logits[accepted]))]
    for _ in range(4):
        got.append(int(np.argmax(r.forward_batch([got[-1]]))))
    return logits, accepted, got


def test_oracle_verify_batch_equals_the_passes_it_replaces():
    """The reference's speculative rule (tests/speculate.rs:49-60 and on) on
    the oracle: a verify batch's rows give the single passes' logits bit for
    bit, and after accept(k) the runner generates what one that only saw k
    rows does.  The DeltaNet layers walk a ring of DRAFT + 1 slots
    (forward.rs:641-688, 2067-2076); the sequential side works in place."""
    stack = gh.ToyStack(5)
    ctx = 64
    rows, want, tails = sequential_reference(stack, lambda s: gh.OracleBackend(stack, ctx, s))
    for what, batch in spec_batches(rows):
        logits, accepted, got = speculative_run(
            stack, gh.OracleBackend(stack, ctx, DRAFT + 1), batch, rows)
        for r in range(accepted + 1):
            assert np.array_equal(logits[r], want[r]), (what, r)
        assert got == tails[accepted], what
    assert len(set(rows)) > 1
