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

    def linear(self, layer, qkv, z, alpha, beta):
        return np.zeros((qkv.shape[0], gh.N_V * gh.S), np.float32)


class CountingBackend(ZeroBackend):
    def __init__(self):
        self.full_layers, self.lin_layers = [], []

    def full(self, layer, pos, qg, k, v):
        self.full_layers.append(layer)
        return super().full(layer, pos, qg, k, v)

    def linear(self, layer, qkv, z, alpha, beta):
        self.lin_layers.append(layer)
        return super().linear(layer, qkv, z, alpha, beta)


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
