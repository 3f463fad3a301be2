"""The oracle's restatement of the reference's projection arithmetic
(Activations::quantize_batch, the scalar q4k / q6k / q80 dots;
crates/llm-core/src/quant.rs:337-372, kernels/mod.rs:245-320) checked the
way the reference checks its own kernels (crates/llm-core/tests/kernels.rs):
the same seeded weights and activations, an f64 reference, and a tolerance
of 1e-5 times the sum of the absolute terms; plus that file's exact checks
(zero inputs give zero, a weight block past k contributes nothing)."""
import numpy as np
import pytest

import oracle as orc
import proj_cases as pc


@pytest.mark.parametrize("ty", pc.TYPES)
def test_awkward_shapes_match_the_f64_reference(ty):
    for i, (k, rows) in enumerate(pc.AWKWARD_SHAPES):
        w, x = pc.shape_case(ty, k, rows, 0x51ED + i)
        got = orc.matvec(ty, w, rows, k, x)[0]
        d, qs, _ = orc.q8k_quantize(x, k)
        stride = orc.row_bytes(ty, k)
        for r in range(rows):
            want, mag = pc.reference_dot(ty, w[r * stride:(r + 1) * stride], d[0], qs[0], k)
            assert abs(float(got[r]) - want) <= max(mag * 1e-5, 1e-12), (ty, k, rows, r)


@pytest.mark.parametrize("ty", pc.TYPES)
def test_a_model_shape_matches_the_f64_reference(ty):
    """(2560, 1024), the attn_k / attn_v shape, on its first 64 rows (the
    pure-Python f64 reference is slow)."""
    k, rows = 2560, 1024
    w, x = pc.shape_case(ty, k, rows, 0x51A9E + 4)
    got = orc.matvec(ty, w, rows, k, x, threads=4)[0]
    d, qs, _ = orc.q8k_quantize(x, k)
    stride = orc.row_bytes(ty, k)
    for r in range(64):
        want, mag = pc.reference_dot(ty, w[r * stride:(r + 1) * stride], d[0], qs[0], k)
        assert abs(float(got[r]) - want) <= max(mag * 1e-5, 1e-12), (ty, r)


def test_activation_quantization_is_the_reference_rule():
    """d = amax / 127, q = round(x * 127 / amax) with ties away from zero,
    clamped to +-127, the tail of the last block zero, bsums per 16."""
    x = np.array([0.5, -1.0, 0.25, 127.0 / 254.0 * 1.0] + [0.0] * 296, np.float32)
    d, qs, bs = orc.q8k_quantize(x, 300)
    assert d.shape == (1, 2) and d[0, 0] == np.float32(1.0) / np.float32(127.0)
    assert list(qs[0, 0, :4]) == [64, -127, 32, 64]  # 63.5 rounds away from zero
    assert not qs[0, 1, 44:].any() and d[0, 1] == 0.0
    assert int(bs[0, 0, 0]) == int(qs[0, 0, :16].astype(np.int32).sum())


@pytest.mark.parametrize("ty", pc.TYPES)
def test_zero_inputs_give_zero_and_blocks_past_k_do_not_contribute(ty):
    """kernels.rs:247-332."""
    k = 512
    nb = k // pc.BLOCK_LEN[ty]
    rng = pc.XorShift(7)
    w = pc.random_weights(ty, rng, nb)
    assert orc.matvec(ty, w, 1, k, np.zeros(k, np.float32))[0, 0] == 0.0
    x = rng.signed_n(k)
    assert orc.matvec(ty, np.zeros_like(w), 1, k, x)[0, 0] == 0.0
    short, long = 256, 261
    rng = pc.XorShift(0xBEEF)
    w = pc.random_weights(ty, rng, -(-long // pc.BLOCK_LEN[ty]))
    x = rng.signed_n(short)
    a = orc.matvec(ty, w[:orc.row_bytes(ty, short)], 1, short, x)[0, 0]
    b = orc.matvec(ty, w, 1, long, np.concatenate([x, np.zeros(5, np.float32)]))[0, 0]
    assert a == b


def test_a_batch_row_equals_the_row_alone():
    """Each row of a batch is quantized and dotted exactly as it would be on
    its own (quant.rs:276-281, kernels/mod.rs:205-217)."""
    k, rows = 1024, 16
    w, _ = pc.shape_case(pc.Q4_K, k, rows, 99)
    rng = pc.XorShift(5)
    xs = rng.signed_n(5 * k).reshape(5, k)
    batch = orc.matvec(pc.Q4_K, w, rows, k, xs)
    for t in range(5):
        assert np.array_equal(batch[t], orc.matvec(pc.Q4_K, w, rows, k, xs[t])[0])
