"""The projections on the device (rl_act_quantize + rl_matvec) against the
oracle's restatement of the reference's scalar kernel tier
(crates/llm-core/src/quant.rs:337-372, kernels/mod.rs:245-320), bit for bit,
on the reference kernel tests' own fixtures and shapes
(crates/llm-core/tests/kernels.rs:23-44): every awkward shape, every model
shape, batches of rows, zero inputs."""
import numpy as np
import pytest
import torch

import oracle as orc
import proj_cases as pc
import rlcuda

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=64, max_batch=1)
    with rlcuda.Context(cfg) as c:
        yield c


def run(ctx, ty, w, rows, k, x):
    dev = torch.device("cuda", 0)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    t = x.shape[0]
    dw = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
    dx = torch.from_numpy(x).to(dev)
    out = torch.full((t, rows), float("nan"), device=dev)
    ctx.act_quantize(dx, t, k)
    ctx.matvec(ty, dw, rows, out)
    ctx.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("ty", pc.TYPES)
def test_awkward_shapes_bit_for_bit(ctx, ty):
    for i, (k, rows) in enumerate(pc.AWKWARD_SHAPES):
        w, x = pc.shape_case(ty, k, rows, 0x51ED + i)
        want = orc.matvec(ty, w, rows, k, x)
        got = run(ctx, ty, w, rows, k, x)
        assert np.array_equal(got, want), (ty, k, rows, np.abs(got - want).max())


@pytest.mark.parametrize("ty", pc.TYPES)
@pytest.mark.parametrize("shape", pc.MODEL_SHAPES)
def test_model_shapes_bit_for_bit(ctx, ty, shape):
    k, rows = shape
    i = pc.MODEL_SHAPES.index(shape)
    w, x = pc.shape_case(ty, k, rows, 0x51A9E + i)
    want = orc.matvec(ty, w, rows, k, x, threads=8)
    got = run(ctx, ty, w, rows, k, x)
    assert np.array_equal(got, want), (ty, shape, np.abs(got - want).max())


@pytest.mark.parametrize("t", [2, 8, 9, 17])
def test_a_batch_gives_each_row_its_single_result(ctx, t):
    """Batches straddling the kernel's group of 8 activation rows."""
    k, rows = 2560, 1024
    for ty in pc.TYPES:
        w, _ = pc.shape_case(ty, k, rows, 0x77 + t)
        rng = pc.XorShift(t)
        xs = (rng.signed_n(t * k) * np.float32(3.0)).reshape(t, k)
        got = run(ctx, ty, w, rows, k, xs)
        assert np.array_equal(got, orc.matvec(ty, w, rows, k, xs, threads=8)), (ty, t)
        assert np.array_equal(got[t - 1], run(ctx, ty, w, rows, k, xs[t - 1])[0]), (ty, t)


def test_a_group_gives_each_weight_its_own_result(ctx):
    """rl_matvec_group: a layer's qg, k and v (and types mixed) in one launch,
    each output the single matvec's bits."""
    dev = torch.device("cuda", 0)
    k = 2560
    parts = []
    for i, (ty, rows) in enumerate([(pc.Q4_K, 1024), (pc.Q6_K, 256), (pc.Q8_0, 96),
                                    (pc.Q4_K, 32)]):
        w, _ = pc.shape_case(ty, k, rows, 0x600 + i)
        parts.append((ty, torch.from_numpy(w).to(dev), rows,
                      torch.full((2, rows), float("nan"), device=dev), w))
    rng = pc.XorShift(11)
    xs = (rng.signed_n(2 * k) * np.float32(3.0)).reshape(2, k)
    ctx.act_quantize(torch.from_numpy(xs).to(dev), 2, k)
    ctx.matvec_group([p[:4] for p in parts])
    ctx.sync()
    for ty, _, rows, out, w in parts:
        assert np.array_equal(out.cpu().numpy(), orc.matvec(ty, w, rows, k, xs)), ty


@pytest.mark.parametrize("t", [1, 3])
def test_the_one_launch_group_matches_the_two_launch_path(ctx, t):
    """rl_matmul_group (quantization inside the launch) gives the bits of
    rl_act_quantize + rl_matvec_group, over groups of mixed types and row
    counts that leave warps with partial row runs."""
    dev = torch.device("cuda", 0)
    for k in (2560, 4096, 300):
        parts = []
        for i, (ty, rows) in enumerate([(pc.Q4_K, 2051), (pc.Q6_K, 130), (pc.Q8_0, 33)]):
            w, _ = pc.shape_case(ty, k, rows, 0x900 + i + k)
            parts.append((ty, torch.from_numpy(w).to(dev), rows,
                          torch.full((t, rows), float("nan"), device=dev), w))
        rng = pc.XorShift(k + t)
        xs = (rng.signed_n(t * k) * np.float32(3.0)).reshape(t, k)
        ctx.matmul_group(torch.from_numpy(xs).to(dev), t, k, [p[:4] for p in parts])
        ctx.sync()
        for ty, _, rows, out, w in parts:
            assert np.array_equal(out.cpu().numpy(), orc.matvec(ty, w, rows, k, xs, threads=8)), \
                (ty, k, t)


@pytest.mark.parametrize("ty", pc.TYPES)
def test_the_one_launch_group_on_awkward_and_long_rows(ctx, ty):
    """rl_matmul_group alone, bit for bit against the oracle: the awkward
    shapes (a Q4_K warp then holds 32 / nb rows, one super-block a lane) and
    rows of more than 32 super-blocks (one Q4_K row a warp, blocks l, l + 32,
    ... a lane)."""
    dev = torch.device("cuda", 0)
    for i, (k, rows) in enumerate(pc.AWKWARD_SHAPES + [(9216, 40), (12800, 7)]):
        w, x = pc.shape_case(ty, k, rows, 0x1AE + i)
        x = np.ascontiguousarray(x, np.float32).reshape(1, k)
        out = torch.full((1, rows), float("nan"), device=dev)
        ctx.matmul_group(torch.from_numpy(x).to(dev), 1, k,
                         [(ty, torch.from_numpy(np.ascontiguousarray(w)).to(dev), rows, out)])
        ctx.sync()
        want = orc.matvec(ty, w, rows, k, x, threads=8)
        got = out.cpu().numpy()
        assert np.array_equal(got, want), (ty, k, rows, np.abs(got - want).max())


def test_zero_inputs_give_zero(ctx):
    k = 512
    for ty in pc.TYPES:
        rng = pc.XorShift(7)
        w = pc.random_weights(ty, rng, k // pc.BLOCK_LEN[ty])
        assert run(ctx, ty, w, 1, k, np.zeros(k, np.float32))[0, 0] == 0.0
        x = rng.signed_n(k)
        assert run(ctx, ty, np.zeros_like(w), 1, k, x)[0, 0] == 0.0


def test_contract_errors(ctx):
    dev = torch.device("cuda", 0)
    w = torch.zeros(1024, dtype=torch.uint8, device=dev)
    out = torch.zeros(4, device=dev)
    with pytest.raises(rlcuda.RlError):
        ctx.matvec(2, w, 1, out)  # not a supported type (and nothing quantized yet, or after)
