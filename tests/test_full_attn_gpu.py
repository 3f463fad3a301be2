"""Parity of the full-attention path (C ABI -> sm_100a kernels) with the
oracle's restatement of Exec::full_attn (forward.rs:1259-1340).

Tolerance: 1e-4 relative per head (max-abs-diff / max-abs-ref), the bar the
build's north star sets for the f32 decode path; the same bar is applied to
the bf16-cache path, whose oracle stores the appended rows rounded to bf16
exactly as the device cache does.
"""
import numpy as np
import pytest

import cases
import rlcuda

TOL = 1e-4
pytestmark = pytest.mark.gpu


def make_ctx(context, kv_dtype=rlcuda.RL_KV_F32, max_batch=16, n_full=1):
    cfg = rlcuda.qwen35_config(n_full=n_full, n_linear=0, context=context, kv_dtype=kv_dtype,
                               max_batch=max_batch)
    return rlcuda.Context(cfg)


def run_case(ctx, case, layer=0):
    if case.pos:
        ctx.write_kv(layer, 0, case.cache)
    ctx.set_weights_full(layer, case.q_norm, case.k_norm)
    t = case.qg.shape[0]
    return ctx.full_attn_host(layer, case.pos, case.qg.reshape(t, -1), case.k.reshape(t, -1),
                              case.v.reshape(t, -1))


def test_config0_decode_f32_at_2047():
    """one decode step at position 2047 over a filled
    2048-entry f32 cache, seed 0."""
    case = cases.full_case(0, 2047, 1)
    want, kv_want = cases.oracle_full(case, 2048)
    with make_ctx(2048) as ctx:
        got = run_case(ctx, case)
        err = cases.rel_err_per_head(got, want, cases.HD)
        assert err <= TOL, err
        # the appended row is the normalised, rotated key and the raw value
        kv_got = ctx.read_kv(0, 2047, 1)
        assert cases.rel_err_per_head(kv_got, kv_want[:, :, 2047:2048], cases.HD) <= 1e-6


def test_decode_with_norm_weights():
    case = cases.full_case(10, 777, 1, unit_norms=False)
    want, _ = cases.oracle_full(case, 1024)
    with make_ctx(1024) as ctx:
        assert cases.rel_err_per_head(run_case(ctx, case), want, cases.HD) <= TOL


@pytest.mark.parametrize("pos,t", [(0, 1), (0, 5), (1, 1), (7, 3), (31, 1), (32, 1),
                                   (127, 1), (128, 1), (126, 5), (129, 4), (256, 16),
                                   (381, 9), (1000, 16)])
def test_rows_match_the_oracle(pos, t):
    """The reference's own (pos, t) cases (forward.rs:2324-2336), straddling
    its TILE and this kernel's tiles; t > 1 is the causal batch."""
    case = cases.full_case(100 + pos + t, pos, t)
    want, _ = cases.oracle_full(case, pos + t + 3)
    with make_ctx(pos + t + 3) as ctx:
        got = run_case(ctx, case)
    assert cases.rel_err_per_head(got, want, cases.HD) <= TOL


@pytest.mark.parametrize("pos", [4095, 5000, 32767])
def test_decode_bf16_cache(pos):
    """pos 32767 over a 32768-entry cache is the benchmarked decode (the
    metric's workload): the fused single-launch walk with its atomic tile
    dealing over 37+ tiles per split."""
    case = cases.full_case(20, pos, 1, kv_bf16=True)
    want, kv_want = cases.oracle_full(case, pos + 1, kv_bf16=True)
    with make_ctx(pos + 1, rlcuda.RL_KV_BF16) as ctx:
        ctx.profile_reset()
        got = run_case(ctx, case)
        prof = ctx.profile_read()
        assert prof["decode"][1] == 1 and prof["prologue"][1] == 0, prof
        assert cases.rel_err_per_head(got, want, cases.HD) <= TOL
        row = ctx.read_kv(0, pos, 1)
        assert cases.rel_err_per_head(row, kv_want[:, :, pos:pos + 1], cases.HD) <= 1e-6


def test_speculative_verify_rows_bf16():
    """BASELINE config 3's attention shape, shortened: k = 8 rows appended at
    position 4096 of a bf16 cache."""
    case = cases.full_case(3, 4096, 8, kv_bf16=True)
    want, _ = cases.oracle_full(case, 4104, kv_bf16=True)
    with make_ctx(4104, rlcuda.RL_KV_BF16) as ctx:
        # the exact split-KV walk (the tensor-core verify kernel is tested at
        # the tensor-core bar in test_verify_tc_gpu.py)
        ctx.set_option(rlcuda.RL_OPT_VERIFY_TC, 0)
        assert cases.rel_err_per_head(run_case(ctx, case), want, cases.HD) <= TOL


def test_forced_split_counts_agree():
    case = cases.full_case(4, 3000, 2)
    want, _ = cases.oracle_full(case, 3002)
    for splits in (1, 3, 17, 200):
        with make_ctx(3002) as ctx:
            ctx.set_option(rlcuda.RL_OPT_SPLITS, splits)
            got = run_case(ctx, case)
        assert cases.rel_err_per_head(got, want, cases.HD) <= TOL, splits


def test_sequential_decode_steps_chain():
    """Five decode steps through the device path, each appended row read by
    the next: the device cache follows the oracle's."""
    import oracle as orc
    ctx_len = 600
    case = cases.full_case(5, 590, 1)
    r = orc.Rng(55)
    kv = np.zeros((2, 4, ctx_len, 256), np.float32)
    kv[:, :, :590] = case.cache
    cfg = orc.qwen35_config(ctx_len)
    with make_ctx(ctx_len) as ctx:
        ctx.write_kv(0, 0, case.cache)
        for step in range(5):
            pos = 590 + step
            qg = r.normal((1, 16 * 512))
            k = r.normal((1, 4 * 256))
            v = r.normal((1, 4 * 256))
            want = orc.full_attn(cfg, pos, qg, k, v, kv, case.q_norm, case.k_norm, 8)
            got = ctx.full_attn_host(0, pos, qg, k, v)
            assert cases.rel_err_per_head(got, want, 256) <= TOL, step


def test_device_pointer_entry_point_matches_host_entry_point():
    import torch
    case = cases.full_case(6, 300, 3)
    with make_ctx(303) as a, make_ctx(303) as b:
        host = run_case(a, case)
        b.write_kv(0, 0, case.cache)
        qg = torch.from_numpy(case.qg.reshape(3, -1)).cuda()
        k = torch.from_numpy(case.k.reshape(3, -1)).cuda()
        v = torch.from_numpy(case.v.reshape(3, -1)).cuda()
        out = torch.empty(3, 16 * 256, device="cuda")
        torch.cuda.synchronize()
        b.full_attn(0, 300, 3, qg, k, v, out)
        b.sync()
        assert np.array_equal(out.cpu().numpy(), host)


def test_contract_errors():
    with make_ctx(64, max_batch=8) as ctx:
        x = np.zeros((1, 16 * 512), np.float32)
        kv = np.zeros((1, 4 * 256), np.float32)
        with pytest.raises(rlcuda.RlError) as e:
            ctx.full_attn_host(0, 64, x, kv, kv)
        assert e.value.code == rlcuda.RL_ECONTEXT
        with pytest.raises(rlcuda.RlError) as e:
            ctx.full_attn_host(1, 0, x, kv, kv)
        assert e.value.code == rlcuda.RL_EINVAL
        big = np.zeros((9, 16 * 512), np.float32)
        with pytest.raises(rlcuda.RlError) as e:
            ctx.full_attn_host(0, 0, big, np.zeros((9, 1024), np.float32),
                               np.zeros((9, 1024), np.float32))
        assert e.value.code == rlcuda.RL_EINVAL
        with pytest.raises(rlcuda.RlError) as e:
            ctx.accept(0)
        assert e.value.code == rlcuda.RL_EINVAL
        ctx.accept(64)
        with pytest.raises(rlcuda.RlError) as e:
            ctx.accept(1)
        assert e.value.code == rlcuda.RL_ECONTEXT
        ctx.reset()
        assert ctx.pos == 0 and ctx.live == 0
