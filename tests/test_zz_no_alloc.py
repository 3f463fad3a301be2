"""rl_full_attn_noalloc: full attention for callers that cannot allocate.

Some callers of this library cannot allocate device memory or hold a
context: a serving loop that plans every byte up front and must not allocate
once tokens flow, or a plug-in inside another framework's memory budget.
rl_full_attn_noalloc serves them: the caller owns the KV cache and every
input and output, and the kernels' scratch is a fixed static device array.

These tests call it through the C ABI on a cache the test owns, and check
two decode steps in a row against rl_full_attn on a context holding the same
cache, at the 1e-4 relative tolerance the full-attention tests use.  The file
is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

import cases
import oracle as orc
import rlcuda

TOL = 1e-4
pytestmark = pytest.mark.gpu


def _bind():
    L = rlcuda.lib()
    fn = L.rl_full_attn_noalloc
    fn.argtypes = [ctypes.POINTER(rlcuda.Config), ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


@pytest.mark.parametrize("t", [1, 4])
@pytest.mark.parametrize("kv_dtype", [rlcuda.RL_KV_BF16, rlcuda.RL_KV_F32])
def test_noalloc_matches_the_context_entry_point_on_two_steps(kv_dtype, t):
    """t = 1 is a decode step; t = 4 is a batch whose rows see each other's
    appended keys (the context runs it on the exact split-KV walk, with the
    tensor-core verify kernel switched off)."""
    import torch
    fn = _bind()
    context, pos0 = 3000, 2900
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=context, kv_dtype=kv_dtype,
                               max_batch=t)
    r = orc.Rng(2024)
    cache = r.normal((2, 4, pos0, 256))
    q_norm = r.normal(256, 1.0, 0.2)
    k_norm = r.normal(256, 1.0, 0.2)
    tdt = torch.bfloat16 if kv_dtype == rlcuda.RL_KV_BF16 else torch.float32
    dev = torch.device("cuda", 0)
    # the caller's own cache and weights
    k_cache = torch.zeros((4, context, 256), dtype=tdt, device=dev)
    v_cache = torch.zeros((4, context, 256), dtype=tdt, device=dev)
    src = torch.from_numpy(cache).to(dev)
    k_cache[:, :pos0] = src[0].to(tdt)
    v_cache[:, :pos0] = src[1].to(tdt)
    qn = torch.from_numpy(q_norm).to(dev)
    kn = torch.from_numpy(k_norm).to(dev)
    stream = torch.cuda.current_stream(dev)
    with rlcuda.Context(cfg) as ctx:
        ctx.set_option(rlcuda.RL_OPT_VERIFY_TC, 0)
        ctx.write_kv(0, 0, cache)
        ctx.set_weights_full(0, q_norm, k_norm)
        for step in range(2):  # two calls in a row share the static scratch
            pos = pos0 + step * t
            qg = r.normal((t, 16 * 512))
            k = r.normal((t, 4 * 256))
            v = r.normal((t, 4 * 256))
            want = ctx.full_attn_host(0, pos, qg, k, v)
            d_qg, d_k, d_v = (torch.from_numpy(x).to(dev) for x in (qg, k, v))
            out = torch.full((t, 16 * 256), float("nan"), device=dev)
            code = fn(ctypes.byref(cfg), stream.cuda_stream, k_cache.data_ptr(),
                      v_cache.data_ptr(), qn.data_ptr(), kn.data_ptr(), pos, t,
                      d_qg.data_ptr(), d_k.data_ptr(), d_v.data_ptr(), out.data_ptr())
            assert code == 0, rlcuda.lib().rl_last_error(None).decode()
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            err = cases.rel_err_per_head(got, want, 256)
            assert err <= TOL, (step, err)
            # the appended rows landed in the caller's cache, as in the context's
            rows = ctx.read_kv(0, pos, t)
            mine = np.stack([k_cache[:, pos:pos + t].float().cpu().numpy(),
                             v_cache[:, pos:pos + t].float().cpu().numpy()])
            assert np.array_equal(rows, mine), step
        # no kernel of these calls gave up a bounded wait
        assert rlcuda.lib().rl_noalloc_status(stream.cuda_stream) == 0


def test_noalloc_refuses_a_call_whose_scratch_does_not_fit():
    import torch
    fn = _bind()
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=1024, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    dev = torch.device("cuda", 0)
    t = 512  # 512 rows of staged queries alone exceed the scratch
    kc = torch.zeros((4, 1024, 256), dtype=torch.bfloat16, device=dev)
    ones = torch.ones(256, device=dev)
    qg = torch.zeros((t, 16 * 512), device=dev)
    kv = torch.zeros((t, 4 * 256), device=dev)
    out = torch.zeros((t, 16 * 256), device=dev)
    code = fn(ctypes.byref(cfg), torch.cuda.current_stream(dev).cuda_stream, kc.data_ptr(),
              kc.data_ptr(), ones.data_ptr(), ones.data_ptr(), 0, t, qg.data_ptr(),
              kv.data_ptr(), kv.data_ptr(), out.data_ptr())
    assert code == rlcuda.RL_EINVAL
    assert b"RL_NOALLOC_SCRATCH_BYTES" in rlcuda.lib().rl_last_error(None)
