"""A sequence split across GPUs, emulated on one device: each shard is its
own context (rl_set_shard), each walks its range (rl_full_attn_partial) and
rl_merge_partials merges the shards' partials.  The merged row must match
the oracle's single pass over the whole cache (forward.rs:1259-1340), and
the new key/value row must land in the shard that holds its position."""
import functools

import numpy as np
import pytest
import torch

import cases
import rlcuda
import split_kv

TOL = 1e-4
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,seq", [(2, 4096), (3, 3000), (4, 1000), (8, 8192)])
def test_shards_merge_to_the_single_pass_row(world, seq):
    pos = seq - 1
    case = cases.full_case(60 + world, pos, 1, kv_bf16=True)
    want, kv_want = cases.oracle_full(case, seq, kv_bf16=True)
    dev = torch.device("cuda", 0)
    qg = torch.from_numpy(case.qg.reshape(-1)).to(dev)
    k = torch.from_numpy(case.k.reshape(-1)).to(dev)
    v = torch.from_numpy(case.v.reshape(-1)).to(dev)
    ctxs, parts = [], []
    for r in range(world):
        lo, n = split_kv.shard_range(seq, world, r)
        cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=n, kv_dtype=rlcuda.RL_KV_BF16,
                                   max_batch=1)
        ctx = rlcuda.Context(cfg)
        ctx.set_shard(lo, seq)
        m = min(n, max(0, pos - lo))
        if m:
            ctx.write_kv(0, 0, np.ascontiguousarray(case.cache[:, :, lo:lo + m]))
        part = torch.empty((16, 258), device=dev)
        ctx.full_attn_partial(0, pos, qg, k, v, part)
        ctx.sync()
        ctxs.append(ctx)
        parts.append(part)
    out = torch.empty(16 * 256, device=dev)
    ctxs[0].merge_partials(torch.stack(parts), qg, out)
    ctxs[0].sync()
    got = out.cpu().numpy()[None]
    assert cases.rel_err_per_head(got, want, cases.HD) <= TOL
    owner = split_kv.owner_of(pos, seq, world)
    lo, _ = split_kv.shard_range(seq, world, owner)
    row = ctxs[owner].read_kv(0, pos - lo, 1)
    assert cases.rel_err_per_head(row, kv_want[:, :, pos:pos + 1], cases.HD) <= 1e-6
    for c in ctxs:
        c.close()


SEQ_4A = 131072


@functools.lru_cache(maxsize=1)
def _case_4a():
    """Config 4a's shape: one decode row at position 131071 over a bf16 cache
    of 131072 positions (seed 4), and the oracle's single pass over it."""
    pos = SEQ_4A - 1
    case = cases.full_case(4, pos, 1, kv_bf16=True)
    want, kv_want = cases.oracle_full(case, SEQ_4A, kv_bf16=True)
    return case, want, kv_want[:, :, pos:pos + 1].copy()


def test_config4a_single_gpu_pass_at_131072():
    case, want, row_want = _case_4a()
    pos = SEQ_4A - 1
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=SEQ_4A, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    with rlcuda.Context(cfg) as ctx:
        ctx.write_kv(0, 0, case.cache)
        got = ctx.full_attn_host(0, pos, case.qg.reshape(1, -1), case.k.reshape(1, -1),
                                 case.v.reshape(1, -1))
        assert cases.rel_err_per_head(got, want, cases.HD) <= TOL
        assert cases.rel_err_per_head(ctx.read_kv(0, pos, 1), row_want, cases.HD) <= 1e-6


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config4a_shards_at_131072(world):
    """Config 4a at its own size: 131072 positions split over 2, 4 and 8
    emulated shards.  Both exchanges must give the single-pass row: the
    gathered partials merged by rl_merge_partials, and the peer-memory
    exchange (rl_split_publish on every shard, then rl_split_merge on every
    shard)."""
    case, want, row_want = _case_4a()
    pos = SEQ_4A - 1
    dev = torch.device("cuda", 0)
    qg = torch.from_numpy(case.qg.reshape(-1)).to(dev)
    k = torch.from_numpy(case.k.reshape(-1)).to(dev)
    v = torch.from_numpy(case.v.reshape(-1)).to(dev)
    ctxs, parts = [], []
    try:
        for r in range(world):
            lo, n = split_kv.shard_range(SEQ_4A, world, r)
            cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=n,
                                       kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
            ctx = rlcuda.Context(cfg)
            ctxs.append(ctx)
            ctx.set_shard(lo, SEQ_4A)
            m = min(n, max(0, pos - lo))
            if m:
                ctx.write_kv(0, 0, np.ascontiguousarray(case.cache[:, :, lo:lo + m]))
            part = torch.empty((16, 258), device=dev)
            ctx.full_attn_partial(0, pos, qg, k, v, part)
            ctx.sync()
            parts.append(part)
        out = torch.empty(16 * 256, device=dev)
        ctxs[0].merge_partials(torch.stack(parts), qg, out)
        ctxs[0].sync()
        assert cases.rel_err_per_head(out.cpu().numpy()[None], want, cases.HD) <= TOL
        owner = split_kv.owner_of(pos, SEQ_4A, world)
        lo, _ = split_kv.shard_range(SEQ_4A, world, owner)
        assert cases.rel_err_per_head(ctxs[owner].read_kv(0, pos - lo, 1), row_want,
                                      cases.HD) <= 1e-6
        # the same step again over the peer exchange (the appended row is
        # rewritten with the same values)
        for r, c in enumerate(ctxs):
            c.exchange_init(r, world)
        bufs = [c.exchange_buffer() for c in ctxs]
        for c in ctxs:
            c.exchange_connect_ptrs(bufs)
        for c in ctxs:
            c.split_publish(0, pos, qg, k, v)
        for c in ctxs:
            c.sync()
        for r, c in enumerate(ctxs):
            out = torch.empty(16 * 256, device=dev)
            c.split_merge(qg, out)
            c.sync()
            assert cases.rel_err_per_head(out.cpu().numpy()[None], want, cases.HD) <= TOL, r
    finally:
        for c in ctxs:
            c.close()


def test_a_shard_context_refuses_the_single_gpu_entry_point():
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=128, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    with rlcuda.Context(cfg) as ctx:
        ctx.set_shard(128, 512)
        x = np.zeros((1, 16 * 512), np.float32)
        with pytest.raises(rlcuda.RlError):
            ctx.full_attn_host(0, 200, x, np.zeros((1, 1024), np.float32),
                               np.zeros((1, 1024), np.float32))
        with pytest.raises(rlcuda.RlError):
            ctx.set_shard(400, 512)  # 400 + 128 runs past the sequence


@pytest.mark.parametrize("world,seq", [(1, 700), (2, 4096), (4, 3000), (8, 8192)])
def test_peer_exchange_merges_to_the_single_pass_row(world, seq):
    """The exchange over peer memory (rl_split_publish / rl_split_merge),
    shards emulated on one GPU with their buffers connected by pointer:
    every shard publishes (pushing its partial and flag into every shard's
    buffer), then every shard merges.  Two steps, so both slots and both
    epochs are used; every shard's row must be the single-pass row."""
    dev = torch.device("cuda", 0)
    ctxs = []
    for r in range(world):
        lo, n = split_kv.shard_range(seq, world, r)
        cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=n, kv_dtype=rlcuda.RL_KV_BF16,
                                   max_batch=1)
        ctx = rlcuda.Context(cfg)
        ctx.set_shard(lo, seq)
        ctx.exchange_init(r, world)
        ctxs.append(ctx)
    bufs = [c.exchange_buffer() for c in ctxs]
    for c in ctxs:
        c.exchange_connect_ptrs(bufs)
    for step, pos in enumerate((seq - 2, seq - 1)):
        case = cases.full_case(90 + world + step, pos, 1, kv_bf16=True)
        want, _ = cases.oracle_full(case, seq, kv_bf16=True)
        qg = torch.from_numpy(case.qg.reshape(-1)).to(dev)
        k = torch.from_numpy(case.k.reshape(-1)).to(dev)
        v = torch.from_numpy(case.v.reshape(-1)).to(dev)
        for r, c in enumerate(ctxs):
            lo, n = split_kv.shard_range(seq, world, r)
            m = min(n, max(0, pos - lo))
            if m:
                c.write_kv(0, 0, np.ascontiguousarray(case.cache[:, :, lo:lo + m]))
            c.split_publish(0, pos, qg, k, v)
        for c in ctxs:
            c.sync()  # every flag is up before any merge waits on it
        for c in ctxs:
            out = torch.empty(16 * 256, device=dev)
            c.split_merge(qg, out)
            c.sync()
            got = out.cpu().numpy()[None]
            assert cases.rel_err_per_head(got, want, cases.HD) <= TOL, step
    for c in ctxs:
        c.close()


def test_a_peer_that_never_publishes_times_out_and_the_context_recovers():
    """Failure detection without a GPU fault: of two emulated shards only
    shard 0 publishes step 1, so shard 0's merge waits on a flag nothing
    sets.  With a 2 ms limit (RL_OPT_WAIT_LIMIT_US) the wait gives up, the
    next rl_sync reports RL_ETIMEOUT, and the same contexts then run the
    late shard's step and a full second step to the single-pass rows."""
    world, seq = 2, 4096
    dev = torch.device("cuda", 0)
    ctxs = []
    try:
        for r in range(world):
            lo, n = split_kv.shard_range(seq, world, r)
            cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=n,
                                       kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
            c = rlcuda.Context(cfg)
            ctxs.append(c)
            c.set_shard(lo, seq)
            c.exchange_init(r, world)
            c.set_option(rlcuda.RL_OPT_WAIT_LIMIT_US, 2000)
            assert c.get_option(rlcuda.RL_OPT_WAIT_LIMIT_US) == 2000
        bufs = [c.exchange_buffer() for c in ctxs]
        for c in ctxs:
            c.exchange_connect_ptrs(bufs)
        def step_inputs(step, pos):
            case = cases.full_case(140 + step, pos, 1, kv_bf16=True)
            want, _ = cases.oracle_full(case, seq, kv_bf16=True)
            for r, c in enumerate(ctxs):
                lo, n = split_kv.shard_range(seq, world, r)
                m = min(n, max(0, pos - lo))
                if m:
                    c.write_kv(0, 0, np.ascontiguousarray(case.cache[:, :, lo:lo + m]))
            inputs = [torch.from_numpy(x.reshape(-1)).to(dev) for x in (case.qg, case.k, case.v)]
            return pos, want, inputs

        # step 1: shard 1 is late; shard 0 publishes and its merge gives up
        pos, want, (qg, k, v) = step_inputs(0, seq - 2)
        ctxs[0].split_publish(0, pos, qg, k, v)
        ctxs[0].sync()
        out = torch.empty(16 * 256, device=dev)
        ctxs[0].split_merge(qg, out)
        with pytest.raises(rlcuda.RlError) as e:
            ctxs[0].sync()
        assert e.value.code == rlcuda.RL_ETIMEOUT
        ctxs[0].sync()  # the status was reported once and cleared
        # the late shard catches up on step 1: every flag is up for it
        ctxs[1].split_publish(0, pos, qg, k, v)
        ctxs[1].sync()
        ctxs[1].split_merge(qg, out)
        ctxs[1].sync()
        assert cases.rel_err_per_head(out.cpu().numpy()[None], want, cases.HD) <= TOL
        # step 2 runs normally on both
        pos, want, (qg, k, v) = step_inputs(1, seq - 1)
        for c in ctxs:
            c.split_publish(0, pos, qg, k, v)
        for c in ctxs:
            c.sync()
        for r, c in enumerate(ctxs):
            out = torch.empty(16 * 256, device=dev)
            c.split_merge(qg, out)
            c.sync()
            assert cases.rel_err_per_head(out.cpu().numpy()[None], want, cases.HD) <= TOL, r
    finally:
        for c in ctxs:
            c.close()


def test_exchange_contract_errors():
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=128, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    with rlcuda.Context(cfg) as ctx:
        ctx.set_shard(0, 256)
        x = torch.zeros(16 * 512, device="cuda")
        with pytest.raises(rlcuda.RlError):
            ctx.split_merge(x, torch.empty(4096, device="cuda"))  # nothing set up or published
        with pytest.raises(rlcuda.RlError):
            ctx.exchange_init(2, 2)  # rank outside the world
        ctx.exchange_init(0, 1)
        with pytest.raises(rlcuda.RlError):
            ctx.exchange_init(0, 1)  # twice


def test_peer_exchange_across_two_gpus():
    """Two processes, one GPU each, the buffers shared by CUDA IPC handles
    swapped over gloo: the ranks' rows equal the single-pass row."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [here, os.path.join(here, "..", "rust-llm_b200"), os.path.join(here, "..", "oracle"),
         os.environ.get("PYTHONPATH", "")]), NCCL_NVLS_ENABLE="0")
    r = subprocess.run(
        ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
         "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
         "29611", os.path.join(here, "split_exchange_worker.py")],
        env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("exchange ok") == 2, r.stdout[-2000:]
