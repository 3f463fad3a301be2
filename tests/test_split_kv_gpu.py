"""A sequence split across GPUs, emulated on one device: each shard is its
own context (rl_set_shard), each walks its range (rl_full_attn_partial) and
rl_merge_partials merges the shards' partials.  The merged row must match
the oracle's single pass over the whole cache (forward.rs:1259-1340), and
the new key/value row must land in the shard that holds its position."""
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
