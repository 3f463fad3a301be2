"""Worker of test_split_kv_gpu.test_peer_exchange_across_two_gpus: one rank
per GPU holds its range of a 4096-position sequence, the ranks swap their
exchange buffers' CUDA IPC handles over a gloo group, and three decode rows
go through rl_full_attn_split; each rank checks its row against the oracle's
single pass and prints "exchange ok"."""
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

import cases
import rlcuda
import split_kv

SEQ = 4096


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    dev = torch.device("cuda", local)
    lo, n = split_kv.shard_range(SEQ, world, rank)
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=n, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    ctx = rlcuda.Context(cfg, device=local)
    shard = split_kv.GpuShard(ctx, lo, SEQ, exchange=True, rank=rank, world=world)
    for step, pos in enumerate((SEQ - 3, SEQ - 2, SEQ - 1)):
        case = cases.full_case(500 + step, pos, 1, kv_bf16=True)
        want, _ = cases.oracle_full(case, SEQ, kv_bf16=True)
        m = min(n, max(0, pos - lo))
        if m:
            ctx.write_kv(0, 0, np.ascontiguousarray(case.cache[:, :, lo:lo + m]))
        ctx.sync()
        dist.barrier()  # every rank's cache holds this step's prefix
        qg = torch.from_numpy(case.qg.reshape(-1)).to(dev)
        k = torch.from_numpy(case.k.reshape(-1)).to(dev)
        v = torch.from_numpy(case.v.reshape(-1)).to(dev)
        out = torch.empty(16 * 256, device=dev)
        shard.split(0, pos, qg, k, v, out)
        ctx.sync()
        err = cases.rel_err_per_head(out.cpu().numpy()[None], want, cases.HD)
        assert err <= 1e-4, (rank, step, err)
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    print("exchange ok", rank, flush=True)


if __name__ == "__main__":
    main()
