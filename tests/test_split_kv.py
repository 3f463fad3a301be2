"""Host logic of the split-sequence decode (rust-llm_b200/split_kv.py) on CPU:
the range arithmetic, and two gloo ranks gathering and merging per-shard
partials into the row a single pass over the whole cache gives.  The
partials here are computed with numpy from raw queries (the GPU path's
kernels are covered by test_split_kv_gpu.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import split_kv

H, HD, NKV = 16, 256, 4
LOG2E = 1.4426950408889634


@pytest.mark.parametrize("seq,world", [(131072, 8), (131072, 2), (4096, 3), (100, 4), (64, 1),
                                       (65, 2), (1000, 7)])
def test_ranges_cover_the_sequence_once(seq, world):
    seen = np.zeros(seq, np.int32)
    prev_end = 0
    for r in range(world):
        lo, n = split_kv.shard_range(seq, world, r)
        assert lo == prev_end
        if r < world - 1 and lo + n < seq:
            assert n % 64 == 0
        seen[lo:lo + n] += 1
        prev_end = lo + n
    assert prev_end == seq and (seen == 1).all()
    for pos in (0, seq // 2, seq - 1):
        r = split_kv.owner_of(pos, seq, world)
        lo, n = split_kv.shard_range(seq, world, r)
        assert lo <= pos < lo + n


def _partial(q, K, V, n_valid):
    """[H][HD+2]: unnormalised output, max (log2 units), sum, over the first
    n_valid rows of this shard's K/V [NKV][n][HD]."""
    out = np.zeros((H, HD + 2), np.float64)
    for h in range(H):
        if n_valid == 0:
            out[h, HD] = -np.inf
            continue
        s = (K[h // 4, :n_valid] @ q[h]) / 16.0 * LOG2E
        m = s.max()
        w = np.exp2(s - m)
        out[h, :HD] = w @ V[h // 4, :n_valid]
        out[h, HD] = m
        out[h, HD + 1] = w.sum()
    return out


def _merge(parts, gate):
    m = parts[:, :, HD]
    M = m.max(0)
    sc = np.where(np.isinf(m), 0.0, np.exp2(m - M))
    L = (parts[:, :, HD + 1] * sc).sum(0)
    o = (parts[:, :, :HD] * sc[:, :, None]).sum(0) / L[:, None]
    return o * (1.0 / (1.0 + np.exp(-gate)))


class NumpyShard:
    def __init__(self, K, V, lo):
        self.K, self.V, self.lo = K, V, lo

    def partial(self, layer, pos, qg, k, v, out_partial):
        q = qg.numpy().reshape(H, 2 * HD)[:, :HD].astype(np.float64)
        n_valid = max(0, min(pos + 1 - self.lo, self.K.shape[1]))
        out_partial.copy_(torch.from_numpy(_partial(q, self.K, self.V, n_valid)).float())

    def merge(self, parts, qg, out):
        gate = qg.numpy().reshape(H, 2 * HD)[:, HD:].astype(np.float64)
        out.copy_(torch.from_numpy(_merge(parts.double().numpy(), gate).reshape(-1)).float())


def _rank(rank, world, port, seq, pos, res):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        K = rng.standard_normal((NKV, seq, HD))
        V = rng.standard_normal((NKV, seq, HD))
        qg = torch.from_numpy(rng.standard_normal(H * 2 * HD)).float()
        lo, n = split_kv.shard_range(seq, world, rank)
        dec = split_kv.SplitDecoder(NumpyShard(K[:, lo:lo + n], V[:, lo:lo + n], lo), world, rank,
                                    H, HD, make=lambda shape: torch.zeros(shape))
        out = torch.zeros(H * HD)
        dec.step(0, pos, qg, None, None, out)
        res[rank] = out.numpy().copy()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,seq,pos", [(2, 300, 299), (2, 300, 40), (3, 200, 199)])
def test_gloo_ranks_merge_to_the_single_pass_row(world, seq, pos):
    res = mp.get_context("spawn").Manager().dict()  # no fork of a threaded process
    mp.spawn(_rank, args=(world, _free_port(), seq, pos, res), nprocs=world, join=True)
    rng = np.random.default_rng(7)
    K = rng.standard_normal((NKV, seq, HD))
    V = rng.standard_normal((NKV, seq, HD))
    qg = rng.standard_normal(H * 2 * HD).reshape(H, 2 * HD)
    want = _merge(_partial(qg[:, :HD], K, V, pos + 1)[None], qg[:, HD:]).reshape(-1)
    for r in range(world):
        np.testing.assert_allclose(res[r], want, rtol=2e-5, atol=2e-6)


def test_sequence_partition_balances_context():
    """Config 4b's partition: 64 sequences with contexts U[4096, 32768],
    longest first to the least-loaded GPU; every sequence exactly once and the
    heaviest GPU within one longest sequence of the mean."""
    import numpy as np
    lens = [int(x) for x in np.random.default_rng(5).integers(4096, 32769, 64)]
    for world in (1, 2, 4, 8):
        parts = split_kv.partition_sequences(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)
        assert max(loads) <= sum(lens) / world + max(lens)
    assert split_kv.partition_sequences([5, 9, 1], 2) == [[1], [0, 2]]


def _handles_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    got = split_kv.connect_handles(bytes([rank]) * 64, world)
    q.put((rank, got))
    dist.destroy_process_group()


def test_exchange_handles_arrive_in_rank_order():
    """The peer exchange's set-up swaps each rank's 64-byte IPC handle over
    the process group; every rank must see all of them in rank order."""
    world = 3
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_handles_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r] == [bytes([g]) * 64 for g in range(world)]
    assert split_kv.connect_handles(b"x" * 64, 1) == [b"x" * 64]
