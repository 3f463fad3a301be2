"""Batched decode (rl_batch_create / rl_batch_full_attn): one walk launch
gives every sequence the row rl_full_attn would give it on its own context.
Sequences of different lengths (so their CTAs draw different numbers of
tiles), several layers, the exact bf16-cache bar of the single decode: per
head 1e-4 against the oracle on the same bf16-rounded cache, and each
sequence's appended row lands in its own cache."""
import numpy as np
import pytest
import torch

import cases
import rlcuda

TOL = 1e-4
pytestmark = pytest.mark.gpu


def _batch_case(lengths, layers, seed):
    dev = torch.device("cuda", 0)
    ctxs, cs = [], []
    for i, n in enumerate(lengths):
        cfg = rlcuda.qwen35_config(n_full=layers, n_linear=0, context=n + 1,
                                   kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
        ctx = rlcuda.Context(cfg)
        per_layer = []
        for layer in range(layers):
            case = cases.full_case(seed + 37 * i + layer, n, 1, kv_bf16=True,
                                   unit_norms=layer % 2 == 0)
            ctx.write_kv(layer, 0, case.cache)
            ctx.set_weights_full(layer, case.q_norm, case.k_norm)
            per_layer.append(case)
        ctxs.append(ctx)
        cs.append(per_layer)
    return dev, ctxs, cs


@pytest.mark.parametrize("lengths", [[4097, 100, 2000, 64], [777], [30000, 4096, 17, 9000, 12345]])
def test_batch_rows_match_their_single_sequence_rows(lengths):
    layers = 2
    dev, ctxs, cs = _batch_case(lengths, layers, 1000 + len(lengths))
    n = len(lengths)
    pos = torch.tensor(lengths, dtype=torch.int32, device=dev)
    with rlcuda.Batch(ctxs) as b:
        for layer in range(layers):
            qg = torch.from_numpy(np.stack([cs[i][layer].qg.reshape(-1) for i in range(n)])).to(dev)
            k = torch.from_numpy(np.stack([cs[i][layer].k.reshape(-1) for i in range(n)])).to(dev)
            v = torch.from_numpy(np.stack([cs[i][layer].v.reshape(-1) for i in range(n)])).to(dev)
            out = torch.full((n, 16 * 256), float("nan"), device=dev)
            b.full_attn(layer, pos, qg, k, v, out)
            ctxs[0].sync()
            got = out.cpu().numpy()
            for i, length in enumerate(lengths):
                want, kv_want = cases.oracle_full(cs[i][layer], length + 1, kv_bf16=True)
                assert cases.rel_err_per_head(got[i:i + 1], want, cases.HD) <= TOL, (i, layer)
                row = ctxs[i].read_kv(layer, length, 1)
                assert cases.rel_err_per_head(row, kv_want[:, :, length:length + 1],
                                              cases.HD) <= 1e-6
    for c in ctxs:
        c.close()


def test_batch_contract_errors():
    a = rlcuda.Context(rlcuda.qwen35_config(n_full=1, n_linear=0, context=256,
                                            kv_dtype=rlcuda.RL_KV_BF16, max_batch=1))
    f = rlcuda.Context(rlcuda.qwen35_config(n_full=1, n_linear=0, context=256, max_batch=1))
    with pytest.raises(rlcuda.RlError):
        rlcuda.Batch([a, f])  # an f32 cache
    with rlcuda.Batch([a]) as b:
        x = torch.zeros((1, 16 * 512), device="cuda")
        with pytest.raises(rlcuda.RlError):
            b.full_attn(1, torch.zeros(1, dtype=torch.int32, device="cuda"), x,
                        torch.zeros((1, 1024), device="cuda"), torch.zeros((1, 1024), device="cuda"),
                        torch.zeros((1, 4096), device="cuda"))  # no layer 1
    a.close()
    f.close()
