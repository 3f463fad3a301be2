"""The attention-only greedy-token harness.

A 32-layer toy stack with the Qwen3.5 hybrid layout (full attention at
layer il when il % 4 == 3, Gated DeltaNet elsewhere; the reference's
docs/models.md:96) and the attention shapes of the path (16 query heads, 4 KV
heads, head_dim 256; 16 q/k heads and 32 v heads of 128 for DeltaNet).
Everything outside the attention ops is one shared host implementation:
token embedding, per-layer RMS-scaled input, seeded f32 projections into
the attention inputs (qg, k, v for a full layer; qkv, z, alpha, beta for a
DeltaNet layer), the output projection added to the residual stream, and an
argmax head over a 256-token vocabulary.  Two backends supply the attention
ops: the oracle's restatement of Exec::full_attn / Exec::linear_attn
(forward.rs:1259-1340, :1530-1652) and the sm_100a library through its C
ABI.  Because only the attention differs, the greedy tokens of the two runs
must be identical.
"""
import numpy as np

import oracle as orc

N_LAYERS = 32
VOCAB = 256
D_MODEL = 128
N_HEAD, N_KV, HD = 16, 4, 256
CONV_DIM, N_V, S = 8192, 32, 128


def is_full(il: int) -> bool:
    return il % 4 == 3


class ToyStack:
    """Seeded weights of the toy stack.  Projection weights are N(0, 1/d_in)
    so every projected input is roughly unit-variance, as the BASELINE
    configs draw them."""

    def __init__(self, seed: int):
        r = np.random.default_rng(seed)

        def w(n_out, n_in):
            return (r.standard_normal((n_out, n_in)) / np.sqrt(n_in)).astype(np.float32)

        self.embed = r.standard_normal((VOCAB, D_MODEL)).astype(np.float32)
        self.head = w(VOCAB, D_MODEL)
        self.layers = []
        for il in range(N_LAYERS):
            if is_full(il):
                self.layers.append(dict(
                    wqg=w(N_HEAD * 2 * HD, D_MODEL), wk=w(N_KV * HD, D_MODEL),
                    wv=w(N_KV * HD, D_MODEL), wo=w(D_MODEL, N_HEAD * HD) * 0.5,
                    q_norm=(1.0 + 0.1 * r.standard_normal(HD)).astype(np.float32),
                    k_norm=(1.0 + 0.1 * r.standard_normal(HD)).astype(np.float32)))
            else:
                a_log = r.uniform(0.0, np.log(16.0), N_V)
                self.layers.append(dict(
                    wqkv=w(CONV_DIM, D_MODEL), wz=w(N_V * S, D_MODEL), wa=w(N_V, D_MODEL),
                    wb=w(N_V, D_MODEL), wo=w(D_MODEL, N_V * S) * 0.5,
                    conv1d=(0.5 * r.standard_normal((CONV_DIM, 4))).astype(np.float32),
                    ssm_a=(-np.exp(a_log)).astype(np.float32),
                    dt_bias=(0.1 * r.standard_normal(N_V)).astype(np.float32),
                    norm=(1.0 + 0.1 * r.standard_normal(S)).astype(np.float32)))

    def logits(self, backend, rows, pos: int, live: int = 0) -> np.ndarray:
        """One pass of the stack over a batch of rows at positions pos.. (ring
        slot `live` for the DeltaNet layers); the logits of every row.  Every
        host-side product is taken one row at a time, so a row's numbers do
        not depend on the batch around it: a verify batch's row then differs
        from the same token's single pass only through the attention ops."""
        x = self.embed[np.asarray(rows)]                           # [t][d]
        for il, lw in enumerate(self.layers):
            h = np.stack([_rms(r) for r in x])
            if is_full(il):
                o = backend.full(il // 4, pos, _proj(lw["wqg"], h), _proj(lw["wk"], h),
                                 _proj(lw["wv"], h))
            else:
                o = backend.linear(il - (il + 1) // 4, live, _proj(lw["wqkv"], h),
                                   _proj(lw["wz"], h), _proj(lw["wa"], h), _proj(lw["wb"], h))
            x = (x + _proj(lw["wo"], o)).astype(np.float32)
        return np.stack([self.head @ _rms(r) for r in x]).astype(np.float32)

    def run(self, backend, prompt, n_new: int):
        """Feeds the prompt as one batch of rows, then decodes greedily one
        row at a time; returns the n_new generated tokens."""
        r = Runner(self, backend)
        nxt = int(np.argmax(r.forward_batch(prompt)))
        out = [nxt]
        for _ in range(n_new - 1):
            nxt = int(np.argmax(r.forward_batch([nxt])))
            out.append(nxt)
        return out


def _rms(x):
    return (x / np.sqrt((x * x).mean() + 1e-6)).astype(np.float32)


def _proj(w, h):
    return np.stack([w @ r for r in h]).astype(np.float32)


class Runner:
    """The reference Runner's position and ring bookkeeping over a backend
    (forward.rs:641-688): forward_batch runs rows and commits them all;
    verify runs rows and commits none; accept(rows >= 1) moves pos and the
    live ring slot, with no copy, so a rollback is a smaller accept."""

    def __init__(self, stack: ToyStack, backend):
        self.stack, self.backend = stack, backend
        self.slots = getattr(backend, "slots", 1)
        self.pos = self.live = 0
        self.batch = 0

    def verify(self, rows) -> np.ndarray:
        assert len(rows) <= self.slots or self.slots == 1
        out = self.stack.logits(self.backend, rows, self.pos, self.live)
        self.batch = len(rows)
        return out

    def accept(self, rows: int):
        assert 1 <= rows <= self.batch
        self.pos += rows
        self.live = (self.live + rows) % self.slots
        if hasattr(self.backend, "accept"):
            self.backend.accept(rows)
        self.batch = 0

    def forward_batch(self, rows) -> np.ndarray:
        """The logits of the token after the last row."""
        out = self.stack.logits(self.backend, rows, self.pos, self.live)
        self.batch = len(rows)
        self.accept(len(rows))
        return out[-1]


class OracleBackend:
    """The oracle's restatement, with f32 caches and ring states it owns."""

    def __init__(self, stack: ToyStack, context: int, slots: int = 1):
        self.cfg = orc.qwen35_config(context)
        self.stack = stack
        self.slots = slots
        self.kv = [np.zeros((2, N_KV, context, HD), np.float32) for _ in range(N_LAYERS // 4)]
        n_lin = N_LAYERS - N_LAYERS // 4
        self.conv = [np.zeros((slots, CONV_DIM, 3), np.float32) for _ in range(n_lin)]
        self.ssm = [np.zeros((N_V, slots, S, S), np.float32) for _ in range(n_lin)]
        self.full_w = [lw for il, lw in enumerate(stack.layers) if is_full(il)]
        self.lin_w = [lw for il, lw in enumerate(stack.layers) if not is_full(il)]

    def full(self, layer, pos, qg, k, v):
        w = self.full_w[layer]
        return orc.full_attn(self.cfg, pos, qg, k, v, self.kv[layer], w["q_norm"], w["k_norm"],
                             threads=8)

    def linear(self, layer, live, qkv, z, alpha, beta):
        w = self.lin_w[layer]
        return orc.linear_attn(self.cfg, self.slots, live, qkv, z, alpha, beta, self.conv[layer],
                               self.ssm[layer], w["conv1d"], w["ssm_a"], w["dt_bias"], w["norm"],
                               threads=8)


class DeviceBackend:
    """The sm_100a library through rl_full_attn_host / rl_linear_attn_host."""

    def __init__(self, stack: ToyStack, context: int, max_batch: int, kv_dtype=None,
                 slots: int = 1):
        import rlcuda
        kv_dtype = rlcuda.RL_KV_F32 if kv_dtype is None else kv_dtype
        self.slots = slots
        cfg = rlcuda.qwen35_config(n_full=N_LAYERS // 4, n_linear=N_LAYERS - N_LAYERS // 4,
                                   context=context, slots=slots, kv_dtype=kv_dtype,
                                   max_batch=max_batch)
        self.ctx = rlcuda.Context(cfg)
        fi = li = 0
        for il, lw in enumerate(stack.layers):
            if is_full(il):
                self.ctx.set_weights_full(fi, lw["q_norm"], lw["k_norm"])
                fi += 1
            else:
                self.ctx.set_weights_linear(li, lw["conv1d"], lw["ssm_a"], lw["dt_bias"],
                                            lw["norm"])
                li += 1

    def full(self, layer, pos, qg, k, v):
        return self.ctx.full_attn_host(layer, pos, qg, k, v)

    def linear(self, layer, live, qkv, z, alpha, beta):
        return self.ctx.linear_attn_host(layer, live, qkv, z, alpha, beta)

    def accept(self, rows):
        # the context's own pos / live follow the runner's (rl_accept)
        self.ctx.accept(rows)

    def close(self):
        self.ctx.close()
