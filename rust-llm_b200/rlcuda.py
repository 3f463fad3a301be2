"""Python host wrapper over the C ABI of librlcuda.so (include/rlcuda.h).

It mirrors the reference's interface for the attention path: a context that
owns the caches (``Caches``, crates/rust-llm/src/forward.rs:236-254), the two
attention calls ``full_attn`` / ``linear_attn`` (forward.rs:1220, :1484) and
the lifecycle ``reset`` / ``accept`` / ``pos`` (forward.rs:553-688).  Errors
come back as :class:`RlError` carrying the library's status and message, the
way the reference's contract violations panic.

There is no fallback: if librlcuda.so is missing or cannot be loaded this
module raises on import of the library.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# RLCUDA_LIB points at a library built elsewhere (default: the in-tree build)
LIB_PATH = os.environ.get("RLCUDA_LIB") or os.path.join(HERE, "librlcuda.so")

RL_OK, RL_EINVAL, RL_ECONTEXT, RL_ECUDA, RL_ENCCL, RL_ETIMEOUT, RL_EUNSUPPORTED, RL_ENOMEM = (
    0, -1, -2, -3, -4, -5, -6, -7)
RL_KV_F32, RL_KV_BF16 = 0, 1
(RL_OPT_SPLITS, RL_OPT_PREFILL_ROWS, RL_OPT_CHUNK_ROWS, RL_OPT_CLUSTER, RL_OPT_EARLY_TILES,
 RL_OPT_VERIFY_TC, RL_OPT_DN_ROWS, RL_OPT_WAIT_LIMIT_US, RL_OPT_WALK_SPANS,
 RL_OPT_DN_SCAN_TC, RL_OPT_DN_OVERLAP, RL_OPT_DN_LOCAL_TC) = range(12)
PROF_KERNELS = ("prologue", "decode", "merge", "dn_step", "prefill", "dn_chunk", "verify",
                "walk_span")
HOST, DEVICE = 0, 1
RL_IPC_HANDLE_BYTES = 64
RL_EXCHANGE_MAX_GPUS = 8

_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_i = ctypes.c_int


class RlError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rlcuda status {code}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    """rl_config (include/rlcuda.h)."""

    _fields_ = [
        ("n_full", ctypes.c_int32),
        ("n_linear", ctypes.c_int32),
        ("n_head", ctypes.c_int32),
        ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_rot", ctypes.c_int32),
        ("rope_theta", ctypes.c_float),
        ("rms_eps", ctypes.c_float),
        ("d_state", ctypes.c_int32),
        ("n_k_heads", ctypes.c_int32),
        ("n_v_heads", ctypes.c_int32),
        ("conv_kernel", ctypes.c_int32),
        ("context", ctypes.c_int32),
        ("slots", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
    ]

    @property
    def conv_dim(self) -> int:
        return 2 * self.n_k_heads * self.d_state + self.n_v_heads * self.d_state


def qwen35_config(n_full=1, n_linear=1, context=2048, slots=1, kv_dtype=RL_KV_F32,
                  max_batch=16) -> Config:
    """The Qwen3.5-4B attention shapes (the reference's docs/models.md:100-105)."""
    return Config(n_full, n_linear, 16, 4, 256, 64, 1e7, 1e-6, 128, 16, 32, 4, context, slots,
                  kv_dtype, max_batch)


# Every symbol include/rlcuda.h declares, with its ctypes signature.
SIGNATURES = {
    "rl_ctx_create": ([_i, ctypes.POINTER(Config), ctypes.POINTER(_vp)], _i),
    "rl_ctx_destroy": ([_vp], None),
    "rl_last_error": ([_vp], ctypes.c_char_p),
    "rl_set_stream": ([_vp, _vp], _i),
    "rl_get_stream": ([_vp], _vp),
    "rl_reset": ([_vp], _i),
    "rl_set_weights_full": ([_vp, _i, _f32p, _f32p], _i),
    "rl_set_weights_linear": ([_vp, _i, _f32p, _f32p, _f32p, _f32p], _i),
    "rl_full_attn": ([_vp, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
    "rl_full_attn_host": ([_vp, _i, _i, _i, _f32p, _f32p, _f32p, _f32p], _i),
    "rl_linear_attn": ([_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "rl_linear_attn_host": ([_vp, _i, _i, _i, _f32p, _f32p, _f32p, _f32p, _f32p], _i),
    "rl_accept": ([_vp, _i], _i),
    "rl_pos": ([_vp], _i),
    "rl_live": ([_vp], _i),
    "rl_sync": ([_vp], _i),
    "rl_set_option": ([_vp, _i, ctypes.c_int64], _i),
    "rl_get_option": ([_vp, _i], ctypes.c_int64),
    "rl_write_kv": ([_vp, _i, _i, _i, _vp, _i], _i),
    "rl_read_kv": ([_vp, _i, _i, _i, _vp, _i], _i),
    "rl_write_conv": ([_vp, _i, _vp, _i], _i),
    "rl_read_conv": ([_vp, _i, _vp, _i], _i),
    "rl_write_ssm": ([_vp, _i, _vp, _i], _i),
    "rl_read_ssm": ([_vp, _i, _vp, _i], _i),
    "rl_profile_enable": ([_vp, _i], _i),
    "rl_profile_read": ([_vp, _i, ctypes.POINTER(ctypes.c_double),
                         ctypes.POINTER(ctypes.c_int64)], _i),
    "rl_profile_reset": ([_vp], _i),
    "rl_full_attn_noalloc": ([ctypes.POINTER(Config), _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp,
                              _vp, _vp], _i),
    "rl_noalloc_status": ([_vp], _i),
    "rl_act_quantize": ([_vp, _vp, _i, _i], _i),
    "rl_matvec": ([_vp, _i, _vp, _i, _vp], _i),
    "rl_matvec_group": ([_vp, _i, ctypes.POINTER(_i), ctypes.POINTER(_vp), ctypes.POINTER(_i),
                         ctypes.POINTER(_vp)], _i),
    "rl_matmul_group": ([_vp, _vp, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_vp),
                         ctypes.POINTER(_i), ctypes.POINTER(_vp)], _i),
    "rl_set_shard": ([_vp, _i, _i], _i),
    "rl_full_attn_partial": ([_vp, _i, _i, _vp, _vp, _vp, _vp], _i),
    "rl_merge_partials": ([_vp, _i, _vp, _vp, _vp], _i),
    "rl_exchange_init": ([_vp, _i, _i, _vp], _i),
    "rl_exchange_connect": ([_vp, _vp], _i),
    "rl_exchange_connect_ptrs": ([_vp, ctypes.POINTER(ctypes.c_uint64)], _i),
    "rl_exchange_buffer": ([_vp], ctypes.c_uint64),
    "rl_split_publish": ([_vp, _i, _i, _vp, _vp, _vp], _i),
    "rl_split_merge": ([_vp, _vp, _vp], _i),
    "rl_full_attn_split": ([_vp, _i, _i, _vp, _vp, _vp, _vp], _i),
    "rl_batch_create": ([ctypes.POINTER(_vp), _i, ctypes.POINTER(_vp)], _i),
    "rl_batch_full_attn": ([_vp, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "rl_batch_destroy": ([_vp], None),
    "rl_version": ([], ctypes.c_char_p),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads librlcuda.so, raising if it is absent: there is no CPU fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python rust-llm_b200/build.py` "
                "(nvcc, sm_100a); the attention path has no fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _ptr(x) -> int:
    """A device pointer: a torch tensor (its data_ptr) or an int."""
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return int(x)


class Context:
    """One device's attention caches and the calls that run on them."""

    def __init__(self, cfg: Config, device: int = 0):
        self.cfg = cfg
        self.device = device
        h = _vp()
        self._L = lib()
        code = self._L.rl_ctx_create(device, ctypes.byref(cfg), ctypes.byref(h))
        if code:
            raise RlError(code, self._L.rl_last_error(None).decode())
        self._h = h

    # -- lifecycle -------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            self._L.rl_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, code: int):
        if code:
            raise RlError(code, self._L.rl_last_error(self._h).decode())

    @property
    def handle(self):
        return self._h

    def reset(self):
        self._check(self._L.rl_reset(self._h))

    def accept(self, rows: int):
        self._check(self._L.rl_accept(self._h, rows))

    @property
    def pos(self) -> int:
        return self._L.rl_pos(self._h)

    @property
    def live(self) -> int:
        return self._L.rl_live(self._h)

    def sync(self):
        self._check(self._L.rl_sync(self._h))

    def set_stream(self, stream_ptr: int):
        self._check(self._L.rl_set_stream(self._h, stream_ptr))

    def set_option(self, opt: int, value: int):
        self._check(self._L.rl_set_option(self._h, opt, value))

    def get_option(self, opt: int) -> int:
        return int(self._L.rl_get_option(self._h, opt))

    # -- per-kernel timing -----------------------------------------------
    def profile(self, on: bool):
        self._check(self._L.rl_profile_enable(self._h, int(on)))

    def profile_reset(self):
        self._check(self._L.rl_profile_reset(self._h))

    def profile_read(self) -> dict:
        """{kernel: (total_ms, launches)} since the last reset."""
        out = {}
        for k, name in enumerate(PROF_KERNELS):
            ms = ctypes.c_double()
            n = ctypes.c_int64()
            self._check(self._L.rl_profile_read(self._h, k, ctypes.byref(ms), ctypes.byref(n)))
            out[name] = (ms.value, n.value)
        return out

    # -- weights ---------------------------------------------------------
    def set_weights_full(self, layer, q_norm, k_norm):
        q_norm = np.ascontiguousarray(q_norm, np.float32)
        k_norm = np.ascontiguousarray(k_norm, np.float32)
        self._check(self._L.rl_set_weights_full(self._h, layer, _p(q_norm), _p(k_norm)))

    def set_weights_linear(self, layer, conv1d, ssm_a, dt_bias, norm):
        a = [np.ascontiguousarray(x, np.float32) for x in (conv1d, ssm_a, dt_bias, norm)]
        self._check(self._L.rl_set_weights_linear(self._h, layer, *(_p(x) for x in a)))

    # -- the two attention calls ----------------------------------------
    def full_attn_host(self, layer, pos, qg, k, v) -> np.ndarray:
        """Host arrays in, host array out (the Runner drop-in path)."""
        t = qg.shape[0]
        qg, k, v = (np.ascontiguousarray(x, np.float32) for x in (qg, k, v))
        out = np.empty((t, self.cfg.n_head * self.cfg.head_dim), np.float32)
        self._check(self._L.rl_full_attn_host(self._h, layer, pos, t, _p(qg), _p(k), _p(v),
                                              _p(out)))
        return out

    def full_attn(self, layer, pos, t, qg, k, v, out):
        """Device pointers (torch tensors or ints); enqueued, not waited for."""
        self._check(self._L.rl_full_attn(self._h, layer, pos, t, _ptr(qg), _ptr(k), _ptr(v),
                                         _ptr(out)))

    # -- a sequence split across GPUs -----------------------------------
    def set_shard(self, lo: int, seq_context: int):
        self._check(self._L.rl_set_shard(self._h, lo, seq_context))

    def full_attn_partial(self, layer, pos, qg, k, v, partial):
        """Device tensors; partial [n_head][head_dim + 2] f32."""
        self._check(self._L.rl_full_attn_partial(self._h, layer, pos, _ptr(qg), _ptr(k), _ptr(v),
                                                 _ptr(partial)))

    def merge_partials(self, parts, qg, out):
        """parts [n_parts][n_head][head_dim + 2] f32 (device) -> out [n_head*head_dim]."""
        self._check(self._L.rl_merge_partials(self._h, int(parts.shape[0]), _ptr(parts), _ptr(qg),
                                              _ptr(out)))

    # -- split sequence over peer memory (rl_exchange_*) --------------------
    def exchange_init(self, rank: int, world: int) -> bytes:
        """Allocates this GPU's exchange buffer; returns its CUDA IPC handle."""
        h = ctypes.create_string_buffer(RL_IPC_HANDLE_BYTES)
        self._check(self._L.rl_exchange_init(self._h, rank, world, h))
        return h.raw

    def exchange_connect(self, handles):
        """Every rank's handle, in rank order (this rank's own is ignored)."""
        blob = b"".join(handles)
        self._check(self._L.rl_exchange_connect(self._h, blob))

    def exchange_connect_ptrs(self, bufs):
        """Every rank's exchange buffer as a device pointer of this process."""
        arr = (ctypes.c_uint64 * len(bufs))(*bufs)
        self._check(self._L.rl_exchange_connect_ptrs(self._h, arr))

    def exchange_buffer(self) -> int:
        return int(self._L.rl_exchange_buffer(self._h))

    # -- projections ----------------------------------------------------
    def act_quantize(self, x, t: int, k: int):
        """Activations::quantize_batch on device rows x [t][k]."""
        self._check(self._L.rl_act_quantize(self._h, _ptr(x), t, k))

    def matvec(self, ggml_type: int, w, rows: int, out):
        """out [t][rows] = W . x against the last quantized activations."""
        self._check(self._L.rl_matvec(self._h, ggml_type, _ptr(w), rows, _ptr(out)))

    def matvec_group(self, parts):
        """parts: [(ggml_type, w, rows, out)] sharing the last quantized
        activations, one launch."""
        n = len(parts)
        types = (_i * n)(*[p[0] for p in parts])
        ws = (_vp * n)(*[_ptr(p[1]) for p in parts])
        rows = (_i * n)(*[p[2] for p in parts])
        outs = (_vp * n)(*[_ptr(p[3]) for p in parts])
        self._check(self._L.rl_matvec_group(self._h, n, types, ws, rows, outs))

    def matmul_group(self, x, t: int, k: int, parts):
        """Exec::matmul_group: x [t][k] quantized and dotted with every
        (ggml_type, w, rows, out) of parts, one launch."""
        n = len(parts)
        types = (_i * n)(*[p[0] for p in parts])
        ws = (_vp * n)(*[_ptr(p[1]) for p in parts])
        rows = (_i * n)(*[p[2] for p in parts])
        outs = (_vp * n)(*[_ptr(p[3]) for p in parts])
        self._check(self._L.rl_matmul_group(self._h, _ptr(x), t, k, n, types, ws, rows, outs))

    def split_publish(self, layer, pos, qg, k, v):
        self._check(self._L.rl_split_publish(self._h, layer, pos, _ptr(qg), _ptr(k), _ptr(v)))

    def split_merge(self, qg, out):
        self._check(self._L.rl_split_merge(self._h, _ptr(qg), _ptr(out)))

    def full_attn_split(self, layer, pos, qg, k, v, out):
        self._check(self._L.rl_full_attn_split(self._h, layer, pos, _ptr(qg), _ptr(k), _ptr(v),
                                               _ptr(out)))

    def linear_attn_host(self, layer, live, qkv, z, alpha, beta) -> np.ndarray:
        t = qkv.shape[0]
        qkv, z, alpha, beta = (np.ascontiguousarray(x, np.float32) for x in (qkv, z, alpha, beta))
        out = np.empty((t, self.cfg.n_v_heads * self.cfg.d_state), np.float32)
        self._check(self._L.rl_linear_attn_host(self._h, layer, live, t, _p(qkv), _p(z),
                                                _p(alpha), _p(beta), _p(out)))
        return out

    def linear_attn(self, layer, live, t, qkv, z, alpha, beta, out):
        self._check(self._L.rl_linear_attn(self._h, layer, live, t, _ptr(qkv), _ptr(z),
                                           _ptr(alpha), _ptr(beta), _ptr(out)))

    # -- state -----------------------------------------------------------
    def write_kv(self, layer, p0, src):
        """src [2][n_kv][n][hd] f32: a numpy array (host) or a torch CUDA tensor."""
        n = src.shape[2]
        if isinstance(src, np.ndarray):
            src = np.ascontiguousarray(src, np.float32)
            self._check(self._L.rl_write_kv(self._h, layer, p0, n, src.ctypes.data, HOST))
        else:
            self._check(self._L.rl_write_kv(self._h, layer, p0, n, src.data_ptr(), DEVICE))

    def read_kv(self, layer, p0, n) -> np.ndarray:
        c = self.cfg
        out = np.empty((2, c.n_head_kv, n, c.head_dim), np.float32)
        self._check(self._L.rl_read_kv(self._h, layer, p0, n, out.ctypes.data, HOST))
        return out

    def _state_shape(self, ssm: bool):
        c = self.cfg
        if ssm:
            return (c.n_v_heads, c.slots, c.d_state, c.d_state)
        return (c.slots, c.conv_dim, c.conv_kernel - 1)

    def write_conv(self, layer, src):
        src = np.ascontiguousarray(src, np.float32).reshape(self._state_shape(False))
        self._check(self._L.rl_write_conv(self._h, layer, src.ctypes.data, HOST))

    def read_conv(self, layer) -> np.ndarray:
        out = np.empty(self._state_shape(False), np.float32)
        self._check(self._L.rl_read_conv(self._h, layer, out.ctypes.data, HOST))
        return out

    def write_ssm(self, layer, src):
        src = np.ascontiguousarray(src, np.float32).reshape(self._state_shape(True))
        self._check(self._L.rl_write_ssm(self._h, layer, src.ctypes.data, HOST))

    def read_ssm(self, layer) -> np.ndarray:
        out = np.empty(self._state_shape(True), np.float32)
        self._check(self._L.rl_read_ssm(self._h, layer, out.ctypes.data, HOST))
        return out


class Batch:
    """Batched decode over many contexts (rl_batch_*): one walk launch per
    layer for one decode row of every sequence.  Runs on the first context's
    stream; close it before its contexts."""

    def __init__(self, ctxs):
        self.ctxs = list(ctxs)
        self._L = self.ctxs[0]._L
        arr = (_vp * len(self.ctxs))(*[c.handle for c in self.ctxs])
        h = _vp()
        code = self._L.rl_batch_create(arr, len(self.ctxs), ctypes.byref(h))
        if code:
            raise RlError(code, self._L.rl_last_error(self.ctxs[0].handle).decode())
        self._h = h

    def full_attn(self, layer, pos, qg, k, v, out):
        """Device tensors: pos [n] int32, qg [n][n_head*2*hd], k, v [n][n_kv*hd],
        out [n][n_head*hd]."""
        self.ctxs[0]._check(self._L.rl_batch_full_attn(self._h, layer, _ptr(pos), _ptr(qg), _ptr(k),
                                                       _ptr(v), _ptr(out)))

    def close(self):
        if getattr(self, "_h", None):
            self._L.rl_batch_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
