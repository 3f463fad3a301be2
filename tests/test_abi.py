"""The C ABI library loads and exports every symbol include/rlcuda.h declares
(CPU only: no compute calls), and the host-side contract checks that need no
device answer as the reference's contract does."""
import os
import re
import subprocess

import pytest

import rlcuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "rlcuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rl_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    import build  # rust-llm_b200/build.py
    build.build()
    assert os.path.exists(rlcuda.LIB_PATH)
    assert rlcuda.lib().rl_version().decode().startswith("rlcuda")


def test_every_declared_symbol_is_exported_and_bound():
    names = header_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", rlcuda.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (rl_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    unbound = [n for n in names if n not in rlcuda.SIGNATURES]
    assert not unbound, unbound
    L = rlcuda.lib()
    for n in names:
        assert getattr(L, n) is not None


def test_null_context_is_an_error_not_a_crash():
    L = rlcuda.lib()
    assert L.rl_pos(None) == -1
    assert L.rl_live(None) == -1
    assert L.rl_accept(None, 1) == rlcuda.RL_EINVAL
    assert L.rl_reset(None) == rlcuda.RL_EINVAL
    assert b"NULL" in L.rl_last_error(None)
    L.rl_ctx_destroy(None)


def test_unsupported_shapes_are_refused_before_any_device_work():
    cfg = rlcuda.qwen35_config()
    cfg.head_dim = 128
    with pytest.raises(rlcuda.RlError) as e:
        rlcuda.Context(cfg)
    assert e.value.code == rlcuda.RL_EUNSUPPORTED
    cfg = rlcuda.qwen35_config()
    cfg.kv_dtype = 7
    with pytest.raises(rlcuda.RlError) as e:
        rlcuda.Context(cfg)
    assert e.value.code == rlcuda.RL_EINVAL


def test_noalloc_refuses_misaligned_or_bad_arguments_before_any_launch():
    """rl_full_attn_noalloc checks its arguments before it touches the
    device, so these run without a GPU: the pointers are never dereferenced."""
    import ctypes
    L = rlcuda.lib()
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=1024, kv_dtype=rlcuda.RL_KV_BF16,
                               max_batch=1)
    good = 0x10000

    def call(cfg=cfg, **over):
        p = dict(k_cache=good, v_cache=good, q_norm=good, k_norm=good, qg=good, k=good, v=good,
                 out=good)
        p.update(over)
        return L.rl_full_attn_noalloc(ctypes.byref(cfg), None, p["k_cache"], p["v_cache"],
                                      p["q_norm"], p["k_norm"], 10, 1, p["qg"], p["k"], p["v"],
                                      p["out"])

    for name in ("k_cache", "v_cache", "q_norm", "k_norm", "qg", "k", "v", "out"):
        assert call(**{name: good + 8}) == rlcuda.RL_EINVAL, name
        assert name.encode() in L.rl_last_error(None), name
    bad = rlcuda.qwen35_config(n_full=1, n_linear=0, context=1024, kv_dtype=rlcuda.RL_KV_BF16)
    bad.n_rot = 8
    assert call(cfg=bad) == rlcuda.RL_EINVAL
    assert b"multiple of 16" in L.rl_last_error(None)
