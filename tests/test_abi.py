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
