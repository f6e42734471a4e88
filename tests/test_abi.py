"""The C-ABI library: it loads, exports every symbol include/kq.h declares, and the Python shim
binds exactly those. No compute call is made here (no GPU needed)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "kq.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kq_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("kq_model_create", "kq_step", "kq_feed", "kq_qmat_matvec", "kq_qmat_dequant", "kq_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import kq
    path = kq.LIB_PATH
    assert os.path.exists(path), "libkq.so not built"
    lib = ctypes.CDLL(path)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_shim_binds_exactly_the_header():
    import kq
    assert sorted(kq.SIGNATURES) == declared_symbols()


def test_version_and_error_without_gpu_work():
    import kq
    assert kq.lib().kq_version() >= 100
    assert isinstance(kq.last_error(), str)


def test_no_silent_cpu_path_without_device():
    """On a host without a GPU the engine must fail loudly, never compute on the CPU."""
    import kq
    if kq.lib().kq_device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises((RuntimeError, ValueError, MemoryError)):
        kq.Engine(kq.Config.default(n_layers=1, vocab=1024, ctx=64))
    with pytest.raises((RuntimeError, ValueError, MemoryError)):
        kq.QMat(12, 8, 256)


def test_config_default_is_baseline_config2():
    import kq
    c = kq.Config.default()
    assert (c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab) == (4096, 32, 32, 8, 128, 12288, 151936)
    assert (c.t_q, c.t_k, c.t_v, c.t_o, c.t_gate, c.t_up, c.t_down, c.t_emb, c.t_out) == (12, 12, 14, 12, 12, 12, 14, 12, 14)
    assert abs(c.rope_theta - 1e6) < 1 and abs(c.eps - 1e-6) < 1e-12
