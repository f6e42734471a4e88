"""GPU: the whole dense GQA decode step (config-2 architecture) against the CPU oracle through the
C ABI: greedy tokens identical, logits and hidden state within 1e-3 relative L2, K/V cache rows."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TINY = dict(D=512, NL=2, NH=4, NKV=1, HD=128, NFF=1024, vocab=4096, ctx=512)


def kq_cfg(kq, t):
    return kq.Config.default(dim=t["D"], n_layers=t["NL"], n_heads=t["NH"], n_kv_heads=t["NKV"], head_dim=t["HD"],
                             ffn=t["NFF"], vocab=t["vocab"], ctx=t["ctx"])


@pytest.fixture(params=["persistent", "launches"], autouse=True)
def decode_path(request, monkeypatch):
    """Every test runs on both decode paths: the persistent one-kernel-per-token decode
    (KQ_PERSIST=1) and the per-operation launches in a CUDA graph (the default); the variable is
    read when a model is created."""
    monkeypatch.setenv("KQ_PERSIST", "1" if request.param == "persistent" else "0")
    return request.param


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


@pytest.mark.parametrize("t", [TINY, dict(TINY, NH=8, NKV=2, D=1024, NFF=2048, NL=3), dict(TINY, NH=8, NKV=8, NL=1),
                               dict(TINY, NH=16, NKV=2, D=2048, NFF=4096, NL=2, vocab=2048)])
def test_step_logits_and_greedy(kq, oracle, t):
    e = kq.Engine(kq_cfg(kq, t), seed=0)
    o = oracle.Model(seed=0, **t)
    ids = [int(v) for v in oracle.gen_tokens(12, t["vocab"], 1, 1)]
    got = e.generate(ids, 16)
    ref = o.generate(ids, 16)
    assert got == ref
    assert rel_l2(e.ylog, o.logits()) < 1e-3
    assert rel_l2(e.hidden(), o.hidden()) < 1e-3
    # K/V cache rows of the last layer
    n = len(ids) + 15
    Kg = e.get_kv(t["NL"] - 1, 0, n).view(np.float16).astype(np.float32)
    Ko = o.kcache(t["NL"] - 1, n).view(np.float16).astype(np.float32)
    assert rel_l2(Kg, Ko) < 1e-3
    Vg = e.get_kv(t["NL"] - 1, 1, n).view(np.float16).astype(np.float32)
    Vo = o.vcache(t["NL"] - 1, n).view(np.float16).astype(np.float32)
    assert rel_l2(Vg, Vo) < 1e-3


def test_long_context_attention(kq, oracle):
    t = dict(TINY, NL=1, ctx=1100)
    e = kq.Engine(kq_cfg(kq, t), seed=0)
    o = oracle.Model(seed=0, **t)
    for npos in (127, 128, 129, 1000):
        e.reset(); o.reset()
        e.fill_kv(npos, 3); o.fill_kv(npos, 3)
        a = e.step(11, npos)
        b = o.step(11, npos)
        assert a == b
        assert rel_l2(e.ylog, o.logits()) < 1e-3


def test_device_loop_matches_host_steps(kq, oracle):
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    ids = [3, 1, 4, 1, 5]
    ref = e.generate(ids, 10)
    e.reset()
    for i, tk in enumerate(ids[:-1]):
        e.feed(tk, i)
    got = e.decode_loop(ids[-1], len(ids) - 1, 10)
    assert got == ref


def test_engine_argument_errors(kq):
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    with pytest.raises(ValueError):
        e.step(-1, 0)
    with pytest.raises(ValueError):
        e.step(TINY["vocab"], 0)
    with pytest.raises(OverflowError):
        e.step(0, TINY["ctx"])
    with pytest.raises(ValueError):
        e.set_tensor(0, kq.T_Q, np.zeros(10, np.uint8))
