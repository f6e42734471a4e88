"""GPU: prefill (kq_feed_batch) as batched tensor-core passes of up to 128 tokens, each a linear
chain with a causal mask, against the CPU oracle fed token by token (the reference's
feed_batch, gpu4.py:109-110). Bars: every layer's K/V cache rows within 1e-3 relative L2, the
greedy steps that follow identical, and the decode-step path (KQ_VERIFY_SEQ=1) unchanged."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

CFG = dict(D=1024, NL=2, NH=8, NKV=2, HD=128, NFF=2048, vocab=4096, ctx=512)


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


def engine(kq, t):
    cfg = kq.Config.default(dim=t["D"], n_layers=t["NL"], n_heads=t["NH"], n_kv_heads=t["NKV"], head_dim=t["HD"],
                            ffn=t["NFF"], vocab=t["vocab"], ctx=t["ctx"])
    return kq.Engine(cfg, seed=0)


@pytest.mark.parametrize("n,pos0", [(2, 0), (37, 0), (128, 0), (200, 0), (300, 40)])
def test_prefill_cache_matches_oracle(kq, oracle, n, pos0):
    e = engine(kq, CFG)
    o = oracle.Model(seed=0, **CFG)
    rng = np.random.default_rng(n)
    toks = [int(v) for v in rng.integers(0, CFG["vocab"], n)]
    if pos0:
        e.fill_kv(pos0, 4)
        o.fill_kv(pos0, 4)
    e.feed_batch(toks, pos0)
    for i, t in enumerate(toks):
        o.step(t, pos0 + i, head=False)
    end = pos0 + n
    for layer in range(CFG["NL"]):
        for which in (0, 1):
            g = e.get_kv(layer, which, end).view(np.float16).astype(np.float32)
            ref = (o.kcache if which == 0 else o.vcache)(layer, end).view(np.float16).astype(np.float32)
            assert rel_l2(g, ref) < 1e-3, (layer, which)
    # greedy steps continue from the prefilled cache
    a = b = int(rng.integers(0, CFG["vocab"]))
    for i in range(8):
        a = e.step(a, end + i)
        b = o.step(b, end + i)
        assert a == b, i


def test_generate_uses_prefill_and_matches_oracle(kq, oracle):
    t = dict(CFG, ctx=256)
    e = engine(kq, t)
    o = oracle.Model(seed=0, **t)
    ids = [int(v) for v in np.random.default_rng(7).integers(0, t["vocab"], 150)]
    assert e.generate(ids, 24) == o.generate(ids, 24)


def test_prefill_rejects_bad_input(kq):
    e = engine(kq, CFG)
    with pytest.raises(ValueError):
        e.feed_batch([1, CFG["vocab"]], 0)
    with pytest.raises(OverflowError):
        e.feed_batch([1] * 20, CFG["ctx"] - 10)
