"""GPU: batched decode of many sequences (kq_batch_caches / kq_batch_feed / kq_batch_step) against
each sequence decoded alone by the whole-model path (kq_feed_batch + kq_step). Every sequence
has its own K/V cache; one step runs one token of each sequence through the batched pass with
attention over each token's own cache. Bar: identical greedy ids, step by step, and the cache
rows within 1e-3 relative L2."""
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


def engine(kq):
    t = CFG
    cfg = kq.Config.default(dim=t["D"], n_layers=t["NL"], n_heads=t["NH"], n_kv_heads=t["NKV"], head_dim=t["HD"],
                            ffn=t["NFF"], vocab=t["vocab"], ctx=t["ctx"])
    return kq.Engine(cfg, seed=0)


def test_batched_steps_match_single_sequences(kq):
    rng = np.random.default_rng(12)
    lens = [37, 150, 5, 90]
    prompts = [[int(v) for v in rng.integers(0, CFG["vocab"], n)] for n in lens]
    nsteps = 6
    # reference: each sequence alone
    ref = []
    single = engine(kq)
    for p in prompts:
        single.reset()
        single.feed_batch(p[:-1], 0)
        toks, t = [], p[-1]
        for i in range(nsteps):
            t = single.step(t, len(p) - 1 + i)
            toks.append(t)
        ref.append(toks)
    single.close()
    # batched: sequences 3, 0, 2, 1 of four caches
    e = engine(kq)
    e.batch_caches(4)
    order = [3, 0, 2, 1]
    for s in order:
        e.batch_feed(s, prompts[s][:-1], 0)
    cur = [prompts[s][-1] for s in order]
    pos = [len(prompts[s]) - 1 for s in order]
    got = [[] for _ in order]
    for i in range(nsteps):
        cur = e.batch_step(order, cur, pos)
        for j in range(len(order)):
            got[j].append(cur[j])
        pos = [p + 1 for p in pos]
    for j, s in enumerate(order):
        assert got[j] == ref[s], (s, got[j], ref[s])


def test_batched_step_arguments(kq):
    e = engine(kq)
    with pytest.raises(ValueError):
        e.batch_step([0], [1], [0])            # no caches yet
    e.batch_caches(2)
    with pytest.raises(ValueError):
        e.batch_step([0, 0], [1, 2], [3, 3])   # one token per sequence
    with pytest.raises(ValueError):
        e.batch_step([2], [1], [0])            # sequence out of range
    with pytest.raises(OverflowError):
        e.batch_step([1], [1], [CFG["ctx"]])
