"""GPU, at the configurations' own sizes: the full config-2 model (32 layers, hidden 4096, 32/8
heads, FFN 12288, vocab 151936, Q4_K/Q6_K) against the CPU oracle through the C ABI.

  * greedy identity: a 512-token prompt of uniform random ids, then 256 greedy steps; the token
    sequences must be identical and every step's logits within 1e-3 relative L2. The smallest
    top-2 logit margin of the oracle over the 256 steps is reported (a margin far above the
    logit error means the identity is not luck).
  * decode attention at context 4096 (the benchmark's length, 64 key splits by default) on a
    one-layer model of the config-2 widths.
  * acceptance at the full vocabulary (151936 ids, 149 summation blocks of the blocked softmax)
    over the config-3 draft tree [4, 2, 2, 1] at temperature 0.7: bit-exact with the oracle.
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

RTOL = 1e-3
VOCAB = 151936


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


def tree_from_branching(branching):
    parents, level = [-1], [0]
    for b in branching:
        nxt = []
        for v in level:
            for _ in range(b):
                parents.append(v)
                nxt.append(len(parents) - 1)
        level = nxt
    return parents


def test_config2_greedy_identity_256_steps(kq, oracle, record_property):
    prompt_len, steps = 512, 256
    ids = [int(v) for v in oracle.gen_tokens(prompt_len, VOCAB, 1, 1)]
    e = kq.Engine(kq.Config.default(), seed=0)
    o = oracle.Model(seed=0)
    try:
        e.feed_batch(ids[:-1], 0)                     # the prompt through the batched pass
        for i, t in enumerate(ids[:-1]):              # the oracle token by token (cpu4.py:227-236)
            o.step(t, i, head=False)
        pos, te, to = prompt_len - 1, ids[-1], ids[-1]
        got, ref, margins, errs = [], [], [], []
        for k in range(steps):
            a = e.step(te, pos)
            b = o.step(to, pos)
            zo = o.logits()
            top2 = np.partition(zo, -2)[-2:]
            margins.append(float(top2[1] - top2[0]))
            errs.append(rel_l2(e.ylog, zo))
            got.append(a)
            ref.append(b)
            if a != b:
                break
            te, to, pos = a, b, pos + 1
    finally:
        e.close()
        o.close()
    k_min = int(np.argmin(margins))
    record_property("min_top2_margin", margins[k_min])
    record_property("max_logit_rel_l2", max(errs))
    print("config-2 greedy: %d steps, smallest oracle top-2 margin %.4g (step %d), logits rel-L2 first %.3g "
          "median %.3g largest %.3g (step %d)" % (len(got), margins[k_min], k_min, errs[0], float(np.median(errs)),
                                                  max(errs), int(np.argmax(errs))))
    assert got == ref, ("first divergence at step %d; oracle top-2 margin there %.4g" % (len(got) - 1, margins[-1]))
    assert len(got) == steps
    assert max(errs) < RTOL, max(errs)


@pytest.mark.parametrize("npos", [4031, 4095, 4096])
def test_decode_attention_at_context_4096(kq, oracle, npos):
    """One layer of the config-2 widths, K/V filled to npos positions, one decode step at npos:
    the position range of the benchmark (K/V pre-filled to 4031 plus the timed steps)."""
    t = dict(NL=1, vocab=4096, ctx=4097)
    e = kq.Engine(kq.Config.default(n_layers=1, vocab=4096, ctx=4097), seed=0)
    o = oracle.Model(seed=0, **t)
    try:
        e.fill_kv(npos, 3)
        o.fill_kv(npos, 3)
        a = e.step(11, npos)
        b = o.step(11, npos)
        assert rel_l2(e.ylog, o.logits()) < RTOL
        assert rel_l2(e.hidden(), o.hidden()) < RTOL
        assert a == b
    finally:
        e.close()
        o.close()


@pytest.mark.parametrize("splits", ["1", "7", "18", "64"])
@pytest.mark.parametrize("npos", [31, 4095])
def test_decode_attention_splits(kq, oracle, monkeypatch, splits, npos):
    """The decode step's tensor-core attention over key-split counts from 1 to 64, at a short
    context (most splits empty) and at the benchmark's, three consecutive steps."""
    monkeypatch.setenv("KQ_DSPLIT", splits)
    t = dict(NL=1, vocab=4096, ctx=4100)
    e = kq.Engine(kq.Config.default(n_layers=1, vocab=4096, ctx=4100), seed=0)
    o = oracle.Model(seed=0, **t)
    try:
        e.fill_kv(npos, 3)
        o.fill_kv(npos, 3)
        for k in range(3):
            a = e.step(11 + k, npos + k)
            b = o.step(11 + k, npos + k)
            assert rel_l2(e.hidden(), o.hidden()) < RTOL
            assert rel_l2(e.ylog, o.logits()) < RTOL
            assert a == b
    finally:
        e.close()
        o.close()


@pytest.mark.parametrize("temperature", [0.7, 0.0])
def test_accept_bit_exact_at_full_vocabulary(kq, oracle, temperature):
    """Config-3's acceptance over a vocabulary of 151936 ids: tree [4, 2, 2, 1] (45 nodes),
    draft distributions softmax of N(0, 2) logits, seeded uniforms; half the drafts are sampled
    from their parent's q so that some are accepted."""
    e = kq.Engine(kq.Config.default(dim=512, n_layers=1, n_heads=4, n_kv_heads=1, ffn=1024, ctx=256), seed=0)
    try:
        rng = np.random.default_rng(2)
        npos = 100
        e.fill_kv(npos, 5)
        parents = tree_from_branching([4, 2, 2, 1])
        n = len(parents)
        assert n == 45
        g = rng.normal(0.0, 2.0, (n, VOCAB)).astype(np.float32)
        toks = [int(rng.integers(0, VOCAB))]
        for c in range(1, n):
            if c % 2:
                q = np.exp(g[parents[c]].astype(np.float64) - g[parents[c]].max())
                toks.append(int(rng.choice(VOCAB, p=q / q.sum())))
            else:
                toks.append(int(rng.integers(0, VOCAB)))
        _, z = e.verify(toks, parents, npos)
        u_acc = rng.random(n).astype(np.float32)
        u_fin = rng.random(n).astype(np.float32)
        path, out = e.accept(toks, parents, g, temperature, u_acc, u_fin)
        opath, oout = oracle.accept(z, g, toks, parents, temperature, u_acc, u_fin)
        assert path == opath
        assert out == oout
        for j in range(1, len(path)):
            assert parents[path[j]] == path[j - 1]
            assert out[j - 1] == toks[path[j]]
    finally:
        e.close()
