"""GPU: speculative verification over a draft tree (kq_verify), on-device acceptance (kq_accept)
and K/V compaction (kq_commit) against the CPU oracle (or_verify / or_accept / or_commit).

Bars: verify logits within 1e-3 relative L2 of the oracle, a linear chain verified in one call
reproduces the greedy decode steps token for token, acceptance bit-exact given identical logits
and uniforms (greedy and stochastic), compacted K/V rows equal to the oracle's."""
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
    monkeypatch.setenv("KQ_PERSIST", "1" if request.param == "persistent" else "0")
    return request.param


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


def tree_from_branching(branching):
    """Parent pointers of a breadth-first tree: node 0, then branching[0] children of it, ..."""
    parents = [-1]
    level = [0]
    for b in branching:
        nxt = []
        for v in level:
            for _ in range(b):
                parents.append(v)
                nxt.append(len(parents) - 1)
        level = nxt
    return parents


def draft_tokens(parents, vocab, rng):
    return [int(v) for v in rng.integers(0, vocab, len(parents))]


def test_tree_verify_matches_oracle(kq, oracle):
    t = dict(TINY, NH=8, NKV=2, D=1024, NFF=2048, NL=2)
    e = kq.Engine(kq_cfg(kq, t), seed=0)
    o = oracle.Model(seed=0, **t)
    npos = 150
    e.fill_kv(npos, 3)
    o.fill_kv(npos, 3)
    parents = tree_from_branching([3, 2, 1])
    toks = draft_tokens(parents, t["vocab"], np.random.default_rng(5))
    best, logits = e.verify(toks, parents, npos)
    obest, ologits = o.verify(toks, parents, npos)
    for i in range(len(parents)):
        assert rel_l2(logits[i], ologits[i]) < 1e-3, i
        top2 = np.sort(ologits[i])[-2:]
        if top2[1] - top2[0] > 1e-3 * np.abs(ologits[i]).max():
            assert best[i] == obest[i], i
    # the K/V rows of the tree slots
    n = npos + len(parents)
    Kg = e.get_kv(t["NL"] - 1, 0, n).view(np.float16).astype(np.float32)
    Ko = o.kcache(t["NL"] - 1, n).view(np.float16).astype(np.float32)
    assert rel_l2(Kg, Ko) < 1e-3


@pytest.mark.parametrize("seq", [1, 0])
def test_chain_verify_reproduces_greedy_steps(kq, monkeypatch, seq):
    """A linear chain verified in one call against the same steps decoded one by one: identical
    ids node by node (KQ_VERIFY_SEQ=1: each node is a decode step), or, for the batched
    tensor-core pass, logits within 1e-3 and identical ids wherever the top-2 margin is clear."""
    monkeypatch.setenv("KQ_VERIFY_SEQ", str(seq))
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    npos = 40
    e.fill_kv(npos, 4)
    chain, step_logits = [17], []
    for i in range(6):
        chain.append(e.step(chain[-1], npos + i))
        step_logits.append(e.ylog)
    e.fill_kv(npos, 4)
    parents = [-1] + list(range(len(chain) - 1))
    best, logits = e.verify(chain, parents, npos)
    if seq:
        assert list(best[:-1]) == chain[1:]
    for i, ref in enumerate(step_logits):
        assert rel_l2(logits[i], ref) < 1e-3
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 1e-2 * np.abs(ref).max():
            assert best[i] == chain[i + 1]


@pytest.mark.parametrize("form", ["1", "0"])   # KQ_ACCEPT_GRID: the cooperative multi-CTA kernel, the one-CTA kernel
@pytest.mark.parametrize("temperature", [0.0, 0.7, 1.3])
@pytest.mark.parametrize("branching,seed", [([4, 2, 2, 1], 1), ([2, 2, 2], 2), ([1] * 8, 3), ([], 4)])
def test_accept_bit_exact_with_oracle(kq, oracle, monkeypatch, temperature, branching, seed, form):
    monkeypatch.setenv("KQ_ACCEPT_GRID", form)
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    rng = np.random.default_rng(100 + seed)
    npos = 60
    e.fill_kv(npos, 5)
    parents = tree_from_branching(branching)
    n = len(parents)
    g = rng.normal(0.0, 2.0, (n, TINY["vocab"])).astype(np.float32)
    # drafts sampled from each parent's q (so that some are accepted), others uniform
    toks = [int(rng.integers(0, TINY["vocab"]))]
    for c in range(1, n):
        q = np.exp(g[parents[c]] - g[parents[c]].max())
        toks.append(int(rng.choice(TINY["vocab"], p=q / q.sum())) if c % 2 else int(rng.integers(0, TINY["vocab"])))
    _, z = e.verify(toks, parents, npos)
    u_acc = rng.random(n).astype(np.float32)
    u_fin = rng.random(n).astype(np.float32)
    path, out = e.accept(toks, parents, g, temperature, u_acc, u_fin)
    opath, oout = oracle.accept(z, g, toks, parents, temperature, u_acc, u_fin)
    assert path == opath
    assert out == oout
    assert len(out) == len(path)
    for j in range(1, len(path)):
        assert parents[path[j]] == path[j - 1]
        assert out[j - 1] == toks[path[j]]


def test_accept_resident_draft_equals_host_draft(kq):
    """Draft logits already on the device (kq_draft_upload + kq_accept_resident) give the same
    decision as the host copy."""
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    rng = np.random.default_rng(21)
    e.fill_kv(50, 5)
    parents = tree_from_branching([3, 2])
    n = len(parents)
    toks = [int(v) for v in rng.integers(0, TINY["vocab"], n)]
    g = rng.normal(0.0, 2.0, (n, TINY["vocab"])).astype(np.float32)
    ua, uf = rng.random(n).astype(np.float32), rng.random(n).astype(np.float32)
    e.verify(toks, parents, 50, want_logits=False)
    a = e.accept(toks, parents, g, 0.9, ua, uf)
    e.upload_draft(g)
    b = e.accept(toks, parents, None, 0.9, ua, uf, resident=True)
    assert a == b
    ptr, ld = e.draft_logits_device()
    assert ptr and ld == TINY["vocab"]


def test_accept_full_path_when_draft_equals_target(kq, oracle):
    """q = p: every draft is accepted (u * q(d) < p(d) for u < 1)."""
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    npos = 30
    e.fill_kv(npos, 6)
    parents = tree_from_branching([1] * 5)
    toks = [3, 9, 27, 81, 243, 729]
    _, z = e.verify(toks, parents, npos)
    T = 0.7
    g = (z / np.float32(T)).astype(np.float32)   # softmax(g) == softmax(z / T) up to rounding
    rng = np.random.default_rng(9)
    u_acc = (rng.random(len(toks)) * 0.5).astype(np.float32)
    u_fin = rng.random(len(toks)).astype(np.float32)
    path, out = e.accept(toks, parents, g, T, u_acc, u_fin)
    opath, oout = oracle.accept(z, g, toks, parents, T, u_acc, u_fin)
    assert (path, out) == (opath, oout)
    assert path == list(range(len(toks)))


def test_greedy_accept_of_greedy_chain_takes_all(kq, monkeypatch):
    monkeypatch.setenv("KQ_VERIFY_SEQ", "1")   # node-by-node verification reproduces decode exactly
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    npos = 25
    e.fill_kv(npos, 7)
    chain = [5]
    for i in range(5):
        chain.append(e.step(chain[-1], npos + i))
    e.fill_kv(npos, 7)
    parents = [-1] + list(range(len(chain) - 1))
    best, _ = e.verify(chain, parents, npos, want_logits=False)
    path, out = e.accept(chain, parents, temperature=0.0)
    assert path == list(range(len(chain)))
    assert out == chain[1:] + [int(best[-1])]


def test_commit_matches_oracle_and_decoding_continues(kq, oracle):
    t = TINY
    e = kq.Engine(kq_cfg(kq, t), seed=0)
    o = oracle.Model(seed=0, **t)
    npos = 80
    e.fill_kv(npos, 8)
    o.fill_kv(npos, 8)
    parents = tree_from_branching([3, 2, 2])
    rng = np.random.default_rng(11)
    toks = draft_tokens(parents, t["vocab"], rng)
    e.verify(toks, parents, npos, want_logits=False)
    o.verify(toks, parents, npos)
    path = [0]                                 # root to leaf through each node's last child
    while any(parents[c] == path[-1] for c in range(len(parents))):
        path.append(max(c for c in range(len(parents)) if parents[c] == path[-1]))
    assert len(path) == 4 and all(parents[path[j]] == path[j - 1] for j in range(1, len(path)))
    e.commit(path, npos)
    o.commit(path, npos)
    n = npos + len(path)
    for layer in range(t["NL"]):
        for which in (0, 1):
            g = e.get_kv(layer, which, n).view(np.float16).astype(np.float32)
            ref = (o.kcache if which == 0 else o.vcache)(layer, n).view(np.float16).astype(np.float32)
            assert rel_l2(g[npos * 128:], ref[npos * 128:]) < 1e-3
    # decoding continues after the accepted tokens
    nxt = toks[path[-1]]
    a = e.step(nxt, npos + len(path))
    b = o.step(nxt, npos + len(path))
    assert a == b


def test_argument_errors(kq):
    e = kq.Engine(kq_cfg(kq, TINY), seed=0)
    with pytest.raises(ValueError):
        e.verify([1, 2, 3], [-1, 0, 5], 10)            # parent after child
    with pytest.raises(ValueError):
        e.verify([1, 2], [0, 0], 10)                   # root must have parent -1
    with pytest.raises(ValueError):
        e.verify([1] * 129, [-1] + list(range(128)), 10)
    with pytest.raises(ValueError):
        e.verify([1, TINY["vocab"]], [-1, 0], 10)      # bad token
    with pytest.raises(OverflowError):
        e.verify([1, 2, 3], [-1, 0, 1], TINY["ctx"] - 2)
    e.verify([1, 2, 3], [-1, 0, 1], 10, want_logits=False)
    with pytest.raises(ValueError):
        e.accept([1, 2], [-1, 0])                      # not the verified tree
    with pytest.raises(ValueError):
        e.accept([1, 2, 3], [-1, 0, 1], temperature=0.7)   # stochastic needs q and uniforms
    with pytest.raises(ValueError):
        e.commit([0, 2, 1], 10)                        # node ids must increase
