"""The oracle's dense GQA decoder (config-2 architecture) against independent numpy restatements
of each reference building block, on a tiny configuration (no GPU)."""
import numpy as np
import pytest

from conftest import rel_l2

TINY = dict(D=512, NL=2, NH=4, NKV=1, HD=128, NFF=1024, vocab=2048, ctx=64)


def test_rmsnorm_matches_reference_formula(oracle):
    # kcpu4.c:123-139: fp64 sum of squares, s = 1/sqrtf((float)(sum/D) + eps), xn = (h*s)*w
    import ctypes as C
    D = 4096
    h = oracle.gen_normal(D, 0.0, 3.0, 1, 1)
    y = oracle.gen_normal(D, 0.0, 1.0, 1, 2)
    w = oracle.gen_normal(D, 1.0, 0.02, 0, 3)
    hh, xn = h.copy(), np.empty(D, np.float32)
    oracle.lib().or_rmsnorm(oracle.ptr(hh), oracle.ptr(y), 1, oracle.ptr(w), oracle.ptr(xn), D, np.float32(1e-6))
    ref_h = (h + y).astype(np.float32)
    acc = 0.0
    for v in ref_h.astype(np.float64):
        acc += v * v
    s = np.float32(1.0) / np.sqrt(np.float32(acc / D) + np.float32(1e-6), dtype=np.float32)
    ref = (ref_h * s).astype(np.float32) * w
    assert np.array_equal(hh, ref_h)
    assert np.array_equal(xn, ref.astype(np.float32))


def test_decoder_step_matches_numpy(oracle):
    """One token through the tiny model, recomputed in numpy fp64 from the same tensors."""
    m = oracle.Model(seed=0, **TINY)
    c = m.cfg
    tok, pos = 17, 0
    m.step(tok, pos)
    logits = m.logits()
    # numpy restatement
    def mat(layer, kind, R, Cc, ty):
        W = np.ctypeslib.as_array(oracle.lib().or_model_tensor(m.h, layer, kind), shape=(R * (Cc // 256) * oracle.BLOCK[ty],))
        return oracle.decode_blocks(W.reshape(-1, oracle.BLOCK[ty]), ty).reshape(R, Cc).astype(np.float64)
    QD, KD = c.NH * c.HD, c.NKV * c.HD
    h = mat(-1, oracle.T_EMB, c.vocab, c.D, c.t_emb)[tok]
    rh = c.HD // 2
    inv = np.float64(c.rope_theta) ** (-2.0 * np.arange(rh) / c.HD)
    cs, sn = np.cos(pos * inv).astype(np.float32), np.sin(pos * inv).astype(np.float32)
    def norm(x, w):
        return x / np.sqrt(np.mean(x * x) + 1e-6) * w
    y = np.zeros(c.D)
    for l in range(c.NL):
        an = oracle.gen_normal(c.D, 1.0, 0.02, 0, oracle.stream(l, oracle.T_ATTN_NORM)).astype(np.float64)
        fn = oracle.gen_normal(c.D, 1.0, 0.02, 0, oracle.stream(l, oracle.T_FFN_NORM)).astype(np.float64)
        h = h + y
        xn = norm(h, an)
        q = mat(l, oracle.T_Q, QD, c.D, c.t_q) @ xn
        k = mat(l, oracle.T_K, KD, c.D, c.t_k) @ xn
        v = mat(l, oracle.T_V, KD, c.D, c.t_v) @ xn
        def rope(x):
            x = x.reshape(-1, c.HD)
            a, b = x[:, :rh], x[:, rh:]
            return np.concatenate([a * cs - b * sn, a * sn + b * cs], 1)
        qr, kr = rope(q), rope(k)
        kh = kr.astype(np.float16).astype(np.float64)
        vh = v.reshape(-1, c.HD).astype(np.float16).astype(np.float64)
        G = c.NH // c.NKV
        att = np.zeros((c.NH, c.HD))
        for hh in range(c.NH):
            kv = hh // G
            s = (kh[kv] @ qr[hh]) / np.sqrt(c.HD)          # one position: softmax = 1
            att[hh] = vh[kv]
        y = mat(l, oracle.T_O, c.D, QD, c.t_o) @ att.reshape(-1)
        h = h + y
        xn = norm(h, fn)
        g = mat(l, oracle.T_GATE, c.NFF, c.D, c.t_gate) @ xn
        u = mat(l, oracle.T_UP, c.NFF, c.D, c.t_up) @ xn
        y = mat(l, oracle.T_DOWN, c.D, c.NFF, c.t_down) @ (g / (1 + np.exp(-g)) * u)
    h = h + y
    on = oracle.gen_normal(c.D, 1.0, 0.02, 0, oracle.stream(-1, oracle.T_OUTNORM)).astype(np.float64)
    ref = mat(-1, oracle.T_OUT, c.vocab, c.D, c.t_out) @ norm(h, on)
    assert rel_l2(logits, ref) < 1e-5
    assert rel_l2(m.hidden(), h) < 1e-5


def test_attention_over_many_positions(oracle):
    """Scores, softmax and P.V over a pre-filled fp16 cache (kcpu4.c:244-282) vs numpy."""
    m = oracle.Model(seed=0, **dict(TINY, NL=1))
    c = m.cfg
    npos = 40
    m.fill_kv(npos, 5)
    m.step(3, npos)              # attends over positions 0..npos
    K = m.kcache(0, npos + 1).reshape(npos + 1, c.NKV, c.HD).view(np.float16).astype(np.float64)
    V = m.vcache(0, npos + 1).reshape(npos + 1, c.NKV, c.HD).view(np.float16).astype(np.float64)
    assert np.isfinite(K).all() and np.isfinite(V).all()
    # the freshly stored row is what the step produced; the pre-filled rows are the generator's
    K2 = oracle.Model(seed=0, **dict(TINY, NL=1))
    K2.fill_kv(npos, 5)
    assert np.array_equal(K2.kcache(0, npos), m.kcache(0, npos))


def test_greedy_generate_is_deterministic(oracle):
    m = oracle.Model(seed=0, **TINY)
    a = m.generate([5, 6, 7, 8], 6)
    b = m.generate([5, 6, 7, 8], 6)
    assert a == b and len(a) == 6 and all(0 <= t < TINY["vocab"] for t in a)


def test_bad_token_rejected(oracle):
    m = oracle.Model(seed=0, **TINY)
    with pytest.raises(ValueError):
        m.step(TINY["vocab"], 0)
    with pytest.raises(ValueError):
        m.step(0, TINY["ctx"])


def test_oracle_exp_accuracy(oracle):
    """kq_exp (the acceptance rule's e^t) is within 2 ulp of e^t on [-87, 0] and 0 below."""
    import ctypes as C
    L = oracle.lib()
    ts = np.linspace(-87.0, 0.0, 4001).astype(np.float32)
    got = np.array([L.or_kq_exp(float(t)) for t in ts], np.float64)
    ref = np.exp(ts.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 2 * 2.0 ** -24
    assert L.or_kq_exp(-87.5) == 0.0 and L.or_kq_exp(-np.inf) == 0.0


def test_oracle_accept_rules(oracle):
    """Greedy and stochastic acceptance on small hand-made trees."""
    V = 2048
    rng = np.random.default_rng(3)
    z = rng.normal(0, 3, (4, V)).astype(np.float32)
    parents = [-1, 0, 0, 1]
    best0, best1 = int(np.argmax(z[0])), int(np.argmax(z[1]))
    # greedy: the second child of the root matches, then node 3 does not
    toks = [7, (best0 + 1) % V, best0, (int(np.argmax(z[2])) + 1) % V]
    path, out = oracle.accept(z, None, toks, parents, 0.0)
    assert path == [0, 2] and out == [best0, int(np.argmax(z[2]))]
    # greedy chain through node 1 and node 3
    toks = [7, best0, 5, best1]
    path, out = oracle.accept(z, None, toks, parents, 0.0)
    assert path == [0, 1, 3] and out == [best0, best1, int(np.argmax(z[3]))]
    # stochastic with q == p at temperature 1: u < 1 accepts every draft
    path, out = oracle.accept(z, z, [7, 11, 13, 17], parents, 1.0, np.full(4, 0.999, np.float32),
                              np.zeros(4, np.float32))
    assert path == [0, 1, 3]
    # stochastic with u = 1: nothing is accepted; the root's sample is a valid token
    path, out = oracle.accept(z, z, [7, 11, 13, 17], parents, 1.0, np.ones(4, np.float32),
                              np.full(4, 0.5, np.float32))
    assert path == [0] and len(out) == 1 and 0 <= out[0] < V


def test_oracle_chain_verify_equals_steps(oracle):
    t = dict(D=512, NL=1, NH=4, NKV=1, HD=128, NFF=1024, vocab=2048, ctx=64)
    m = oracle.Model(seed=0, **t)
    m.fill_kv(10, 1)
    chain = [3]
    for i in range(4):
        chain.append(m.step(chain[-1], 10 + i))
    m.fill_kv(10, 1)
    best, _ = m.verify(chain, [-1, 0, 1, 2, 3], 10)
    assert list(best[:-1]) == chain[1:]


def test_ffn_block_matches_numpy(oracle):
    """or_ffn_block (config-1's block: kcpu4.c:287-295 without the residual add) against a numpy
    fp64 restatement from the same tensors: rmsnorm, gate/up, silu(g) * u, down."""
    t = dict(TINY, NL=1)
    m = oracle.Model(seed=0, **t)
    D, F = t["D"], t["NFF"]
    X = np.stack([oracle.gen_normal(D, 0.0, 1.0, 1, 40 + i) for i in range(3)])
    Y = m.ffn_block(0, X)

    def mat(kind, R, Cc, ty):
        W = np.ctypeslib.as_array(oracle.lib().or_model_tensor(m.h, 0, kind), shape=(R * (Cc // 256) * oracle.BLOCK[ty],))
        return oracle.decode_blocks(W.reshape(-1, oracle.BLOCK[ty]), ty).reshape(R, Cc).astype(np.float64)
    Wg, Wu, Wd = mat(oracle.T_GATE, F, D, 12), mat(oracle.T_UP, F, D, 12), mat(oracle.T_DOWN, D, F, 14)
    gamma = oracle.gen_normal(D, 1.0, 0.02, 0, oracle.stream(0, oracle.T_FFN_NORM)).astype(np.float64)
    for i in range(3):
        x = X[i].astype(np.float64)
        xn = x / np.sqrt(np.mean(x * x) + 1e-6) * gamma
        g, u = Wg @ xn, Wu @ xn
        ref = Wd @ (g / (1.0 + np.exp(-g)) * u)
        assert rel_l2(Y[i], ref) < 1e-5, i
    m.close()
