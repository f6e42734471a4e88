"""The oracle's acceptance rule (oracle/kq_oracle.c or_accept, which the GPU acceptance kernels
match bit for bit) against the reference's speculative sampling with a deterministic draft
(spec_accept, scripts/kindi_q4/kindi/spec.py:769-787), in distribution: for draft chains over a
12-token vocabulary, the histograms of how many drafts are kept and of the token emitted after
them, over seeded trials of each side, must be homogeneous (chi-square, p > 1e-3; both sides
seeded, so the outcome is fixed). The reference's histograms are in tests/golden/accept_golden.json
(made by tests/golden/make_accept_golden.py). A one-hot draft distribution q turns the oracle's
general rule (accept child c iff u * q(d) < p(d), else p <- normalised max(0, p - q)) into the
reference's (keep d with probability p(d), else draw from p without d). Host-side: no GPU."""
import json
import os

import numpy as np
import pytest
from scipy.stats import chi2_contingency

HERE = os.path.dirname(os.path.abspath(__file__))
TRIALS = 20000


@pytest.fixture(scope="module")
def golden_accept():
    with open(os.path.join(HERE, "golden", "accept_golden.json")) as f:
        return json.load(f)


def run_oracle(oracle, P, drafts, seed):
    V = P.shape[1]
    k = len(drafts)
    with np.errstate(divide="ignore"):
        z = np.log(P).astype(np.float32)             # softmax(z) = P; zero probabilities: -inf
    g = np.full((k + 1, V), -1e4, np.float32)        # q of node i's child: one-hot at drafts[i]
    for i, d in enumerate(drafts):
        g[i, d] = 0.0
    tokens = [0] + list(drafts)
    parents = [-1] + list(range(k))
    rng = np.random.default_rng(seed)
    kept = np.zeros(k + 1, np.int64)
    final = np.zeros(V, np.int64)
    for _ in range(TRIALS):
        u = rng.random((2, k + 1)).astype(np.float32)
        path, out = oracle.accept(z, g, tokens, parents, 1.0, u[0], u[1])
        kept[len(path) - 1] += 1
        final[out[-1]] += 1
    return kept, final


def homogeneous(a, b):
    t = np.array([a, b], np.float64)
    t = t[:, t.sum(axis=0) > 0]
    if t.shape[1] < 2:
        return 1.0
    return chi2_contingency(t)[1]


def test_oracle_matches_reference_distribution(oracle, golden_accept):
    assert golden_accept["V"] == 12
    for ci, c in enumerate(golden_accept["cases"]):
        P = np.array(c["P"], np.float64)
        kept, final = run_oracle(oracle, P, c["drafts"], 500 + ci)
        pk = homogeneous(c["kept_hist"], kept)
        pf = homogeneous(c["final_hist"], final)
        assert pk > 1e-3 and pf > 1e-3, (c["name"], pk, pf, c["kept_hist"], kept.tolist())
        if c["name"] == "never":
            assert kept[0] == TRIALS and final[c["drafts"][0]] == 0
        if c["name"] == "always":
            assert kept[-1] == TRIALS
