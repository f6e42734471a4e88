"""Generates tests/golden/accept_golden.json from the REFERENCE speculative-sampling rule.

Run once on a host that has the reference tree (read-only):
    python tests/golden/make_accept_golden.py /path/to/reference      (or set KQ_REFERENCE)

Source of truth: spec_accept, scripts/kindi_q4/kindi/spec.py:769-787 (speculative sampling with a
deterministic draft: draft i kept with probability p_i(d_i); at the first rejection a token drawn
from p_i without d_i, renormalised; all kept: a token drawn from p_k). It draws from numpy's
RandomState, so its outputs cannot match another implementation bit for bit; the fixture holds,
per scenario, the target distributions, the drafts and the histograms of (a) how many drafts were
kept and (b) the token emitted after them, over many seeded trials. tests/test_accept_reference.py
compares the oracle's acceptance (oracle/kq_oracle.c or_accept, which the GPU kernels match bit
for bit) with these histograms. The module imports a GPU array library at its top that this host
lacks; spec_accept does not use it, so the import is satisfied by an inert stand-in module in
sys.modules for the duration of this script (the same device as make_ngram_golden.py).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_ngram_golden import _InertModule  # noqa: E402

V = 12
TRIALS = 40000


def scenarios():
    rng = np.random.default_rng(91)
    out = []
    for name, k, w in (("chain3", 3, 0.6), ("chain1", 1, 0.3), ("chain5", 5, 0.75)):
        # drafts the target favours (weight w on the drafted token), so that several are kept
        d = rng.integers(0, V, k).tolist()
        P = (1.0 - w) * rng.dirichlet(np.full(V, 0.6), k + 1)
        for i in range(k):
            P[i, d[i]] += w
        P[k] /= P[k].sum()
        out.append((name, P, d))
    P = rng.dirichlet(np.full(V, 1.0), 3)          # a draft the target never takes: always rejected
    d = [int(np.argmin(P[0]))]
    P[0, d[0]] = 0.0
    P[0] /= P[0].sum()
    out.append(("never", P[:2], d))
    P = rng.dirichlet(np.full(V, 1.0), 3)          # drafts the target is sure of: always kept
    d = [3, 7]
    P[0] = np.eye(V)[3]
    P[1] = np.eye(V)[7]
    out.append(("always", P, d))
    return out


def main(ref_root):
    for name in ("cupy", "cupyx", "cupy.cuda", "cupy.cuda.runtime"):
        sys.modules.setdefault(name, _InertModule(name))
    sys.path.insert(0, os.path.join(ref_root, "scripts", "kindi_q4"))
    from kindi.spec import spec_accept   # the reference rule

    cases = []
    for si, (name, P, d) in enumerate(scenarios()):
        rng = np.random.RandomState(1000 + si)
        idx = np.arange(V)
        kept = np.zeros(len(d) + 1, np.int64)
        final = np.zeros(V, np.int64)
        for _ in range(TRIALS):
            out = spec_accept(lambda i: (idx, P[i]), d, rng)
            a = len(out) - 1
            kept[a] += 1
            final[out[-1]] += 1
        cases.append({"name": name, "P": P.tolist(), "drafts": d, "trials": TRIALS,
                      "kept_hist": kept.tolist(), "final_hist": final.tolist()})
    path = os.path.join(HERE, "accept_golden.json")
    with open(path, "w") as f:
        json.dump({"source": "scripts/kindi_q4/kindi/spec.py:769-787 spec_accept", "V": V, "cases": cases}, f)
    print("wrote", path, len(cases), "scenarios x", TRIALS, "trials")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KQ_REFERENCE")
    if not root:
        sys.exit("usage: make_accept_golden.py /path/to/reference (or set KQ_REFERENCE)")
    main(root)
