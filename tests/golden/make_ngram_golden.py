"""Generates tests/golden/ngram_golden.json from the REFERENCE prompt-lookup drafter.

Run once on a host that has the reference tree (read-only):
    python tests/golden/make_ngram_golden.py /path/to/reference      (or set KQ_REFERENCE)

Source of truth: NgramDraft, scripts/kindi_q4/kindi/spec.py:801-841, driven through its own
methods (reset, push, truncate, propose). The module imports a GPU array library at its top that
this host lacks; NgramDraft does not use it, so the import is satisfied by an inert stand-in
module installed in sys.modules for the duration of this script (nothing of the reference is
changed or copied).

Cases: drafter sizes (nmax, nmin) in {(4, 1), (3, 2), (1, 1), (6, 3)}; histories of 0..160 tokens
over small vocabularies (so suffixes repeat), some with -1 (unknown) and -2 tokens; after a reset,
a scripted mix of propose(k) for k in {0, 1, 3, 8}, push(t) and truncate(L) (L up to 3 past the
end), each result recorded. The fixture is small (< 300 KB) and the GPU box never needs the
reference tree.
"""
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class _Inert(object):
    def __init__(self, *a, **k):
        pass

    def __call__(self, *a, **k):
        return _Inert()

    def __getattr__(self, name):
        return _Inert()

    def __iter__(self):
        return iter(())

    def __getitem__(self, key):
        return _Inert()


class _InertModule(types.ModuleType):
    def __getattr__(self, name):
        return _Inert()


def main(ref_root):
    for name in ("cupy", "cupyx", "cupy.cuda", "cupy.cuda.runtime"):
        sys.modules.setdefault(name, _InertModule(name))
    sys.path.insert(0, os.path.join(ref_root, "scripts", "kindi_q4"))
    from kindi.spec import NgramDraft   # the reference drafter

    rng = np.random.default_rng(77)
    cases = []
    for nmax, nmin in ((4, 1), (3, 2), (1, 1), (6, 3)):
        for c in range(12):
            vocab = int(rng.choice([3, 5, 12, 50]))
            n = int(rng.integers(0, 161))
            hist = rng.integers(0, vocab, n).tolist()
            if c % 3 == 1 and n:
                for i in rng.integers(0, n, max(1, n // 20)).tolist():
                    hist[i] = -1
            if c % 4 == 2 and n:
                hist[int(rng.integers(0, n))] = -2
            d = NgramDraft(nmax=nmax, nmin=nmin)
            d.reset(list(hist))
            ops = []
            for _ in range(40):
                r = rng.random()
                if r < 0.55:
                    k = int(rng.choice([0, 1, 3, 8]))
                    ops.append(["propose", k, [int(t) for t in d.propose(k)]])
                elif r < 0.85:
                    t = int(rng.integers(0, vocab)) if rng.random() > 0.05 else -1
                    d.push(t)
                    ops.append(["push", t, len(d.h)])
                else:
                    L = int(rng.integers(0, len(d.h) + 4))
                    d.truncate(L)
                    ops.append(["truncate", L, len(d.h)])
            cases.append({"nmax": nmax, "nmin": nmin, "hist": [int(t) for t in hist], "ops": ops})
    out = os.path.join(HERE, "ngram_golden.json")
    with open(out, "w") as f:
        json.dump({"source": "scripts/kindi_q4/kindi/spec.py:801-841 NgramDraft", "cases": cases}, f,
                  separators=(",", ":"))
    print("wrote", out, sum(len(c["ops"]) for c in cases), "operations in", len(cases), "cases")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KQ_REFERENCE")
    if not root:
        sys.exit("usage: make_ngram_golden.py /path/to/reference (or set KQ_REFERENCE)")
    main(root)
