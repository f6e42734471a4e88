"""The library's prompt-lookup drafter (kq_ngram_* behind kq.NgramDraft) against the reference's
NgramDraft (scripts/kindi_q4/kindi/spec.py:801-841): every proposal, push and truncation of the
scripted cases in tests/golden/ngram_golden.json (made by tests/golden/make_ngram_golden.py from
the reference itself) must match. Host-side code: no GPU."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def kq():
    import kq as K   # host-side entry points: the library loads without a GPU
    return K


@pytest.fixture(scope="module")
def cases():
    with open(os.path.join(HERE, "golden", "ngram_golden.json")) as f:
        return json.load(f)["cases"]


def test_replays_reference_cases(kq, cases):
    n_prop = 0
    for ci, c in enumerate(cases):
        d = kq.NgramDraft(nmax=c["nmax"], nmin=c["nmin"])
        d.reset(c["hist"])
        assert len(d) == len(c["hist"])
        for oi, (op, arg, want) in enumerate(c["ops"]):
            if op == "propose":
                assert d.propose(arg) == want, (ci, oi, arg)
                n_prop += 1
            elif op == "push":
                d.push(arg)
                assert len(d) == want, (ci, oi)
            else:
                d.truncate(arg)
                assert len(d) == want, (ci, oi)
        d.close()
    assert n_prop > 500


def test_reference_example_and_chain_use(kq):
    """The latest earlier occurrence wins; the proposal is a chain for kq_verify."""
    d = kq.NgramDraft()
    d.reset([7, 1, 2, 3, 9, 1, 2, 3, 5, 1, 2, 3])
    assert d.propose(2) == [5, 1]            # suffix [1, 2, 3]: latest earlier occurrence at 5..7
    d.push(4)
    assert d.propose(3) == []                # [.., 3, 4] never occurred before
    d.truncate(8)                            # back to [7, 1, 2, 3, 9, 1, 2, 3]: the index still
    assert d.propose(3) == []                # points past the end for every suffix (not re-resolved)
    d.reset([7, 1, 2, 3, 9, 1, 2, 3])
    assert d.propose(3) == [9, 1, 2]
    toks = [3] + d.propose(3)
    parents = [-1] + list(range(len(toks) - 1))
    assert parents == [-1, 0, 1, 2] and toks == [3, 9, 1, 2]


def test_unknown_tokens(kq):
    d = kq.NgramDraft(nmax=2, nmin=1)
    d.reset([1, 2, -1, 1, 2])
    assert d.propose(3) == []                # continuation of [1, 2] holds -1: no proposal
    d.reset([4, -2, 6, 4])
    assert d.propose(3) == [6, 4]            # other negative tokens are left out
    d.reset([3, 3, -1])
    assert d.propose(2) == []                # the suffix holds -1 at every n


def test_argument_errors(kq):
    with pytest.raises(ValueError):
        kq.NgramDraft(nmax=0, nmin=0)
    with pytest.raises(ValueError):
        kq.NgramDraft(nmax=2, nmin=3)
    with pytest.raises(ValueError):
        kq.NgramDraft(nmax=65, nmin=1)
    d = kq.NgramDraft()
    d.reset(np.arange(10))
    with pytest.raises(ValueError):
        d.propose(-1)
    with pytest.raises(ValueError):
        d.truncate(-1)
    assert d.propose(0) == []
