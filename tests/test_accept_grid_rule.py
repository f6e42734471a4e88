"""The inverse-CDF selection of the multi-CTA acceptance kernel (kq_accept.cuh k_accept_grid),
restated in numpy float32 next to the one-CTA kernel's sequential walk (k_accept), on random and
rounding-adversarial inputs: both pick the same id.

One-CTA walk: from block 0, skip blocks while prefix + bs[b] <= target (prefix accumulating the
block sums in order); scan the first other block id by id from the prefix; if rounding leaves the
target above every running sum of it, go on with the next blocks; none: the largest id with
p > 0 (0 if none). Grid form: every block b computes its own in-order prefix, blocks with
prefix + bs[b] > target scan, and the smallest found id wins (ids grow with b)."""
import numpy as np
import pytest

BLK = 1024
f32 = np.float32


def block_sums(p):
    nb = (len(p) + BLK - 1) // BLK
    return [f32(np.sum(p[b * BLK:(b + 1) * BLK], dtype=np.float32)) for b in range(nb)]


def scan(p, b, prefix, target):
    run = prefix
    for i in range(b * BLK, min(len(p), (b + 1) * BLK)):
        run = f32(run + p[i])
        if run > target:
            return i
    return None


def fallback(p):
    nz = np.nonzero(p > 0)[0]
    return int(nz[-1]) if len(nz) else 0


def pick_sequential(p, bs, target):
    nb, prefix, cand = len(bs), f32(0), 0
    while True:
        b = cand
        while b < nb and not (f32(prefix + bs[b]) > target):
            prefix = f32(prefix + bs[b])
            b += 1
        if b >= nb:
            return fallback(p)
        i = scan(p, b, prefix, target)
        if i is not None:
            return i
        prefix = f32(prefix + bs[b])
        cand = b + 1


def pick_grid(p, bs, target):
    found = []
    for b in range(len(bs)):
        prefix = f32(0)
        for b2 in range(b):
            prefix = f32(prefix + bs[b2])
        if f32(prefix + bs[b]) > target:
            i = scan(p, b, prefix, target)
            if i is not None:
                found.append(i)
    return min(found) if found else fallback(p)


@pytest.mark.parametrize("V", [4096, 5000, 1024 * 7 + 3])
@pytest.mark.parametrize("seed", range(6))
def test_grid_pick_equals_sequential_walk(V, seed):
    rng = np.random.default_rng(seed)
    p = rng.exponential(1.0, V).astype(np.float32) * (rng.random(V) < 0.5)   # zeros and a long tail
    p = (p / np.float32(p.sum())).astype(np.float32)
    bs = block_sums(p)
    W = f32(0)
    for s in bs:
        W = f32(W + s)
    prefixes = np.cumsum(np.array(bs, np.float64))
    targets = [f32(u * W) for u in rng.random(8)]
    # adversarial: targets just below a block boundary, where the tree sum and the running sum
    # of the block round differently
    for b in range(len(bs)):
        targets.append(np.nextafter(f32(prefixes[b]), f32(0), dtype=np.float32))
        targets.append(f32(prefixes[b]))
    targets += [f32(W), np.nextafter(f32(W), f32(2), dtype=np.float32)]
    for t in targets:
        t = f32(t)
        assert pick_grid(p, bs, t) == pick_sequential(p, bs, t), (V, seed, float(t))


def test_all_zero_and_single_id():
    p = np.zeros(3000, np.float32)
    bs = block_sums(p)
    assert pick_grid(p, bs, f32(0)) == pick_sequential(p, bs, f32(0)) == 0
    p[2500] = 1.0
    bs = block_sums(p)
    for t in (f32(0), f32(0.5), f32(1.0)):
        assert pick_grid(p, bs, t) == pick_sequential(p, bs, t)
