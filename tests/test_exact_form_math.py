"""The arithmetic of the batched GEMM's exact form (kq_tmm.cuh, Q4_K row tiles), restated in numpy
and checked against the oracle on the CPU.

A Q4_K weight is (d * sc) * q - dmin * mn (q4kernels.h:19-30; oracle/kq_oracle.c). The exact form
puts q * sc (an integer <= 945, exact in fp16) in the MMA's A operand, multiplies it with the fp16
hi and lo parts of the activations, accumulates each 256-column super-block in fp32, scales the
super-block by d, and subtracts dmin * mn_b times the fp32 sum of the activations over each
32-column sub-block b. These tests pin the field decoding against the oracle's dequantisation, the
fp16 identity the dequantising warps use, and the whole decomposition against the oracle's fp32
matvec."""
import numpy as np
import pytest

from conftest import rel_l2

Q4K = 12


def q4k_fields(W, R, Cc):
    """d, dmin [R][G]; sc, mn [R][G][8]; q [R][G][8][32] from GGUF Q4_K blocks (144 bytes)."""
    G = Cc // 256
    blk = W.reshape(R, G, 144)
    d = blk[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = blk[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    s = blk[..., 4:16].astype(np.int32)
    sc = np.empty((R, G, 8), np.int32)
    mn = np.empty((R, G, 8), np.int32)
    sc[..., :4] = s[..., 0:4] & 63
    mn[..., :4] = s[..., 4:8] & 63
    sc[..., 4:] = (s[..., 8:12] & 15) | ((s[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)
    qs = blk[..., 16:144].astype(np.int32).reshape(R, G, 4, 32)
    q = np.empty((R, G, 8, 32), np.int32)
    q[:, :, 0::2, :] = qs & 15   # 32-byte chunk c: low nibbles = sub-block 2c, high = 2c + 1
    q[:, :, 1::2, :] = qs >> 4
    return d, dmin, sc, mn, q


def test_fp16_offset_identity():
    """(1024 + q) * sc - 1024 * sc, rounded once, is q * sc for every nibble and 6-bit scale; the
    byte pair (q, 0x64) is the fp16 1024 + q; 1024 * sc is an fp16 value."""
    q = np.arange(16)
    for sc in range(64):
        assert float(np.float16(1024 * sc)) == 1024 * sc
        exact = ((1024 + q) * sc - 1024 * sc).astype(np.float64)
        assert np.array_equal(exact.astype(np.float16).astype(np.float64), q * sc)
        assert (q * sc).max() < 2048
    bits = (np.uint16(0x6400) | q.astype(np.uint16)).view(np.float16)
    assert np.array_equal(bits.astype(np.float64), 1024 + q)


@pytest.mark.parametrize("R,Cc,seed", [(64, 1024, 3), (32, 4096, 7)])
def test_fields_reproduce_oracle_dequant(oracle, R, Cc, seed):
    W = oracle.gen_matrix(R, Cc, Q4K, 0, seed)
    d, dmin, sc, mn, q = q4k_fields(W, R, Cc)
    ds = (d[..., None] * sc.astype(np.float32)).astype(np.float32)      # fp32 d * sc
    dm = (dmin[..., None] * mn.astype(np.float32)).astype(np.float32)   # fp32 dmin * mn
    w = (ds[..., None] * q.astype(np.float32) - dm[..., None]).astype(np.float32).reshape(R, Cc)
    for r in (0, R // 2, R - 1):
        ref = oracle.dequant_row(W, R, Cc, Q4K, r)
        assert np.allclose(w[r], ref, rtol=1e-6, atol=0), r


@pytest.mark.parametrize("R,Cc,M,seed", [(64, 1024, 5, 3), (128, 4096, 9, 11)])
def test_exact_decomposition_matches_oracle(oracle, R, Cc, M, seed):
    W = oracle.gen_matrix(R, Cc, Q4K, 0, seed)
    d, dmin, sc, mn, q = q4k_fields(W, R, Cc)
    G = Cc // 256
    X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 50 + t) for t in range(M)])
    xh = X.astype(np.float16)
    xl = (X - xh.astype(np.float32)).astype(np.float16)
    A = (q * sc[..., None]).astype(np.float16)                         # the A operand
    assert np.array_equal(A.astype(np.int64), q * sc[..., None])
    A64 = A.astype(np.float64).reshape(R, G, 256)
    Dh = np.einsum("rgc,tgc->rgt", A64, xh.astype(np.float64).reshape(M, G, 256)).astype(np.float32)
    Dl = np.einsum("rgc,tgc->rgt", A64, xl.astype(np.float64).reshape(M, G, 256)).astype(np.float32)
    y = np.zeros((R, M), np.float32)
    for g in range(G):                                                  # read-back: acc += d * (hi + lo)
        y = (y + d[:, g, None] * (Dh[:, g] + Dl[:, g])).astype(np.float32)
    sums = X.reshape(M, G, 8, 32).sum(axis=-1, dtype=np.float32)      # the packers' sub-block sums
    dm = (dmin[..., None] * mn.astype(np.float32)).astype(np.float32)
    y = (y - np.einsum("rgb,tgb->rt", dm.astype(np.float64), sums.astype(np.float64))).astype(np.float32)
    for t in range(M):
        assert rel_l2(y[:, t], oracle.matvec(W, R, Cc, Q4K, X[t])) < 2e-6, t
