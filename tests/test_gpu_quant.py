"""GPU: bit-exact dequantisation and the fused-dequant GEMV against the CPU oracle, through the
C ABI (kq_qmat_*). The reference's bar: dequantisation bit-exact (q4kernels.h:12-33), matrix
products within 1e-3 relative L2 of Kindi's CPU path (here also checked at 1e-5)."""
import numpy as np
import pytest

from conftest import rel_l2, same_bits_or_both_nan

pytestmark = pytest.mark.gpu

RTOL_L2 = 1e-3        # north-star tolerance for GEMV outputs
TIGHT_L2 = 2e-5       # what the exact int8 digit-plane arithmetic actually achieves


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


@pytest.mark.parametrize("ty", [12, 14])
@pytest.mark.parametrize("case", ["refcase", "synth", "edge"])
def test_dequant_bit_exact_on_golden(kq, golden, ty, case):
    raw = golden["%s_raw_%d" % (case, ty)]
    R, Cc = raw.shape[0], raw.shape[1] * 256 if raw.ndim == 3 else 1024
    if raw.ndim == 1:
        R = 64
    m = kq.QMat(ty, R, Cc).upload(raw.reshape(-1))
    assert same_bits_or_both_nan(m.dequant(), golden["%s_dense_%d" % (case, ty)].reshape(R, Cc))


@pytest.mark.parametrize("ty", [12, 14])
def test_device_generator_matches_oracle(kq, oracle, ty):
    R, Cc = 24, 2048
    m = kq.QMat(ty, R, Cc).fill_synthetic(0, 7)
    W = oracle.gen_matrix(R, Cc, ty, 0, 7)
    ref = oracle.decode_blocks(W.reshape(-1, oracle.BLOCK[ty]), ty).reshape(R, Cc)
    assert same_bits_or_both_nan(m.dequant(), ref)


SHAPES = [(12, 12288, 4096), (14, 4096, 12288), (14, 1024, 4096), (12, 4096, 4096), (12, 8, 256),
          (14, 16, 512), (12, 40, 1024), (14, 64, 2048), (12, 128, 6144), (14, 8, 4096)]


@pytest.mark.parametrize("ty,R,Cc", SHAPES)
def test_matvec_parity(kq, oracle, ty, R, Cc):
    W = oracle.gen_matrix(R, Cc, ty, 0, 100 + R)
    x = oracle.gen_normal(Cc, 0.0, 1.0, 1, R)
    m = kq.QMat(ty, R, Cc).upload(W)
    y = m.matvec(x)
    ref = oracle.matvec(W, R, Cc, ty, x)
    e = rel_l2(y, ref)
    assert e < RTOL_L2
    assert e < TIGHT_L2, e


def test_matvec_golden_reference_case(kq, golden):
    for ty in (12, 14):
        raw = golden["refcase_raw_%d" % ty]
        m = kq.QMat(ty, 16, 512).upload(raw.reshape(-1))
        assert rel_l2(m.matvec(golden["refcase_x_%d" % ty]), golden["refcase_y_%d" % ty]) < TIGHT_L2


def test_matvec_edge_activations(kq, oracle):
    """Zero, tiny, huge-range and non-finite activations."""
    R, Cc = 16, 1024
    W = oracle.gen_matrix(R, Cc, 12, 0, 5)
    m = kq.QMat(12, R, Cc).upload(W)
    assert np.array_equal(m.matvec(np.zeros(Cc, np.float32)), oracle.matvec(W, R, Cc, 12, np.zeros(Cc, np.float32)))
    x = oracle.gen_normal(Cc, 0.0, 1.0, 1, 9)
    x[:256] *= 1e-30
    x[256:512] *= 1e20
    assert rel_l2(m.matvec(x), oracle.matvec(W, R, Cc, 12, x)) < TIGHT_L2
    x[3] = np.nan
    assert np.isnan(m.matvec(x)).all()


Q6_SHAPES = [(14, 4096, 12288), (14, 1024, 4096), (14, 16, 512), (14, 64, 2048), (14, 8, 4096), (14, 24, 256),
             (14, 40, 1024), (14, 8, 12288)]


@pytest.mark.parametrize("path", ["0", "1"])
@pytest.mark.parametrize("ty,R,Cc", Q6_SHAPES)
def test_matvec_parity_q6k_both_paths(kq, oracle, monkeypatch, ty, R, Cc, path):
    """Q6_K through the dp4a GEMV (KQ_GEMV_MMA6=0) and through the tensor-core one (=1; by
    default it serves Q6_K only inside mixed launches)."""
    monkeypatch.setenv("KQ_GEMV_MMA6", path)
    W = oracle.gen_matrix(R, Cc, ty, 0, 300 + R)
    x = oracle.gen_normal(Cc, 0.0, 1.0, 1, 7 + R)
    m = kq.QMat(ty, R, Cc).upload(W)
    assert rel_l2(m.matvec(x), oracle.matvec(W, R, Cc, ty, x)) < TIGHT_L2


@pytest.mark.parametrize("path", ["0", "1"])
@pytest.mark.parametrize("qbyte,sign", [(0x00, 1.0), (0xFF, -1.0), (0xFF, 1.0)])
def test_matvec_q6k_extreme_magnitudes(kq, oracle, monkeypatch, qbyte, sign, path):
    """Q6_K blocks at the ends of every range: all weights q - 32 = -32 (or +31), every scale
    -128, activations all +-127 (the largest first digit): the int32 sums of the tensor-core and
    the dp4a paths must not overflow."""
    monkeypatch.setenv("KQ_GEMV_MMA6", path)
    R, Cc = 64, 4096
    blk = np.zeros(210, np.uint8)
    blk[:192] = qbyte                      # ql, qh
    blk[192:208] = 0x80                    # int8 scales -128
    blk[208:210] = np.frombuffer(np.float16(1e-3).tobytes(), np.uint8)
    W = np.tile(blk, R * (Cc // 256))
    m = kq.QMat(14, R, Cc).upload(W)
    x = np.full(Cc, 127.0 * sign, np.float32)
    ref = oracle.matvec(W, R, Cc, 14, x)
    assert np.isfinite(ref).all()
    assert rel_l2(m.matvec(x), ref) < RTOL_L2   # identical addends: the oracle's fp32 sums drift


@pytest.mark.parametrize("path", ["0", "1"])
@pytest.mark.parametrize("ty", [12, 14])
def test_matvec_edge_activations_both_types(kq, oracle, monkeypatch, ty, path):
    """Zero, tiny, huge-range and non-finite activations on a launch of each type and path."""
    monkeypatch.setenv("KQ_GEMV_MMA6", path)
    R, Cc = 64, 4096
    W = oracle.gen_matrix(R, Cc, ty, 0, 6)
    m = kq.QMat(ty, R, Cc).upload(W)
    assert np.array_equal(m.matvec(np.zeros(Cc, np.float32)), oracle.matvec(W, R, Cc, ty, np.zeros(Cc, np.float32)))
    x = oracle.gen_normal(Cc, 0.0, 1.0, 1, 10)
    x[:256] *= 1e-30
    x[256:1024] *= 1e20
    assert rel_l2(m.matvec(x), oracle.matvec(W, R, Cc, ty, x)) < TIGHT_L2
    x[3000] = np.inf
    assert not np.isfinite(m.matvec(x)).any()


def test_matvec_nan_weights_propagate(kq, golden):
    raw = golden["edge_raw_12"]
    m = kq.QMat(12, 8, 256).upload(raw.reshape(-1))
    y = m.matvec(np.ones(256, np.float32))
    assert np.isnan(y[1])          # all-0xFF block: d = NaN
    assert np.isfinite(y[0]) and y[0] == 0.0


def test_bad_shapes_rejected(kq):
    with pytest.raises(ValueError):
        kq.QMat(12, 7, 256)
    with pytest.raises(ValueError):
        kq.QMat(12, 8, 300)
    with pytest.raises(ValueError):
        kq.QMat(13, 8, 256)
    with pytest.raises(ValueError):
        kq.QMat(12, 8, 16384)          # wider than one CTA's digit-plane prologue supports
    m = kq.QMat(12, 8, 256)
    with pytest.raises(ValueError):
        m.upload(np.zeros(100, np.uint8))


# The tensor-core GEMM of the batched passes (kq_qmat_matmul, M >= 2): split-precision fp16
# operands with fp32 accumulation, checked row by row against the oracle's fp32 matvec. Shapes
# cover one and many row tiles of 128, partial tiles, single and split-K launches, both types.
MM_SHAPES = [(12, 128, 256), (14, 128, 512), (12, 256, 4096), (14, 1024, 4096), (12, 6144, 4096),
             (14, 4096, 12288), (12, 200, 1024), (14, 24, 2048), (12, 12288, 4096),
             (14, 4096, 3072), (14, 4096, 1536)]   # the down shards of 4- and 8-way tensor parallelism


# Token counts: config-1's speculative-verify widths 4, 8, 16 (and M = 1, the GEMV, above), the
# 45 nodes of config-3's draft tree, and others for partial MMA tiles. The three large shapes
# (config-1's 12288 x 4096 Q4_K and 4096 x 12288 Q6_K, and 6144 x 4096) run the config widths and 45.
@pytest.mark.parametrize("M", [2, 4, 5, 8, 16, 45, 64])
@pytest.mark.parametrize("ty,R,Cc", MM_SHAPES)
def test_matmul_parity(kq, oracle, ty, R, Cc, M):
    if R * Cc > 4096 * 4096 and M not in (4, 8, 16, 45):
        pytest.skip("large shapes at the config widths")
    W = oracle.gen_matrix(R, Cc, ty, 0, 300 + R)
    X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 1000 * M + i) for i in range(M)])
    m = kq.QMat(ty, R, Cc).upload(W)
    Y = m.matmul(X)
    assert Y.shape == (M, R)
    for i in range(M):
        ref = oracle.matvec(W, R, Cc, ty, X[i])
        e = rel_l2(Y[i], ref)
        assert e < RTOL_L2, (i, e)
        assert e < TIGHT_L2, (i, e)


# The same products through the split-weight form only (KQ_TMM_EXACT=0): Q4_K row tiles otherwise
# take the exact form (q * sc in the MMA, d and the minimum term applied outside it).
@pytest.mark.parametrize("M", [4, 16, 45])
@pytest.mark.parametrize("ty,R,Cc", [(12, 256, 4096), (12, 200, 1024), (12, 12288, 4096), (14, 1024, 4096)])
def test_matmul_parity_split_form(kq, oracle, monkeypatch, ty, R, Cc, M):
    monkeypatch.setenv("KQ_TMM_EXACT", "0")
    W = oracle.gen_matrix(R, Cc, ty, 0, 300 + R)
    X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 1000 * M + i) for i in range(M)])
    Y = kq.QMat(ty, R, Cc).upload(W).matmul(X)
    for i in range(M):
        assert rel_l2(Y[i], oracle.matvec(W, R, Cc, ty, X[i])) < TIGHT_L2, i


@pytest.mark.parametrize("form", ["0", "1"])
@pytest.mark.parametrize("qbyte,sign", [(0x00, 1.0), (0xFF, -1.0), (0xFF, 1.0), (0x0F, 1.0)])
def test_matmul_q4k_extreme_magnitudes(kq, oracle, monkeypatch, qbyte, sign, form):
    """Q4_K blocks at the ends of every range: every scale and minimum 63, nibbles 0 or 15 (or 15
    and 0), large d and dmin, activations all +-127 over 8 tokens: q * sc = 945 is the largest A
    value of the exact form; both forms against the oracle."""
    monkeypatch.setenv("KQ_TMM_EXACT", form)
    R, Cc, M = 256, 4096, 8
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(30.0).tobytes(), np.uint8)      # d
    blk[2:4] = np.frombuffer(np.float16(7.5).tobytes(), np.uint8)       # dmin
    blk[4:16] = 0xFF                                                    # scales, minimums: 63
    blk[16:144] = qbyte
    W = np.tile(blk, R * (Cc // 256))
    X = np.stack([np.full(Cc, 127.0 * sign * (1 + (i % 3)), np.float32) for i in range(M)])
    Y = kq.QMat(12, R, Cc).upload(W).matmul(X)
    for i in range(M):
        ref = oracle.matvec(W, R, Cc, 12, X[i])
        assert np.isfinite(ref).all()
        assert rel_l2(Y[i], ref) < RTOL_L2, i   # identical addends: the oracle's fp32 sums drift


def test_matmul_edge_activations_exact_form(kq, oracle):
    """Zero rows, tiny and huge-range rows, a row with an infinity, in one Q4_K batch: the range
    scaling and the sub-block sums see the same packed values."""
    R, Cc = 384, 4096
    W = oracle.gen_matrix(R, Cc, 12, 0, 21)
    X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 400 + i) for i in range(5)])
    X[0] = 0.0
    X[1, :256] *= 1e-30
    X[1, 256:1024] *= 1e20
    X[2] *= 1e-6
    X[3, 3000] = np.inf
    Y = kq.QMat(12, R, Cc).upload(W).matmul(X)
    assert np.array_equal(Y[0], oracle.matvec(W, R, Cc, 12, X[0]))
    for i in (1, 2, 4):
        assert rel_l2(Y[i], oracle.matvec(W, R, Cc, 12, X[i])) < TIGHT_L2, i
    assert not np.isfinite(Y[3]).all()


def test_matmul_rows_independent_of_batch(kq, oracle):
    """Each token's row depends only on its own activations: the same x gives the same products
    whatever the other tokens of the batch are (the MMA N dimension only carries tokens)."""
    R, Cc = 512, 2048
    W = oracle.gen_matrix(R, Cc, 12, 0, 9)
    m = kq.QMat(12, R, Cc).upload(W)
    X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 50 + i) for i in range(8)])
    Y8 = m.matmul(X)
    X2 = X.copy()
    X2[1:] = np.stack([oracle.gen_normal(Cc, 0.0, 3.0, 1, 90 + i) for i in range(7)])
    Y2 = m.matmul(X2)
    assert np.array_equal(Y8[0], Y2[0])


def test_gemv_rule_only_binds_the_single_token_gemv(kq, oracle):
    """1536 and 3072 columns (the down-projection shards of 8- and 4-way tensor parallelism) are
    valid matrices for the batched GEMM but not for the single-token GEMV, whose rows reduce over
    power-of-two warp segments or whole warps: matvec refuses them with ValueError."""
    for Cc in (1536, 3072):
        W = oracle.gen_matrix(16, Cc, 14, 0, 7)
        m = kq.QMat(14, 16, Cc).upload(W)
        with pytest.raises(ValueError):
            m.matvec(np.ones(Cc, np.float32))
        X = np.stack([oracle.gen_normal(Cc, 0.0, 1.0, 1, 3 + i) for i in range(2)])
        Y = m.matmul(X)
        for i in range(2):
            assert rel_l2(Y[i], oracle.matvec(W, 16, Cc, 14, X[i])) < TIGHT_L2
