"""The CPU oracle against the reference's own golden data (no GPU).

tests/golden/quant_golden.npz was produced from the reference (tests/golden/make_golden.py):
its numpy block decoder (scripts/kindi_q4/kindi/q4pack.py:52-76) and its native kc_dequant /
kc_matvec (kcpu4.c:337-341) built from the reference sources. These tests pin the oracle's block
decode (q4kernels.h:12-33) and fused dot (q4kernels.h:37-71) bit for bit, and the shared
synthetic generator byte for byte."""
import numpy as np
import pytest

from conftest import same_bits_or_both_nan


@pytest.mark.parametrize("ty", [12, 14])
def test_decode_matches_reference_unit_case(golden, oracle, ty):
    # tests/kindi_q4/test_quant.py:14-29: random blocks, d forced to 0.013
    raw = golden["refcase_raw_%d" % ty]
    dense = oracle.decode_blocks(raw.reshape(-1, oracle.BLOCK[ty]), ty).reshape(golden["refcase_dense_%d" % ty].shape)
    assert same_bits_or_both_nan(dense, golden["refcase_dense_%d" % ty])


@pytest.mark.parametrize("ty", [12, 14])
def test_matvec_matches_reference_unit_case(golden, oracle, ty):
    raw = golden["refcase_raw_%d" % ty]
    rows, cols = raw.shape[0], raw.shape[1] * 256
    y = oracle.matvec(raw.reshape(-1), rows, cols, ty, golden["refcase_x_%d" % ty])
    assert same_bits_or_both_nan(y, golden["refcase_y_%d" % ty])
    # the reference test's own tolerance against an fp64 product (test_quant.py:32)
    dense = golden["refcase_dense_%d" % ty].astype(np.float64)
    np.testing.assert_allclose(y, dense @ golden["refcase_x_%d" % ty].astype(np.float64), atol=0.00015, rtol=0.00001)


@pytest.mark.parametrize("ty", [12, 14])
def test_generator_and_decode_pinned(golden, oracle, ty):
    W = oracle.gen_matrix(64, 1024, ty, 0, 7)
    assert np.array_equal(W, golden["synth_raw_%d" % ty]), "synthetic generator drifted"
    dense = oracle.decode_blocks(W.reshape(-1, oracle.BLOCK[ty]), ty).reshape(64, 1024)
    assert same_bits_or_both_nan(dense, golden["synth_dense_%d" % ty])
    y = oracle.matvec(W, 64, 1024, ty, golden["synth_x_%d" % ty])
    assert same_bits_or_both_nan(y, golden["synth_y_%d" % ty])


@pytest.mark.parametrize("ty", [12, 14])
def test_edge_blocks(golden, oracle, ty):
    raw = golden["edge_raw_%d" % ty]
    dense = oracle.decode_blocks(raw.reshape(-1, oracle.BLOCK[ty]), ty).reshape(8, 256)
    assert same_bits_or_both_nan(dense, golden["edge_dense_%d" % ty])


def test_pack_layout_addressing(oracle):
    # q4kernels.h:8-10: the 8-row interleaved pack layout addresses the same blocks
    for ty in (12, 14):
        W = oracle.gen_matrix(16, 512, ty, 3, 11)
        Wp = oracle.to_pack_layout(W, 16, 512, ty)
        x = oracle.gen_normal(512, 0.0, 1.0, 1, 5)
        assert np.array_equal(oracle.matvec(W, 16, 512, ty, x, layout=0), oracle.matvec(Wp, 16, 512, ty, x, layout=1))


@pytest.mark.skipif(not __import__("os").path.exists(
    __import__("os").path.join(__import__("os").path.dirname(__file__), "..", "oracle", "_ref", "libkcpu4.so")),
    reason="oracle/_ref (reference kcpu4.c) not built")
@pytest.mark.parametrize("ty,R,Cc", [(12, 64, 4096), (14, 32, 12288), (12, 8, 256), (14, 40, 768)])
def test_oracle_bit_identical_to_reference_library(oracle, ty, R, Cc):
    W = oracle.gen_matrix(R, Cc, ty, 9, 77)
    x = oracle.gen_normal(Cc, 0.0, 1.0, 1, 3)
    Wp = oracle.to_pack_layout(W, R, Cc, ty)
    assert same_bits_or_both_nan(oracle.matvec(W, R, Cc, ty, x), oracle.ref_matvec(Wp, R, Cc, ty, x))
    for row in (0, R - 1):
        assert same_bits_or_both_nan(oracle.dequant_row(W, R, Cc, ty, row), oracle.ref_dequant(Wp, R, Cc, ty, row))
