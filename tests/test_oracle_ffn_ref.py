"""The oracle's MLP block (oracle/kq_oracle.c or_ffn_block, config-1's block, which the GPU tests
compare the CUDA path with) against the reference's own: ffn of scripts/kindi_q4/kindi/kcpu4.c
(:287-295, with its rmsfold, fold, gemv and q4_dot), compiled unmodified from the reference tree
and reached through oracle/ref_ffn.c (oracle/_ref/libkcpu4_ffn.so). Same weights (the oracle
model's layer tensors, regenerated from the same seeded streams), same rows: the outputs must be
bit-identical. Skipped when the reference library was not built (no reference tree)."""
import numpy as np
import pytest

from conftest import same_bits_or_both_nan


@pytest.fixture(scope="module")
def ref_ffn(oracle):
    if oracle.ref_ffn_lib() is None:
        pytest.skip("oracle/_ref/libkcpu4_ffn.so not built (reference tree absent)")
    return oracle


def layer_ffn_tensors(O, cfg, seed, layer):
    D, F = cfg["D"], cfg["NFF"]
    Wg = O.gen_matrix(F, D, cfg["t_gate"], seed, O.stream(layer, O.T_GATE))
    Wu = O.gen_matrix(F, D, cfg["t_up"], seed, O.stream(layer, O.T_UP))
    Wd = O.gen_matrix(D, F, cfg["t_down"], seed, O.stream(layer, O.T_DOWN))
    norm = O.gen_normal(D, 1.0, 0.02, seed, O.stream(layer, O.T_FFN_NORM))
    return Wg, Wu, Wd, norm


@pytest.mark.parametrize("D,F,layer,M", [(512, 1024, 1, 4), (2048, 6144, 0, 2), (4096, 12288, 3, 1)])
def test_oracle_ffn_block_equals_reference(ref_ffn, D, F, layer, M):
    O = ref_ffn
    cfg = dict(O.CFG2, D=D, NFF=F, NL=layer + 1, NH=D // 128, NKV=max(1, D // 512), vocab=1024, ctx=64)
    seed = 5
    m = O.Model(seed=seed, **cfg)
    try:
        X = np.stack([O.gen_normal(D, 0.0, 1.0, 9, 70 + i) for i in range(M)])
        Y = m.ffn_block(layer, X)
    finally:
        m.close()
    Wg, Wu, Wd, norm = layer_ffn_tensors(O, cfg, seed, layer)
    for i in range(M):
        ref = O.ref_ffn_block(Wg, Wu, Wd, (cfg["t_gate"], cfg["t_up"], cfg["t_down"]), D, F, norm, X[i])
        assert np.isfinite(ref).all()
        assert same_bits_or_both_nan(Y[i], ref), (i, float(np.abs(Y[i] - ref).max()))
