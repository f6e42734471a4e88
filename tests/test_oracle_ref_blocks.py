"""Blocks of the oracle (oracle/kq_oracle.c, which the GPU tests compare the CUDA path with)
against the reference's own CPU engine, scripts/kindi_q4/kindi/kcpu4.c compiled unmodified from
the reference tree and reached through oracle/ref_blocks.c (oracle/_ref/libkcpu4_blocks.so):
  - the MLP block (or_ffn_block, config-1's block) against the reference's ffn (:287-295, with
    its rmsfold, fold, gemv and q4_dot);
  - the embedding row, final norm, head GEMV and greedy argmax of a step (the oracle model with no
    layers) against the reference's kc_step (:303-335) on a model of no layers.
Same weights (the oracle model's tensors, regenerated from the same seeded streams), same inputs:
the outputs must be bit-identical. Skipped when the reference library was not built (no
reference tree)."""
import numpy as np
import pytest

from conftest import same_bits_or_both_nan


@pytest.fixture(scope="module")
def ref_blocks(oracle):
    if oracle.ref_blocks_lib() is None:
        pytest.skip("oracle/_ref/libkcpu4_blocks.so not built (reference tree absent)")
    return oracle


def layer_ffn_tensors(O, cfg, seed, layer):
    D, F = cfg["D"], cfg["NFF"]
    Wg = O.gen_matrix(F, D, cfg["t_gate"], seed, O.stream(layer, O.T_GATE))
    Wu = O.gen_matrix(F, D, cfg["t_up"], seed, O.stream(layer, O.T_UP))
    Wd = O.gen_matrix(D, F, cfg["t_down"], seed, O.stream(layer, O.T_DOWN))
    norm = O.gen_normal(D, 1.0, 0.02, seed, O.stream(layer, O.T_FFN_NORM))
    return Wg, Wu, Wd, norm


@pytest.mark.parametrize("D,F,layer,M", [(512, 1024, 1, 4), (2048, 6144, 0, 2), (4096, 12288, 3, 1)])
def test_oracle_ffn_block_equals_reference(ref_blocks, D, F, layer, M):
    O = ref_blocks
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


@pytest.mark.parametrize("D,V,temb,thead", [(512, 4096, 12, 14), (4096, 151936, 12, 14), (1024, 2048, 14, 12)])
def test_oracle_head_step_equals_reference(ref_blocks, D, V, temb, thead):
    O = ref_blocks
    cfg = dict(O.CFG2, D=D, NL=0, NH=D // 128, NKV=max(1, D // 512), vocab=V, ctx=64, t_emb=temb, t_out=thead)
    seed = 3
    Wemb = O.gen_matrix(V, D, temb, seed, O.stream(-1, O.T_EMB))
    Whead = O.gen_matrix(V, D, thead, seed, O.stream(-1, O.T_OUT))
    norm = O.gen_normal(D, 1.0, 0.02, seed, O.stream(-1, O.T_OUTNORM))
    m = O.Model(seed=seed, **cfg)
    try:
        for tok in (0, 1, V // 3, V - 1):
            best = m.step(tok, 0, head=True)
            logits = m.logits()
            rbest, rlogits = O.ref_head_step(Wemb, temb, Whead, thead, D, V, norm, tok)
            assert same_bits_or_both_nan(logits, rlogits), tok
            assert best == rbest, tok
            m.reset()
    finally:
        m.close()
