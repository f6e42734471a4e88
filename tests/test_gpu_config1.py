"""GPU: config-1, the mixed Q4_K_M MLP block at the speculative-verify widths M = 1, 4, 8, 16,
against the CPU oracle through the C ABI (kq_ffn_block vs or_ffn_block).

The block is a config-2 layer's: RMSNorm (eps 1e-6, gamma ~ N(1, 0.02)) over hidden 4096, gate and
up Q4_K 4096 -> 12288 with SwiGLU, down Q6_K 12288 -> 4096; activations ~ N(0, 1). M = 1 runs the
decode GEMVs, M >= 2 the batched tensor-core pass. Bar: every row within 1e-3 relative L2 (the
north-star tolerance); each row must also equal the row computed alone (rows are independent)."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

RTOL = 1e-3
CFG1 = dict(NL=2, vocab=4096, ctx=64)


@pytest.fixture(scope="module")
def models():
    import kq
    from oracle import oracle as O
    assert kq.lib().kq_device_count() > 0, "no GPU"
    e = kq.Engine(kq.Config.default(n_layers=CFG1["NL"], vocab=CFG1["vocab"], ctx=CFG1["ctx"]), seed=0)
    o = O.Model(seed=0, **CFG1)
    yield e, o, O
    e.close()
    o.close()


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("layer", [0, 1])
def test_mlp_block_matches_oracle(models, M, layer):
    e, o, O = models
    X = np.stack([O.gen_normal(4096, 0.0, 1.0, 1, 500 + 17 * M + i) for i in range(M)])
    Y = e.ffn_block(layer, X)
    R = o.ffn_block(layer, X)
    assert Y.shape == (M, 4096)
    for i in range(M):
        err = rel_l2(Y[i], R[i])
        assert err < RTOL, (i, err)


def test_mlp_block_row_independent_of_batch(models):
    """The first row of a 16-row block equals the same row in a 4-row block (the batched pass is
    batch-invariant per token, as the reference's token-by-token loop is)."""
    e, o, O = models
    X = np.stack([O.gen_normal(4096, 0.0, 1.0, 1, 900 + i) for i in range(16)])
    a = e.ffn_block(0, X)
    b = e.ffn_block(0, X[:4])
    assert np.array_equal(a[:4], b)


def test_mlp_block_argument_errors(models):
    e, o, O = models
    with pytest.raises(ValueError):
        e.ffn_block(2, np.zeros((1, 4096), np.float32))      # no such layer
    with pytest.raises(ValueError):
        e.ffn_block(0, np.zeros((129, 4096), np.float32))    # wider than one pass
    with pytest.raises(ValueError):
        e.ffn_block(0, np.zeros((2, 1024), np.float32))      # wrong width
