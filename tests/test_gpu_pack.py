"""GPU: an engine loaded from a Kindi Q4 pack (make_engine(pack, ctx), kq_model_load_pack) equals
the synthetic model the pack was written from, and decodes the oracle's greedy tokens.

The pack (tests/kindi_pack.py) holds the generator's tensors in the reference's on-disk format:
8-row interleaved Q4_K/Q6_K blocks at 16 KiB-aligned offsets in weights.bin, norm weights in
f32.bin, index.json and kindi_pack.json with sizes and SHA-256 digests."""
import numpy as np
import pytest

import kindi_pack as KP

pytestmark = pytest.mark.gpu

T = dict(D=512, NL=2, NH=4, NKV=1, HD=128, NFF=1024, vocab=4096)


@pytest.fixture(scope="module")
def kq():
    import kq as K
    assert K.lib().kq_device_count() > 0, "no GPU"
    return K


@pytest.mark.parametrize("norm_name,types", [("ffn_norm.weight", None),
                                             ("post_attention_norm.weight", dict(q=14, k=14, o=14, down=12, emb=14, out=12))])
def test_pack_engine_equals_synthetic_model(kq, oracle, tmp_path, norm_name, types):
    out = str(tmp_path / "pack")
    KP.write_dense_pack(out, types=types, ffn_norm_name=norm_name, **T)
    e = kq.make_engine(out, ctx=128, log=lambda *a: None)
    c = e.config
    s = kq.Engine(kq.Config.default(dim=512, n_layers=2, n_heads=4, n_kv_heads=1, ffn=1024, vocab=4096, ctx=128,
                                    t_q=c.t_q, t_k=c.t_k, t_v=c.t_v, t_o=c.t_o, t_gate=c.t_gate, t_up=c.t_up,
                                    t_down=c.t_down, t_emb=c.t_emb, t_out=c.t_out), seed=0)
    ids = [7, 99, 1234, 5, 4000, 17]
    got = e.generate(ids, 12)
    z = e.ylog
    assert got == s.generate(ids, 12)
    assert np.array_equal(z, s.ylog)                      # same weights bit for bit: same arithmetic
    o = oracle.Model(seed=0, ctx=128, **dict(T, t_q=c.t_q, t_k=c.t_k, t_v=c.t_v, t_o=c.t_o, t_gate=c.t_gate,
                                             t_up=c.t_up, t_down=c.t_down, t_emb=c.t_emb, t_out=c.t_out))
    assert got == o.generate(ids, 12)
    e.close()
    s.close()


def test_rejected_pack_allocates_nothing(kq, tmp_path):
    out = str(tmp_path / "bad")
    man = KP.write_dense_pack(out, **T)
    man["dimensions"]["full_attention_interval"] = 4
    KP.write_manifest(out, man)
    with pytest.raises(ValueError, match="hybrid"):
        kq.make_engine(out, log=lambda *a: None)
