"""CPU: the Kindi Q4 pack reader (kq_pack_read_config) on packs written in the reference's format
by tests/kindi_pack.py. No GPU: the pack is validated on the host before anything is allocated,
as the reference's verify_pack does (scripts/kindi_q4/kindi/q4pack.py:86-108), and every
rejection carries the reference's message."""
import json
import os

import pytest

import kindi_pack as KP


@pytest.fixture()
def pack(tmp_path):
    out = str(tmp_path / "pack")
    man = KP.write_dense_pack(out)
    return out, man


@pytest.fixture(scope="module")
def kq():
    import kq as K
    return K


def test_valid_pack_gives_its_configuration(kq, pack):
    out, _ = pack
    c = kq.read_pack_config(out, ctx=128)
    assert (c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab, c.ctx) == (512, 2, 4, 1, 128, 1024, 4096, 128)
    assert (c.t_q, c.t_k, c.t_v, c.t_o, c.t_gate, c.t_up, c.t_down, c.t_emb, c.t_out) == (12, 12, 14, 12, 12, 12, 14, 12, 14)
    assert abs(c.rope_theta - 1e6) < 1 and abs(c.eps - 1e-6) < 1e-12


def test_post_attention_norm_name_accepted(kq, tmp_path):
    out = str(tmp_path / "p2")
    KP.write_dense_pack(out, ffn_norm_name="post_attention_norm.weight", types=dict(q=14, down=12))
    c = kq.read_pack_config(out)
    assert (c.t_q, c.t_down) == (14, 12)


def _expect(kq, out, msg):
    with pytest.raises(ValueError) as ei:
        kq.read_pack_config(out)
    assert msg in str(ei.value), str(ei.value)


def test_unsupported_format(kq, pack):
    out, man = pack
    man["pack_format"] = "kindi-tern-v2"
    KP.write_manifest(out, man)
    _expect(kq, out, "Unsupported pack")


def test_hybrid_profile_rejected(kq, pack):
    out, man = pack
    man["dimensions"]["full_attention_interval"] = 4
    KP.write_manifest(out, man)
    _expect(kq, out, "hybrid")


def test_size_mismatch(kq, pack):
    out, _ = pack
    with open(os.path.join(out, "weights.bin"), "ab") as f:
        f.write(b"\0")
    _expect(kq, out, "Pack size mismatch: weights.bin")


def test_checksum_mismatch_and_size_only_mode(kq, pack, monkeypatch):
    out, _ = pack
    p = os.path.join(out, "f32.bin")
    b = bytearray(open(p, "rb").read())
    b[5] ^= 1
    open(p, "wb").write(bytes(b))
    _expect(kq, out, "Pack checksum mismatch: f32.bin")
    monkeypatch.setenv("KINDI_Q4_VERIFY", "size")   # the reference's fast mode checks sizes only
    kq.read_pack_config(out)
    monkeypatch.setenv("KINDI_Q4_VERIFY", "bogus")
    _expect(kq, out, "KINDI_Q4_VERIFY must be full or size")


def test_manifest_path_must_be_a_bare_name(kq, pack):
    out, man = pack
    man["files"]["../weights.bin"] = man["files"]["weights.bin"]
    KP.write_manifest(out, man)
    _expect(kq, out, "Invalid manifest path")


def test_unaligned_tensor_offset(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    idx["tensors"]["blk.0.attn_q.weight"]["offset"] += 4096
    KP.write_index(out, man, idx)
    _expect(kq, out, "Invalid packed tensor span: blk.0.attn_q.weight")


def test_span_past_the_file(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    rec = idx["tensors"]["output.weight"]
    rec["offset"] = man["files"]["weights.bin"]["size"] // KP.PAGE * KP.PAGE
    KP.write_index(out, man, idx)
    _expect(kq, out, "Invalid packed tensor span: output.weight")


def test_byte_count_must_match_the_shape(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    idx["tensors"]["blk.1.ffn_down.weight"]["bytes"] -= 210
    KP.write_index(out, man, idx)
    _expect(kq, out, "Invalid packed tensor dimensions: blk.1.ffn_down.weight")


def test_missing_tensor(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    del idx["tensors"]["blk.1.attn_k.weight"]
    KP.write_index(out, man, idx)
    _expect(kq, out, "Missing/extra tensors")


def test_wrong_shape(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    rec = idx["tensors"]["blk.0.attn_v.weight"]
    rec["rows"], rec["ne0"] = 64, 1024            # same byte count, wrong shape
    KP.write_index(out, man, idx)
    _expect(kq, out, "Unexpected shape: blk.0.attn_v.weight")


def test_float_tensor_span(kq, pack):
    out, man = pack
    idx = KP.read_index(out)
    idx["tensors"]["blk.0.attn_norm.weight"]["f32_off"] = 2
    KP.write_index(out, man, idx)
    _expect(kq, out, "Invalid float tensor span: blk.0.attn_norm.weight")


def test_malformed_json(kq, pack):
    out, _ = pack
    with open(os.path.join(out, "kindi_pack.json"), "w") as f:
        f.write('{"pack_format": "kindi-q4-v1", ')
    _expect(kq, out, "malformed JSON")


def test_runtime_limits_apply(kq, tmp_path):
    """A well-formed pack the runtime cannot run (head_dim 64) is refused before any allocation."""
    out = str(tmp_path / "p3")
    KP.write_dense_pack(out, HD=64, NH=8, NKV=2)
    _expect(kq, out, "head_dim must be 128")


def test_missing_directory(kq, tmp_path):
    _expect(kq, str(tmp_path / "nope"), "cannot read kindi_pack.json")
    assert json.dumps({"ok": 1})
