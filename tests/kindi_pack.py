"""Test helper: writes a Kindi Q4 pack directory for the dense GQA decoder in the reference's
on-disk format (scripts/kindi_q4/kindi/q4pack.py:110-180), with every tensor taken from the
shared synthetic generator (the oracle's `or_gen_*`, the same bytes kq_model_fill_synthetic
generates), so a model loaded from the pack must equal the synthetic model bit for bit.

Format, as the reference's convert() writes it:
  weights.bin   each Q4_K/Q6_K matrix in the 8-row interleave [R/8][C/256][8][block], its offset
                a multiple of 16 KiB, zero padded to a multiple of 16 KiB
  f32.bin       float tensors (the norm weights), little-endian float32
  index.json    {"tensors": {gguf name: {rows, ne0, dims, type, folded, offset, bytes,
                padded_bytes} or {rows, ne0, dims, type: 0, folded, f32_off}}}
  kindi_pack.json  pack_format "kindi-q4-v1", head "output.weight", hadamard_block 1,
                dimensions, layout, files {name: {size, sha256}}
The dimensions are the dense profile the B200 runtime accepts (full_attention_interval 1).
"""
import hashlib
import json
import os

from oracle import oracle as O

PAGE = 16384


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(4 << 20), b""):
            h.update(b)
    return h.hexdigest()


def write_dense_pack(out, D=512, NL=2, NH=4, NKV=1, HD=128, NFF=1024, vocab=4096, rope_theta=1e6, eps=1e-6,
                     types=None, seed=0, ffn_norm_name="ffn_norm.weight"):
    """Writes the pack into the new directory `out` and returns the manifest dict."""
    ty = dict(q=12, k=12, v=14, o=12, gate=12, up=12, down=14, emb=12, out=14)
    if types:
        ty.update(types)
    os.makedirs(out)
    index = {}
    wpath, fpath = os.path.join(out, "weights.bin"), os.path.join(out, "f32.bin")
    with open(wpath, "wb") as wf, open(fpath, "wb") as ff:
        def quant(name, R, Cc, t, layer, kind):
            raw = O.gen_matrix(R, Cc, t, seed, O.stream(layer, kind))        # GGUF row-major bytes
            tiled = O.to_pack_layout(raw, R, Cc, t)                         # q4pack.py:151-158
            off = wf.tell()
            wf.write(tiled.tobytes())
            nbytes = tiled.nbytes
            padded = (nbytes + PAGE - 1) // PAGE * PAGE
            wf.write(bytes(padded - nbytes))
            index[name] = dict(rows=R, ne0=Cc, dims=[R, Cc], type=t, folded=False, offset=off, bytes=nbytes,
                               padded_bytes=padded)

        def floats(name, layer, kind):
            v = O.gen_normal(D, 1.0, 0.02, seed, O.stream(layer, kind)).astype("<f4")
            index[name] = dict(rows=1, ne0=D, dims=[D], type=0, folded=False, f32_off=ff.tell())
            ff.write(v.tobytes())

        quant("token_embd.weight", vocab, D, ty["emb"], -1, O.T_EMB)
        quant("output.weight", vocab, D, ty["out"], -1, O.T_OUT)
        floats("output_norm.weight", -1, O.T_OUTNORM)
        for l in range(NL):
            p = "blk.%d." % l
            floats(p + "attn_norm.weight", l, O.T_ATTN_NORM)
            quant(p + "attn_q.weight", NH * HD, D, ty["q"], l, O.T_Q)
            quant(p + "attn_k.weight", NKV * HD, D, ty["k"], l, O.T_K)
            quant(p + "attn_v.weight", NKV * HD, D, ty["v"], l, O.T_V)
            quant(p + "attn_output.weight", D, NH * HD, ty["o"], l, O.T_O)
            floats(p + ffn_norm_name, l, O.T_FFN_NORM)
            quant(p + "ffn_gate.weight", NFF, D, ty["gate"], l, O.T_GATE)
            quant(p + "ffn_up.weight", NFF, D, ty["up"], l, O.T_UP)
            quant(p + "ffn_down.weight", D, NFF, ty["down"], l, O.T_DOWN)
    with open(os.path.join(out, "index.json"), "w") as f:
        json.dump({"tensors": index}, f, sort_keys=True)
    dims = dict(layers=NL, width=D, ffn=NFF, heads=NH, kv_heads=NKV, head_dim=HD, rope_dim=HD, rope_base=rope_theta,
                norm_eps=eps, full_attention_interval=1)
    names = ("weights.bin", "f32.bin", "index.json")
    man = dict(pack_format="kindi-q4-v1", model="synthetic dense GQA", head="output.weight", hadamard_block=1,
               dimensions=dims, quantization="mixed Q4_K/Q6_K; original blocks preserved",
               layout="8-row-block-interleave",
               files={n: dict(size=os.path.getsize(os.path.join(out, n)), sha256=_sha256(os.path.join(out, n)))
                      for n in names})
    write_manifest(out, man)
    return man


def write_manifest(out, man):
    with open(os.path.join(out, "kindi_pack.json"), "w") as f:
        f.write(json.dumps(man, indent=2) + "\n")


def refresh_file_record(out, man, name):
    """Re-record one file's size and digest after a test edited it."""
    p = os.path.join(out, name)
    man["files"][name] = dict(size=os.path.getsize(p), sha256=_sha256(p))
    write_manifest(out, man)


def read_index(out):
    return json.load(open(os.path.join(out, "index.json")))


def write_index(out, man, index):
    with open(os.path.join(out, "index.json"), "w") as f:
        json.dump(index, f, sort_keys=True)
    refresh_file_record(out, man, "index.json")

