"""Generates tests/golden/quant_golden.npz from the REFERENCE implementation.

Run once on a host that has the reference tree (read-only) and oracle/_ref built:
    python tests/golden/make_golden.py /path/to/reference      (or set KQ_REFERENCE)

Sources of truth:
  - the reference's numpy block decoder, scripts/kindi_q4/kindi/q4pack.py:52-76 (decode_blocks)
  - the reference's native kc_dequant / kc_matvec, scripts/kindi_q4/kindi/kcpu4.c:337-341,
    compiled from its own sources into oracle/_ref by oracle/Makefile

Cases:
  refcase_*  the exact case of tests/kindi_q4/test_quant.py:10-32 (default_rng(35), 16 x 512
             random blocks, d (and dmin) forced to fp16 0.013, x ~ normal)
  synth_*    matrices from the shared synthetic generator (oracle/kq_oracle.c or_gen_matrix),
             seed 0, stream 7, 64 x 1024, with x ~ normal(default_rng(36))
  edge_*     hand-made blocks: all-zero, fp16 subnormal / max d, every 6-bit scale at 63
The fixture is small (< 400 KB) and the GPU box never needs the reference tree.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "scripts", "kindi_q4"))
    from kindi.q4pack import decode_blocks, BLOCK  # the reference's numpy decoder
    assert O.ref_lib() is not None, "build oracle/_ref first (make -C oracle)"
    out = {}
    # --- the reference's own unit-test case (test_quant.py:14-32)
    rng = np.random.default_rng(35)
    for ty in (12, 14):
        rows, cols = 16, 512
        bs = BLOCK[ty]
        raw = rng.integers(0, 256, (rows, cols // 256, bs), dtype=np.uint8)
        for offset in ([0, 2] if ty == 12 else [208]):
            raw[:, :, offset:offset + 2] = np.array([0.013], dtype='<f2').view(np.uint8)
        dense = decode_blocks(raw, ty).reshape(rows, cols)
        tile = O.to_pack_layout(raw.reshape(-1), rows, cols, ty)
        kc_rows = np.stack([O.ref_dequant(tile, rows, cols, ty, r) for r in range(rows)])
        assert np.array_equal(kc_rows, dense)
        x = rng.normal(size=cols).astype(np.float32)
        y = O.ref_matvec(tile, rows, cols, ty, x)
        out["refcase_raw_%d" % ty] = raw
        out["refcase_dense_%d" % ty] = dense
        out["refcase_x_%d" % ty] = x
        out["refcase_y_%d" % ty] = y
    # --- synthetic generator matrices
    rng = np.random.default_rng(36)
    for ty in (12, 14):
        R, Cc = 64, 1024
        W = O.gen_matrix(R, Cc, ty, 0, 7)
        dense = decode_blocks(W.reshape(-1, BLOCK[ty]), ty).reshape(R, Cc)
        x = rng.normal(size=Cc).astype(np.float32)
        y = O.ref_matvec(O.to_pack_layout(W, R, Cc, ty), R, Cc, ty, x)
        out["synth_raw_%d" % ty] = W
        out["synth_dense_%d" % ty] = dense
        out["synth_x_%d" % ty] = x
        out["synth_y_%d" % ty] = y
    # --- edge blocks (8 rows x 1 block each)
    for ty in (12, 14):
        bs = BLOCK[ty]
        raw = np.zeros((8, 1, bs), np.uint8)
        raw[1, 0, :] = 0xFF                                   # all bits set (d = NaN for both types)
        raw[2, 0, :] = 0x55
        halfs = [np.float16(6.0e-8), np.float16(65504.0), np.float16(-1.5), np.float16(0.013), np.float16(1e-4)]
        for r, hv in zip(range(3, 8), halfs):
            raw[r, 0, :] = np.random.default_rng(r).integers(0, 256, bs, dtype=np.uint8)
            hb = np.array([hv], dtype='<f2').view(np.uint8)
            for off in ([0, 2] if ty == 12 else [208]):
                raw[r, 0, off:off + 2] = hb
            if ty == 12 and r == 7:
                raw[r, 0, 4:16] = 0xFF                        # every 6-bit scale and min = 63
        dense = decode_blocks(raw, ty).reshape(8, 256)
        tile = O.to_pack_layout(raw.reshape(-1), 8, 256, ty)
        kc_rows = np.stack([O.ref_dequant(tile, 8, 256, ty, r) for r in range(8)])
        assert np.array_equal(kc_rows.view(np.uint32), dense.view(np.uint32))
        out["edge_raw_%d" % ty] = raw
        out["edge_dense_%d" % ty] = dense
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "quant_golden.npz"))


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KQ_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py /path/to/reference   (or set KQ_REFERENCE)")
    main(root)
