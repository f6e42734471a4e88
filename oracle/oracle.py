"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loaded by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm to check
or time the CUDA library against a CPU restatement of the Kindi Q4 path. The product package never
imports this module.

  liboracle.so       kq_oracle.c: restated block decode, matvec, dense GQA decoder, generator
  _ref/libkcpu4.so   the reference's own kcpu4.c compiled from its sources (when it was built)
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
Q4K, Q6K = 12, 14
BLOCK = {Q4K: 144, Q6K: 210}

PF = C.POINTER(C.c_float)
PU8 = C.POINTER(C.c_uint8)
PU16 = C.POINTER(C.c_uint16)
PI32 = C.POINTER(C.c_int32)

# tensor kinds of the synthetic stream numbering (kq_oracle.c)
T_EMB, T_OUT, T_OUTNORM, T_ATTN_NORM, T_Q, T_K, T_V, T_O, T_FFN_NORM, T_GATE, T_UP, T_DOWN = range(12)


def stream(layer, kind):
    return (layer + 1) * 32 + kind


class OCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("D", "NL", "NH", "NKV", "HD", "NFF", "vocab", "ctx")] + \
               [("rope_theta", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int) for n in ("t_q", "t_k", "t_v", "t_o", "t_gate", "t_up", "t_down", "t_emb", "t_out")]


def ptr(a, t=PF):
    return a.ctypes.data_as(t)


def build():
    """Compile liboracle.so (and oracle/_ref when the reference sources exist)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.or_decode_block.argtypes = [PU8, C.c_int, PF]
        L.or_matvec_raw.argtypes = [PU8, C.c_int, C.c_int, C.c_int, C.c_int, PF, PF]
        L.or_dequant_raw.argtypes = [PU8, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, PF]
        L.or_gen_matrix.argtypes = [PU8, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_uint64]
        L.or_gen_normal.argtypes = [PF, C.c_int64, C.c_float, C.c_float, C.c_uint64, C.c_uint64]
        L.or_gen_tokens.argtypes = [PI32, C.c_int64, C.c_int, C.c_uint64, C.c_uint64]
        L.or_gen_uniform.argtypes = [PF, C.c_int64, C.c_uint64, C.c_uint64]
        L.or_gen_half_normal.argtypes = [PU16, C.c_int64, C.c_uint64, C.c_uint64]
        L.or_model_create.argtypes = [C.POINTER(OCfg), C.c_uint64, C.c_int]
        L.or_model_create.restype = C.c_void_p
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_model_reset.argtypes = [C.c_void_p]
        L.or_model_fill_kv.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
        L.or_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.or_step.restype = C.c_int
        L.or_model_logits.argtypes = [C.c_void_p]
        L.or_model_logits.restype = PF
        L.or_model_hidden.argtypes = [C.c_void_p]
        L.or_model_hidden.restype = PF
        L.or_model_swiglu.argtypes = [C.c_void_p]
        L.or_model_swiglu.restype = PF
        L.or_model_kcache.argtypes = [C.c_void_p, C.c_int]
        L.or_model_kcache.restype = PU16
        L.or_model_vcache.argtypes = [C.c_void_p, C.c_int]
        L.or_model_vcache.restype = PU16
        L.or_model_tensor.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.or_model_tensor.restype = PU8
        L.or_rmsnorm.argtypes = [PF, PF, C.c_int, PF, PF, C.c_int, C.c_float]
        L.or_attn_scale.argtypes = [C.c_int]
        L.or_attn_scale.restype = C.c_float
        L.or_verify.argtypes = [C.c_void_p, PI32, PI32, C.c_int, C.c_int, PF, PI32]
        L.or_verify.restype = C.c_int
        L.or_ffn_block.argtypes = [C.c_void_p, C.c_int, PF, C.c_int, PF]
        L.or_ffn_block.restype = C.c_int
        L.or_commit.argtypes = [C.c_void_p, PI32, C.c_int, C.c_int]
        L.or_commit.restype = C.c_int
        L.or_accept.argtypes = [PF, PF, PI32, PI32, C.c_int, C.c_int, C.c_float, PF, PF, PI32, PI32]
        L.or_accept.restype = C.c_int
        L.or_kq_exp.argtypes = [C.c_float]
        L.or_kq_exp.restype = C.c_float
        L.or_set_threads.argtypes = [C.c_int]
        L.or_get_threads.restype = C.c_int
        assert L.or_sizeof_cfg() == C.sizeof(OCfg)
        _lib = L
    return _lib


# ----------------------------------------------------------------------------- primitives
def decode_blocks(raw, ty):
    """raw [..., BLOCK[ty]] uint8 -> float32 [..., 256] via or_decode_block."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, BLOCK[ty])
    out = np.empty((raw.shape[0], 256), np.float32)
    L = lib()
    for i in range(raw.shape[0]):
        L.or_decode_block(ptr(raw[i], PU8), ty, ptr(out[i]))
    return out


def gen_matrix(R, Cc, ty, seed, strm, layout=0):
    W = np.empty(R * (Cc // 256) * BLOCK[ty], np.uint8)
    lib().or_gen_matrix(ptr(W, PU8), R, Cc, ty, layout, seed, strm)
    return W


def gen_normal(n, mu, sigma, seed, strm):
    y = np.empty(n, np.float32)
    lib().or_gen_normal(ptr(y), n, mu, sigma, seed, strm)
    return y


def gen_tokens(n, V, seed, strm):
    y = np.empty(n, np.int32)
    lib().or_gen_tokens(ptr(y, PI32), n, V, seed, strm)
    return y


def gen_uniform(n, seed, strm):
    y = np.empty(n, np.float32)
    lib().or_gen_uniform(ptr(y), n, seed, strm)
    return y


def matvec(W, R, Cc, ty, x, layout=0):
    y = np.empty(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    lib().or_matvec_raw(ptr(W, PU8), R, Cc, ty, layout, ptr(x), ptr(y))
    return y


def dequant_row(W, R, Cc, ty, row, layout=0):
    y = np.empty(Cc, np.float32)
    lib().or_dequant_raw(ptr(W, PU8), R, Cc, ty, layout, row, ptr(y))
    return y


def to_pack_layout(W, R, Cc, ty):
    """GGUF row-major [R][G][bs] -> Kindi pack [R/8][G][8][bs] (q4pack.py:151-158)."""
    bs = BLOCK[ty]
    return np.ascontiguousarray(W.reshape(R // 8, 8, Cc // 256, bs).transpose(0, 2, 1, 3)).reshape(-1)


# ----------------------------------------------------------------------------- dense decoder
CFG2 = dict(D=4096, NL=32, NH=32, NKV=8, HD=128, NFF=12288, vocab=151936, ctx=4096,
            rope_theta=1e6, eps=1e-6, t_q=Q4K, t_k=Q4K, t_v=Q6K, t_o=Q4K, t_gate=Q4K, t_up=Q4K,
            t_down=Q6K, t_emb=Q4K, t_out=Q6K)


def make_cfg(**kw):
    d = dict(CFG2)
    d.update(kw)
    return OCfg(**d)


class Model(object):
    """The dense GQA decoder restated on the CPU, weights generated from `seed`."""

    def __init__(self, seed=0, layout=0, **cfg):
        self.cfg = make_cfg(**cfg)
        self.L = lib()
        self.h = self.L.or_model_create(C.byref(self.cfg), seed, layout)
        if not self.h:
            raise MemoryError("oracle model allocation failed")

    def close(self):
        if self.h:
            self.L.or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self.L.or_model_reset(self.h)

    def fill_kv(self, npos, seed):
        self.L.or_model_fill_kv(self.h, npos, seed)

    def step(self, tok, pos, head=True):
        r = self.L.or_step(self.h, int(tok), int(pos), 1 if head else 0)
        if r == -3:
            raise ValueError("oracle: bad token or position")
        return r

    def logits(self):
        return np.ctypeslib.as_array(self.L.or_model_logits(self.h), shape=(self.cfg.vocab,)).copy()

    def hidden(self):
        return np.ctypeslib.as_array(self.L.or_model_hidden(self.h), shape=(self.cfg.D,)).copy()

    def swiglu(self):
        """The SwiGLU output (silu(gate) * up, NFF floats) of the last layer of the last step."""
        return np.ctypeslib.as_array(self.L.or_model_swiglu(self.h), shape=(self.cfg.NFF,)).copy()

    def kcache(self, layer, npos):
        n = npos * self.cfg.NKV * self.cfg.HD
        return np.ctypeslib.as_array(self.L.or_model_kcache(self.h, layer), shape=(n,)).copy()

    def vcache(self, layer, npos):
        n = npos * self.cfg.NKV * self.cfg.HD
        return np.ctypeslib.as_array(self.L.or_model_vcache(self.h, layer), shape=(n,)).copy()

    def verify(self, tokens, parents, pos):
        """Draft-tree verification (or_verify): (argmax ids [n], logits [n][vocab])."""
        t = np.ascontiguousarray(tokens, np.int32)
        par = np.ascontiguousarray(parents, np.int32)
        n = len(t)
        logits = np.empty((n, self.cfg.vocab), np.float32)
        best = np.empty(n, np.int32)
        if self.L.or_verify(self.h, ptr(t, PI32), ptr(par, PI32), n, int(pos), ptr(logits), ptr(best, PI32)):
            raise ValueError("oracle: bad verify arguments")
        return best, logits

    def ffn_block(self, layer, X):
        """or_ffn_block: the MLP block of `layer` on the rows of X [M, D]."""
        X = np.ascontiguousarray(X, np.float32)
        Y = np.empty_like(X)
        if self.L.or_ffn_block(self.h, int(layer), ptr(X), X.shape[0], ptr(Y)):
            raise ValueError("oracle: bad MLP block arguments")
        return Y

    def commit(self, path, pos):
        p = np.ascontiguousarray(path, np.int32)
        if self.L.or_commit(self.h, ptr(p, PI32), len(p) - 1, int(pos)):
            raise ValueError("oracle: bad commit arguments")

    def generate(self, ids, n):
        """Greedy: kcpu4's Engine.generate order (cpu4.py:227-236)."""
        self.reset()
        for i, t in enumerate(ids[:-1]):
            self.step(t, i, head=False)
        pos = len(ids)
        out = [self.step(ids[-1], pos - 1)]
        while len(out) < n:
            out.append(self.step(out[-1], pos))
            pos += 1
        return out


def accept(z, g, tokens, parents, temperature, u_acc=None, u_fin=None):
    """or_accept: (path, emitted tokens) for target logits z [n][V], draft logits g [n][V]
    (ignored when temperature == 0) and uniforms u_acc / u_fin [n]."""
    z = np.ascontiguousarray(z, np.float32)
    n, V = z.shape
    g = np.ascontiguousarray(g if g is not None else np.zeros_like(z), np.float32)
    t = np.ascontiguousarray(tokens, np.int32)
    par = np.ascontiguousarray(parents, np.int32)
    ua = np.ascontiguousarray(u_acc if u_acc is not None else np.zeros(n), np.float32)
    uf = np.ascontiguousarray(u_fin if u_fin is not None else np.zeros(n), np.float32)
    tau = np.float32(1.0) / np.float32(temperature) if temperature > 0 else np.float32(0.0)
    path = np.empty(n + 1, np.int32)
    out = np.empty(n + 1, np.int32)
    no = lib().or_accept(ptr(z), ptr(g), ptr(t, PI32), ptr(par, PI32), n, V, float(tau), ptr(ua), ptr(uf),
                         ptr(path, PI32), ptr(out, PI32))
    if no < 0:
        raise ValueError("oracle: bad accept arguments")
    return [int(v) for v in path[:no]], [int(v) for v in out[:no]]


# ----------------------------------------------------------------------------- reference library
class RefMat(C.Structure):
    """The reference's Mat (kcpu4.c:26)."""
    _fields_ = [("W", PU8), ("S", PF), ("R", C.c_int), ("C", C.c_int), ("type", C.c_int),
                ("offset", C.c_uint64), ("bytes", C.c_uint64)]


_ref = None


def ref_lib():
    """The reference's kcpu4.c built from its own sources into oracle/_ref, or None."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libkcpu4.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.kc_matvec.argtypes = [C.POINTER(RefMat), PF, PF]
        L.kc_dequant.argtypes = [C.POINTER(RefMat), C.c_int, PF]
        _ref = L
    return _ref


def ref_matvec(Wpack, R, Cc, ty, x):
    """kc_matvec on a matrix in the Kindi pack layout."""
    L = ref_lib()
    m = RefMat(ptr(Wpack, PU8), None, R, Cc, ty, 0, Wpack.nbytes)
    y = np.empty(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    L.kc_matvec(C.byref(m), ptr(x), ptr(y))
    return y


def ref_dequant(Wpack, R, Cc, ty, row):
    L = ref_lib()
    m = RefMat(ptr(Wpack, PU8), None, R, Cc, ty, 0, Wpack.nbytes)
    y = np.empty(Cc, np.float32)
    L.kc_dequant(C.byref(m), row, ptr(y))
    return y


_ref_blocks = None


def ref_blocks_lib():
    """oracle/_ref/libkcpu4_blocks.so (ref_blocks.c over the reference's own kcpu4.c), or None."""
    global _ref_blocks
    if _ref_blocks is None:
        path = os.path.join(HERE, "_ref", "libkcpu4_blocks.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.ref_ffn_block.restype = C.c_int
        L.ref_ffn_block.argtypes = [PU8, PU8, PU8, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, PF, PF, PF]
        L.ref_head_step.restype = C.c_int
        L.ref_head_step.argtypes = [PU8, C.c_int, PU8, C.c_int, C.c_int, C.c_int, PF, C.c_int, PF]
        _ref_blocks = L
    return _ref_blocks


def ref_ffn_block(Wg, Wu, Wd, types, D, NFF, norm, x):
    """The reference's MLP block (kcpu4.c:287-295 ffn) on GGUF row-major weights (converted to the
    Kindi pack layout it reads), one token x [D] -> y [D]."""
    tg, tu, td = types
    pg, pu, pd = (to_pack_layout(Wg, NFF, D, tg), to_pack_layout(Wu, NFF, D, tu), to_pack_layout(Wd, D, NFF, td))
    norm = np.ascontiguousarray(norm, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(D, np.float32)
    rc = ref_blocks_lib().ref_ffn_block(ptr(pg, PU8), ptr(pu, PU8), ptr(pd, PU8), tg, tu, td, D, NFF, ptr(norm), ptr(x), ptr(y))
    if rc:
        raise MemoryError("ref_ffn_block scratch")
    return y


def ref_head_step(Wemb, t_emb, Whead, t_head, D, V, out_norm, tok):
    """The reference's kc_step on a model of no layers (embedding row, final norm, head GEMV,
    argmax): (best token, logits [V]); weights GGUF row-major, converted to the pack layout."""
    pe, ph = to_pack_layout(Wemb, V, D, t_emb), to_pack_layout(Whead, V, D, t_head)
    out_norm = np.ascontiguousarray(out_norm, np.float32)
    logits = np.empty(V, np.float32)
    best = ref_blocks_lib().ref_head_step(ptr(pe, PU8), t_emb, ptr(ph, PU8), t_head, D, V, ptr(out_norm), int(tok),
                                          ptr(logits))
    if best < 0:
        raise RuntimeError("ref_head_step failed (%d)" % best)
    return best, logits
