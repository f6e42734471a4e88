"""kq -- Python face of the B200 Kindi-Q4 runtime (libkq.so, C ABI in include/kq.h).

The host runtime is C++/CUDA; this module is a thin ctypes shim with the same engine interface
as the reference's Q4 engines (scripts/kindi_q4/kindi/cpu4.py:94-236 and gpu4.py:50-110):

    e = make_engine(pack, ctx)  # engine.make_engine -> gpu4.Engine (or Engine(config) synthetic)
    e.reset(); e.feed(tok, pos); e.feed_batch(toks, pos)
    e.step(tok, pos) -> greedy id; e.generate(ids, n) -> list; e.ylog -> logits

Argument errors raise ValueError, positions past the context OverflowError, allocation failures
MemoryError and CUDA failures RuntimeError, as in the reference engines. There is no CPU
fallback: importing kq without libkq.so raises ImportError, and every call runs on the GPU.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkq.so")
Q4_K, Q6_K = 12, 14
BLOCK = {Q4_K: 144, Q6_K: 210}
T_EMB, T_OUT, T_OUTNORM, T_ATTN_NORM, T_Q, T_K, T_V, T_O, T_FFN_NORM, T_GATE, T_UP, T_DOWN = range(12)

OK, ERR_ARG, ERR_BACKEND, ERR_OVERFLOW, ERR_MEMORY, ERR_TIMEOUT = 0, -1, -2, -3, -4, -5


class Config(C.Structure):
    """kq_config (include/kq.h)."""
    _fields_ = [(n, C.c_int) for n in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "ctx")] + \
               [("rope_theta", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int) for n in ("t_q", "t_k", "t_v", "t_o", "t_gate", "t_up", "t_down", "t_emb", "t_out",
                                       "max_tokens")]

    @classmethod
    def default(cls, **kw):
        c = cls()
        lib().kq_config_default(C.byref(c))
        for k, v in kw.items():
            if not hasattr(c, k):
                raise ValueError("unknown config field %r" % k)
            setattr(c, k, v)
        return c

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


PF = C.POINTER(C.c_float)
PI32 = C.POINTER(C.c_int32)
PU16 = C.POINTER(C.c_uint16)

# Every symbol include/kq.h declares, with its ctypes signature (restype, argtypes).
SIGNATURES = {
    "kq_version": (C.c_int, []),
    "kq_error": (C.c_char_p, []),
    "kq_device_count": (C.c_int, []),
    "kq_config_default": (None, [C.POINTER(Config)]),
    "kq_model_create": (C.c_void_p, [C.POINTER(Config), C.c_int]),
    "kq_model_free": (None, [C.c_void_p]),
    "kq_pack_read_config": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(Config)]),
    "kq_model_load_pack": (C.c_void_p, [C.c_char_p, C.c_int, C.c_int]),
    "kq_tp_unique_id": (C.c_int, [C.c_char_p]),
    "kq_batch_caches": (C.c_int, [C.c_void_p, C.c_int]),
    "kq_batch_feed": (C.c_int, [C.c_void_p, C.c_int, PI32, C.c_int, C.c_int]),
    "kq_batch_step": (C.c_int, [C.c_void_p, PI32, PI32, PI32, C.c_int, PI32]),
    "kq_model_create_tp": (C.c_void_p, [C.POINTER(Config), C.c_int, C.c_int, C.c_int, C.c_char_p]),
    "kq_model_tp": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kq_model_fill_synthetic": (C.c_int, [C.c_void_p, C.c_uint64]),
    "kq_model_set_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "kq_model_reset": (C.c_int, [C.c_void_p]),
    "kq_model_fill_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64]),
    "kq_model_get_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, PU16]),
    "kq_feed": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "kq_step": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "kq_feed_batch": (C.c_int, [C.c_void_p, PI32, C.c_int, C.c_int]),
    "kq_generate": (C.c_int, [C.c_void_p, PI32, C.c_int, C.c_int, PI32]),
    "kq_logits": (C.c_int, [C.c_void_p, C.c_int, PF]),
    "kq_hidden": (C.c_int, [C.c_void_p, PF]),
    "kq_decode_loop": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, PI32]),
    "kq_time_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, PF]),
    "kq_step_kernels": (C.c_int, [C.c_void_p]),
    "kq_phase_times": (C.c_int, [C.c_void_p, PF]),
    "kq_ffn_block": (C.c_int, [C.c_void_p, C.c_int, PF, C.c_int, PF]),
    "kq_time_ffn_block": (C.c_int, [C.c_void_p, C.c_int, C.c_int, PF]),
    "kq_qmat_create": (C.c_void_p, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "kq_qmat_free": (None, [C.c_void_p]),
    "kq_qmat_upload": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "kq_qmat_fill_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64]),
    "kq_qmat_dequant": (C.c_int, [C.c_void_p, C.c_int, C.c_int, PF]),
    "kq_qmat_matvec": (C.c_int, [C.c_void_p, PF, PF]),
    "kq_qmat_matmul": (C.c_int, [C.c_void_p, PF, C.c_int, PF]),
    "kq_qmat_matvec_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kq_time_matvec": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_int, PF]),
    "kq_qmat_bytes": (C.c_size_t, [C.c_void_p]),
    "kq_qmat_argmax_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kq_verify": (C.c_int, [C.c_void_p, PI32, PI32, C.c_int, C.c_int, PF, PI32]),
    "kq_accept": (C.c_int, [C.c_void_p, PI32, PI32, C.c_int, PF, C.c_float, PF, PF, PI32, PI32, PI32]),
    "kq_accept_resident": (C.c_int, [C.c_void_p, PI32, PI32, C.c_int, C.c_float, PF, PF, PI32, PI32, PI32]),
    "kq_draft_logits": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]),
    "kq_draft_upload": (C.c_int, [C.c_void_p, PF, C.c_int]),
    "kq_commit": (C.c_int, [C.c_void_p, PI32, C.c_int, C.c_int]),
    "kq_ngram_create": (C.c_void_p, [C.c_int, C.c_int]),
    "kq_ngram_free": (None, [C.c_void_p]),
    "kq_ngram_reset": (C.c_int, [C.c_void_p, PI32, C.c_int]),
    "kq_ngram_push": (C.c_int, [C.c_void_p, C.c_int32]),
    "kq_ngram_truncate": (C.c_int, [C.c_void_p, C.c_int]),
    "kq_ngram_propose": (C.c_int, [C.c_void_p, C.c_int, PI32]),
    "kq_ngram_length": (C.c_int, [C.c_void_p]),
}

_lib = None


def lib():
    """The loaded libkq.so. Raises ImportError when it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("libkq.so is not built (run `make -C oxcoder-9b_b200` or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error():
    return lib().kq_error().decode(errors="replace")


def check(rc):
    """Map a kq status code to the reference engines' exception types."""
    if rc >= 0:
        return rc
    msg = last_error()
    if rc == ERR_ARG:
        raise ValueError(msg)
    if rc == ERR_OVERFLOW:
        raise OverflowError(msg)
    if rc == ERR_MEMORY:
        raise MemoryError(msg)
    raise RuntimeError(msg or ("kq error %d" % rc))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, t=PF):
    return a.ctypes.data_as(t)


# ----------------------------------------------------------------------------- matrices
class QMat(object):
    """A Q4_K / Q6_K matrix resident on the GPU (kc_matvec / kc_dequant hooks)."""

    def __init__(self, type_, rows, cols, device=0):
        self.type, self.rows, self.cols = int(type_), int(rows), int(cols)
        h = lib().kq_qmat_create(self.type, self.rows, self.cols, device)
        if not h:
            msg = last_error()
            raise (MemoryError if "alloc" in msg else ValueError)(msg)
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().kq_qmat_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def nbytes(self):
        return int(lib().kq_qmat_bytes(self.h))

    def upload(self, gguf_bytes):
        b = np.ascontiguousarray(gguf_bytes, dtype=np.uint8)
        check(lib().kq_qmat_upload(self.h, b.ctypes.data, b.nbytes))
        return self

    def fill_synthetic(self, seed, stream):
        check(lib().kq_qmat_fill_synthetic(self.h, seed, stream))
        return self

    def dequant(self, row=0, nrows=None):
        nrows = self.rows - row if nrows is None else nrows
        out = np.empty((nrows, self.cols), np.float32)
        check(lib().kq_qmat_dequant(self.h, row, nrows, _ptr(out)))
        return out

    def matvec(self, x):
        x = _f32(x)
        if x.shape != (self.cols,):
            raise ValueError("x must have %d elements" % self.cols)
        y = np.empty(self.rows, np.float32)
        check(lib().kq_qmat_matvec(self.h, _ptr(x), _ptr(y)))
        return y

    def matmul(self, X):
        X = _f32(X)
        if X.ndim != 2 or X.shape[1] != self.cols:
            raise ValueError("X must be [M, %d]" % self.cols)
        Y = np.empty((X.shape[0], self.rows), np.float32)
        check(lib().kq_qmat_matmul(self.h, _ptr(X), X.shape[0], _ptr(Y)))
        return Y


def time_matvec(mats, n):
    """Mean ms per launch of the matvec rotating over `mats` (CUDA events)."""
    arr = (C.c_void_p * len(mats))(*[m.h for m in mats])
    ms = C.c_float()
    check(lib().kq_time_matvec(arr, len(mats), n, C.byref(ms)))
    return ms.value


# ----------------------------------------------------------------------------- engine
def tp_unique_id():
    """A fresh NCCL unique id (128 bytes) for kq.Engine(tp=(rank, world, id)); one rank makes it
    and every rank passes the same bytes."""
    buf = C.create_string_buffer(128)
    check(lib().kq_tp_unique_id(buf))
    return buf.raw


class Engine(object):
    """Dense GQA decoder on one B200 (the gpu4.Engine interface).

    config: a Config (default: the BASELINE config-2 model). seed: fill every tensor from the
    seeded synthetic generator (None leaves the weights to set_tensor). tp=(rank, world, id):
    this process's shard of a tensor-parallel model over `world` GPUs (one process per GPU, the
    same 128-byte NCCL id from tp_unique_id() on every rank); it returns when all ranks joined."""

    def __init__(self, config=None, device=0, seed=0, tp=None, pack=None, **overrides):
        if pack is not None:
            if config is not None or tp is not None:
                raise ValueError("a pack engine takes its configuration from the pack")
            self.config = read_pack_config(pack, overrides.pop("ctx", 4096))
            if overrides:
                raise ValueError("unexpected arguments for a pack engine: %s" % sorted(overrides))
            seed = None
        else:
            self.config = config if config is not None else Config.default(**overrides)
        self.ctx = self.config.ctx
        self.vocab = self.config.vocab
        self.tp = tp
        if pack is not None:
            h = lib().kq_model_load_pack(os.fsencode(pack), self.ctx, device)
        elif tp is not None:
            rank, world, uid = tp
            if len(uid) != 128:
                raise ValueError("the NCCL id is 128 bytes")
            h = lib().kq_model_create_tp(C.byref(self.config), device, int(rank), int(world), bytes(uid))
        else:
            h = lib().kq_model_create(C.byref(self.config), device)
        if not h:
            msg = last_error()
            raise (MemoryError if "alloc" in msg else ValueError)(msg)
        self.h = h
        self.device = device
        if seed is not None:
            check(lib().kq_model_fill_synthetic(self.h, seed))
        self._ylog = None

    def close(self):
        if getattr(self, "h", None):
            lib().kq_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- tensors
    def set_tensor(self, layer, kind, data):
        a = np.ascontiguousarray(data)
        check(lib().kq_model_set_tensor(self.h, layer, kind, a.ctypes.data, a.nbytes))

    def fill_kv(self, npos, seed):
        check(lib().kq_model_fill_kv(self.h, npos, seed))

    def get_kv(self, layer, which, npos):
        """K (which 0) or V (1) cache rows [0, npos) as fp16 bits in the order [pos][kv][hd]; a
        tensor-parallel shard returns its own KV heads."""
        nkv = self.config.n_kv_heads // (self.tp[1] if self.tp is not None else 1)
        out = np.empty(npos * nkv * self.config.head_dim, np.uint16)
        check(lib().kq_model_get_kv(self.h, layer, which, npos, _ptr(out, PU16)))
        return out

    # ---- engine API (cpu4.Engine / gpu4.Engine)
    def _validate(self, tok, pos):
        if tok < 0 or tok >= self.vocab or pos < 0:
            raise ValueError("Invalid token or position")
        if pos >= self.ctx:
            raise OverflowError("position %d is past the context (%d)" % (pos, self.ctx))

    def reset(self):
        check(lib().kq_model_reset(self.h))

    def feed(self, tok, pos):
        self._validate(tok, pos)
        check(lib().kq_feed(self.h, int(tok), int(pos)))

    def feed_batch(self, toks, pos):
        t = np.ascontiguousarray(toks, dtype=np.int32)
        for i, tok in enumerate(t):
            self._validate(int(tok), pos + i)
        check(lib().kq_feed_batch(self.h, _ptr(t, PI32), len(t), int(pos)))

    def step(self, tok, pos):
        self._validate(tok, pos)
        self._ylog = None
        return check(lib().kq_step(self.h, int(tok), int(pos)))

    def generate(self, ids, n):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        for i, tok in enumerate(ids):
            self._validate(int(tok), i)
        if len(ids) + n - 1 > self.ctx:
            raise OverflowError("generation runs past the context")
        out = np.empty(n, np.int32)
        check(lib().kq_generate(self.h, _ptr(ids, PI32), len(ids), n, _ptr(out, PI32)))
        return [int(t) for t in out]

    def decode_loop(self, tok, pos, n):
        """n greedy steps on the device without host round trips."""
        self._validate(tok, pos)
        out = np.empty(n, np.int32)
        check(lib().kq_decode_loop(self.h, int(tok), int(pos), int(n), _ptr(out, PI32)))
        return [int(t) for t in out]

    # ---- speculative verification (kq_verify / kq_accept / kq_commit)
    def verify(self, tokens, parents, pos, want_logits=True):
        """Runs a draft tree (node 0 = last accepted token at `pos`); (argmax ids, logits or None)."""
        t = np.ascontiguousarray(tokens, np.int32)
        par = np.ascontiguousarray(parents, np.int32)
        if t.shape != par.shape:
            raise ValueError("tokens and parents must have the same length")
        n = len(t)
        best = np.empty(n, np.int32)
        logits = np.empty((n, self.vocab), np.float32) if want_logits else None
        check(lib().kq_verify(self.h, _ptr(t, PI32), _ptr(par, PI32), n, int(pos),
                              _ptr(logits) if logits is not None else None, _ptr(best, PI32)))
        return best, logits

    def accept(self, tokens, parents, draft_logits=None, temperature=0.0, u_acc=None, u_fin=None, resident=False):
        """On-device acceptance over the last verify pass: (accepted node path, emitted tokens).
        resident=True: the draft logits are the rows already on the device (upload_draft, or a
        drafter writing draft_logits_device()), not copied from the host."""
        t = np.ascontiguousarray(tokens, np.int32)
        par = np.ascontiguousarray(parents, np.int32)
        n = len(t)
        g = _f32(draft_logits) if draft_logits is not None and not resident else None
        ua = _f32(u_acc) if u_acc is not None else None
        uf = _f32(u_fin) if u_fin is not None else None
        path = np.empty(n + 1, np.int32)
        out = np.empty(n + 1, np.int32)
        plen = C.c_int32()
        pua = _ptr(ua) if ua is not None else None
        puf = _ptr(uf) if uf is not None else None
        if resident:
            no = check(lib().kq_accept_resident(self.h, _ptr(t, PI32), _ptr(par, PI32), n, float(temperature), pua, puf,
                                                _ptr(path, PI32), _ptr(out, PI32), C.byref(plen)))
        else:
            no = check(lib().kq_accept(self.h, _ptr(t, PI32), _ptr(par, PI32), n, _ptr(g) if g is not None else None,
                                       float(temperature), pua, puf, _ptr(path, PI32), _ptr(out, PI32), C.byref(plen)))
        return [int(v) for v in path[:plen.value]], [int(v) for v in out[:no]]

    def upload_draft(self, draft_logits):
        """Copy draft logits (n x vocab) into the device buffer accept(resident=True) reads."""
        g = _f32(draft_logits)
        check(lib().kq_draft_upload(self.h, _ptr(g), g.shape[0]))

    def draft_logits_device(self):
        """(device pointer, row length) of the resident draft-logit buffer, for a GPU drafter."""
        p, ld = C.c_void_p(), C.c_int()
        check(lib().kq_draft_logits(self.h, C.byref(p), C.byref(ld)))
        return p.value, ld.value

    # ---- batched decode of many sequences
    def batch_caches(self, n_seq):
        """Allocate (zeroed) K/V caches for n_seq sequences."""
        check(lib().kq_batch_caches(self.h, int(n_seq)))

    def batch_feed(self, seq, toks, pos):
        """Prefill sequence `seq` with toks from position pos."""
        t = np.ascontiguousarray(toks, np.int32)
        check(lib().kq_batch_feed(self.h, int(seq), _ptr(t, PI32), len(t), int(pos)))

    def batch_step(self, seqs, toks, pos):
        """One token for each of the distinct sequences seqs (token toks[i] at position pos[i]):
        their greedy ids."""
        sq = np.ascontiguousarray(seqs, np.int32)
        t = np.ascontiguousarray(toks, np.int32)
        p = np.ascontiguousarray(pos, np.int32)
        out = np.empty(len(t), np.int32)
        check(lib().kq_batch_step(self.h, _ptr(sq, PI32), _ptr(t, PI32), _ptr(p, PI32), len(t), _ptr(out, PI32)))
        return [int(v) for v in out]

    def commit(self, path, pos):
        """K/V compaction of an accepted path (path[0] = 0)."""
        p = np.ascontiguousarray(path, np.int32)
        check(lib().kq_commit(self.h, _ptr(p, PI32), len(p) - 1, int(pos)))

    def ffn_block(self, layer, X):
        """The MLP block of `layer` (rmsnorm, gate/up + SwiGLU, down) on the rows of X [M, dim]."""
        X = _f32(X)
        if X.ndim != 2 or X.shape[1] != self.config.dim:
            raise ValueError("X must be [M, %d]" % self.config.dim)
        Y = np.empty_like(X)
        check(lib().kq_ffn_block(self.h, int(layer), _ptr(X), X.shape[0], _ptr(Y)))
        return Y

    def time_ffn_block(self, M, n):
        """Mean ms per MLP block of M rows over n blocks (successive layers' weights)."""
        ms = C.c_float()
        check(lib().kq_time_ffn_block(self.h, int(M), int(n), C.byref(ms)))
        return ms.value

    def phase_times(self):
        """ms per category of the batched passes since the last call (model created with
        KQ_PHASE_TIMES=1): {"gemm", "attention", "allreduce", "other"}."""
        out = np.zeros(4, np.float32)
        check(lib().kq_phase_times(self.h, _ptr(out)))
        return dict(zip(("gemm", "attention", "allreduce", "other"), [float(v) for v in out]))

    def step_kernels(self):
        """Kernels one decode step launches (kernel nodes of the step graph)."""
        return check(lib().kq_step_kernels(self.h))

    def time_decode(self, tok, pos, n):
        ms = C.c_float()
        check(lib().kq_time_decode(self.h, int(tok), int(pos), int(n), C.byref(ms)))
        return ms.value

    @property
    def ylog(self):
        """Logits of the last step (Engine.ylog[:ylog_n])."""
        out = np.empty(self.vocab, np.float32)
        check(lib().kq_logits(self.h, 0, _ptr(out)))
        return out

    @property
    def ylog_n(self):
        return self.vocab

    ylog_map = None

    def hidden(self):
        out = np.empty(self.config.dim, np.float32)
        check(lib().kq_hidden(self.h, _ptr(out)))
        return out


# ----------------------------------------------------------------------------- drafter
class NgramDraft(object):
    """The library's prompt-lookup drafter (kq_ngram_*) behind the interface of the reference's
    NgramDraft (scripts/kindi_q4/kindi/spec.py:801-841): reset(hist), truncate(L), push(t) and
    propose(k) -> up to k token ids that followed the latest earlier occurrence of the longest
    matching suffix (lengths nmax .. nmin). Host-side; no GPU. Negative L or k raise ValueError
    (the reference would apply Python's slice rules to them)."""

    def __init__(self, nmax=4, nmin=1):
        self.nmax, self.nmin = nmax, nmin
        self._d = lib().kq_ngram_create(int(nmax), int(nmin))
        if not self._d:
            raise ValueError(last_error())

    def close(self):
        if getattr(self, "_d", None):
            lib().kq_ngram_free(self._d)
            self._d = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, hist):
        h = np.ascontiguousarray(np.asarray(hist, dtype=np.int64).astype(np.int32))
        check(lib().kq_ngram_reset(self._d, _ptr(h, PI32), int(h.size)))

    def truncate(self, L):
        check(lib().kq_ngram_truncate(self._d, int(L)))

    def push(self, t):
        check(lib().kq_ngram_push(self._d, int(t)))

    def propose(self, k):
        k = int(k)
        out = np.empty(max(k, 1), np.int32)
        n = check(lib().kq_ngram_propose(self._d, k, _ptr(out, PI32)))
        return [int(v) for v in out[:n]]

    def __len__(self):
        return lib().kq_ngram_length(self._d)


def read_pack_config(pack, ctx=4096):
    """Validate a Kindi Q4 pack directory without touching the GPU (kq_pack_read_config) and
    return its Config at context ctx. Raises ValueError with the reference's messages
    ("Unsupported pack", "Pack size mismatch: ...", "Invalid packed tensor span: ...", ...)."""
    c = Config()
    check(lib().kq_pack_read_config(os.fsencode(pack), int(ctx), C.byref(c)))
    return c


def make_engine(pack=None, ctx=4096, clusters=None, log=print, device=0, seed=0, **overrides):
    """engine.make_engine (engine.py:369-381) for the Q4 path on one GPU. `pack`: a Kindi Q4 pack
    directory (validated, then loaded); a Config, or None, builds the synthetic model of that
    configuration (the default: config-2) from `seed`. The approximate head (`clusters`) is not
    part of the Q4 path, as in the reference."""
    if clusters is not None:
        raise ValueError("Q4 approximate-head paths are not validated")
    if isinstance(pack, (str, bytes, os.PathLike)):
        if overrides:
            raise ValueError("a pack engine takes its configuration from the pack")
        log("kq: loading Q4 pack %s (ctx %d, device %d)" % (os.fspath(pack), ctx, device))
        return Engine(pack=pack, ctx=ctx, device=device)
    if ctx is not None:
        overrides["ctx"] = ctx
    return Engine(pack, device=device, seed=seed, **overrides)
