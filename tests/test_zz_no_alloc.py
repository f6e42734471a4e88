"""GPU: kq_qmat_argmax_noalloc -- the argmax form of the GEMV with its scratch in a static device
array, so the call allocates nothing -- against the existing entry point kq_qmat_matvec_dev
followed by an argmax on the host (lowest index among equal maxima, the head's tie rule).

The file name sorts last, so in a full `-m gpu` run this also runs after every other GPU test in
the same process; it needs no state from them and passes alone in a fresh process too."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144          # KQ_NOALLOC_MAX_ROWS in include/kq.h
NEAR_TIE_REL = 1e-6        # tolerance: an index whose product is this close to the max is accepted

SHAPES = [(14, 151936, 4096), (12, 2048, 12288), (12, 8, 256), (14, 4096, 2048)]


@pytest.fixture(scope="module")
def env():
    import torch
    import kq as K
    assert K.lib().kq_device_count() > 0 and torch.cuda.is_available(), "no GPU"
    return K, torch


def _noalloc(K, m, x, idx):
    return K.lib().kq_qmat_argmax_noalloc(m.h, C.c_void_p(x.data_ptr()), C.c_void_p(idx.data_ptr()), None)


def _existing(K, torch, m, x):
    y = torch.empty(m.rows, dtype=torch.float32, device="cuda")
    K.check(K.lib().kq_qmat_matvec_dev(m.h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), None))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _agrees(idx, y):
    top = int(np.argmax(y))
    if idx == top:
        return True
    return 0 <= idx < y.size and y[idx] >= y[top] - NEAR_TIE_REL * abs(y[top])


@pytest.mark.parametrize("ty,R,Cc", SHAPES)
def test_two_calls_in_a_row_match_existing_entry_point(env, ty, R, Cc):
    K, torch = env
    m = K.QMat(ty, R, Cc).fill_synthetic(0, 91 + R % 7)
    g = torch.Generator(device="cuda").manual_seed(R + Cc)
    x1 = torch.randn(Cc, generator=g, device="cuda", dtype=torch.float32)
    x2 = torch.randn(Cc, generator=g, device="cuda", dtype=torch.float32)
    idx = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    # back to back on one stream, no synchronisation between: the second and third calls see the
    # scratch (ticket, partials) exactly as the previous call left it
    K.check(_noalloc(K, m, x1, idx[0:1]))
    K.check(_noalloc(K, m, x2, idx[1:2]))
    K.check(_noalloc(K, m, x1, idx[2:3]))
    torch.cuda.synchronize()
    got = idx.cpu().numpy().tolist()
    y1, y2 = _existing(K, torch, m, x1), _existing(K, torch, m, x2)
    assert _agrees(got[0], y1), (got[0], int(np.argmax(y1)))
    assert _agrees(got[1], y2), (got[1], int(np.argmax(y2)))
    assert got[2] == got[0]
    m.matvec(np.zeros(Cc, np.float32))   # synchronising call: raises if a device wait gave up
    m.close()


def test_ties_take_the_lowest_index(env):
    K, torch = env
    m = K.QMat(12, 4096, 4096).fill_synthetic(0, 5)
    x = torch.zeros(4096, dtype=torch.float32, device="cuda")   # every product is 0
    idx = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    K.check(_noalloc(K, m, x, idx[0:1]))
    K.check(_noalloc(K, m, x, idx[1:2]))
    torch.cuda.synchronize()
    assert idx.cpu().numpy().tolist() == [0, 0]
    m.close()


def test_calls_leave_free_device_memory_unchanged(env):
    K, torch = env
    m = K.QMat(14, 151936, 4096).fill_synthetic(0, 6)
    x = torch.randn(4096, device="cuda", dtype=torch.float32)
    idx = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    K.check(_noalloc(K, m, x, idx))            # first call on the device: scratch look-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(20):
        K.check(_noalloc(K, m, x, idx))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    m.close()


def test_sizes_beyond_the_scratch_are_rejected(env):
    K, torch = env
    m = K.QMat(12, MAX_ROWS + 8, 256)
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    idx = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    rc = _noalloc(K, m, x, idx)
    assert rc == K.ERR_ARG
    assert "static scratch" in K.last_error() and str(MAX_ROWS) in K.last_error()
    torch.cuda.synchronize()
    assert int(idx.cpu()[0]) == -7             # nothing was launched
    ok = K.QMat(12, MAX_ROWS, 256).fill_synthetic(0, 8)   # exactly at the limit is accepted
    K.check(_noalloc(K, ok, x, idx))
    torch.cuda.synchronize()
    assert int(idx.cpu()[0]) == 0
    assert K.lib().kq_qmat_argmax_noalloc(None, C.c_void_p(x.data_ptr()), C.c_void_p(idx.data_ptr()), None) == K.ERR_ARG
    assert K.lib().kq_qmat_argmax_noalloc(ok.h, None, C.c_void_p(idx.data_ptr()), None) == K.ERR_ARG
    m.close()
    ok.close()
