"""GPU, 2+ devices: the tensor-parallel model (kq_model_create_tp) against the whole model.

Each rank is a process on its own GPU holding its shard (KV heads, FFN slice, vocabulary slice)
joined by NCCL; the batched pass all-reduces the o and down partials and all-gathers the head's
argmax. Bars: every rank's K/V cache heads after a prefill within 1e-3 rel-L2 of the same heads
of the whole model on one GPU, the greedy steps that follow identical, and batched decode of three
sequences (kq_batch_*) giving the whole model's ids. Worlds 2, 4 and 8 each skip when the
host has fewer GPUs. The FFN of 12288 gives the per-rank down-projection widths of config-4:
6144, 3072 and 1536 input columns."""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

CFG = dict(D=1024, NL=2, NH=32, NKV=8, HD=128, NFF=12288, vocab=4096, ctx=512)
HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "oxcoder-9b_b200")


def _cfg(kq, t):
    return kq.Config.default(dim=t["D"], n_layers=t["NL"], n_heads=t["NH"], n_kv_heads=t["NKV"], head_dim=t["HD"],
                             ffn=t["NFF"], vocab=t["vocab"], ctx=t["ctx"])


def _run(kq, e, prompt, npos, nsteps):
    e.fill_kv(npos, 4)
    e.feed_batch(prompt, npos)
    end = npos + len(prompt)
    toks, t = [], prompt[-1]
    for i in range(nsteps):
        t = e.step(t, end + i)
        toks.append(t)
    kv = [[e.get_kv(l, w, end) for w in (0, 1)] for l in range(CFG["NL"])]
    # batched decode of three sequences (prompt prefixes of different lengths)
    e.batch_caches(3)
    lens = [len(prompt), 41, 17]
    for sq, n in enumerate(lens):
        e.batch_feed(sq, prompt[:n - 1], 0)
    cur, pos, bt = [prompt[n - 1] for n in lens], [n - 1 for n in lens], []
    for i in range(4):
        cur = e.batch_step([0, 1, 2], cur, pos)
        bt.append(list(cur))
        pos = [p + 1 for p in pos]
    return toks, kv, bt


def _rank_main(rank, world, uid, prompt, npos, nsteps, q):
    try:
        sys.path.insert(0, PKG)
        import kq
        e = kq.Engine(_cfg(kq, CFG), device=rank, seed=0, tp=(rank, world, uid))
        q.put((rank, _run(kq, e, prompt, npos, nsteps)))
        e.close()
    except Exception as ex:   # reported to the parent
        q.put((rank, repr(ex)))


@pytest.fixture(scope="module")
def kq():
    import kq as K
    return K


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_prefill_and_steps_match_whole_model(kq, world):
    if kq.lib().kq_device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    rng = np.random.default_rng(3)
    prompt = [int(v) for v in rng.integers(0, CFG["vocab"], 70)]
    npos, nsteps = 30, 6
    uid = kq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, uid, prompt, npos, nsteps, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
    whole = kq.Engine(_cfg(kq, CFG), device=0, seed=0)
    toks, kv, bt = _run(kq, whole, prompt, npos, nsteps)
    nkv_l, hd, end = CFG["NKV"] // world, CFG["HD"], npos + len(prompt)
    for r in range(world):
        assert res[r][0] == toks, (r, res[r][0], toks)
        assert res[r][2] == bt, (r, res[r][2], bt)
        for l in range(CFG["NL"]):
            for w in (0, 1):
                got = res[r][1][l][w].view(np.float16).astype(np.float32).reshape(end, nkv_l, hd)
                ref = kv[l][w].view(np.float16).astype(np.float32).reshape(end, CFG["NKV"], hd)[:, r * nkv_l:(r + 1) * nkv_l]
                assert rel_l2(got, ref) < 1e-3, (r, l, w)


def _loss_rank(rank, uid, q_out, q_in):
    """Rank 1 stops taking part after the prefill (it keeps its process and memory until rank 0
    is done); rank 0's next step must end with a timeout, not hang."""
    try:
        sys.path.insert(0, PKG)
        import time
        import kq
        e = kq.Engine(_cfg(kq, CFG), device=rank, seed=0, tp=(rank, 2, uid))
        e.feed_batch(list(range(1, 40)), 0)            # collectives of both ranks complete
        if rank == 1:
            q_out.put((1, "left"))
            q_in.get(timeout=240)                      # rank 0 finished; no collective of ours in flight
            e.close()
            return
        assert q_in.get(timeout=120) == "rank 1 left"
        t0 = time.time()
        try:
            e.step(5, 39)                              # its all-reduce has no partner
            res = "no error"
        except Exception as ex:
            res = repr(ex)
        dt = time.time() - t0
        try:
            e.step(5, 39)
            again = "no error"
        except Exception as ex:
            again = repr(ex)
        e.close()
        q_out.put((0, (res, dt, again)))
    except Exception as ex:
        q_out.put((rank, "error: " + repr(ex)))


def test_tp_silent_peer_times_out(kq):
    """Failure detection on the NCCL path (the reference bounds its cross-GPU wait and reports
    it: kindi.cu:1007-1014, tp.py:788-792): a rank whose peer stops answering gets
    KQ_ERR_TIMEOUT after KQ_TP_TIMEOUT_MS, its communicator aborted, instead of blocking in
    NCCL. NVLS stays off (NCCL_NVLS_ENABLE=0) and the silent rank leaves between steps."""
    if kq.lib().kq_device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = {"NCCL_NVLS_ENABLE": "0", "KQ_TP_TIMEOUT_MS": "3000"}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        uid = kq.tp_unique_id()
        ctx = mp.get_context("spawn")
        q_out, q0, q1 = ctx.Queue(), ctx.Queue(), ctx.Queue()
        p0 = ctx.Process(target=_loss_rank, args=(0, uid, q_out, q0))
        p1 = ctx.Process(target=_loss_rank, args=(1, uid, q_out, q1))
        p0.start()
        p1.start()
        first = q_out.get(timeout=300)
        assert first == (1, "left"), first
        q0.put("rank 1 left")
        r0 = q_out.get(timeout=300)
        q1.put("done")
        p0.join(timeout=60)
        p1.join(timeout=60)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    assert r0[0] == 0 and not isinstance(r0[1], str), r0
    res, dt, again = r0[1]
    assert "did not answer" in res, res
    assert 2.5 < dt < 60, dt
    assert "aborted" in again, again
