"""CPU, world size 2 over gloo: the tensor-parallel decomposition the library runs on NCCL,
checked with the oracle on the host. Rank r holds the column slice r of a row-split matrix (o,
down: input columns of its heads / FFN slice) and its vocabulary slice of the head:
  - the all-reduced sum of the ranks' partial products equals the whole matrix-vector product;
  - the row slices of a column-split matrix (q/k/v, gate/up) are the whole product's rows;
  - the argmax gathered over vocabulary slices (best per rank, then the first rank holding the
    maximum) equals the whole argmax with the lowest index on ties."""
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        sys.path.insert(0, ROOT)
        from oracle import oracle as O
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world)
        R, C, ty = 256, 2048, 12
        G = C // 256
        W = O.gen_matrix(R, C, ty, 0, 41)                                   # GGUF row-major bytes
        blocks = np.frombuffer(bytes(W), np.uint8).reshape(R, G, O.BLOCK[ty])
        x = O.gen_normal(C, 0.0, 1.0, 1, 5)
        full = O.matvec(W, R, C, ty, x)
        # row-split matrix: this rank's input columns (whole super-blocks), partials all-reduced
        gl = G // world
        part = O.matvec(np.ascontiguousarray(blocks[:, rank * gl:(rank + 1) * gl]).reshape(-1), R, gl * 256, ty,
                        x[rank * gl * 256:(rank + 1) * gl * 256])
        t = torch.from_numpy(np.asarray(part, np.float32).copy())
        dist.all_reduce(t)
        err_sum = float(np.linalg.norm(t.numpy() - full) / np.linalg.norm(full))
        # column-split matrix: this rank's rows
        rl = R // world
        rows = O.matvec(np.ascontiguousarray(blocks[rank * rl:(rank + 1) * rl]).reshape(-1), rl, C, ty, x)
        rows_equal = bool(np.array_equal(np.asarray(rows, np.float32), np.asarray(full, np.float32)[rank * rl:(rank + 1) * rl]))
        # vocabulary-split argmax with a tie across the ranks' slices
        V = 1000
        z = np.random.default_rng(7).standard_normal(V).astype(np.float32)
        z[123] = z[777] = np.float32(9.0)
        vl = V // world
        sl = z[rank * vl:(rank + 1) * vl]
        loc = int(np.argmax(sl))
        vals = [torch.zeros(1) for _ in range(world)]
        ids = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(vals, torch.tensor([float(sl[loc])]))
        dist.all_gather(ids, torch.tensor([rank * vl + loc]))
        best_v, best_i = vals[0].item(), int(ids[0].item())
        for r in range(1, world):
            if vals[r].item() > best_v:
                best_v, best_i = vals[r].item(), int(ids[r].item())
        dist.destroy_process_group()
        q.put((rank, err_sum, rows_equal, best_i, int(np.argmax(z))))
    except Exception as ex:
        q.put((rank, repr(ex), None, None, None))


def test_tensor_parallel_decomposition_gloo():
    pytest.importorskip("torch")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
    for rank, err, rows_equal, best, ref in res:
        assert not isinstance(err, str), err
        assert err < 1e-6, (rank, err)
        assert rows_equal, rank
        assert best == ref == 123, (rank, best, ref)
