"""Tensor parallelism over one prompt on two GPUs: each rank (one process per GPU) runs the late-layer pass over its
value heads, attention kv heads and projector columns, the columns gathered into every rank's block inputs by the
library's NVLink peer kernels, and the same pass on one GPU over the same seeded inputs. The rank's results must be
its slices of the one-GPU pass's, bit for bit (the reference's rule for per-rank heads, tests/kernel_test.cpp:
1498-1577): every DeltaNet state and conv state, the decay sums, its attention caches, every layer's gathered block
input, the mask and the hazard record; and no bounded wait gave up. Two passes in a row, so the second runs on
counters the first advanced. Skipped with fewer than two GPUs."""
import os
import socket

import pytest

gpu = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape_kw, q):
    import sys
    import ctypes as C
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "radiance-ridgefill_b200"))
    import torch
    import torch.distributed as dist
    import late_pass as LP
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    out = {"rank": rank}
    try:
        team = LP.Team(world, rank, dist)
        shape = LP.LateShape(**shape_kw)
        dev = f"cuda:{rank}"
        tp = LP.LatePass(shape, dev, seed=3, team=team)
        one = LP.LatePass(shape, dev, seed=3)
        stream = torch.cuda.Stream(device=dev)
        for _ in range(2):
            tp.run(stream.cuda_stream)
            one.run(stream.cuda_stream)
        stream.synchronize()
        lib = team.lib
        lib.ridgefill_device_error.restype = C.c_int
        out["device_error"] = lib.ridgefill_device_error(1)
        (v0, v1), (k0, k1), (a0, a1) = tp.geo["v"], tp.geo["k"], tp.geo["a"]
        G, hv, hk, D = shape.n_gdn, shape.hv, shape.hk, shape.head
        heads_v = torch.cat([torch.arange(j * hv + v0, j * hv + v1) for j in range(G)]).to(dev)
        ch = torch.cat([torch.arange(k0 * D, k1 * D), torch.arange((hk + k0) * D, (hk + k1) * D),
                        torch.arange((2 * hk + v0) * D, (2 * hk + v1) * D)]).to(dev)
        checks = {
            "state": torch.equal(tp.state, one.state[:, heads_v]),
            "nd": torch.equal(tp.nd, one.nd[:, heads_v]),
            "applied": torch.equal(tp.applied, one.applied[:, heads_v]),
            "block_inputs": all(torch.equal(a, b) for a, b in zip(tp.x, one.x)),
            "conv_state": all(torch.equal(a, b[:, :, ch]) for a, b in zip(tp.conv_state, one.conv_state)),
            "caches": all(torch.equal(a, b[:, :, a0:a1]) for a, b in zip(tp.cache, one.cache)),
            "mask": torch.equal(tp.mask, one.mask) and torch.equal(tp.bounds, one.bounds),
            "hazard": torch.equal(tp.meta, one.meta) and torch.equal(tp.count, one.count),
        }
        out["checks"] = checks
        out["heads"] = (v0, v1, a0, a1)
        team.close()
    except Exception as e:   # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put(out)
    dist.barrier()
    dist.destroy_process_group()


@gpu
@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_ranks_hold_slices_of_the_one_gpu_pass(cuda, world):
    torch = cuda
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    shape_kw = dict(T=640, layers="GGAG", seqlens=(200, 440))
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape_kw, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for res in results:
        assert "error" not in res, res
        assert res["device_error"] == 0, res
        assert all(res["checks"].values()), res
    assert sorted(r["heads"][:2] for r in results) == [(0, 16), (16, 32)]
