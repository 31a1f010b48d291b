"""More than one rank, on the CPU: the head spans of tensor parallelism (the reference's rule,
tests/kernel_test.cpp:1458-1466) and, over two gloo ranks, that each rank's fill over its own span of heads
(views of the operands) is byte for byte its slice of the one-rank fill, and that the bench's job time is
the slowest rank's. The oracle computes; the device rows' own slice test is in test_gdn_device.py."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

import harness as H

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "radiance-ridgefill_b200"))
import shard  # noqa: E402


@pytest.mark.parametrize("hk,hv,world,want", [
    (16, 48, 1, [(0, 48)]),
    (16, 48, 2, [(0, 24), (24, 48)]),
    (16, 48, 3, [(18, 33), (33, 48), (0, 18)]),   # kernel_test.cpp:1462-1463
    (16, 48, 4, [(0, 12), (12, 24), (24, 36), (36, 48)]),
    (16, 32, 2, [(0, 16), (16, 32)]),
    (4, 8, 3, [(4, 6), (6, 8), (0, 4)]),
])
def test_head_spans(hk, hv, world, want):
    spans = [shard.head_span(hk, hv, r, world) for r in range(world)]
    assert [v for v, _ in spans] == want
    covered = sorted(x for (v0, v1), _ in spans for x in range(v0, v1))
    assert covered == list(range(hv))
    for (v0, v1), (k0, k1) in spans:   # the span's k heads are exactly the ones its v heads read
        assert v0 == k0 * (hv // hk) and v1 == k1 * (hv // hk)


def test_head_span_refusals():
    with pytest.raises(ValueError):
        shard.head_span(3, 8, 0, 2)
    with pytest.raises(ValueError):
        shard.head_span(2, 4, 0, 3)
    with pytest.raises(ValueError):
        shard.head_span(4, 8, 2, 2)


def test_max_over_ranks_without_a_group():
    assert shard.max_over_ranks([1.5, 2]) == [1.5, 2.0]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        T, hk, hv = 130, 4, 8
        q, k, v, g, beta, state = H.gdn_inputs(77, T, hk, hv, "fast", slots=2)
        idx, cu = [1], [0, T]
        (v0, v1), (k0, k1) = shard.head_span(hk, hv, rank, world)
        # this rank's views: its k heads, its v heads, its heads of g, beta and the state
        mine, o = H.oracle_gdn(k[:, k0:k1], v[:, v0:v1], g[:, v0:v1], beta[:, v0:v1], state[:, v0:v1], idx, cu,
                               q=q[:, k0:k1])
        np.save(os.path.join(out_dir, f"state{rank}.npy"), mine)
        np.save(os.path.join(out_dir, f"o{rank}.npy"), o)
        np.save(os.path.join(out_dir, f"span{rank}.npy"), np.array([v0, v1]))
        slow = shard.max_over_ranks([1.0 + rank, 10.0 - rank], dist)
        np.save(os.path.join(out_dir, f"max{rank}.npy"), np.array(slow))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_fill_their_slices_of_one_rank(tmp_path):
    import torch.multiprocessing as mp
    H.oracle()   # built here, loaded by each rank
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    T, hk, hv = 130, 4, 8
    q, k, v, g, beta, state = H.gdn_inputs(77, T, hk, hv, "fast", slots=2)
    full, full_o = H.oracle_gdn(k, v, g, beta, state, [1], [0, T], q=q)
    for r in range(world):
        v0, v1 = np.load(tmp_path / f"span{r}.npy")
        part, part_o = np.load(tmp_path / f"state{r}.npy"), np.load(tmp_path / f"o{r}.npy")
        assert np.array_equal(part.view(np.uint32), full[:, v0:v1].view(np.uint32))
        assert np.array_equal(part_o, full_o[:, v0:v1])
        assert list(np.load(tmp_path / f"max{r}.npy")) == [2.0, 10.0]
