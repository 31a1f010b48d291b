"""The tensor-parallel split on the CPU: each rank's slices of the pass's weights put together in rank order are
the whole (projector columns, the DeltaNet channels of each rank's heads, its a|b rows, its attention kv rows), the
spans are the reference's (shard.head_span), and the attention kv heads go one to a rank while there are heads."""
import types

import pytest
import torch

import harness  # noqa: F401  (puts the package on the path)
import late_pass as LP
import shard


def _team(world, rank):
    return types.SimpleNamespace(world=world, rank=rank)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rank_slices_partition_the_weights(world):
    s = LP.LateShape(T=64, d=256, layers="GGA", hk=8, hv=16)
    x = LP.late_inputs(s, "cpu", 4)
    parts = [LP.local_inputs(s, x, _team(world, r)) for r in range(world)]
    D = s.head
    for li in range(len(s.layers)):
        assert torch.equal(torch.cat([p[0]["w_proj"][li] for p in parts]), x["w_proj"][li])
        assert torch.equal(torch.cat([p[0]["s_proj"][li] for p in parts], dim=1), x["s_proj"][li])
    spans = [p[1]["v"] for p in parts]
    assert spans == [shard.head_span(s.hk, s.hv, r, world)[0] for r in range(world)]
    assert [p[1]["cols"] for p in parts] == [(r * s.d // world, (r + 1) * s.d // world) for r in range(world)]
    for j in range(s.n_gdn):
        # every rank's mixed-projection rows are the q, k and v channels of its heads, in that order
        q = torch.cat([p[0]["w_in"][j][:(p[1]["k"][1] - p[1]["k"][0]) * D] for p in parts])
        assert torch.equal(q, x["w_in"][j][:s.hk * D])
        v_rows = torch.cat([p[0]["w_in"][j][2 * (p[1]["k"][1] - p[1]["k"][0]) * D:] for p in parts])
        assert torch.equal(v_rows, x["w_in"][j][2 * s.hk * D:])
        a_rows = torch.cat([p[0]["w_ab"][j][:p[1]["v"][1] - p[1]["v"][0]] for p in parts])
        assert torch.equal(a_rows, x["w_ab"][j][:s.hv])
    states = torch.cat([p[0]["state"].view(1, s.n_gdn, -1, D, D) for p in parts], dim=2).view(1, -1, D, D)
    assert torch.equal(states, x["state"])
    heads = [p[1]["a"] for p in parts]
    assert heads[:2] == [(0, 1), (1, 2)] and all(h == (0, 0) for h in heads[2:])


def test_a_split_that_leaves_ragged_blocks_is_refused():
    s = LP.LateShape(T=64, d=96, layers="G", hk=2, hv=4)
    x = LP.late_inputs(s, "cpu", 1)
    with pytest.raises(ValueError):
        LP.local_inputs(s, x, _team(4, 0))   # 24 columns a rank: not whole 16-column blocks
