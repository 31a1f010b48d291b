"""How the RidgeFill pass spreads over GPUs (one process per GPU).

Two forms, both without a collective on the data path:

* independent prompts (the bench's form): every rank runs the whole pass over its own chunk; the job's
  throughput is the rows of all ranks over the slowest rank's time (`max_over_ranks`).
* tensor parallelism over value heads (the reference's form): the DeltaNet fill, the state correction, the
  state read and the decay sums are per value head, and a rank holds a contiguous span of heads with the
  k-heads they read (`head_span`). A rank's launches take views of the full operands over its span; each
  head is computed as at TP1, so the ranks' results are byte for byte the slices of the TP1 result.

The span rule is the reference's (tests/kernel_test.cpp:1458-1466, ridgefill_projector.h plan_rank): even
worlds give rank r heads [r H / W, (r + 1) H / W); at TP3 the K heads split as evenly as they go with the
remainder to the last rank first (radiance's remainder placement: 16 K heads -> 5 / 5 / 6), and the spans
run from the last rank: with 48 value heads ranks 0 / 1 / 2 hold [18, 33), [33, 48), [0, 18).
"""
from __future__ import annotations


def k_head_counts(n_head_k: int, world: int) -> list[int]:
    """K heads per rank: n_head_k / world each, the remainder one each to the last ranks."""
    if world <= 0 or n_head_k < world:
        raise ValueError(f"{n_head_k} k-heads over {world} ranks")
    base, extra = divmod(n_head_k, world)
    return [base + (1 if r >= world - extra else 0) for r in range(world)]


def head_span(n_head_k: int, n_head_v: int, rank: int, world: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """(v0, v1), (k0, k1): the value heads and the k heads rank `rank` of `world` holds.

    Even divisions are rank-ordered; an uneven one places the ranks holding the extra head first in head
    order (the remainder ranks take the lowest heads), the others after them in rank order."""
    if n_head_v % n_head_k:
        raise ValueError("value heads must be a multiple of k heads")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    per_v = n_head_v // n_head_k
    counts = k_head_counts(n_head_k, world)
    extra = n_head_k % world
    order = list(range(world - extra, world)) + list(range(world - extra)) if extra else list(range(world))
    k0 = 0
    for r in order:
        if r == rank:
            return (k0 * per_v, (k0 + counts[r]) * per_v), (k0, k0 + counts[r])
        k0 += counts[r]
    raise AssertionError("unreachable")


def max_over_ranks(values, dist=None):
    """The elementwise maximum of a list of floats over the process group (the job's time is its slowest
    rank's); the values themselves without a group. Every rank calls it at the same point."""
    vals = [float(v) for v in values]
    if dist is None or not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return vals
    import torch
    backend = dist.get_backend()
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
