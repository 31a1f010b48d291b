"""The bench's pass (radiance-ridgefill_b200/ridgefill_step.py) issued on two streams -- Step.run_pipelined: the
projector path from the top of the pass and select after the mask on one, mask, undo, fill, rho, apply and the
hazard record on the other -- writes every buffer bit for bit as the same pass issued in order on one stream
(Step.run), over three consecutive passes that carry the state, ND, the applied correction and the hazard record
from pass to pass, at 4,096 rows of the bench's shapes."""
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "radiance-ridgefill_b200"))

OUTPUTS = ("codes", "a_scale", "x_proj", "x", "mask", "bounds", "state", "applied", "nd", "meta", "count")
SEEDED = ("h_s", "w", "k", "v", "g", "beta", "ab", "x", "state", "C", "nd", "applied", "meta")   # the rest start empty


def test_pipelined_pass_equals_the_ordered_pass(cuda, product_lib):
    torch = cuda
    import ridgefill_step as RS
    ordered = RS.Step(RS.StepShape(T=4096), seed=5)
    piped = RS.Step(RS.StepShape(T=4096), seed=5)
    for name in SEEDED:
        assert torch.equal(getattr(ordered, name), getattr(piped, name)), f"{name}: seeded inputs differ"
    main = torch.cuda.Stream(priority=-1)
    side = torch.cuda.Stream(priority=0)
    for _ in range(3):
        ordered.run(main.cuda_stream)
        piped.run_pipelined(main, side)
    torch.cuda.synchronize()
    assert int(ordered.mask.sum()) > 0   # the pass approximates rows, so select and rho have work
    for name in OUTPUTS:
        assert torch.equal(getattr(ordered, name), getattr(piped, name)), name
