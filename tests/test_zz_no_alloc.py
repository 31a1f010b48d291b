"""ridgefill_gdn_fill_noalloc -- the DeltaNet fill for callers that cannot allocate device memory where
they launch it (an FFI host without a device allocator, an engine step whose memory is fixed before the
pass). It takes the row's operands without a workspace and uses the 64 MiB workspace compiled into the
library. Called here through the C ABI three times in a row with different shapes (the shared workspace
keeps the previous call's contents, laid out for another shape): one 1,000-row sequence with the state
alone; two sequences of 300 and 400 rows over other heads with the output o; the first shape again. Each
result is checked against the ridgefill_gdn_fill row given an allocated workspace: the same kernels on the
same inputs, so the state and o must be bit for bit the same. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu


def _operands(torch, seed, T, hk, hv, cu, idx, with_o):
    q, k, v, g, beta, state = H.gdn_inputs(seed, T, hk, hv, "slow")
    t = {"k": torch.from_numpy(k.view(np.int16)).cuda(), "v": torch.from_numpy(v.view(np.int16)).cuda(),
         "g": torch.from_numpy(g).cuda(), "beta": torch.from_numpy(beta).cuda(),
         "idx": torch.tensor(idx, dtype=torch.int32).cuda(), "cu": torch.tensor(cu, dtype=torch.int32).cuda(),
         "q": torch.from_numpy(q.view(np.int16)).cuda() if with_o else None}
    return t, state


def _tensors(t, S, O):
    return [H.dev(t["q"], abi.BF16), H.dev(t["k"], abi.BF16), H.dev(t["v"], abi.BF16), H.dev(t["g"]), H.dev(t["beta"]),
            H.dev(S), H.dev(t["idx"]), H.dev(t["cu"]), H.dev(O, abi.BF16)]


def _noalloc(lib, tensors, params, torch) -> int:
    fn = lib.lib.ridgefill_gdn_fill_noalloc
    fn.argtypes = [C.POINTER(abi.RadArgs), C.c_void_p]
    fn.restype = C.c_int
    args, keep = abi.Plugin.args(tensors, params)   # no scratch operand
    rc = fn(C.byref(args), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    del keep
    return rc


CALLS = [   # (seed, T, hk, hv, cu_seqlens, state slots, output o)
    (101, 1000, 2, 4, [0, 1000], [1], False),
    (202, 700, 4, 8, [0, 300, 700], [2, 0], True),
    (303, 1000, 2, 4, [0, 1000], [1], False),
]


def test_noalloc_fill_matches_the_row_on_calls_in_a_row(cuda, product_lib):
    torch = cuda
    for call, (seed, T, hk, hv, cu, idx, with_o) in enumerate(CALLS):
        params = H.gdn_params(T, hk, hv)
        t, state = _operands(torch, seed, T, hk, hv, cu, idx, with_o)
        S_row, S_na = torch.from_numpy(state.copy()).cuda(), torch.from_numpy(state.copy()).cuda()
        O_row = torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda") if with_o else None
        O_na = torch.full((T, hv, 128), 0x7FC1, dtype=torch.int16, device="cuda") if with_o else None
        assert H.launch(product_lib, "ridgefill_gdn_fill", _tensors(t, S_row, O_row), params) == abi.OK
        assert _noalloc(product_lib, _tensors(t, S_na, O_na), params, torch) == abi.OK, f"call {call}"
        assert torch.equal(S_na, S_row), f"call {call}: state"
        if with_o:
            assert torch.equal(O_na, O_row), f"call {call}: o"
        untouched = [s for s in range(state.shape[0]) if s not in idx]
        got = S_na.cpu().numpy()
        assert all(np.array_equal(got[s], state[s]) for s in untouched)


def test_noalloc_refuses_past_its_workspace(cuda, product_lib):
    """A call whose workspace would exceed 64 MiB is refused with RAD_E_SHAPE before any launch (its state is
    left alone): 8,192 rows at 32 heads, and 2,048 rows at 20 heads with o (the output form's limit is 19)."""
    torch = cuda
    for T, hk, hv, with_o in ((8192, 16, 32, False), (2048, 4, 20, True)):
        t, state = _operands(torch, 7, T, hk, hv, [0, T], [1], with_o)
        S = torch.from_numpy(state.copy()).cuda()
        O = torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda") if with_o else None
        assert _noalloc(product_lib, _tensors(t, S, O), H.gdn_params(T, hk, hv), torch) == abi.E_SHAPE
        assert np.array_equal(S.cpu().numpy(), state)


def test_noalloc_fits_its_stated_limits(cuda, product_lib):
    """The stated limits fit: one 2,048-row sequence at 40 value heads (state alone) and at 19 with o."""
    torch = cuda
    for T, hk, hv, with_o in ((2048, 8, 40, False), (2048, 1, 19, True)):
        t, state = _operands(torch, 9, T, hk, hv, [0, T], [1], with_o)
        S = torch.from_numpy(state.copy()).cuda()
        O = torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda") if with_o else None
        assert _noalloc(product_lib, _tensors(t, S, O), H.gdn_params(T, hk, hv), torch) == abi.OK
