"""ridgefill_gdn_fill_noalloc -- the DeltaNet fill for callers that cannot allocate device memory where
they launch it (an FFI host without a device allocator, an engine step whose memory is fixed before the
pass). It takes the row's operands without a workspace and uses the 64 MiB workspace compiled into the
library. Called here through the C ABI, twice in a row with different inputs (the shared workspace keeps
the first call's contents), each result checked against the ridgefill_gdn_fill row given an allocated
workspace, within the state tolerance the fill's tests use. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu
STATE_TOL = 1e-3


def _operands(torch, seed, T, hk, hv):
    q, k, v, g, beta, state = H.gdn_inputs(seed, T, hk, hv, "slow")
    t = {"k": torch.from_numpy(k.view(np.int16)).cuda(), "v": torch.from_numpy(v.view(np.int16)).cuda(),
         "g": torch.from_numpy(g).cuda(), "beta": torch.from_numpy(beta).cuda(),
         "idx": torch.tensor([1], dtype=torch.int32).cuda(), "cu": torch.tensor([0, T], dtype=torch.int32).cuda()}
    return t, state


def _tensors(t, S):
    return [abi.absent(), H.dev(t["k"], abi.BF16), H.dev(t["v"], abi.BF16), H.dev(t["g"]), H.dev(t["beta"]), H.dev(S),
            H.dev(t["idx"]), H.dev(t["cu"]), abi.absent()]


def _noalloc(lib, tensors, params, torch) -> int:
    fn = lib.lib.ridgefill_gdn_fill_noalloc
    fn.argtypes = [C.POINTER(abi.RadArgs), C.c_void_p]
    fn.restype = C.c_int
    args, keep = abi.Plugin.args(tensors, params)   # no scratch operand
    rc = fn(C.byref(args), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    del keep
    return rc


def test_noalloc_fill_matches_the_row_on_two_calls_in_a_row(cuda, product_lib):
    torch = cuda
    T, hk, hv = 1000, 2, 4
    params = H.gdn_params(T, hk, hv)
    for call, seed in enumerate((101, 202)):
        t, state = _operands(torch, seed, T, hk, hv)
        S_row = torch.from_numpy(state.copy()).cuda()
        S_na = torch.from_numpy(state.copy()).cuda()
        assert H.launch(product_lib, "ridgefill_gdn_fill", _tensors(t, S_row), params) == abi.OK
        assert _noalloc(product_lib, _tensors(t, S_na), params, torch) == abi.OK, f"call {call}"
        got, want = S_na.cpu().numpy(), S_row.cpu().numpy()
        assert H.rel_l2(got[1], want[1]) <= STATE_TOL, f"call {call}"
        assert np.array_equal(got[0], state[0]) and np.array_equal(got[2], state[2])


def test_noalloc_refuses_past_its_workspace(cuda, product_lib):
    """A call whose workspace would exceed 64 MiB is refused with RAD_E_SHAPE before any launch (its
    state is left alone)."""
    torch = cuda
    T, hk, hv = 8192, 16, 32          # 129 chunk slots x 32 heads x 49,680 B = 205.1 MB > 64 MiB
    t, state = _operands(torch, 7, T, hk, hv)
    S = torch.from_numpy(state.copy()).cuda()
    assert _noalloc(product_lib, _tensors(t, S), H.gdn_params(T, hk, hv), torch) == abi.E_SHAPE
    assert np.array_equal(S.cpu().numpy(), state)
