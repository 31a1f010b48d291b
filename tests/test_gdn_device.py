"""ridgefill_gdn_fill on B200 against the sequential gated delta rule in float64 (the oracle): the final
state within 1e-3 relative L2 (the tolerance the task states for the fp32 DeltaNet state), untouched
slots and skipped sequences bit for bit, and at the full 32,768-row configuration the size-independent
property that splitting a sequence at a chunk boundary (two calls, the state carried) is the same
arithmetic as one call, bit for bit."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu
STATE_TOL = 1e-3
O_TOL = 1e-2   # o is bf16; relative L2 over every written row and head


def run_fill(product_lib, torch, k, v, g, beta, state, idx, cu, hk, hv, q=None, o=False):
    T = k.shape[0]
    K = torch.from_numpy(k.view(np.int16)).cuda()
    V = torch.from_numpy(v.view(np.int16)).cuda()
    G, BT = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda()
    S = torch.from_numpy(state.copy()).cuda()
    I = torch.tensor(np.asarray(idx, np.int32)).cuda()
    CU = torch.tensor(np.asarray(cu, np.int32)).cuda()
    Q = torch.from_numpy(q.view(np.int16)).cuda() if q is not None else None
    O = torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda") if o else None
    rc = H.launch(product_lib, "ridgefill_gdn_fill",
                  [H.dev(Q, abi.BF16), H.dev(K, abi.BF16), H.dev(V, abi.BF16), H.dev(G), H.dev(BT), H.dev(S), H.dev(I),
                   H.dev(CU), H.dev(O, abi.BF16)], H.gdn_params(T, hk, hv))
    return rc, S.cpu().numpy(), (O.cpu().numpy().view(np.uint16) if o else None)


@pytest.mark.parametrize("T,hk,hv,decay", [(64, 1, 1, "fast"), (130, 2, 4, "fast"), (1000, 2, 4, "slow"),
                                           (777, 1, 2, "very slow"), (2048, 16, 32, "fast")])
def test_fill_state_matches_sequential_rule(cuda, product_lib, T, hk, hv, decay):
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(T + hv, T, hk, hv, decay)
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, [1], [0, T], hk, hv)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, [1], [0, T])
    err = H.rel_l2(got[1], want[1])
    assert err <= STATE_TOL, err
    assert np.array_equal(got[0], state[0]) and np.array_equal(got[2], state[2])   # other slots untouched


def test_fill_varlen_sequences_and_skipped_slots(cuda, product_lib):
    """Three sequences of 1, 100 and 300 rows (chunks anchored at each start), the second with no state
    (slot -1: skipped, its rows read by nobody), slots in reverse order."""
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(5, 401, 2, 4, "slow", slots=4)
    cu, idx = [0, 1, 101, 401], [3, -1, 0]
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, idx, cu, 2, 4)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, idx, cu)
    for slot in (3, 0):
        assert H.rel_l2(got[slot], want[slot]) <= STATE_TOL
    assert np.array_equal(got[1], state[1]) and np.array_equal(got[2], state[2])


def test_fill_empty_sequence_keeps_state(cuda, product_lib):
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(6, 64, 1, 2, "fast")
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, [2, 1], [0, 0, 64], 1, 2)
    assert rc == abi.OK and np.array_equal(got[2], state[2])
    want, _ = H.oracle_gdn(k, v, g, beta, state, [2, 1], [0, 0, 64])
    assert H.rel_l2(got[1], want[1]) <= STATE_TOL


def test_fill_full_size_split_is_one_call(cuda, product_lib):
    """The single-layer fill at full size: T = 32,768, 16 q/k heads, 32 v heads. Two calls over [0, T/2) and [T/2, T)
    with the state carried equal one call over [0, T) bit for bit (chunks are anchored at the call's
    sequence start and T/2 is a chunk boundary); two heads checked against the float64 rule."""
    torch = cuda
    T, hk, hv = 32768, 16, 32
    q, k, v, g, beta, state = H.gdn_inputs(32, T, hk, hv, "fast", slots=1)
    rc, one, _ = run_fill(product_lib, torch, k, v, g, beta, state, [0], [0, T], hk, hv)
    assert rc == abi.OK
    h = T // 2
    rc1, mid, _ = run_fill(product_lib, torch, k[:h], v[:h], g[:h], beta[:h], state, [0], [0, h], hk, hv)
    rc2, two, _ = run_fill(product_lib, torch, k[h:], v[h:], g[h:], beta[h:], mid, [0], [0, T - h], hk, hv)
    assert rc1 == rc2 == abi.OK
    assert np.array_equal(one.view(np.uint32), two.view(np.uint32))
    want, _ = H.oracle_gdn(k, v, g, beta, state, [0], [0, T], heads=(5, 7))
    assert H.rel_l2(one[0, 5:7], want[0, 5:7]) <= STATE_TOL
    # every head against the float32 rule (the f64 one takes minutes at this size); per head, the same bound
    want32, _ = H.oracle_gdn(k, v, g, beta, state, [0], [0, T], f64=False)
    errs = [H.rel_l2(one[0, h], want32[0, h]) for h in range(hv)]
    assert max(errs) <= STATE_TOL, errs


@pytest.mark.parametrize("T,hk,hv,dk,o", [(512, 4, 8, 32, False), (300, 2, 4, 32, True), (200, 1, 3, 64, True),
                                          (129, 2, 2, 16, False)])
def test_small_heads_follow_the_rule(cuda, product_lib, T, hk, hv, dk, o):
    """Head dims of at most 64 (the reference's CPU mini model has 32) run the per-row form: state within the
    same 1e-3 relative L2 of the float64 rule, o within 1e-2, over two sequences with one slot skipped."""
    torch = cuda
    rng = np.random.default_rng(T + dk)
    k = rng.standard_normal((T, hk, dk)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q = rng.standard_normal((T, hk, dk)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((T, hv, dk)).astype(np.float32)
    g = -np.log1p(np.exp(rng.standard_normal((T, hv)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, hv))))).astype(np.float32)
    state = (0.1 * rng.standard_normal((3, hv, dk, dk))).astype(np.float32)
    kb, vb, qb = H.f32_to_bf16_bits(k), H.f32_to_bf16_bits(v), H.f32_to_bf16_bits(q)
    cu, idx = [0, T // 3, T], [2, -1]
    S = torch.from_numpy(state.copy()).cuda()
    O = torch.zeros((T, hv, dk), dtype=torch.int16, device="cuda") if o else None
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    Kd, Vd, Qd = t16(kb), t16(vb), (t16(qb) if o else None)
    G, B = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda()
    I, CU = torch.tensor(idx, dtype=torch.int32).cuda(), torch.tensor(cu, dtype=torch.int32).cuda()
    params = [H.pint("M", T), H.pint("n_head_k", hk), H.pint("n_head_v", hv), H.pint("head_k", dk), H.pint("head_v", dk),
              H.pint("chunk", 64)]
    assert H.launch(product_lib, "ridgefill_gdn_fill", [H.dev(Qd, abi.BF16), H.dev(Kd, abi.BF16), H.dev(Vd, abi.BF16), H.dev(G),
                                                        H.dev(B), H.dev(S), H.dev(I), H.dev(CU), H.dev(O, abi.BF16)],
                    params) == abi.OK
    want, want_o = H.oracle_gdn(kb, vb, g, beta, state, idx, cu, q=qb if o else None)
    got = S.cpu().numpy()
    assert H.rel_l2(got[2], want[2]) <= STATE_TOL
    assert np.array_equal(got[0], state[0]) and np.array_equal(got[1], state[1])
    if o:
        got_o = O.cpu().numpy().view(np.uint16)
        assert not got_o[T // 3:].any()   # the skipped sequence's rows are left as they were
        rows = slice(0, T // 3)
        assert H.rel_l2(H.bf16_bits_to_f32(got_o[rows]), H.bf16_bits_to_f32(want_o[rows])) <= O_TOL


@pytest.mark.parametrize("T,hk,hv,decay", [(64, 1, 1, "fast"), (130, 2, 4, "slow"), (777, 1, 2, "very slow"),
                                           (2048, 16, 32, "fast")])
def test_fill_output_matches_sequential_rule(cuda, product_lib, T, hk, hv, decay):
    """The output form: o_t = scale * S_t q_t for every row (scale 1/sqrt(128)), and the same state."""
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(T + 3 * hv, T, hk, hv, decay)
    rc, got, o = run_fill(product_lib, torch, k, v, g, beta, state, [1], [0, T], hk, hv, q=q, o=True)
    assert rc == abi.OK
    want, want_o = H.oracle_gdn(k, v, g, beta, state, [1], [0, T], q=q)
    assert H.rel_l2(got[1], want[1]) <= STATE_TOL
    err = H.rel_l2(H.bf16_bits_to_f32(o), H.bf16_bits_to_f32(want_o))
    assert err <= O_TOL, err


def test_fill_output_varlen_and_skipped(cuda, product_lib):
    """Output form over three sequences (1, 100 and 300 rows), the second without a state slot: its o rows
    are left as they were (zero here), the others match the rule."""
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(9, 401, 2, 4, "fast", slots=4)
    cu, idx = [0, 1, 101, 401], [3, -1, 0]
    rc, got, o = run_fill(product_lib, torch, k, v, g, beta, state, idx, cu, 2, 4, q=q, o=True)
    assert rc == abi.OK
    want, want_o = H.oracle_gdn(k, v, g, beta, state, idx, cu, q=q)
    assert not o[1:101].any()
    for r0, r1 in ((0, 1), (101, 401)):
        assert H.rel_l2(H.bf16_bits_to_f32(o[r0:r1]), H.bf16_bits_to_f32(want_o[r0:r1])) <= O_TOL
    for slot in (3, 0):
        assert H.rel_l2(got[slot], want[slot]) <= STATE_TOL


@pytest.mark.parametrize("with_o", [False, True])
def test_fill_head_spans_are_slices_of_one_call(cuda, product_lib, with_o):
    """Tensor parallelism over value heads (shard.head_span, the reference's spans, uneven at TP3): each rank's
    call over views of its heads writes, byte for byte, its slice of the one-rank call's state (and o)."""
    import shard
    torch = cuda
    T, hk, hv = 700, 16, 48
    q, k, v, g, beta, state = H.gdn_inputs(11, T, hk, hv, "fast", slots=2)
    K = torch.from_numpy(k.view(np.int16)).cuda()
    V = torch.from_numpy(v.view(np.int16)).cuda()
    Q = torch.from_numpy(q.view(np.int16)).cuda()
    G, BT = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda()
    I, CU = torch.tensor([1], dtype=torch.int32).cuda(), torch.tensor([0, T], dtype=torch.int32).cuda()

    def call(S, O, ks, vs):
        ops = [H.dev(Q[:, ks], abi.BF16) if with_o else abi.absent(), H.dev(K[:, ks], abi.BF16), H.dev(V[:, vs], abi.BF16),
               H.dev(G[:, vs]), H.dev(BT[:, vs]), H.dev(S[:, vs]), H.dev(I), H.dev(CU),
               H.dev(O[:, vs], abi.BF16) if with_o else abi.absent()]
        return H.launch(product_lib, "ridgefill_gdn_fill", ops, H.gdn_params(T, ks.stop - ks.start, vs.stop - vs.start))

    S1, O1 = torch.from_numpy(state.copy()).cuda(), torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda")
    assert call(S1, O1, slice(0, hk), slice(0, hv)) == abi.OK
    for world in (2, 3):
        S, O = torch.from_numpy(state.copy()).cuda(), torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda")
        for r in range(world):
            (v0, v1), (k0, k1) = shard.head_span(hk, hv, r, world)
            assert call(S, O, slice(k0, k1), slice(v0, v1)) == abi.OK
        assert torch.equal(S.view(torch.int32), S1.view(torch.int32)), world
        assert torch.equal(O, O1), world


def test_fill_refusals(cuda, product_lib):
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(7, 64, 1, 2, "fast")
    K = torch.from_numpy(k.view(np.int16)).cuda()
    V = torch.from_numpy(v.view(np.int16)).cuda()
    G, BT, S = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda(), torch.from_numpy(state).cuda()
    I, CU = torch.tensor([1], dtype=torch.int32).cuda(), torch.tensor([0, 64], dtype=torch.int32).cuda()
    ops = [abi.absent(), H.dev(K, abi.BF16), H.dev(V, abi.BF16), H.dev(G), H.dev(BT), H.dev(S), H.dev(I), H.dev(CU), abi.absent()]
    assert H.launch(product_lib, "ridgefill_gdn_fill", ops, H.gdn_params(64, 1, 2)) == abi.OK
    assert H.launch(product_lib, "ridgefill_gdn_fill", ops, H.gdn_params(64, 1, 2), scratch_bytes=0) == abi.E_INVAL
    p = H.gdn_params(64, 1, 2)
    p[5] = H.pint("chunk", 32)
    assert H.launch(product_lib, "ridgefill_gdn_fill", ops, p) == abi.E_UNSUPPORTED
    bad = list(ops)
    bad[3] = H.dev(G.to(torch.bfloat16))
    assert H.launch(product_lib, "ridgefill_gdn_fill", bad, H.gdn_params(64, 1, 2)) == abi.E_DTYPE
    bad = list(ops)
    bad[0] = H.dev(K, abi.BF16)   # q without o
    assert H.launch(product_lib, "ridgefill_gdn_fill", bad, H.gdn_params(64, 1, 2)) == abi.E_INVAL


def test_waits_give_up_and_the_context_survives(cuda, product_lib):
    """Failure detection without a fault: the library's two waits, run against a barrier phase and a flag
    that nothing completes, give up after their limit with the fill's error code, and the same context then
    runs a fill correctly."""
    import ctypes
    torch = cuda
    lib = product_lib.lib
    lib.ridgefill_device_error(1)   # clear
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.full((2,), 7, dtype=torch.int32, device="cuda")
    fn = lib.ridgefill_wait_selftest
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    assert fn(flag.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream) == abi.OK
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    assert lib.ridgefill_device_error(1) == 0x201
    assert lib.ridgefill_device_error(0) == 0
    q, k, v, g, beta, state = H.gdn_inputs(3, 300, 2, 4, "fast")
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, [1], [0, 300], 2, 4)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, [1], [0, 300])
    assert H.rel_l2(got[1], want[1]) <= STATE_TOL


def test_fill_state_is_affine_in_its_start(cuda, product_lib):
    """The segment composition on the device, in one varlen call of three sequences: rows [0, m) from S_0, rows
    [m, n) from zero, and rows [m, n) again with v = 0 from the identity (its end state is the segment's transition
    M). S_mid M + S_2 equals the one-sequence call's end state, and the f64 rule's, within 3e-3 relative L2 (three
    fills' 1e-3 bounds composed)."""
    torch = cuda
    n, m, hk, hv = 300, 131, 2, 4
    _, k, v, g, beta, state = H.gdn_inputs(41, n, hk, hv, decay="very slow", slots=1)
    rows = np.r_[0:n, m:n]
    v3 = v[rows].copy()
    v3[n:] = 0
    st3 = np.zeros((3, hv, 128, 128), np.float32)
    st3[0] = state[0]
    st3[2] = np.eye(128, dtype=np.float32)
    rc, got3, _ = run_fill(product_lib, torch, k[rows], v3, g[rows], beta[rows], st3, [0, 1, 2], [0, m, n, 2 * n - m], hk, hv)
    assert rc == abi.OK
    composed = np.einsum("hij,hjk->hik", got3[0].astype(np.float64), got3[2].astype(np.float64)) + got3[1]
    rc, full, _ = run_fill(product_lib, torch, k, v, g, beta, state, [0], [0, n], hk, hv)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, [0], [0, n])
    assert H.rel_l2(composed, full[0]) <= 3e-3
    assert H.rel_l2(composed, want[0]) <= 3e-3


# ------------------------------------------------------------------ the per-head form (>= 64 chains, state only)
# A state-only call of at least 64 chains (v-heads x sequences) runs one CTA a head, the transform beside the chain
# in each CTA; the tests above stay below that and exercise the cooperative form.

@pytest.mark.parametrize("T,hk,hv,decay", [(600, 16, 64, "fast"), (333, 32, 64, "slow"), (1100, 8, 96, "very slow")])
def test_head_form_matches_sequential_rule(cuda, product_lib, T, hk, hv, decay):
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(T + hv + 1, T, hk, hv, decay)
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, [1], [0, T], hk, hv)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, [1], [0, T])
    errs = [H.rel_l2(got[1, h], want[1, h]) for h in range(hv)]
    assert max(errs) <= STATE_TOL, max(errs)
    assert np.array_equal(got[0], state[0]) and np.array_equal(got[2], state[2])


def test_head_form_varlen_sequences_and_skipped_slots(cuda, product_lib):
    """Four sequences of 1, 100, 300 and 64 rows over 24 v-heads (96 chains): chunks anchored at each start, the
    second sequence with no state (slot -1) and the last with a slot outside the pool, both skipped."""
    torch = cuda
    q, k, v, g, beta, state = H.gdn_inputs(15, 465, 6, 24, "slow", slots=4)
    cu, idx = [0, 1, 101, 401, 465], [3, -1, 0, 9]
    rc, got, _ = run_fill(product_lib, torch, k, v, g, beta, state, idx, cu, 6, 24)
    assert rc == abi.OK
    want, _ = H.oracle_gdn(k, v, g, beta, state, idx, cu)
    for slot in (3, 0):
        assert H.rel_l2(got[slot], want[slot]) <= STATE_TOL
    assert np.array_equal(got[1], state[1]) and np.array_equal(got[2], state[2])


def test_head_form_agrees_with_the_cooperative_form(cuda, product_lib):
    """The same 64 v-heads over 2,000 rows: one call (the per-head form) against four calls of 16 heads each (the
    cooperative form), every head within the state tolerance of the other form."""
    torch = cuda
    T, hk, hv = 2000, 32, 64
    q, k, v, g, beta, state = H.gdn_inputs(23, T, hk, hv, "fast", slots=1)
    rc, one, _ = run_fill(product_lib, torch, k, v, g, beta, state, [0], [0, T], hk, hv)
    assert rc == abi.OK
    per = hv // 4
    parts = []
    for p in range(4):
        hs, ks = slice(p * per, (p + 1) * per), slice(p * per // 2, (p + 1) * per // 2)
        rc, got, _ = run_fill(product_lib, torch, np.ascontiguousarray(k[:, ks]), np.ascontiguousarray(v[:, hs]),
                              np.ascontiguousarray(g[:, hs]), np.ascontiguousarray(beta[:, hs]),
                              np.ascontiguousarray(state[:, hs]), [0], [0, T], per // 2, per)
        assert rc == abi.OK
        parts.append(got[0])
    coop = np.concatenate(parts, axis=0)
    errs = [H.rel_l2(one[0, h], coop[h]) for h in range(hv)]
    assert max(errs) <= STATE_TOL, max(errs)


def test_head_form_full_size_split_is_one_call(cuda, product_lib):
    """32,768 rows over 64 v-heads: two calls over [0, T/2) and [T/2, T) with the state carried equal one call bit
    for bit; four heads against the float32 rule."""
    torch = cuda
    T, hk, hv = 32768, 32, 64
    q, k, v, g, beta, state = H.gdn_inputs(33, T, hk, hv, "fast", slots=1)
    rc, one, _ = run_fill(product_lib, torch, k, v, g, beta, state, [0], [0, T], hk, hv)
    assert rc == abi.OK
    h = T // 2
    rc1, mid, _ = run_fill(product_lib, torch, k[:h], v[:h], g[:h], beta[:h], state, [0], [0, h], hk, hv)
    rc2, two, _ = run_fill(product_lib, torch, k[h:], v[h:], g[h:], beta[h:], mid, [0], [0, T - h], hk, hv)
    assert rc1 == rc2 == abi.OK
    assert np.array_equal(one.view(np.uint32), two.view(np.uint32))
    for h0 in (0, 21, 42, 63):
        want32, _ = H.oracle_gdn(k, v, g, beta, state, [0], [0, T], f64=False, heads=(h0, h0 + 1))
        assert H.rel_l2(one[0, h0], want32[0, h0]) <= STATE_TOL

