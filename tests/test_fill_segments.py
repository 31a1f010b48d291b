"""The fill's state is affine in its start state, the property a segment-parallel fill rests on: for a sequence
split at row m, S_end = S_mid M + S_2, where S_mid is the rule over [0, m) from S_0, S_2 the rule over [m, n) from
zero, and M the rule over [m, n) from the identity with v = 0 (the product, in row order, of the rows' transitions
exp(g_t) (I - beta_t k_t k_t^T), acting on the k side of the [dv, dk] state). Checked on the oracle's f64
sequential rule (oracle/ridgefill_oracle.cpp), at a chunk boundary and inside a chunk."""
import numpy as np
import pytest

import harness as H


@pytest.mark.parametrize("m", [64, 128, 131])
def test_split_sequence_composes(m):
    T, hk, hv = 300, 2, 4
    _, k, v, g, beta, state = H.gdn_inputs(7, T, hk, hv, decay="very slow", slots=1)
    full, _ = H.oracle_gdn(k, v, g, beta, state, [0], [0, T])
    mid, _ = H.oracle_gdn(k[:m], v[:m], g[:m], beta[:m], state, [0], [0, m])
    s2, _ = H.oracle_gdn(k[m:], v[m:], g[m:], beta[m:], np.zeros_like(state), [0], [0, T - m])
    eye = np.broadcast_to(np.eye(128, dtype=np.float32), state.shape).copy()
    M, _ = H.oracle_gdn(k[m:], np.zeros_like(v[m:]), g[m:], beta[m:], eye, [0], [0, T - m])
    carried = np.einsum("hij,hjk->hik", mid[0].astype(np.float64), M[0].astype(np.float64))
    assert H.rel_l2(carried + s2[0], full[0]) <= 1e-5
    assert np.linalg.norm(carried) > 0.1 * np.linalg.norm(full[0])   # the carried part matters at this decay
