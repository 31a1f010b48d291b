"""The reference's split scan of the last prefill sequence, issued as one sequence of device rows
(arch/qwen4exp_blocks.h:137-157, STRADDLE_SPLIT): the scan over [s, b') (the fill with bounds[0:2] as its
cu_seqlens), the decay sums over the same rows (ridgefill_rho_update, M = b'), the correction applied
(ridgefill_state_correct apply with the N|D pool), then the scan over [b', e) (bounds[2:4]) from the corrected
state. Checked against the same sequence on the host: the fill's float64 sequential rule (the oracle) and the host
rows of rho and the correction, on the same seeded inputs:

    decay sums N, D          1e-4 relative (the reference's bound), rho = clamp(N/D, 0, 1) within 1e-5
    applied scale            1e-5 relative
    final state              1e-3 relative L2 (the fill's bound)

and, with alpha = 0 (the apply adds nothing), the split sequence's final state bit for bit equal to one fill over
[s, e): the split point b' - s is a multiple of the 64-row chunk, so both cut the rows into the same chunks.
Shapes: 4 v-heads (the cooperative fill) and 64 v-heads (the per-head fill), a sequence starting at row 0 and one
starting at row 40."""
import numpy as np
import pytest

import harness as H
from harness import Buf, abi, pint, pstr, pf64
from test_gdn_device import run_fill

pytestmark = pytest.mark.gpu
SLOTS, SLOT, D = 3, 1, 128


def _inputs(seed, T, hk, hv):
    q, k, v, g, beta, state = H.gdn_inputs(seed, T, hk, hv, slots=SLOTS)
    r = np.random.default_rng(seed + 1)
    a = H.f32_to_bf16_bits((2.0 * r.standard_normal((T, hv))).astype(np.float32))
    mask = (r.uniform(size=T) >= 0.3).astype(np.int32)   # 30 % of the rows exact
    a_log = (-4.0 + 6.5 * r.uniform(size=hv)).astype(np.float32)
    dt_bias = (-3.0 + 4.0 * r.uniform(size=hv)).astype(np.float32)
    C = (0.01 * r.standard_normal((hv, D, D))).astype(np.float32)
    return k, v, g, beta, state, a, mask, a_log, dt_bias, C


def _split_sequence(lib, domain, fill, inp, bounds, alpha):
    """fill [s, b'), rho over [s, b'), apply, fill [b', e): the final state, the N|D pool and the applied scales."""
    k, v, g, beta, state, a, mask, a_log, dt_bias, C = inp
    T, hv = a.shape
    s, b, _, e = bounds
    st = fill(state, [s, b])
    bnd = Buf(abi.I32, [4])
    bnd.flat()[:] = bounds
    ab, mk, al, dt = Buf(abi.BF16, [T, hv]), Buf(abi.I32, [T]), Buf(abi.F32, [hv]), Buf(abi.F32, [hv])
    ab.flat()[:] = a.ravel()
    mk.flat()[:] = mask
    al.flat()[:] = a_log
    dt.flat()[:] = dt_bias
    nd, sidx = Buf(abi.F32, [SLOTS, hv, 1, 2]), Buf(abi.I32, [1, 1])
    sidx.flat()[0] = SLOT
    rho = lib.find_row("ridgefill_rho_update", domain)
    assert H.run_row(lib, rho, [ab, mk, al, dt, nd, sidx, bnd], [pint("M", b), pint("n_head", hv)]) == abi.OK
    pool, applied, cb = Buf(abi.F32, [SLOTS, hv, D, D]), Buf(abi.F32, [SLOTS, hv, 1, 1]), Buf(abi.F32, [hv, D, D])
    pool.flat()[:] = st.ravel()
    cb.flat()[:] = C.ravel()
    idx = Buf(abi.I32, [1, 2])
    idx.flat()[:] = [SLOT, 999]
    corr = lib.find_row("ridgefill_state_correct", domain)
    assert H.run_row(lib, corr, [pool, idx, applied, idx, cb, nd, idx, bnd],
                     [pint("M", 1), pstr("mode", "apply"), pf64("alpha", alpha), pint("n_head", hv), pint("sd0", D),
                      pint("sd1", D)]) == abi.OK
    st = fill(pool.flat().reshape(SLOTS, hv, D, D).copy(), [b, e])
    return st, nd.flat().reshape(SLOTS, hv, 2).copy(), applied.flat().reshape(SLOTS, hv).copy()


@pytest.mark.parametrize("hv,s", [(4, 0), (4, 40), (64, 0), (64, 40)])
def test_split_scan_sequence_matches_the_host(cuda, product_lib, oracle_lib, hv, s):
    torch = cuda
    hk, T = hv // 2, 240
    b, e = s + 128, T
    inp = _inputs(7 + hv + s, T, hk, hv)
    k, v, g, beta = inp[:4]

    def dev_fill(st, cu):
        rc, out, _ = run_fill(product_lib, torch, k, v, g, beta, st, [SLOT], cu, hk, hv)
        assert rc == abi.OK
        return out

    def host_fill(st, cu):
        return H.oracle_gdn(k, v, g, beta, st, [SLOT], cu)[0]

    bounds = [s, b, b, e]
    got, nd_d, ap_d = _split_sequence(product_lib, abi.DOMAIN_DEVICE, dev_fill, inp, bounds, 0.5)
    want, nd_h, ap_h = _split_sequence(oracle_lib, abi.DOMAIN_HOST, host_fill, inp, bounds, 0.5)
    n_d, d_d, n_h, d_h = nd_d[SLOT, :, 0], nd_d[SLOT, :, 1], nd_h[SLOT, :, 0], nd_h[SLOT, :, 1]
    assert np.all(np.abs(n_d - n_h) <= 1e-4 * np.maximum(np.abs(n_h), 1e-30) + 1e-30), (n_d, n_h)
    assert np.all(np.abs(d_d - d_h) <= 1e-4 * np.abs(d_h)), (d_d, d_h)
    rho_d, rho_h = np.clip(n_d / d_d, 0, 1), np.clip(n_h / d_h, 0, 1)
    assert np.all(np.abs(rho_d - rho_h) <= 1e-5), (rho_d, rho_h)
    assert np.all(np.abs(ap_d - ap_h) <= 1e-5 * np.maximum(np.abs(ap_h), 1e-30)), (ap_d, ap_h)
    assert np.any(ap_d[SLOT] != 0)   # the correction did something
    for slot in range(SLOTS):   # the other slots: untouched by every step
        if slot != SLOT:
            assert np.array_equal(got[slot], inp[4][slot])
    assert H.rel_l2(got[SLOT], want[SLOT]) <= 1e-3
    # alpha = 0: the apply adds nothing and the two scans are one fill over [s, e), bit for bit
    flat, _, _ = _split_sequence(product_lib, abi.DOMAIN_DEVICE, dev_fill, inp, bounds, 0.0)
    one = dev_fill(inp[4], [s, e])
    assert np.array_equal(flat, one)
