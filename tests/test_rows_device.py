"""The reference's seven row ops: the sm_100a device rows against the CPU oracle, after the reference's
own `gpu` cases (tests/kernel_test.cpp:1580-1927) -- every buffer compared bit for bit (padding
included), rho within the reference's 1e-5. The refusal cases run on CPU too: a device row refuses an
operand the oracle refuses, with the same code, before it touches the GPU."""
import numpy as np
import pytest

import cases as K
import harness as H
from harness import abi, Buf

gpu = pytest.mark.gpu


def rows(op, product_lib, oracle_lib):
    return product_lib.find_row(op, abi.DOMAIN_DEVICE), oracle_lib.find_row(op, abi.DOMAIN_HOST)


# ----------------------------------------------------------------- refusals (CPU and GPU)

def _refusal_cases():
    table = [1.0, 2.0]
    mc = K.MaskCall([0, 1, 0, 1], 4, 0, 4, table)
    yield "mask", mc.copy(mode="classy"), abi.E_INVAL
    yield "mask", mc.copy(share=1.5), abi.E_INVAL
    yield "mask", mc.copy(table=None), abi.E_INVAL
    yield "mask", mc.copy(table=None, mode="random"), abi.E_INVAL


@pytest.mark.parametrize("case", list(range(4)))
def test_mask_refusals_match_oracle(case, product_lib, oracle_lib):
    _, c, want = list(_refusal_cases())[case]
    dev, host = rows("ridgefill_mask", product_lib, oracle_lib)
    assert K.run_mask(oracle_lib, host, c)[0] == want
    assert H.run_host(product_lib, dev, _mask_bufs(c), _mask_params(c)) == want


def _mask_bufs(c):
    b = len(c.ids)
    cu, tok, pos, mask, bounds = Buf(abi.I32, [2]), Buf(abi.I32, [b]), Buf(abi.I32, [b]), Buf(abi.I32, [c.n]), Buf(abi.I32, [4])
    cu.flat()[:2] = [c.s, c.e]
    score = Buf(abi.F32, [len(c.table)]) if c.table is not None else None
    return [cu, tok, pos, score, mask, bounds, None]


def _mask_params(c):
    return [H.pint("M", len(c.ids)), H.pf64("share", c.share), H.pint("seed", c.seed), H.pstr("mode", c.mode)]


def test_operand_refusals_match_oracle(product_lib, oracle_lib):
    """tests/kernel_test.cpp:871-960 and 1182-1217: every refusal of the shared parse, same code on the
    device rows as on the oracle (no case here reaches a launch)."""
    mk_d, mk_h = rows("ridgefill_mask", product_lib, oracle_lib)
    cu, cu1, cu_f = Buf(abi.I32, [2]), Buf(abi.I32, [1]), Buf(abi.F32, [2])
    cu.flat()[1] = 4
    tok, pos, short_pos = Buf(abi.I32, [4]), Buf(abi.I32, [4]), Buf(abi.I32, [3])
    pos16, score, score16 = Buf(abi.BF16, [4]), Buf(abi.F32, [2]), Buf(abi.BF16, [2])
    mask, bounds, bounds3 = Buf(abi.I32, [4]), Buf(abi.I32, [4]), Buf(abi.I32, [3])
    p = [H.pint("M", 4), H.pf64("share", 0.5), H.pint("seed", 0), H.pstr("mode", "class")]
    no_seed = [p[0], p[1], p[3]]
    mask_cases = [
        ([cu, tok, pos, score, mask, bounds], no_seed, abi.E_INVAL),
        ([None, tok, pos, score, mask, bounds], p, abi.E_INVAL),
        ([cu, None, pos, score, mask, bounds], p, abi.E_INVAL),
        ([cu, tok, None, score, mask, bounds], p, abi.E_INVAL),
        ([cu, tok, pos, score, None, bounds], p, abi.E_INVAL),
        ([cu, tok, pos, score, mask, None], p, abi.E_INVAL),
        ([cu_f, tok, pos, score, mask, bounds], p, abi.E_DTYPE),
        ([cu, tok, pos16, score, mask, bounds], p, abi.E_DTYPE),
        ([cu, tok, pos, score16, mask, bounds], p, abi.E_DTYPE),
        ([cu1, tok, pos, score, mask, bounds], p, abi.E_SHAPE),
        ([cu, tok, short_pos, score, mask, bounds], p, abi.E_SHAPE),
        ([cu, tok, pos, score, mask, bounds3], p, abi.E_SHAPE),
    ]
    for bufs, params, want in mask_cases:
        assert H.run_host(oracle_lib, mk_h, bufs, params) == want
        assert H.run_host(product_lib, mk_d, bufs, params) == want
    big = K.MaskCall([1] * (49153), 49153, 0, 49153, [1.0] * 8, mode="none")
    assert H.run_host(product_lib, mk_d, _mask_bufs(big), _mask_params(big)) == abi.E_SHAPE   # past shared memory

    sc_d, sc_h = rows("ridgefill_state_correct", product_lib, oracle_lib)
    k = K.CorrectRun(3, 2, 4, 4, [0], 0)
    cp = [H.pint("M", 1), H.pstr("mode", "apply"), H.pf64("alpha", 1.0), H.pint("n_head", 2), H.pint("sd0", 4), H.pint("sd1", 4)]
    bad_heads = list(cp)
    bad_heads[3] = H.pint("n_head", 3)
    redo = list(cp)
    redo[1] = H.pstr("mode", "redo")
    two = K.slot_index([0, 1])
    b1, bf, bgap = Buf(abi.I32, [1]), Buf(abi.F32, [4]), Buf(abi.I32, [2], [2])
    base = [k.state, k.sidx, k.applied, k.aidx, k.c, None, None]
    correct_cases = [
        (base, redo, abi.E_INVAL),
        (base, bad_heads, abi.E_SHAPE),
        ([k.state, k.sidx, k.applied, two, k.c, None, None], cp, abi.E_SHAPE),
        ([k.state, k.sidx, k.applied, k.aidx, k.c, k.nd, None], cp, abi.E_INVAL),
        ([k.state, None, k.applied, k.aidx, k.c, None, None], cp, abi.E_INVAL),
        (base + [b1], cp, abi.E_SHAPE), (base + [bf], cp, abi.E_DTYPE), (base + [bgap], cp, abi.E_STRIDE),
    ]
    for bufs, params, want in correct_cases:
        assert H.run_host(oracle_lib, sc_h, bufs, params) == want
        assert H.run_host(product_lib, sc_d, bufs, params) == want

    sr_d, sr_h = rows("ridgefill_state_read", product_lib, oracle_lib)
    rp = [H.pint("M", 1), H.pint("n_head", 2), H.pint("sd0", 4), H.pint("sd1", 4)]
    rp_heads = [rp[0], H.pint("n_head", 3), rp[2], rp[3]]
    read_cases = [([k.state, k.sidx, Buf(abi.F32, [31])], rp, abi.E_SHAPE),
                  ([k.state, k.sidx, Buf(abi.BF16, [1, 2, 4, 4])], rp, abi.E_DTYPE),
                  ([k.state, None, Buf(abi.F32, [1, 2, 4, 4])], rp, abi.E_INVAL),
                  ([k.state, k.sidx, Buf(abi.F32, [1, 2, 4, 4])], rp_heads, abi.E_SHAPE)]
    for bufs, params, want in read_cases:
        assert H.run_host(oracle_lib, sr_h, bufs, params) == want
        assert H.run_host(product_lib, sr_d, bufs, params) == want

    rh_d, rh_h = rows("ridgefill_rho_update", product_lib, oracle_lib)
    assert H.run_host(oracle_lib, rh_h, [], [H.pint("M", 8), H.pint("n_head", 4)]) == abi.E_INVAL
    assert H.run_host(product_lib, rh_d, [], [H.pint("M", 8), H.pint("n_head", 4)]) == abi.E_INVAL

    sl_d, sl_h = rows("ridgefill_select", product_lib, oracle_lib)
    dr_d, dr_h = rows("ridgefill_drop_rows", product_lib, oracle_lib)
    m, m_f32 = K.mask_buf([1, 0, 1]), Buf(abi.F32, [3])
    x, x_f32, x_wide = Buf(abi.BF16, [3, 4]), Buf(abi.F32, [3, 4]), Buf(abi.BF16, [3, 5])
    x_short, x_gap = Buf(abi.BF16, [2, 4]), Buf(abi.BF16, [3, 4], [8, 2])
    x_rank3, x_i4, q = Buf(abi.BF16, [3, 4, 1]), Buf(abi.I4, [3, 4]), Buf(abi.I8, [3, 6])
    P = [H.pint("M", 3)]
    sel_cases = [([None, x, None, None, x, None, None], abi.E_INVAL), ([m, None, None, None, x, None, None], abi.E_INVAL),
                 ([m, x, None, None, None, None, None], abi.E_INVAL), ([m, x, q, None, x, None, None], abi.E_INVAL),
                 ([m, x, None, None, x, q, None], abi.E_INVAL), ([m_f32, x, None, None, x, None, None], abi.E_DTYPE),
                 ([m, x, None, None, x_f32, None, None], abi.E_DTYPE), ([m, x_i4, None, None, x_i4, None, None], abi.E_DTYPE),
                 ([m, x, None, None, x_wide, None, None], abi.E_SHAPE), ([m, x, None, None, x_short, None, None], abi.E_SHAPE),
                 ([m, x_short, None, None, x, None, None], abi.E_SHAPE),
                 ([m, x_rank3, None, None, x_rank3, None, None], abi.E_SHAPE),
                 ([m, x, None, None, x_gap, None, None], abi.E_STRIDE)]
    for bufs, want in sel_cases:
        assert H.run_host(oracle_lib, sl_h, bufs, P) == want
        assert H.run_host(product_lib, sl_d, bufs, P) == want
    ids, ids_short, ids_f32 = Buf(abi.I32, [3, 8]), Buf(abi.I32, [2, 8]), Buf(abi.F32, [3, 8])
    ids_gap, ids_flat = Buf(abi.I32, [3, 8], [16, 2]), Buf(abi.I32, [24])
    drop_cases = [([m, ids], 9, abi.E_SHAPE), ([m, ids], -1, abi.E_INVAL), ([m, ids_short], 2, abi.E_SHAPE),
                  ([m, ids_flat], 2, abi.E_SHAPE), ([m, ids_f32], 2, abi.E_DTYPE), ([m_f32, ids], 2, abi.E_DTYPE),
                  ([m, ids_gap], 2, abi.E_STRIDE)]
    for bufs, top_k, want in drop_cases:
        params = [H.pint("M", 3), H.pint("top_k", top_k)]
        assert H.run_host(oracle_lib, dr_h, bufs, params) == want
        assert H.run_host(product_lib, dr_d, bufs, params) == want
    assert H.run_host(product_lib, dr_d, [m, ids], [H.pint("M", 3)]) == abi.E_INVAL


# ----------------------------------------------------------------- device == oracle

@gpu
def test_described_operands_launch(cuda, product_lib):
    """Every device row accepts the operands its own description builds (kernel_test.cpp:364-376)."""
    from test_abi import DEVICE_OPS, described_params
    import ctypes as C
    r = H.Rng(1234)
    for op in DEVICE_OPS:
        row = product_lib.find_row(op, abi.DOMAIN_DEVICE)
        sc = product_lib.schema(op)
        params = described_params(op)
        pp = (abi.RadParam * len(params))(*params)
        m = dict((p.key.decode(), p.ival) for p in params).get("M", 0)
        bufs, prev = [], 0
        for i in range(sc.n_operands):
            d = abi.RadOpdDesc()
            assert row.opd_shape(pp, len(params), i, C.byref(d)) == abi.OK
            if d.flags & abi.OPD_F_ABSENT:
                bufs.append(None)
                continue
            shape = [d.shape[j] for j in range(d.rank)]
            b = Buf(d.dtype, shape)
            n = b.numel()
            hi = d.idx_max if d.idx_max > 0 else prev
            f = b.flat()
            if d.fill == abi.FILL_INDEX and d.flags & abi.OPD_F_IDX_CU:
                f[:n] = [i * m // (n - 1) if n > 1 else m for i in range(n)]
            elif d.fill == abi.FILL_INDEX and d.flags & abi.OPD_F_IDX_UNIQUE:
                f[:n] = np.random.default_rng(i).permutation(hi)[:n]
            elif d.fill == abi.FILL_INDEX:
                f[:n] = [r.below(hi) for _ in range(n)]
            elif d.dtype in (abi.F32, abi.BF16):
                vals = [0.01 + 0.98 * r.uniform() if d.fill == abi.FILL_SIGMOID else r.normal() for _ in range(n)]
                f[:n] = H.f32_to_bf16_bits(np.asarray(vals, np.float32)) if d.dtype == abi.BF16 else vals
            elif d.dtype == abi.I8:
                f[:n] = [int(r.below(255)) - 127 for _ in range(n)]
            bufs.append(b)
            prev = shape[0]
        if op == "ridgefill_gdn_fill":   # sigmoid-filled g is a positive log decay: make it a decay
            bufs[3].flat()[:] = -np.abs(bufs[3].flat())
        assert H.run_device(product_lib, row, bufs, params) == abi.OK, op


def _correct_steps():
    return [("undo", 1.0, False), ("apply", 0.7, True), ("undo", 1.0, False), ("apply", 1.0, False), ("apply", 0.0, True)]


@gpu
@pytest.mark.parametrize("heads", [48, 24, 18, 15, 12])
def test_state_correct_device_matches_oracle(cuda, product_lib, oracle_lib, heads):
    """kernel_test.cpp:1586-1636: padded 128 x 128 slots, shared and separate slot pools, every step."""
    dev, host = rows("ridgefill_state_correct", product_lib, oracle_lib)
    r = H.Rng(31 + heads)
    k = K.random_correct(r, heads)
    sep = k.copy()
    sep.applied = Buf(abi.F32, [4, heads, 1, 1])
    sep.applied.flat()[:] = [0.5 + r.normal() for _ in range(sep.applied.numel())]
    sep.nd = Buf(abi.F32, [7, heads, 1, 2])
    nd = sep.nd.flat()
    for i in range(0, sep.nd.numel(), 2):
        nd[i + 1] = np.float32(1.0 + 50.0 * r.uniform())
        nd[i] = np.float32(nd[i + 1] * 1.2 * r.uniform())
    sep.sidx, sep.aidx, sep.nidx = K.slot_index([3, 0, 5, 2]), K.slot_index([1, 3, 0, 4]), K.slot_index([5, 6, 2, 0])
    for h in (k, sep):
        for mode, alpha, with_nd in _correct_steps():
            d = h.copy()
            assert K.run_correct(oracle_lib, host, h, mode, alpha, with_nd) == abi.OK
            assert K.run_correct(product_lib, dev, d, mode, alpha, with_nd) == abi.OK
            assert np.array_equal(h.state.bytes, d.state.bytes)
            assert np.array_equal(h.applied.bytes, d.applied.bytes) and np.array_equal(h.nd.bytes, d.nd.bytes)


@gpu
def test_state_correct_bounds_device_matches_oracle(cuda, product_lib, oracle_lib):
    dev, host = rows("ridgefill_state_correct", product_lib, oracle_lib)
    r = H.Rng(101)
    k = K.random_correct(r, 24)
    for mode in ("undo", "apply"):
        for b in ((), (9, 9, 9, 12), (10, 4, 4, 12), (3, 9, 9, 12)):
            h, d = k.copy(), k.copy()
            assert K.run_correct(oracle_lib, host, h, mode, 0.7, mode == "apply", b) == abi.OK
            assert K.run_correct(product_lib, dev, d, mode, 0.7, mode == "apply", b) == abi.OK
            assert np.array_equal(h.state.bytes, d.state.bytes) and np.array_equal(h.applied.bytes, d.applied.bytes)
            empty = len(b) > 0 and b[1] <= b[0]
            assert np.array_equal(d.state.bytes, k.state.bytes) == empty


@gpu
@pytest.mark.parametrize("heads", [48, 24, 18, 15, 12])
def test_state_read_device_matches_oracle(cuda, product_lib, oracle_lib, heads):
    dev, host = rows("ridgefill_state_read", product_lib, oracle_lib)
    r = H.Rng(61 + heads)
    k = K.random_correct(r, heads, seq_slots=[0])
    idx = K.slot_index([4, -1, 1, 7, 4])
    rh, oh = K.run_state_read(oracle_lib, host, k, idx)
    rd, od = K.run_state_read(product_lib, dev, k, idx)
    assert rh == rd == abi.OK and np.array_equal(oh.bytes, od.bytes)
    per = heads * 128 * 128
    f = od.flat()
    assert np.all(f[per: 2 * per] == 0) and np.all(f[3 * per: 4 * per] == 0)


@gpu
def test_mask_device_matches_oracle(cuda, product_lib, oracle_lib):
    """kernel_test.cpp:1682-1720 widened past the reference's 8,192-row budget: random windows, every
    mode, heavy ties, ids outside the table, n to 40,000."""
    dev, host = rows("ridgefill_mask", product_lib, oracle_lib)
    r = H.Rng(41)
    levels = [-np.inf, -np.inf, 1.0, 2.0, 2.5, 3.0]
    table = [levels[r.below(6)] for _ in range(1000)]
    runs = 0
    for n in (1, 7, 300, 2048, 8192, 9000, 40000):
        for layout in range(4):
            c = K.random_window(r, n, layout, limit=32768)
            c.table, c.seed, c.first_pos = table, 12345, 4096
            for mode in ("none", "class", "random", "all", "step"):
                for share in (0.25, 1.0, 0.3):
                    c.mode, c.share, c.components, c.n_zeros = mode, share, 3 if runs % 2 else 1, 0 if runs % 3 else 513
                    h, d = K.run_mask(oracle_lib, host, c), K.run_mask(product_lib, dev, c)
                    assert h[0] == d[0] == abi.OK
                    assert np.array_equal(h[1], d[1]) and np.array_equal(h[2], d[2]) and np.array_equal(h[3], d[3]), \
                        (n, layout, mode, share)
                    runs += 1
    c = K.random_window(r, 4000, 1)
    c.table, c.mode, c.seed, c.first_pos = table, "random", 99, 2048
    once, again = K.run_mask(product_lib, dev, c), K.run_mask(product_lib, dev, c)
    other = K.run_mask(product_lib, dev, c.copy(first_pos=6144))
    assert np.array_equal(once[1], again[1])
    assert (other[1] == 1).sum() == (once[1] == 1).sum() and not np.array_equal(other[1], once[1])


@gpu
def test_mask_device_fail_safe(cuda, product_lib, oracle_lib):
    """cu_last out of order: the device row takes the window empty inside the clamped [s, e]
    (kernel_test.cpp:1745-1769); the host row refuses."""
    dev, host = rows("ridgefill_mask", product_lib, oracle_lib)
    for s, e, want in ((-3, 10, [0, 0, 0, 10]), (12, 8, [8, 8, 8, 8]), (2, 21, [2, 2, 2, 16])):
        c = K.MaskCall([1] * 14, 16, s, e, [1.0] * 8, mode="none")
        rc, mask, bounds, _ = K.run_mask(product_lib, dev, c)
        assert rc == abi.OK and np.all(mask == 0) and list(bounds) == want
        assert K.run_mask(oracle_lib, host, c)[0] == abi.E_INVAL


@gpu
def test_mask_device_matches_rowsel_fixture(cuda, product_lib):
    import json
    fx = json.loads((H.GOLDEN / "rowsel_keys.json").read_text())
    table = np.full(fx["vocab"], -np.inf, np.float32)
    table[fx["kept_ids"]] = fx["kept_scores"]
    dev = product_lib.find_row("ridgefill_mask", abi.DOMAIN_DEVICE)
    for doc in fx["docs"]:
        w = len(doc["token_ids"])
        rc, mask, _, _ = K.run_mask(product_lib, dev, K.MaskCall(doc["token_ids"], w, 0, w, table, fx["share"], 0, "class"))
        assert rc == abi.OK and list(np.flatnonzero(mask == 0)) == doc["rows"]


@gpu
def test_hazard_device_matches_oracle(cuda, product_lib, oracle_lib):
    dev, host = rows("ridgefill_hazard", product_lib, oracle_lib)
    r = H.Rng(7)
    for _ in range(64):
        c = K.HazardCall()
        c.e = 1 + r.below(2048)
        c.s = r.below(c.e)
        c.first_pos, c.span = r.below(40000), r.below(3000)
        c.b = c.s + r.below(c.e - c.s + 1) if r.below(2) else 0
        c.m0, c.m1, c.count = float(r.below(45000)), float(r.below(40000)), float(r.below(100))
        assert K.run_hazard(oracle_lib, host, c) == K.run_hazard(product_lib, dev, c)
    bad = K.HazardCall(s=10, e=5, span=2048, m0=4096.0)   # the device row counts nothing instead of refusing
    rc, m0, m1, count = K.run_hazard(product_lib, dev, bad)
    assert rc == abi.OK and count == 0.0 and m1 == 0.0


@gpu
def test_rho_device_matches_oracle(cuda, product_lib, oracle_lib):
    """kernel_test.cpp:1773-1800: TP1..TP4 head counts, bf16 a as the first half of a|b, two chunks;
    rho within 1e-5, exactly 1 when no row is exact, always in [0, 1]."""
    dev, host = rows("ridgefill_rho_update", product_lib, oracle_lib)
    r = H.Rng(51)
    worst = 0.0
    for heads in (48, 24, 18, 15, 12):
        for exact in (0.056, 0.5, 0.0):
            h = K.random_rho(r, 2048, heads, exact, True)
            h.pitch = 2 * heads
            d = h.copy()
            for _ in range(2):
                assert K.run_rho(oracle_lib, host, h) == abi.OK
                assert K.run_rho(product_lib, dev, d) == abi.OK
            for k in range(heads):
                worst = max(worst, abs(K.nd_rho(h, k) - K.nd_rho(d, k)))
                if exact == 0.0:
                    assert K.nd_rho(d, k) == 1.0
                assert 0.0 <= K.nd_rho(d, k) <= 1.0
    assert worst <= 1e-5, worst


@gpu
@pytest.mark.parametrize("n", [32768, 32767])
def test_rho_device_at_the_full_chunk(cuda, product_lib, oracle_lib, n):
    """The pass's size: 32,768 rows (and an odd 32,767) x 32 heads, 30 % of the rows exact, two chunks; rho within
    the reference's 1e-5 of the sequential host rule, whatever the composition over row runs does to rounding."""
    dev, host = rows("ridgefill_rho_update", product_lib, oracle_lib)
    r = H.Rng(n)
    h = K.random_rho(r, n, 32, 0.30, True)
    h.pitch = 64
    d = h.copy()
    for _ in range(2):
        assert K.run_rho(oracle_lib, host, h) == abi.OK
        assert K.run_rho(product_lib, dev, d) == abi.OK
    worst = max(abs(K.nd_rho(h, k) - K.nd_rho(d, k)) for k in range(32))
    assert worst <= 1e-5, worst


@gpu
def test_rho_bounds_device_is_the_slice(cuda, product_lib, oracle_lib):
    """With bounds {s, ..} the device row equals itself run on rows [s, n) bit for bit, and the oracle
    within 1e-5 (kernel_test.cpp:1807-1832)."""
    dev, host = rows("ridgefill_rho_update", product_lib, oracle_lib)
    r = H.Rng(91)
    base = K.random_rho(r, 2048, 24, 0.1, True)
    base.pitch = 48
    base.nd = [0.5 + (i % 7) for i in range(len(base.nd))]
    worst = 0.0
    for s in (-3, 0, 5, 1000, 2047, 2048, 4000):
        d, h = base.copy(), base.copy()
        d.bounds = h.bounds = [s, 2048, 2048, 2048]
        cl = min(max(s, 0), 2048)
        sl = base.copy()
        sl.n = 2048 - cl
        sl.a = base.a[cl * 24:]
        sl.mask = base.mask[cl:]
        assert K.run_rho(product_lib, dev, d) == abi.OK
        assert K.run_rho(oracle_lib, host, h) == abi.OK
        assert K.run_rho(product_lib, dev, sl) == abi.OK
        assert np.array_equal(np.asarray(d.nd, np.float32).view(np.uint32), np.asarray(sl.nd, np.float32).view(np.uint32))
        worst = max(worst, max(abs(K.nd_rho(h, k) - K.nd_rho(d, k)) for k in range(24)))
    assert worst <= 1e-5


@gpu
def test_select_device_matches_oracle(cuda, product_lib, oracle_lib):
    dev, host = rows("ridgefill_select", product_lib, oracle_lib)
    r = H.Rng(111)
    for n in (1, 300, 8192, 32768):
        for variant in range(3):
            exact = r.uniform()
            mask = [2 if r.uniform() < 0.02 else (0 if r.uniform() < exact else 1) for _ in range(n)]
            codes = abi.F8E4M3 if variant == 1 else abi.I8
            xw, qw = 64 * (1 + variant), 33 + 16 * variant
            k = {"mask": K.mask_buf(mask), "xs": Buf(abi.BF16, [n, xw], [xw + 8, 1]), "qs": Buf(codes, [n, qw]),
                 "ss": Buf(abi.F32, [n + 1, 3]), "x": Buf(abi.BF16, [n + 1, xw]), "q": Buf(codes, [n, qw], [qw + 5, 1]),
                 "s": Buf(abi.F32, [n, 3], [4, 1])}
            K.fill_pattern(k["xs"], 4 + variant)
            K.fill_pattern(k["qs"], 5)
            K.fill_pattern(k["ss"], 6)
            for name in ("x", "q", "s"):
                K.fill_sentinel(k[name])
            if variant == 2:
                k["qs"] = k["ss"] = k["q"] = k["s"] = None
            h = {a: (b.copy() if b is not None else None) for a, b in k.items()}
            d = {a: (b.copy() if b is not None else None) for a, b in k.items()}
            assert K.run_select(oracle_lib, host, h) == abi.OK
            assert K.run_select(product_lib, dev, d) == abi.OK
            for name in ("x", "q", "s"):
                if d[name] is not None:
                    assert np.array_equal(h[name].bytes, d[name].bytes)
            assert K.selected_exactly(k["xs"], k["x"], d["x"], mask)


@gpu
def test_drop_rows_device_matches_oracle(cuda, product_lib, oracle_lib):
    dev, host = rows("ridgefill_drop_rows", product_lib, oracle_lib)
    r = H.Rng(121)
    for n in (1, 300, 8192, 32768):
        for top_k in (0, 1, 7, 300):
            mask = [2 if r.uniform() < 0.02 else (0 if r.uniform() < 0.3 else 1) for _ in range(n)]
            ids = Buf(abi.I32, [n + 1, top_k + 4], [top_k + 7, 1])
            ids.flat()[:] = np.random.default_rng(n + top_k).integers(0, 1 << 20, len(ids.flat()))
            h, d = ids.copy(), ids.copy()
            assert K.run_drop(oracle_lib, host, K.mask_buf(mask), h, top_k) == abi.OK
            assert K.run_drop(product_lib, dev, K.mask_buf(mask), d, top_k) == abi.OK
            assert np.array_equal(h.bytes, d.bytes) and K.dropped_exactly(ids, d, mask, top_k)


@gpu
def test_each_ranks_heads_compute_their_slice_of_tp1(cuda, product_lib):
    """kernel_test.cpp:1498-1577 on the device rows: a rank's state_correct / rho at its head extent
    (TP2 / TP3 uneven / TP4) is bit-identical to the same heads of the TP1 call."""
    dev_c = product_lib.find_row("ridgefill_state_correct", abi.DOMAIN_DEVICE)
    dev_r = product_lib.find_row("ridgefill_rho_update", abi.DOMAIN_DEVICE)
    r = H.Rng(4848)
    H_, D = 48, 128
    full = K.random_correct(r, H_)
    tp1 = full.copy()
    for mode, alpha, nd in _correct_steps()[:3]:
        assert K.run_correct(product_lib, dev_c, tp1, mode, alpha, nd) == abi.OK
    rho1 = K.random_rho(r, 512, H_, 0.1, True)
    rho1.pitch = 2 * H_
    assert K.run_rho(product_lib, dev_r, rho1) == abi.OK
    for spans in ([(0, 24), (24, 24)], [(18, 15), (33, 15), (0, 18)], [(0, 12), (12, 12), (24, 12), (36, 12)]):
        for h0, hw in spans:
            part = K.CorrectRun(6, hw, D, D, [4, -1, 1, 5], 8)
            for s in range(6):
                for h in range(hw):
                    for name in ("applied",):
                        part.applied.flat()[s * hw + h] = full.applied.flat()[s * H_ + h0 + h]
                    part.nd.flat()[(s * hw + h) * 2:(s * hw + h) * 2 + 2] = full.nd.flat()[(s * H_ + h0 + h) * 2:(s * H_ + h0 + h) * 2 + 2]
                    src = full.state.flat()[full.st_at(s, h0 + h, 0, 0):][: D * full.state.strides[2]]
                    dst0 = part.st_at(s, h, 0, 0)
                    for i in range(D):
                        part.state.flat()[dst0 + i * part.state.strides[2]: dst0 + i * part.state.strides[2] + D] = \
                            src[i * full.state.strides[2]: i * full.state.strides[2] + D]
            part.c.flat()[:] = full.c.flat()[h0 * D * D:(h0 + hw) * D * D]
            for mode, alpha, nd in _correct_steps()[:3]:
                assert K.run_correct(product_lib, dev_c, part, mode, alpha, nd) == abi.OK
            for s in range(6):
                for h in range(hw):
                    a0, b0 = part.st_at(s, h, 0, 0), tp1.st_at(s, h0 + h, 0, 0)
                    for i in (0, 63, 127):
                        pa = part.state.flat()[a0 + i * part.state.strides[2]: a0 + i * part.state.strides[2] + D]
                        pb = tp1.state.flat()[b0 + i * tp1.state.strides[2]: b0 + i * tp1.state.strides[2] + D]
                        assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))
            rp = rho1.copy()
            rp.heads, rp.pitch = hw, 2 * hw
            rp.a = list(np.asarray(rho1.a, np.float32).reshape(512, H_)[:, h0:h0 + hw].reshape(-1))
            rp.a_log, rp.dt_bias = rho1.a_log[h0:h0 + hw], rho1.dt_bias[h0:h0 + hw]
            rp.nd = [0.0] * (rp.slots * hw * 2)
            assert K.run_rho(product_lib, dev_r, rp) == abi.OK
            got = np.asarray(rp.nd, np.float32).reshape(rp.slots, hw, 2)
            want = np.asarray(rho1.nd, np.float32).reshape(rho1.slots, H_, 2)[:, h0:h0 + hw]
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
