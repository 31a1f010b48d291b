"""Pins of the CPU oracle (oracle/ridgefill_oracle.cpp) before anything is checked against it:
 - the reference's own test harness (tests/kernel_test.cpp, compiled here from its source into
   oracle/_ref) passes against the oracle library, golden fixtures included;
 - the oracle equals the reference's host rows (compiled from kernels/host_ref.cpp) bit for bit on
   random operands of every op;
 - the golden fixtures made from the reference's own Python (tests/golden/make_golden.py) hold.
"""
import json
import os
import subprocess

import numpy as np
import pytest

import cases as K
import harness as H
from harness import abi, Buf


def test_reference_harness_passes_on_oracle(oracle_lib):
    if not H.REF_TEST.exists():
        pytest.skip("oracle/_ref/kernel_test is not built (make -C oracle ref needs the reference sources)")
    env = dict(os.environ, RIDGEFILL_RHO_FIXTURE=str(H.GOLDEN / "rho_numpy.txt"),
               RIDGEFILL_ROWSEL_FIXTURE=str(H.GOLDEN / "rowsel_keys.json"))
    res = subprocess.run([str(H.REF_TEST), str(H.ORACLE_SO), "host"], capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    assert "FAIL" not in res.stderr
    checks = [l for l in res.stderr.splitlines() if "check(s)" in l]
    assert checks and int(checks[-1].split()[0]) >= 900
    assert "== fnlev.rules" in res.stderr and "rho vs NumPy" in res.stderr


def _both():
    ref = H.reference()
    if ref is None:
        pytest.skip("oracle/_ref/ridgefill_ref.so is not built")
    return H.oracle(), ref


def test_oracle_equals_reference_mask():
    o, ref = _both()
    r = H.Rng(41)
    table = [[-np.inf, -np.inf, 1.0, 2.0, 2.5, 3.0][r.below(6)] for _ in range(1000)]
    runs = 0
    for n in (1, 7, 300, 2048, 5000):
        for layout in range(4):
            c = K.random_window(r, n, layout)
            c.table, c.seed, c.first_pos = table, 12345, 4096
            for mode in ("none", "class", "random", "all", "step"):
                for share in (0.25, 0.5, 1.0):
                    c.mode, c.share, c.components, c.n_zeros = mode, share, 3 if runs % 2 else 1, 0 if runs % 3 else 33
                    a = K.run_mask(o, o.find_row("ridgefill_mask", 0), c)
                    b = K.run_mask(ref, ref.find_row("ridgefill_mask", 0), c)
                    assert a[0] == b[0]
                    for x, y in zip(a[1:], b[1:]):
                        assert np.array_equal(x, y)
                    runs += 1
    assert runs == 300


def test_oracle_equals_reference_rho_and_correct():
    o, ref = _both()
    r = H.Rng(51)
    for heads in (48, 12):
        for exact in (0.0, 0.3):
            base = K.random_rho(r, 700, heads, exact, True)
            base.pitch = 2 * heads
            for bounds in ([], [5, 600, 600, 700], [-3], [900, 0]):
                a, b = base.copy(), base.copy()
                a.bounds = b.bounds = bounds
                for _ in range(2):
                    assert K.run_rho(o, o.find_row("ridgefill_rho_update", 0), a) == abi.OK
                    assert K.run_rho(ref, ref.find_row("ridgefill_rho_update", 0), b) == abi.OK
                assert np.array_equal(np.asarray(a.nd, np.float32).view(np.uint32), np.asarray(b.nd, np.float32).view(np.uint32))
    for heads in (24, 15):
        k = K.random_correct(r, heads, sd=32, pad=4)
        for mode, alpha, nd, bounds in (("undo", 1.0, False, ()), ("apply", 0.7, True, ()), ("apply", 1.0, False, (2, 6, 6, 9)),
                                        ("undo", 1.0, False, (5, 5)), ("apply", 0.0, True, ())):
            a, b = k.copy(), k.copy()
            assert K.run_correct(o, o.find_row("ridgefill_state_correct", 0), a, mode, alpha, nd, bounds) == abi.OK
            assert K.run_correct(ref, ref.find_row("ridgefill_state_correct", 0), b, mode, alpha, nd, bounds) == abi.OK
            assert np.array_equal(a.state.bytes, b.state.bytes) and np.array_equal(a.applied.bytes, b.applied.bytes)
            k = a


def test_oracle_equals_reference_select_drop_read_hazard():
    o, ref = _both()
    r = H.Rng(111)
    for n in (1, 300, 2000):
        mask = [2 if r.uniform() < 0.02 else (0 if r.uniform() < 0.4 else 1) for _ in range(n)]
        for variant in range(3):
            xw, qw = 64 * (1 + variant), 33 + 16 * variant
            k = {"mask": K.mask_buf(mask), "xs": Buf(abi.BF16, [n, xw], [xw + 8, 1]), "qs": Buf(abi.I8, [n, qw]),
                 "ss": Buf(abi.F32, [n + 1, 3]), "x": Buf(abi.BF16, [n + 1, xw]), "q": Buf(abi.I8, [n, qw], [qw + 5, 1]),
                 "s": Buf(abi.F32, [n, 3], [4, 1])}
            for i, name in enumerate(("xs", "qs", "ss")):
                K.fill_pattern(k[name], 4 + i + variant)
            for name in ("x", "q", "s"):
                K.fill_sentinel(k[name])
            if variant == 2:
                k["qs"] = k["ss"] = k["q"] = k["s"] = None
            a = {n_: (v.copy() if v is not None else None) for n_, v in k.items()}
            b = {n_: (v.copy() if v is not None else None) for n_, v in k.items()}
            assert K.run_select(o, o.find_row("ridgefill_select", 0), a) == abi.OK
            assert K.run_select(ref, ref.find_row("ridgefill_select", 0), b) == abi.OK
            for name in ("x", "q", "s"):
                if a[name] is not None:
                    assert np.array_equal(a[name].bytes, b[name].bytes)
        for top_k in (0, 1, 7, 300):
            ids = Buf(abi.I32, [n + 1, top_k + 4], [top_k + 7, 1])
            ids.flat()[:] = [r.below(1 << 20) for _ in range(len(ids.flat()))]
            a, b = ids.copy(), ids.copy()
            assert K.run_drop(o, o.find_row("ridgefill_drop_rows", 0), K.mask_buf(mask), a, top_k) == abi.OK
            assert K.run_drop(ref, ref.find_row("ridgefill_drop_rows", 0), K.mask_buf(mask), b, top_k) == abi.OK
            assert np.array_equal(a.bytes, b.bytes)
    k = K.random_correct(r, 12, sd=16, pad=3)
    idx = K.slot_index([4, -1, 1, 7, 4])
    ra, oa = K.run_state_read(o, o.find_row("ridgefill_state_read", 0), k, idx)
    rb, ob = K.run_state_read(ref, ref.find_row("ridgefill_state_read", 0), k, idx)
    assert ra == rb == abi.OK and np.array_equal(oa.bytes, ob.bytes)
    for _ in range(64):
        c = K.HazardCall()
        c.e = 1 + r.below(2048)
        c.s = r.below(c.e)
        c.first_pos, c.span = r.below(40000), r.below(3000)
        c.b = c.s + r.below(c.e - c.s + 1) if r.below(2) else 0
        c.m0, c.m1, c.count = float(r.below(45000)), float(r.below(40000)), float(r.below(100))
        assert K.run_hazard(o, o.find_row("ridgefill_hazard", 0), c) == K.run_hazard(ref, ref.find_row("ridgefill_hazard", 0), c)


# ----------------------------------------------------------------- golden fixtures

def read_rho_fixture():
    words = (H.GOLDEN / "rho_numpy.txt").read_text().split()
    assert words[:2] == ["ridgefill-rho-fixture", "1"]
    heads, chunks = int(words[3]), int(words[5])
    pos = 8

    def lst(name):
        nonlocal pos
        assert words[pos] == name, (words[pos], name)
        n = int(words[pos + 1])
        vals = [float(x) for x in words[pos + 2: pos + 2 + n]]
        pos += 2 + n
        return vals

    a_log, dt_bias = lst("A_log"), lst("dt_bias")
    out = []
    for _ in range(chunks):
        assert words[pos] == "chunk"
        rows = int(words[pos + 3])
        pos += 4
        out.append((rows, lst("a"), lst("mask"), lst("N"), lst("D"), lst("rho")))
    return heads, a_log, dt_bias, out


def test_oracle_matches_rho_fixture(oracle_lib):
    """tests/rho_ref.py's closed form over three chunks, ND carried: |rho diff| <= 1e-5, rel N/D <= 1e-4
    (the reference's own bound, tests/kernel_test.cpp:1318-1342)."""
    heads, a_log, dt_bias, chunks = read_rho_fixture()
    nd = [0.0] * (4 * heads * 2)
    row = oracle_lib.find_row("ridgefill_rho_update", 0)
    for rows, a, mask, N, D, rho in chunks:
        c = K.RhoRun()
        c.n, c.heads, c.slot, c.a, c.mask, c.a_log, c.dt_bias, c.nd = rows, heads, 0, a, [int(m) for m in mask], a_log, dt_bias, nd
        assert K.run_rho(oracle_lib, row, c) == abi.OK
        nd = c.nd
        for h in range(heads):
            n, d = nd[h * 2], nd[h * 2 + 1]
            assert abs(n - N[h]) / N[h] <= 1e-4 and abs(d - D[h]) / D[h] <= 1e-4
            assert abs(K.nd_rho(c, h) - rho[h]) <= 1e-5


def test_oracle_matches_rowsel_fixture(oracle_lib):
    """ridgefill_mask class mode over each 2,048-row document keeps exactly the fixture's rows, and the
    same rows + 64 when the window starts at row 64 (tests/kernel_test.cpp:1404-1456)."""
    fx = json.loads((H.GOLDEN / "rowsel_keys.json").read_text())
    table = np.full(fx["vocab"], -np.inf, np.float32)
    table[fx["kept_ids"]] = fx["kept_scores"]
    best = int(fx["kept_ids"][int(np.argmax(table[fx["kept_ids"]]))])
    row = oracle_lib.find_row("ridgefill_mask", 0)
    for doc in fx["docs"]:
        ids, want = doc["token_ids"], doc["rows"]
        w = len(ids)
        rc, mask, bounds, _ = K.run_mask(oracle_lib, row, K.MaskCall(ids, w, 0, w, table, fx["share"], 0, "class"))
        assert rc == abi.OK and list(np.flatnonzero(mask == 0)) == want and len(want) == doc["k"]
        rc, mask, bounds, _ = K.run_mask(oracle_lib, row, K.MaskCall([best] * 64 + ids, w + 64, 64, w + 64, table,
                                                                     fx["share"], 0, "class"))
        assert rc == abi.OK and list(np.flatnonzero(mask[64:] == 0) + 64) == [r + 64 for r in want]
        assert np.all(mask[:64] == 0) and list(bounds) == [64, w + 64, w + 64, w + 64]


def test_oracle_matches_quantise_i8_fixture(oracle_lib):
    """The folder's weight encoder (tools/ridgefill_projector.py quantise_i8) reproduced bit for bit."""
    fx = np.load(H.GOLDEN / "quantise_i8.npz")
    codes, scale = H.oracle_quantise_weight(H.bf16_bits_to_f32(fx["w_bf16"]))
    assert np.array_equal(codes, fx["codes"]) and np.array_equal(scale, fx["scale"])
    assert np.all(H.bf16_bits_to_f32(scale[3, 1]) == 1.0)   # the all-zero group


def test_oracle_gemm_definition():
    """The GEMM oracle against an independent float64 evaluation of the same definition on small shapes:
    the int32 block sums exactly, y within one bf16 ulp (the f32 fold rounds per block)."""
    rng = np.random.default_rng(5)
    for M, N, K, group in ((3, 32, 256, 128), (17, 48, 384, 384), (8, 16, 128, 128)):
        a = rng.integers(-127, 128, (M, K)).astype(np.int8)
        b = rng.integers(-127, 128, (N, K)).astype(np.int8)
        sa = rng.uniform(1e-3, 1e-2, (M, K // group)).astype(np.float32)
        sb = rng.uniform(1e-3, 1e-2, (K // group, N)).astype(np.float32)
        bias = H.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
        y, acc = H.oracle_gemm(a, sa, b, sb, None, group, with_acc=True)
        blocks = np.einsum("mjk,njk->mnj", a.astype(np.int64).reshape(M, -1, group), b.astype(np.int64).reshape(N, -1, group))
        assert np.array_equal(acc, blocks)
        exact = np.einsum("mnj,mj,jn->mn", blocks.astype(np.float64), sa.astype(np.float64), sb.astype(np.float64))
        got = H.bf16_bits_to_f32(y).astype(np.float64)
        assert np.all(np.abs(got - exact) <= np.abs(exact) * 2.0 ** -7 + 1e-30)
        yb = H.oracle_gemm(a, sa, b, sb, bias, group)
        want = H.f32_to_bf16_bits(H.bf16_bits_to_f32(y) + H.bf16_bits_to_f32(bias)[None, :])
        assert np.array_equal(yb, want)


@pytest.mark.parametrize("bias_f32,res,act", [(False, False, 0), (True, True, 0), (False, True, 1), (True, False, 1)])
def test_oracle_gemm_bias_definition(bias_f32, res, act):
    """ridgefill_gemm_nt_bias's oracle against numpy on small shapes (kernels/rows.cpp:155-160): the rounding
    points of y = res + act(a @ b^T + bias) restated independently, bit for bit (the dots are exact in
    float64 for these sizes), with row sampling giving the same rows."""
    rng = np.random.default_rng(11 + act)
    M, N, K = 9, 40, 136
    a = H.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    b = H.f32_to_bf16_bits(rng.standard_normal((N, K)).astype(np.float32))
    bias = rng.standard_normal(N).astype(np.float32)
    bias = bias if bias_f32 else H.f32_to_bf16_bits(bias)
    r = H.f32_to_bf16_bits(rng.standard_normal((M, N)).astype(np.float32)) if res else None
    y, z = H.oracle_gemm_bias(a, b, bias, r, act=act)
    dot = H.bf16_bits_to_f32(a).astype(np.float64) @ H.bf16_bits_to_f32(b).astype(np.float64).T
    bv = bias if bias_f32 else H.bf16_bits_to_f32(bias)
    x = H.f32_to_bf16_bits(dot.astype(np.float32) + bv[None, :])
    if act:
        xv = H.bf16_bits_to_f32(x).astype(np.float64)
        x = H.f32_to_bf16_bits((xv / (1.0 + np.exp(-xv))).astype(np.float32))
    assert np.array_equal(z, x)
    if res:
        x = H.f32_to_bf16_bits(H.bf16_bits_to_f32(x) + H.bf16_bits_to_f32(r))
    assert np.array_equal(y, x)
    y2, _ = H.oracle_gemm_bias(a, b, bias, r, act=act, rows=(3, 7))
    assert np.array_equal(y2[3:7], y[3:7]) and not y2[:3].any()


def test_oracle_gdn_f32_tracks_f64():
    """The timed f32 baseline stays within the state tolerance of the f64 reference value."""
    rng = np.random.default_rng(9)
    T, Hk, Hv, d = 200, 2, 4, 128
    k = rng.standard_normal((T, Hk, d)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, Hv, d)).astype(np.float32)
    g = -np.log1p(np.exp(rng.standard_normal((T, Hv)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, Hv))))).astype(np.float32)
    state = np.zeros((2, Hv, d, d), np.float32)
    kb, vb = H.f32_to_bf16_bits(k), H.f32_to_bf16_bits(v)
    s64, _ = H.oracle_gdn(kb, vb, g, beta, state, [1], [0, T])
    s32, _ = H.oracle_gdn(kb, vb, g, beta, state, [1], [0, T], f64=False)
    assert np.linalg.norm(s32 - s64) / np.linalg.norm(s64) < 1e-5
    assert np.all(s64[0] == 0)   # slot 0 untouched


def _conv_prep_numpy(x, w, a_log, dt_bias, state, cu, a, b, idx, ctx, bias, hk, hv):
    """ridgefill_gdn_conv_prep restated in numpy (float64 arithmetic, the definition's rounding points)."""
    xf = H.bf16_bits_to_f32(x).astype(np.float64)
    wf = H.bf16_bits_to_f32(w).astype(np.float64)
    bf = H.bf16_bits_to_f32(bias).astype(np.float64) if bias is not None else np.zeros(x.shape[1])
    T, C = x.shape
    st = state.copy()
    q = np.zeros((T, hk, 128), np.float64); k = np.zeros_like(q); v = np.zeros((T, hv, 128))
    g = np.zeros((T, hv)); beta = np.zeros((T, hv))
    for i in range(len(cu) - 1):
        s0 = min(max(cu[i], 0), T); e0 = min(max(cu[i + 1], s0), T)
        slot = idx[i]
        in_pool = 0 <= slot < st.shape[0]
        hist = H.bf16_bits_to_f32(st[slot]).astype(np.float64) if (in_pool and ctx is not None and ctx[i] > 0) else np.zeros((3, C))
        rows = np.concatenate([hist, xf[s0:e0]], 0)
        for t in range(s0, e0):
            win = rows[t - s0: t - s0 + 4]                   # rows t-3 .. t
            u = bf + (wf * win.T).sum(1)
            y = u / (1 + np.exp(-u))
            yq, yk, yv = y[:hk * 128].reshape(hk, 128), y[hk * 128:2 * hk * 128].reshape(hk, 128), y[2 * hk * 128:].reshape(hv, 128)
            q[t] = yq / np.sqrt((yq ** 2).sum(1, keepdims=True) + 1e-6)
            k[t] = yk / np.sqrt((yk ** 2).sum(1, keepdims=True) + 1e-6)
            v[t] = yv
            av = H.bf16_bits_to_f32(a[t]).astype(np.float64) + dt_bias
            sp = np.where(av > 20, av, np.log1p(np.exp(np.minimum(av, 20))))
            g[t] = -np.exp(a_log.astype(np.float64)) * sp
            beta[t] = 1 / (1 + np.exp(-H.bf16_bits_to_f32(b[t]).astype(np.float64)))
        if in_pool:
            allrows = np.concatenate([H.bf16_bits_to_f32(st[slot]) if (ctx is not None and ctx[i] > 0) else np.zeros((3, C), np.float32),
                                      H.bf16_bits_to_f32(x[s0:e0])], 0)
            st[slot] = H.f32_to_bf16_bits(allrows[-3:].astype(np.float32))
    return q, k, v, g, beta, st


def test_oracle_conv_prep_definition():
    """The conv_prep oracle against a numpy restatement on small ragged batches with history: q, k, v within one
    bf16 ulp, g and beta within 1e-5 relative, the conv state bit for bit, rows outside the sequences untouched."""
    rng = np.random.default_rng(21)
    hk, hv, T = 1, 2, 40
    C = 2 * hk * 128 + hv * 128
    x = H.f32_to_bf16_bits(rng.standard_normal((T, C)).astype(np.float32))
    w = H.f32_to_bf16_bits((0.5 * rng.standard_normal((C, 4))).astype(np.float32))
    bias = H.f32_to_bf16_bits((0.1 * rng.standard_normal(C)).astype(np.float32))
    a_log = (0.5 * rng.standard_normal(hv)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(hv)).astype(np.float32)
    a = H.f32_to_bf16_bits((3 * rng.standard_normal((T, hv))).astype(np.float32))
    a[0, 0] = H.f32_to_bf16_bits(np.array([30.0], np.float32))[0]   # above the softplus threshold
    b = H.f32_to_bf16_bits(rng.standard_normal((T, hv)).astype(np.float32))
    state = H.f32_to_bf16_bits(rng.standard_normal((4, 3, C)).astype(np.float32))
    cu = np.array([0, 1, 3, 20, 37], np.int32)          # lengths 1, 2, 17, 17; rows 37.. outside
    idx = np.array([2, 0, 7, 1], np.int32)               # slot 7 is outside the pool
    ctx = np.array([5, 0, 3, 9], np.int32)
    for bb in (bias, None):
        q, k, v, g, beta, st = H.oracle_conv_prep(x, w, a_log, dt_bias, state, cu, a, b, idx, ctx, bias=bb, hk=hk, hv=hv)
        nq, nk, nv, ng, nb, nst = _conv_prep_numpy(x, w, a_log, dt_bias, state, cu, a, b, idx, ctx, bb, hk, hv)
        for got, want in ((q, nq), (k, nk), (v, nv)):
            gf = H.bf16_bits_to_f32(got).astype(np.float64)
            assert np.all(np.abs(gf - want) <= np.abs(want) * 2.0 ** -8 + 1e-30)
        assert np.allclose(g[:37], ng[:37], rtol=1e-5, atol=0) and np.allclose(beta[:37], nb[:37], rtol=1e-5, atol=0)
        assert np.array_equal(st, nst)
        assert not q[37:].any() and not g[37:].any()


def _attn_kv_numpy(k, v, w, pos, slots, cache, R, theta, eps, planes):
    """ridgefill_attn_kv_fill written plainly in numpy (f64 norm, f64 rotation products): an independent
    statement of the op to hold the oracle to, up to its f32 rounding order."""
    T, hkv, D = k.shape
    x = H.bf16_bits_to_f32(k).astype(np.float64)
    wf = (H.bf16_bits_to_f32(w) if w.dtype == np.uint16 else w).astype(np.float64)
    r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) / D + eps)
    kn = H.bf16_bits_to_f32(H.f32_to_bf16_bits((x * r * wf).astype(np.float32))).astype(np.float64)
    half = R // 2
    j = np.arange(half)
    inv = theta ** (-2.0 * j / R)
    p = np.stack([pos] * 3) if pos.ndim == 1 else pos
    ang = p[planes, :].T.astype(np.float64) * inv                       # [T, half]
    c, s = np.cos(ang).astype(np.float32)[:, None, :], np.sin(ang).astype(np.float32)[:, None, :]
    kr = kn.copy()
    kr[..., :half] = kn[..., :half] * c - kn[..., half:R] * s
    kr[..., half:R] = kn[..., half:R] * c + kn[..., :half] * s
    out = H.f32_to_bf16_bits(kr.astype(np.float32))
    cache = cache.copy()
    for t in range(T):
        if 0 <= slots[t] < cache.shape[1]:
            cache[0, slots[t]] = out[t]
            cache[1, slots[t]] = v[t]
    return cache, out


@pytest.mark.parametrize("mode,sections,three,w_f32", [("neox", (0, 0, 0), False, False), ("imrope", (11, 11, 10), True, True),
                                                       ("mrope", (8, 12, 12), True, False)])
def test_oracle_attn_kv_definition(mode, sections, three, w_f32):
    """The oracle's K/V cache write against a plain numpy statement of the op: k in the cache within one bf16 ulp
    plus 2^-22 of the largest k (the f32 rounding order of the norm and the rotation differs, and a rotation whose
    two products cancel keeps their f32 rounding), v, the skipped slots and untouched rows bit
    for bit, and the rotary pair -> position plane rule of each rope mode."""
    rng = np.random.default_rng(5)
    T, hkv, R, slots_n = 96, 2, 64, 150
    k = H.f32_to_bf16_bits(rng.standard_normal((T, hkv, 256)).astype(np.float32) * 3)
    v = H.f32_to_bf16_bits(rng.standard_normal((T, hkv, 256)).astype(np.float32))
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    if not w_f32:
        w = H.f32_to_bf16_bits(w)
    pos = (rng.integers(0, 40000, (3, T)) if three else np.arange(1000, 1000 + T)).astype(np.int32)
    slots = rng.permutation(slots_n)[:T].astype(np.int32)
    slots[::7] = -1
    slots[3] = slots_n + 5
    cache = rng.integers(0, 1 << 16, (2, slots_n, hkv, 256)).astype(np.uint16)
    got, ko = H.oracle_attn_kv(k, v, w, pos, slots, cache, R, 1e7, mode=mode, sections=sections, k_out=True)
    half = R // 2
    j = np.arange(half)
    if mode == "mrope":
        planes = np.where(j < sections[0], 0, np.where(j < sections[0] + sections[1], 1, 2))
    elif mode == "imrope":
        planes = np.where((j % 3 == 1) & (j < 3 * sections[1]), 1, np.where((j % 3 == 2) & (j < 3 * sections[2]), 2, 0))
    else:
        planes = np.zeros(half, int)
    want, out = _attn_kv_numpy(k, v, w, pos, slots, cache, R, 1e7, 1e-6, planes)
    def close(x, y):   # one bf16 ulp, plus the f32 rounding of a rotation product where the pair cancels
        a, b = H.bf16_bits_to_f32(x).astype(np.float64), H.bf16_bits_to_f32(y).astype(np.float64)
        return np.all(np.abs(a - b) <= np.ldexp(np.maximum(np.abs(a), np.abs(b)), -8) + np.ldexp(np.abs(b).max(), -22))
    assert close(ko, out), "k_out"
    assert np.mean(ko == out) > 0.99
    assert np.array_equal(got[1], want[1]), "v plane"
    stored = np.zeros(slots_n, bool)
    stored[slots[(slots >= 0) & (slots < slots_n)]] = True
    assert np.array_equal(got[0][~stored], cache[0][~stored]), "rows no slot names are untouched"
    assert close(got[0][stored], want[0][stored]), "k plane"
