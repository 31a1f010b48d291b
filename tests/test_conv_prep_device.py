"""ridgefill_gdn_conv_prep on B200 against the CPU oracle (oracle/ridgefill_oracle.cpp oracle_gdn_conv_prep): q, k, v
within 2 bf16 ulp (the bf16 bound stated for this library's outputs; the device's exp and the warp's sum of squares
may differ from the host's in the last f32 bits), g and beta within 1e-5 relative (f32 exp / log1p), the conv state
bit for bit, and rows outside every sequence untouched. Shapes: ragged batches with history, short sequences (one
and two rows), slots outside the pool, a bias and none, and the real layer (16 qk / 32 v heads x 128)."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu
SENT = 0x5A5A


def _case(seed, T, hk, hv, slots=4, bias=True):
    rng = np.random.default_rng(seed)
    C = 2 * hk * 128 + hv * 128
    d = {
        "x": H.f32_to_bf16_bits(rng.standard_normal((T, C)).astype(np.float32)),
        "w": H.f32_to_bf16_bits((0.5 * rng.standard_normal((C, 4))).astype(np.float32)),
        "bias": H.f32_to_bf16_bits((0.1 * rng.standard_normal(C)).astype(np.float32)) if bias else None,
        "a_log": (0.5 * rng.standard_normal(hv)).astype(np.float32),
        "dt_bias": (0.5 * rng.standard_normal(hv)).astype(np.float32),
        "a": H.f32_to_bf16_bits((3 * rng.standard_normal((T, hv))).astype(np.float32)),
        "b": H.f32_to_bf16_bits(rng.standard_normal((T, hv)).astype(np.float32)),
        "state": H.f32_to_bf16_bits(rng.standard_normal((slots, 3, C)).astype(np.float32)),
    }
    return d


def _run(product_lib, torch, d, cu, idx, ctx, hk, hv, with_q=True):
    T, C = d["x"].shape
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    X, W = t16(d["x"]), t16(d["w"])
    B0 = t16(d["bias"]) if d["bias"] is not None else None
    AL, DT = torch.from_numpy(d["a_log"]).cuda(), torch.from_numpy(d["dt_bias"]).cuda()
    ST = t16(d["state"])
    CU = torch.tensor(np.asarray(cu, np.int32)).cuda()
    A, Bg = t16(d["a"]), t16(d["b"])
    I = torch.tensor(np.asarray(idx, np.int32)).cuda()
    CX = torch.tensor(np.asarray(ctx, np.int32)).cuda() if ctx is not None else None
    Q = torch.full((T, hk, 128), SENT, dtype=torch.int16, device="cuda")
    K = torch.full((T, hk, 128), SENT, dtype=torch.int16, device="cuda")
    V = torch.full((T, hv, 128), SENT, dtype=torch.int16, device="cuda")
    G = torch.full((T, hv), -7.0, dtype=torch.float32, device="cuda")
    BE = torch.full((T, hv), -7.0, dtype=torch.float32, device="cuda")
    ops = [H.dev(X, abi.BF16), H.dev(W, abi.BF16), H.dev(B0, abi.BF16) if B0 is not None else abi.absent(), H.dev(AL),
           H.dev(DT), H.dev(ST, abi.BF16), H.dev(CU), H.dev(A, abi.BF16), H.dev(Bg, abi.BF16), H.dev(I),
           H.dev(CX) if CX is not None else abi.absent(), H.dev(Q, abi.BF16) if with_q else abi.absent(), H.dev(K, abi.BF16),
           H.dev(V, abi.BF16),
           H.dev(G), H.dev(BE)]
    params = [H.pint("M", T), H.pint("n_head_k", hk), H.pint("n_head_v", hv), H.pint("head_k", 128), H.pint("head_v", 128),
              H.pint("conv", 4)]
    rc = H.launch(product_lib, "ridgefill_gdn_conv_prep", ops, params)
    u16 = lambda t: t.cpu().numpy().view(np.uint16)   # noqa: E731
    return rc, u16(Q), u16(K), u16(V), G.cpu().numpy(), BE.cpu().numpy(), u16(ST)


def _check(d, got, cu, idx, ctx, hk, hv):
    T = d["x"].shape[0]
    init = (np.full((T, hk, 128), SENT, np.uint16), np.full((T, hk, 128), SENT, np.uint16), np.full((T, hv, 128), SENT, np.uint16),
            np.full((T, hv), -7.0, np.float32), np.full((T, hv), -7.0, np.float32))
    want = H.oracle_conv_prep(d["x"], d["w"], d["a_log"], d["dt_bias"], d["state"], cu, d["a"], d["b"], idx, ctx, bias=d["bias"],
                              hk=hk, hv=hv, out=init)
    rc, q, k, v, g, beta, st = got
    assert rc == abi.OK
    for name, x, y in (("q", q, want[0]), ("k", k, want[1]), ("v", v, want[2])):
        same = x == y
        xf, yf = H.bf16_bits_to_f32(x).astype(np.float64), H.bf16_bits_to_f32(y).astype(np.float64)
        close = np.abs(xf - yf) <= np.ldexp(np.maximum(np.abs(xf), np.abs(yf)), -7)
        assert np.all(same | close), f"{name}: {int((~(same | close)).sum())} outside 2 bf16 ulp"
    for name, x, y in (("g", g, want[3]), ("beta", beta, want[4])):
        assert np.allclose(x, y, rtol=1e-5, atol=0), name
    assert np.array_equal(st, want[5]), "conv state"


def test_ragged_batch_with_history(cuda, product_lib):
    torch = cuda
    hk, hv = 2, 4
    d = _case(3, 200, hk, hv)
    cu = [0, 1, 3, 70, 133, 190]      # lengths 1, 2, 67, 63, 57; rows 190.. outside every sequence
    idx = [2, 0, 9, 1, 3]             # slot 9 lies outside the pool: zero history, nothing written
    ctx = [4, 0, 6, 2, 0]
    for bias in (True, False):
        dd = dict(d, bias=d["bias"] if bias else None)
        _check(dd, _run(product_lib, torch, dd, cu, idx, ctx, hk, hv), cu, idx, ctx, hk, hv)


def test_without_ctx_lens_every_sequence_starts_fresh(cuda, product_lib):
    torch = cuda
    hk, hv = 1, 2
    d = _case(5, 97, hk, hv)
    cu, idx = [0, 40, 97], [[1], [0]]
    _check(d, _run(product_lib, torch, d, cu, idx, None, hk, hv), cu, np.asarray(idx).reshape(-1), None, hk, hv)


def test_layer_shape(cuda, product_lib):
    """The DeltaNet layer's shape: 16 qk / 32 v heads x 128 (C 8,192), one 4,096-row sequence continuing a context."""
    torch = cuda
    hk, hv = 16, 32
    d = _case(7, 4096, hk, hv, slots=2)
    cu, idx, ctx = [0, 4096], [1], [100]
    _check(d, _run(product_lib, torch, d, cu, idx, ctx, hk, hv), cu, idx, ctx, hk, hv)


def test_split_calls_carry_the_window(cuda, product_lib):
    """A sequence run as two calls (the second continuing the first through the conv state) gives the one call's
    q, k, v, g, beta bit for bit."""
    torch = cuda
    hk, hv = 2, 2
    d = _case(11, 300, hk, hv)
    one = _run(product_lib, torch, d, [0, 300], [0], [1], hk, hv)
    first = dict(d, x=d["x"][:117], a=d["a"][:117], b=d["b"][:117])
    p1 = _run(product_lib, torch, first, [0, 117], [0], [1], hk, hv)
    second = dict(d, x=d["x"][117:], a=d["a"][117:], b=d["b"][117:], state=p1[6])
    p2 = _run(product_lib, torch, second, [0, 183], [0], [1], hk, hv)
    for i in range(1, 6):
        assert np.array_equal(np.concatenate([p1[i], p2[i]]), one[i])
    assert np.array_equal(p2[6], one[6])


def test_refusals(cuda, product_lib):
    torch = cuda
    d = _case(1, 8, 1, 1)
    rc = _run(product_lib, torch, d, [0, 8], [0], None, 1, 1)[0]
    assert rc == abi.OK
    X = torch.zeros((8, 384), dtype=torch.int16, device="cuda")
    params = [H.pint("M", 8), H.pint("n_head_k", 1), H.pint("n_head_v", 1), H.pint("head_k", 128), H.pint("head_v", 128),
              H.pint("conv", 3)]
    ops = [H.dev(X, abi.BF16)] + [abi.absent()] * 15
    assert H.launch(product_lib, "ridgefill_gdn_conv_prep", ops, params) == abi.E_INVAL   # operands missing


def test_conv_prep_feeds_the_fill(cuda, product_lib):
    """The block's path on the device: conv_prep's q, k, v, g, beta straight into ridgefill_gdn_fill (state-only and
    with o). Against the sequential rule on those same device outputs the fill keeps its own bounds (state 1e-3
    relative L2, o 1e-2); against the oracle's whole chain (oracle conv_prep, then the rule) the two-ulp differences
    conv_prep may carry are allowed to grow to 1e-2 in the state and 2e-2 in o."""
    torch = cuda
    hk, hv, T = 2, 4, 300
    d = _case(17, T, hk, hv, bias=True)
    d["a_log"] = (0.3 * np.random.default_rng(1).standard_normal(hv) - 1.0).astype(np.float32)
    cu, idx, ctx = [0, 130, 300], [0, 1], [0, 3]
    got = _run(product_lib, torch, d, cu, idx, ctx, hk, hv)
    assert got[0] == abi.OK
    q, k, v, g, beta = got[1:6]
    want = H.oracle_conv_prep(d["x"], d["w"], d["a_log"], d["dt_bias"], d["state"], cu, d["a"], d["b"], idx, ctx, bias=d["bias"],
                              hk=hk, hv=hv)
    state0 = (0.1 * np.random.default_rng(2).standard_normal((2, hv, 128, 128))).astype(np.float32)
    from test_gdn_device import run_fill, STATE_TOL, O_TOL
    for with_o in (False, True):
        rc, got_state, got_o = run_fill(product_lib, torch, k, v, g, beta, state0, [0, 1], cu, hk, hv,
                                        q=q if with_o else None, o=with_o)
        assert rc == abi.OK
        same_state, same_o = H.oracle_gdn(k, v, g, beta, state0, [0, 1], cu, q=q if with_o else None)
        chain_state, chain_o = H.oracle_gdn(want[1], want[2], want[3], want[4], state0, [0, 1], cu,
                                            q=want[0] if with_o else None)
        for sl in (0, 1):
            assert H.rel_l2(got_state[sl], same_state[sl]) <= STATE_TOL
            assert H.rel_l2(got_state[sl], chain_state[sl]) <= 1e-2
        if with_o:
            o = H.bf16_bits_to_f32(got_o)
            assert H.rel_l2(o, H.bf16_bits_to_f32(same_o)) <= O_TOL
            assert H.rel_l2(o, H.bf16_bits_to_f32(chain_o)) <= 2e-2


def test_block_input_path_from_h(cuda, product_lib):
    """The DeltaNet block from its input h on the device, every stage a row of this library fed the previous row's
    device output: activation codes of h (group 128), the int8 mixed projection h -> x [T, 2 Hk 128 + Hv 128] with
    no bias, the bf16 a|b projection h -> [T, 2 Hv] (a and b read as column views of that one output), conv_prep,
    and the fill with o. Each stage is checked against the oracle on the same inputs: codes, scales and x bit for
    bit, a|b within the bf16 GEMM bound, q, k, v within 2 bf16 ulp, g and beta within 1e-5, the state within 1e-3
    relative L2 and o within 1e-2."""
    torch = cuda
    rng = np.random.default_rng(23)
    T, d, hk, hv = 300, 256, 2, 4
    C = 2 * hk * 128 + hv * 128
    h = H.f32_to_bf16_bits(rng.standard_normal((T, d)).astype(np.float32))
    codes, wscale = H.oracle_quantise_weight((rng.standard_normal((C, d)) / np.sqrt(d)).astype(np.float32))
    scale_kn = np.ascontiguousarray(H.bf16_bits_to_f32(wscale).T)
    w_ab = H.f32_to_bf16_bits((2 * rng.standard_normal((2 * hv, d)) / np.sqrt(d)).astype(np.float32))
    conv = _case(24, T, hk, hv, bias=False)
    conv["a_log"] = (0.3 * rng.standard_normal(hv) - 1.0).astype(np.float32)
    cu, idx, ctx = [0, 170, 300], [2, 0], [4, 0]
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    u16 = lambda t: t.cpu().numpy().view(np.uint16)   # noqa: E731

    Hd = t16(h)
    Qa = torch.empty((T, d), dtype=torch.int8, device="cuda")
    Sa = torch.empty((T, d // 128), dtype=torch.float32, device="cuda")
    assert H.launch(product_lib, "ridgefill_quant_act_i8g", [H.dev(Hd, abi.BF16), H.dev(Qa), H.dev(Sa)],
                    [H.pint("M", T), H.pint("n", d), H.pint("group", 128), H.pstr("dtype", "bf16")]) == abi.OK
    q_ref, s_ref = H.oracle_quant(h, 128)
    assert np.array_equal(Qa.cpu().numpy(), q_ref) and np.array_equal(Sa.cpu().numpy(), s_ref)

    Wc, SW = torch.from_numpy(codes).cuda(), torch.from_numpy(scale_kn).cuda()
    X = torch.full((T, C), SENT, dtype=torch.int16, device="cuda")
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", [H.dev(Qa), H.dev(Sa), H.dev(Wc), H.dev(SW), abi.absent(),
                                                              H.dev(X, abi.BF16), abi.absent()],
                    H.gemm_params(T, C, d, 128)) == abi.OK
    x = u16(X)
    assert np.array_equal(x, H.oracle_gemm(q_ref, s_ref, codes, scale_kn, group=128))

    Wab, Bz = t16(w_ab), torch.zeros(2 * hv, dtype=torch.int16, device="cuda")
    AB = torch.full((T, 2 * hv), SENT, dtype=torch.int16, device="cuda")
    assert H.launch(product_lib, "ridgefill_gemm_nt_bias", [H.dev(Hd, abi.BF16), H.dev(Wab, abi.BF16), H.dev(Bz, abi.BF16),
                                                            abi.absent(), H.dev(AB, abi.BF16)],
                    [H.pint("M", T), H.pint("N", 2 * hv), H.pint("K", d), H.pstr("dtype", "bf16")]) == abi.OK
    ab = u16(AB)
    want_ab, _ = H.oracle_gemm_bias(h, w_ab, np.zeros(2 * hv, np.uint16))
    xf, yf = H.bf16_bits_to_f32(ab).astype(np.float64), H.bf16_bits_to_f32(want_ab).astype(np.float64)
    rms = np.sqrt(np.mean(yf ** 2))
    assert np.all(np.abs(xf - yf) <= 2.0 ** -7 * np.maximum(np.abs(xf), np.abs(yf)) + 2.0 ** -9 * rms)

    Wcv = t16(conv["w"])
    AL, DT = torch.from_numpy(conv["a_log"]).cuda(), torch.from_numpy(conv["dt_bias"]).cuda()
    ST = t16(conv["state"])
    CU, I, CX = (torch.tensor(np.asarray(v_, np.int32)).cuda() for v_ in (cu, idx, ctx))
    q = torch.full((T, hk, 128), SENT, dtype=torch.int16, device="cuda")
    k, v = torch.full_like(q, SENT), torch.full((T, hv, 128), SENT, dtype=torch.int16, device="cuda")
    g = torch.full((T, hv), -7.0, dtype=torch.float32, device="cuda")
    beta = torch.full_like(g, -7.0)
    assert H.launch(product_lib, "ridgefill_gdn_conv_prep",
                    [H.dev(X, abi.BF16), H.dev(Wcv, abi.BF16), abi.absent(), H.dev(AL), H.dev(DT), H.dev(ST, abi.BF16),
                     H.dev(CU), H.dev(AB[:, :hv], abi.BF16), H.dev(AB[:, hv:], abi.BF16), H.dev(I), H.dev(CX),
                     H.dev(q, abi.BF16), H.dev(k, abi.BF16), H.dev(v, abi.BF16), H.dev(g), H.dev(beta)],
                    [H.pint("M", T), H.pint("n_head_k", hk), H.pint("n_head_v", hv), H.pint("head_k", 128),
                     H.pint("head_v", 128), H.pint("conv", 4)]) == abi.OK
    d_ = dict(conv, x=x, a=np.ascontiguousarray(ab[:, :hv]), b=np.ascontiguousarray(ab[:, hv:]))
    _check(d_, (abi.OK, u16(q), u16(k), u16(v), g.cpu().numpy(), beta.cpu().numpy(), u16(ST)), cu, idx, ctx, hk, hv)

    from test_gdn_device import STATE_TOL, O_TOL
    state0 = (0.1 * rng.standard_normal((3, hv, 128, 128))).astype(np.float32)
    S = torch.from_numpy(state0.copy()).cuda()
    O = torch.zeros((T, hv, 128), dtype=torch.int16, device="cuda")
    assert H.launch(product_lib, "ridgefill_gdn_fill", [H.dev(q, abi.BF16), H.dev(k, abi.BF16), H.dev(v, abi.BF16), H.dev(g),
                                                        H.dev(beta), H.dev(S), H.dev(I), H.dev(CU), H.dev(O, abi.BF16)],
                    H.gdn_params(T, hk, hv)) == abi.OK
    want_s, want_o = H.oracle_gdn(u16(k), u16(v), g.cpu().numpy(), beta.cpu().numpy(), state0, idx, cu, q=u16(q))
    got_s = S.cpu().numpy()
    for sl in idx:
        assert H.rel_l2(got_s[sl], want_s[sl]) <= STATE_TOL
    assert np.array_equal(got_s[1], state0[1])   # the slot no sequence names
    assert H.rel_l2(H.bf16_bits_to_f32(u16(O)), H.bf16_bits_to_f32(want_o)) <= O_TOL


@pytest.mark.parametrize("hk,hv", [(2, 4), (3, 6)])
def test_without_q_the_rest_is_bit_for_bit_the_same(cuda, product_lib, hk, hv):
    """With no q operand (what a state-only fill needs) the q columns are not computed and x's q columns are read
    only in each sequence's last three rows (for the conv state): k, v, g, beta and the conv state are bit for bit
    the call with q's, here with x's q columns garbage everywhere else. hk odd puts a q and a k column in one pair."""
    torch = cuda
    d = _case(41, 250, hk, hv)
    cu, idx, ctx = [0, 2, 90, 250], [1, 3, 0], [2, 0, 5]
    with_q = _run(product_lib, torch, d, cu, idx, ctx, hk, hv)
    x = d["x"].copy()
    keep = np.zeros(x.shape[0], bool)
    for a_, b_ in zip(cu[:-1], cu[1:]):
        keep[max(a_, b_ - 3):b_] = True
    x[~keep, :hk * 128] = 0x7FC1   # q columns outside the kept rows: NaN bits nothing may read
    no_q = _run(product_lib, torch, dict(d, x=x), cu, idx, ctx, hk, hv, with_q=False)
    assert with_q[0] == no_q[0] == abi.OK
    for a_, b_ in zip(with_q[2:], no_q[2:]):
        assert np.array_equal(np.asarray(a_).view(np.uint32 if a_.dtype == np.float32 else np.uint16),
                              np.asarray(b_).view(np.uint32 if b_.dtype == np.float32 else np.uint16))
