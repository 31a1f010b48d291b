"""ridgefill_gdn_in_proj on B200: the DeltaNet block's int8 k|v in-projection with conv_prep's convolution, SiLU and
k norm in its epilogue. Checked three ways on the same seeded inputs:
  * against the two device rows it replaces (ridgefill_gemm_nt_q into the k|v columns, then
    ridgefill_gdn_conv_prep): k and v bit for bit (the epilogue sums each k head's squares in conv_prep's order);
  * against the CPU oracle's chain (oracle_gemm_nt_q, then oracle_gdn_conv_prep on the same columns): k and v within
    2 bf16 ulp, the bound conv_prep itself is held to, the tail rows bit for bit;
  * the conv-state update that follows (ridgefill_gdn_conv_prep with columns = 0 over the tail rows) against the
    oracle's state bit for bit, and its gates against the oracle.
Rows outside every sequence keep their contents; tail rows other than each sequence's last three are not written.
Shapes: ragged batches with history (sequences of one and two rows, a slot outside the pool, boundaries on and off
the 125-row CTA tiles), a row count that is not a tile multiple, an odd number of heads (a half-empty last column
tile), and the real layer (16 k, 32 v heads x 128, K 2,048)."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu
SENT = 0x5A5A


def _inputs(seed, T, hk, hv, K, slots=4, bias=True):
    rng = np.random.default_rng(seed)
    N = (hk + hv) * 128
    return {
        "a": rng.integers(-127, 128, (T, K), dtype=np.int8),
        "sa": rng.uniform(1e-3, 3e-3, (T, 1)).astype(np.float32),
        "b": rng.integers(-127, 128, (N, K), dtype=np.int8),
        "sb": rng.uniform(1e-3, 3e-3, (1, N)).astype(np.float32),
        "w": H.f32_to_bf16_bits((0.5 * rng.standard_normal((N, 4))).astype(np.float32)),
        "bias": H.f32_to_bf16_bits((0.1 * rng.standard_normal(N)).astype(np.float32)) if bias else None,
        "state": H.f32_to_bf16_bits(rng.standard_normal((slots, 3, N)).astype(np.float32)),
        "a_log": (0.5 * rng.standard_normal(hv)).astype(np.float32),
        "dt_bias": (0.5 * rng.standard_normal(hv)).astype(np.float32),
        "ga": H.f32_to_bf16_bits((3 * rng.standard_normal((T, hv))).astype(np.float32)),
        "gb": H.f32_to_bf16_bits(rng.standard_normal((T, hv)).astype(np.float32)),
    }


def _t16(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def _u16(t):
    return t.cpu().numpy().view(np.uint16)


def _in_proj(product_lib, torch, d, cu, idx, ctx, hk, hv, group=None, tail=None):
    """The fused row. Returns (rc, k, v, tail) with k, v, tail sentinel-filled before the call."""
    T, K = d["a"].shape
    N = (hk + hv) * 128
    A, SA, B, SB = (torch.from_numpy(d[n]).cuda() for n in ("a", "sa", "b", "sb"))
    W, ST = _t16(torch, d["w"]), _t16(torch, d["state"])
    B0 = _t16(torch, d["bias"]) if d["bias"] is not None else None
    CU = torch.tensor(np.asarray(cu, np.int32)).cuda()
    I = torch.tensor(np.asarray(idx, np.int32)).cuda()
    CX = torch.tensor(np.asarray(ctx, np.int32)).cuda() if ctx is not None else None
    Kt = torch.full((T, hk, 128), SENT, dtype=torch.int16, device="cuda")
    Vt = torch.full((T, hv, 128), SENT, dtype=torch.int16, device="cuda")
    TL = torch.full((T, N), SENT, dtype=torch.int16, device="cuda") if tail is None else tail
    ops = [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(W, abi.BF16), H.dev(B0, abi.BF16) if B0 is not None else abi.absent(),
           H.dev(ST, abi.BF16), H.dev(CU), H.dev(I), H.dev(CX) if CX is not None else abi.absent(), H.dev(Kt, abi.BF16),
           H.dev(Vt, abi.BF16), H.dev(TL, abi.BF16)]
    params = [H.pint("M", T), H.pint("N", N), H.pint("K", K), H.pint("n_head_k", hk), H.pint("n_head_v", hv),
              H.pint("group", group or K), H.pstr("dtype", "i8a8")]
    rc = H.launch(product_lib, "ridgefill_gdn_in_proj", ops, params)
    return rc, _u16(Kt), _u16(Vt), _u16(TL)


def _full(d, x_kv, hk, hv):
    """conv_prep's operands over C = 2 Hk 128 + Hv 128 channels: q columns zero (taps, bias, state), then k|v."""
    T = x_kv.shape[0]
    Cq = hk * 128
    z = lambda *s: np.zeros(s, np.uint16)   # noqa: E731
    x = np.concatenate([z(T, Cq), x_kv], 1)
    w = np.concatenate([z(Cq, 4), d["w"]], 0)
    bias = np.concatenate([z(Cq), d["bias"]]) if d["bias"] is not None else None
    st = np.concatenate([z(d["state"].shape[0], 3, Cq), d["state"]], 2)
    return x, w, bias, st


def _conv_prep_dev(product_lib, torch, d, x, w, bias, st, cu, idx, ctx, hk, hv, columns=1):
    T = x.shape[0]
    X, Wt, ST = _t16(torch, x), _t16(torch, w), _t16(torch, st)
    B0 = _t16(torch, bias) if bias is not None else None
    AL, DT = torch.from_numpy(d["a_log"]).cuda(), torch.from_numpy(d["dt_bias"]).cuda()
    CU = torch.tensor(np.asarray(cu, np.int32)).cuda()
    Ga, Gb = _t16(torch, d["ga"]), _t16(torch, d["gb"])
    I = torch.tensor(np.asarray(idx, np.int32)).cuda()
    CX = torch.tensor(np.asarray(ctx, np.int32)).cuda() if ctx is not None else None
    Kt = torch.full((T, hk, 128), SENT, dtype=torch.int16, device="cuda")
    Vt = torch.full((T, hv, 128), SENT, dtype=torch.int16, device="cuda")
    G = torch.full((T, hv), -7.0, dtype=torch.float32, device="cuda")
    BE = torch.full((T, hv), -7.0, dtype=torch.float32, device="cuda")
    ops = [H.dev(X, abi.BF16), H.dev(Wt, abi.BF16), H.dev(B0, abi.BF16) if B0 is not None else abi.absent(), H.dev(AL),
           H.dev(DT), H.dev(ST, abi.BF16), H.dev(CU), H.dev(Ga, abi.BF16), H.dev(Gb, abi.BF16), H.dev(I),
           H.dev(CX) if CX is not None else abi.absent(), abi.absent(), H.dev(Kt, abi.BF16), H.dev(Vt, abi.BF16),
           H.dev(G), H.dev(BE)]
    params = [H.pint("M", T), H.pint("n_head_k", hk), H.pint("n_head_v", hv), H.pint("head_k", 128), H.pint("head_v", 128),
              H.pint("conv", 4), H.pint("columns", columns)]
    rc = H.launch(product_lib, "ridgefill_gdn_conv_prep", ops, params)
    assert rc == abi.OK
    return _u16(Kt), _u16(Vt), G.cpu().numpy(), BE.cpu().numpy(), _u16(ST)


def _within_2ulp(name, x, y):
    same = x == y
    xf, yf = H.bf16_bits_to_f32(x).astype(np.float64), H.bf16_bits_to_f32(y).astype(np.float64)
    close = np.abs(xf - yf) <= np.ldexp(np.maximum(np.abs(xf), np.abs(yf)), -7)
    assert np.all(same | close), f"{name}: {int((~(same | close)).sum())} outside 2 bf16 ulp"


def _tail_rows(cu, T):
    """Rows that are among their sequence's last three (clamped bounds, the ops' rule)."""
    rows = np.zeros(T, bool)
    for i in range(len(cu) - 1):
        a = min(max(cu[i], 0), T)
        b = min(max(cu[i + 1], a), T)
        rows[max(a, b - 3):b] = True
    return rows


def _check(product_lib, torch, d, cu, idx, ctx, hk, hv):
    T, K = d["a"].shape
    rc, k, v, tail = _in_proj(product_lib, torch, d, cu, idx, ctx, hk, hv)
    assert rc == abi.OK
    # the oracle's chain
    y = H.oracle_gemm(d["a"], d["sa"], d["b"], d["sb"], group=K)
    x, w, bias, st = _full(d, y, hk, hv)
    init = (np.full((T, hk, 128), SENT, np.uint16), np.full((T, hk, 128), SENT, np.uint16), np.full((T, hv, 128), SENT, np.uint16),
            np.full((T, hv), -7.0, np.float32), np.full((T, hv), -7.0, np.float32))
    want = H.oracle_conv_prep(x, w, d["a_log"], d["dt_bias"], st, cu, d["ga"], d["gb"], np.asarray(idx).reshape(-1), ctx,
                              bias=bias, hk=hk, hv=hv, out=init)
    _within_2ulp("k", k, want[1])
    _within_2ulp("v", v, want[2])
    rows = _tail_rows(cu, T)
    assert np.array_equal(tail[rows], y[rows]), "tail rows"
    assert np.all(tail[~rows] == SENT), "rows other than the sequences' last three are not written"
    # the two device rows it replaces: k and v bit for bit
    pk, pv, _, _, _ = _conv_prep_dev(product_lib, torch, d, x, w, bias, st, cu, idx, ctx, hk, hv)
    assert np.array_equal(k, pk), f"k: {int((k != pk).sum())} differ from gemm + conv_prep"
    assert np.array_equal(v, pv), f"v: {int((v != pv).sum())} differ from gemm + conv_prep"
    # the conv-state update and the gates after it, over x holding only the tail rows
    xt = x.copy()
    xt[:, hk * 128:] = np.where(rows[:, None], tail, 0x7FC0)   # rows the update must not read: NaN
    _, _, g, beta, st_new = _conv_prep_dev(product_lib, torch, d, xt, w, bias, st, cu, idx, ctx, hk, hv, columns=0)
    assert np.array_equal(st_new, want[5]), "conv state"
    assert np.allclose(g, want[3], rtol=1e-5, atol=0) and np.allclose(beta, want[4], rtol=1e-5, atol=0), "gates"


def test_ragged_batch_with_history(cuda, product_lib):
    torch = cuda
    hk, hv = 2, 4
    d = _inputs(3, 600, hk, hv, 256, slots=10)
    # boundaries on a CTA tile's edge (125, 375), on a pair tile's (250, 500) and off them (1, 3, 440); rows 585..
    # outside every sequence; one slot per sequence (the update of a shared slot would race), slot 11 outside the pool
    cu = [0, 1, 3, 125, 250, 375, 440, 500, 585]
    idx = [2, 0, 11, 1, 3, 5, 6, 7]
    ctx = [4, 0, 6, 2, 0, 1, 3, 5]
    for bias in (True, False):
        _check(product_lib, torch, dict(d, bias=d["bias"] if bias else None), cu, idx, ctx, hk, hv)


def test_without_ctx_lens_and_odd_heads(cuda, product_lib):
    """No ctx_lens (every sequence starts fresh); 1 k and 2 v heads: N 384, so the pair's last column tile is half
    empty; idx as [n_seq, 1]."""
    torch = cuda
    hk, hv = 1, 2
    d = _inputs(5, 517, hk, hv, 384)
    cu, idx = [0, 40, 291, 517], [[1], [0], [2]]
    _check(product_lib, torch, d, cu, idx, None, hk, hv)


def test_layer_shape(cuda, product_lib):
    """The DeltaNet layer's k|v shape: 16 k, 32 v heads x 128 (N 6,144), K 2,048, two sequences over 4,096 rows, the
    second continuing a context."""
    torch = cuda
    hk, hv = 16, 32
    d = _inputs(7, 4096, hk, hv, 2048, slots=2)
    _check(product_lib, torch, d, [0, 1000, 4096], [0, 1], [0, 100], hk, hv)


def test_tail_view_of_the_mixed_buffer(cuda, product_lib):
    """`tail` as the k|v column view of a wider [T, C] buffer (the block's mixed projection): only its tail rows'
    k|v columns change."""
    torch = cuda
    hk, hv = 2, 2
    T, K = 300, 256
    d = _inputs(11, T, hk, hv, K)
    cu = [0, 177, 300]
    C = 2 * hk * 128 + hv * 128
    mixed = torch.full((T, C), SENT, dtype=torch.int16, device="cuda")
    rc, k, v, _ = _in_proj(product_lib, torch, d, cu, [0, 1], [1, 0], hk, hv, tail=mixed[:, hk * 128:])
    assert rc == abi.OK
    got = _u16(mixed)
    y = H.oracle_gemm(d["a"], d["sa"], d["b"], d["sb"], group=K)
    rows = _tail_rows(cu, T)
    assert np.array_equal(got[rows, hk * 128:], y[rows])
    assert np.all(got[~rows] == SENT) and np.all(got[:, :hk * 128] == SENT)


def test_refusals(cuda, product_lib):
    torch = cuda
    hk, hv = 1, 1
    d = _inputs(1, 16, hk, hv, 256)
    assert _in_proj(product_lib, torch, d, [0, 16], [0], None, hk, hv)[0] == abi.OK
    assert _in_proj(product_lib, torch, d, [0, 16], [0], None, hk, hv, group=128)[0] == abi.E_UNSUPPORTED   # per-row scales only
    bad = dict(d, w=np.zeros((2 * 256, 4), np.uint16))   # taps of the wrong channel count
    assert _in_proj(product_lib, torch, bad, [0, 16], [0], None, hk, hv)[0] == abi.E_SHAPE
    ops = [abi.absent()] * 13
    params = [H.pint("M", 16), H.pint("N", 256), H.pint("K", 256), H.pint("n_head_k", 1), H.pint("n_head_v", 1),
              H.pint("group", 256), H.pstr("dtype", "i8a8")]
    assert H.launch(product_lib, "ridgefill_gdn_in_proj", ops, params) == abi.E_INVAL


@pytest.mark.parametrize("span", [(0, 8, 0, 16), (8, 16, 16, 32), (5, 11, 10, 22)])
def test_head_span_equals_its_slice_of_the_full_call(cuda, product_lib, span):
    """A tensor-parallel rank's call (its k heads k0..k1 and v heads v0..v1: the weight rows, scales, taps and conv
    state of those channels) gives its slice of the full call's k and v, and its tail columns, bit for bit."""
    torch = cuda
    hk, hv = 16, 32
    k0, k1, v0, v1 = span
    d = _inputs(13, 640, hk, hv, 2048, slots=3)
    cu, idx, ctx = [0, 200, 640], [2, 0], [1, 0]
    rc, k, v, tail = _in_proj(product_lib, torch, d, cu, idx, ctx, hk, hv)
    assert rc == abi.OK
    ch = np.concatenate([np.arange(k0 * 128, k1 * 128), np.arange((hk + v0) * 128, (hk + v1) * 128)])
    part = dict(d, b=np.ascontiguousarray(d["b"][ch]), sb=np.ascontiguousarray(d["sb"][:, ch]),
                w=np.ascontiguousarray(d["w"][ch]), bias=np.ascontiguousarray(d["bias"][ch]),
                state=np.ascontiguousarray(d["state"][:, :, ch]))
    rc, kp, vp, tp = _in_proj(product_lib, torch, part, cu, idx, ctx, k1 - k0, v1 - v0)
    assert rc == abi.OK
    assert np.array_equal(kp, k[:, k0:k1]), "k"
    assert np.array_equal(vp, v[:, v0:v1]), "v"
    assert np.array_equal(tp, tail[:, ch]), "tail"


def test_repeated_calls_agree(cuda, product_lib):
    """The same call twice gives the same bits (no order-dependent step in the epilogue)."""
    torch = cuda
    d = _inputs(17, 3000, 16, 32, 2048)
    cu, idx, ctx = [0, 700, 3000], [1, 0], [1, 1]
    first = _in_proj(product_lib, torch, d, cu, idx, ctx, 16, 32)
    for _ in range(3):
        again = _in_proj(product_lib, torch, d, cu, idx, ctx, 16, 32)
        for a, b in zip(first[1:], again[1:]):
            assert np.array_equal(a, b)
