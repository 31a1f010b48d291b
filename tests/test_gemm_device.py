"""The int8 projector on B200 (ridgefill_gemm_nt_q, ridgefill_gemm_nt_q_bias, ridgefill_quant_act_i8g)
against the CPU oracle: the activation codes and scales bit for bit, every int32 block sum bit for bit,
and the bf16 outputs bit for bit (the f32 fold is defined exactly, in block order, with one fma a block:
oracle/ridgefill_oracle.cpp oracle_gemm_nt_q). Shapes: the late pass's per-column projector (group = K),
the folder's i8*bf16[1x128] encoding (group 128) at the real model shape N 2,560 / K 10,240, row
counts that are not tile multiples, and the folder path through the row's own stored-form hooks."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu


def _quant_inputs(rng, M, K):
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0, :128] = 0.0                              # an all-zero group
    x[min(1, M - 1), 128:256] = np.round(x[min(1, M - 1), 128:256] * 2) / 2   # halves: ties
    return H.f32_to_bf16_bits(x)


@pytest.mark.parametrize("M,K,group", [(1, 256, 128), (37, 2048, 128), (300, 2048, 2048), (64, 10240, 128), (5, 10240, 10240),
                                       (7, 4096, 512), (3, 2048, 8), (9, 6144, 1024), (2, 2048, 32), (4, 4096, 4096),
                                       (6, 1024, 256),
                                       # more (row, group) items than warps: each warp codes one item while the next
                                       # one's columns are copied into its other shared-memory slot
                                       (20000, 2048, 2048), (9000, 4096, 512), (3000, 2048, 256)])
def test_quantiser_matches_oracle(cuda, product_lib, M, K, group):
    torch = cuda
    rng = np.random.default_rng(M + K)
    xb = _quant_inputs(rng, M, K)
    q_ref, s_ref = H.oracle_quant(xb, group)
    x = torch.from_numpy(xb.view(np.int16)).cuda()
    q = torch.full((M, K), 99, dtype=torch.int8, device="cuda")
    s = torch.full((M, K // group), -1.0, dtype=torch.float32, device="cuda")
    rc = H.launch(product_lib, "ridgefill_quant_act_i8g", [H.dev(x, abi.BF16), H.dev(q), H.dev(s)],
                  [H.pint("M", M), H.pint("n", K), H.pint("group", group), H.pstr("dtype", "bf16")])
    assert rc == abi.OK
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_quantiser_near_half_integers(cuda, product_lib):
    """The codes are rint(x / s) with the quotient correctly rounded. Rows whose x * (1 / s) rounds to a
    different integer than x / s (both in f32) are present here by construction of the data (checked), and
    the device's codes still equal the oracle's bit for bit."""
    torch = cuda
    M, K, group = 512, 2048, 2048
    rng = np.random.default_rng(5)
    xb = H.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    xf = H.bf16_bits_to_f32(xb)
    sc = (np.abs(xf).max(1) / np.float32(127)).astype(np.float32)
    naive = np.rint((xf * (np.float32(1) / sc)[:, None]).astype(np.float32))
    exact = np.rint((xf / sc[:, None]).astype(np.float32))
    assert int((naive != exact).sum()) >= 100   # the data does reach the half-integer cases
    q_ref, s_ref = H.oracle_quant(xb, group)
    x = torch.from_numpy(xb.view(np.int16)).cuda()
    q = torch.full((M, K), 99, dtype=torch.int8, device="cuda")
    s = torch.full((M, 1), -1.0, dtype=torch.float32, device="cuda")
    rc = H.launch(product_lib, "ridgefill_quant_act_i8g", [H.dev(x, abi.BF16), H.dev(q), H.dev(s)],
                  [H.pint("M", M), H.pint("n", K), H.pint("group", group), H.pstr("dtype", "bf16")])
    assert rc == abi.OK
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def _gemm_case(rng, M, N, K, group):
    a = rng.integers(-127, 128, (M, K)).astype(np.int8)
    b = rng.integers(-127, 128, (N, K)).astype(np.int8)
    sa = rng.uniform(1e-3, 1e-2, (M, K // group)).astype(np.float32)
    sb = rng.uniform(1e-3, 1e-2, (K // group, N)).astype(np.float32)
    bias = H.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
    return a, b, sa, sb, bias


def _run_gemm(product_lib, torch, a, b, sa, sb, bias=None, group=None, acc=False):
    M, K = a.shape
    N = b.shape[0]
    group = group or K
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    SA, SB = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda()
    Y = torch.full((M, N), 0x5A5A, dtype=torch.int16, device="cuda")
    if bias is None and not acc:
        rc = H.launch(product_lib, "ridgefill_gemm_nt_q", [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(Y, abi.BF16),
                                                           abi.absent(), abi.absent()], H.gemm_params(M, N, K, group))
        assert rc == abi.OK
        return Y.cpu().numpy().view(np.uint16), None
    BI = torch.from_numpy(bias.view(np.int16)).cuda() if bias is not None else None
    ACC = torch.full((M, N, K // group), -7, dtype=torch.int32, device="cuda") if acc else None
    rc = H.launch(product_lib, "ridgefill_gemm_nt_q_bias",
                  [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(BI, abi.BF16), H.dev(Y, abi.BF16), H.dev(ACC)],
                  H.gemm_params(M, N, K, group))
    assert rc == abi.OK
    return Y.cpu().numpy().view(np.uint16), (ACC.cpu().numpy() if acc else None)


@pytest.mark.parametrize("M,N,K,group", [
    (1, 256, 256, 256), (64, 256, 256, 128), (130, 512, 384, 128), (128, 2048, 2048, 2048),
    (300, 2048, 2048, 128), (64, 2560, 10240, 128), (257, 272, 1024, 1024)])
def test_gemm_matches_oracle_bitwise(cuda, product_lib, M, N, K, group):
    torch = cuda
    rng = np.random.default_rng(M * 7 + N + K)
    a, b, sa, sb, bias = _gemm_case(rng, M, N, K, group)
    y_ref, acc_ref = H.oracle_gemm(a, sa, b, sb, None, group, with_acc=True)
    y, _ = _run_gemm(product_lib, torch, a, b, sa, sb, group=group)
    assert np.array_equal(y, y_ref), f"{int((y != y_ref).sum())} of {y.size} differ"
    yb, acc = _run_gemm(product_lib, torch, a, b, sa, sb, bias=bias, group=group, acc=True)
    assert np.array_equal(acc, acc_ref)
    assert np.array_equal(yb, H.oracle_gemm(a, sa, b, sb, bias, group))
    # the fused bias equals gemm_nt_q then the add op, bit for bit (arch/ridgefill_layer.h:77-79)
    assert np.array_equal(yb, H.f32_to_bf16_bits(H.bf16_bits_to_f32(y) + H.bf16_bits_to_f32(bias)[None, :]))


def test_gemm_projector_full_size_sampled(cuda, product_lib):
    """The late pass's projector: T = 32,768 rows x d = 2,048, per-row activation and per-column weight
    scales (group = K). Every output row would take the CPU oracle minutes, so 96 sampled rows (each
    128-row tile band represented) are checked bit for bit, and the whole output against a float64
    evaluation on the GPU within one bf16 ulp."""
    torch = cuda
    M, N, K = 32768, 2048, 2048
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    SA = torch.rand((M, 1), device="cuda", generator=g) * 9e-3 + 1e-3
    SB = torch.rand((1, N), device="cuda", generator=g) * 9e-3 + 1e-3
    Y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    rc = H.launch(product_lib, "ridgefill_gemm_nt_q", [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(Y, abi.BF16),
                                                       abi.absent(), abi.absent()], H.gemm_params(M, N, K, K))
    assert rc == abi.OK
    y = Y.cpu().numpy().view(np.uint16)
    rows = np.unique(np.concatenate([np.arange(0, M, 128 * 3) + 17, [0, M - 1]]))[:96]
    y_ref = H.oracle_gemm(A[rows].cpu().numpy(), SA[rows].cpu().numpy(), B.cpu().numpy(), SB.cpu().numpy(), None, K)
    assert np.array_equal(y[rows], y_ref)
    exact = (A.double() @ B.double().T) * SA.double() * SB.double()
    got = torch.from_numpy(H.bf16_bits_to_f32(y)).cuda().double()
    assert bool(((got - exact).abs() <= exact.abs() * 2.0 ** -8 + 1e-30).all())


def test_gemm_through_folder_hooks(cuda, product_lib):
    """The folder path: a bf16 map encoded as the folder does (i8*bf16[1x128]), relaid by the row's own
    hooks, multiplied on the device == the oracle on the canonical planes (arch/ridgefill_int8.h:106-130)."""
    import ctypes as C
    torch = cuda
    rng = np.random.default_rng(79)
    M, N, K = 64, 2560, 10240
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    codes, scale = H.oracle_quantise_weight(w)
    row = product_lib.find_row("ridgefill_gemm_nt_q", abi.DOMAIN_DEVICE)
    params = H.gemm_params(1, N, K, 128)
    pp = (abi.RadParam * len(params))(*params)
    enc = abi.RadEncoding(abi.I8, abi.BF16, 1, 128)
    stored = []
    for opd, plane, dt in ((2, codes, abi.I8), (3, scale, abi.BF16)):
        sel = C.c_int(0 if opd == 2 else 1)
        geom = abi.tensor(dt, plane.shape, plane.ctypes.data)
        lay = abi.RadLayout()
        assert row.layout(pp, len(params), opd, C.byref(enc), C.byref(sel), C.byref(geom), 1, C.byref(lay)) == abi.OK
        out = np.zeros(lay.bytes, np.uint8)
        assert row.relayout(pp, len(params), opd, C.byref(enc), C.byref(sel), C.byref(geom), 1, out.ctypes.data, lay.bytes) == abi.OK
        stored.append(out)
    x = H.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    qa, sa = H.oracle_quant(x, 128)
    sb_canon = H.bf16_bits_to_f32(scale).T.copy()          # the same values, [K/128, N]
    y_ref = H.oracle_gemm(qa, sa, codes, sb_canon, None, 128)
    B = torch.from_numpy(stored[0].view(np.int8).reshape(N, K)).cuda()
    SB = torch.from_numpy(stored[1].view(np.float32).reshape(K // 128, N)).cuda()
    A, SA = torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda()
    Y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    rc = H.launch(product_lib, "ridgefill_gemm_nt_q", [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(Y, abi.BF16),
                                                       abi.absent(), abi.absent()], H.gemm_params(M, N, K, 128))
    assert rc == abi.OK and np.array_equal(Y.cpu().numpy().view(np.uint16), y_ref)
    # and the projection is close to the bf16 product it approximates (the folder's own error budget)
    exact = H.bf16_bits_to_f32(x).astype(np.float64) @ w.astype(np.float64).T
    assert H.rel_l2(H.bf16_bits_to_f32(y_ref), exact) < 0.02


def test_gemm_refusals(cuda, product_lib):
    torch = cuda
    A = torch.zeros((64, 256), dtype=torch.int8, device="cuda")
    B = torch.zeros((256, 256), dtype=torch.int8, device="cuda")
    SA = torch.ones((64, 2), device="cuda")
    SB = torch.ones((2, 256), device="cuda")
    Y = torch.empty((64, 256), dtype=torch.int16, device="cuda")
    base = [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(Y, abi.BF16), abi.absent(), abi.absent()]
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", base, H.gemm_params(64, 256, 256, 128)) == abi.OK
    bad = list(base)
    bad[1] = abi.absent()
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", bad, H.gemm_params(64, 256, 256, 128)) == abi.E_INVAL
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", base, H.gemm_params(64, 256, 256, 96)) == abi.E_SHAPE
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", base, H.gemm_params(64, 256, 256, 256)) == abi.E_SHAPE
    p = H.gemm_params(64, 256, 256, 128)
    p[-1] = H.pstr("dtype", "bf16")
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", base, p) == abi.E_INVAL
    bad = list(base)
    bad[5] = H.dev(SA)
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", bad, H.gemm_params(64, 256, 256, 128)) == abi.E_UNSUPPORTED
    A2 = torch.zeros((64, 272), dtype=torch.int8, device="cuda")[:, 8:264]   # rows 8 bytes off 16
    bad = list(base)
    bad[0] = H.dev(A2)
    assert H.launch(product_lib, "ridgefill_gemm_nt_q", bad, H.gemm_params(64, 256, 256, 128)) == abi.E_STRIDE


def test_sm_budget_changes_nothing_but_the_grid(cuda, product_lib):
    """max_ctas (the SMs a caller leaves the projector beside another stream's kernels) bounds the grid only: 2, 30
    and 116 CTAs write the same bits as the whole GPU, for the per-column and the group-128 forms."""
    torch = cuda
    rng = np.random.default_rng(77)
    for M, N, K, group in ((1000, 512, 1024, 1024), (700, 768, 1024, 128)):
        a, b, sa, sb, bias = _gemm_case(rng, M, N, K, group)
        want, _ = _run_gemm(product_lib, torch, a, b, sa, sb, bias=bias, group=group)
        A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        SA, SB = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda()
        BI = torch.from_numpy(bias.view(np.int16)).cuda()
        for ctas in (2, 30, 116):
            Y = torch.full((M, N), 0x5A5A, dtype=torch.int16, device="cuda")
            rc = H.launch(product_lib, "ridgefill_gemm_nt_q_bias",
                          [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(BI, abi.BF16), H.dev(Y, abi.BF16), abi.absent()],
                          H.gemm_params(M, N, K, group) + [H.pint("max_ctas", ctas)])
            assert rc == abi.OK
            assert np.array_equal(Y.cpu().numpy().view(np.uint16), want), (M, N, K, group, ctas)


@pytest.mark.parametrize("M,N,K,group,ld,c0", [(1000, 512, 1024, 1024, 512, 0), (700, 256, 2048, 2048, 1024, 512),
                                                (300, 768, 1024, 128, 1024, 256), (32768, 2048, 2048, 2048, 2048, 0)])
def test_row_selection_is_the_projector_then_select(cuda, product_lib, M, N, K, group, ld, c0):
    """The rows operand (ridgefill_select's mask): the projector writes its bias-added bf16 rows only where
    rows[m] == 1 (0, 2 and -1 leave the row alone), into a column block [c0, c0 + N) of a wider y as a tensor-
    parallel rank does -- bit for bit what the projector into a scratch matrix followed by ridgefill_select
    writes, every other element of y untouched."""
    torch = cuda
    rng = np.random.default_rng(M + N + c0)
    g = torch.Generator(device="cuda").manual_seed(M + c0)
    A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    SA = torch.rand((M, K // group), device="cuda", generator=g) * 9e-3 + 1e-3
    SB = torch.rand((K // group, N), device="cuda", generator=g) * 9e-3 + 1e-3
    BI = torch.from_numpy(H.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32)).view(np.int16)).cuda()
    rows = torch.from_numpy(rng.choice([0, 1, 1, 1, 2, -1], M).astype(np.int32)).cuda()
    ops = lambda y, r: [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(BI, abi.BF16), H.dev(y, abi.BF16), abi.absent(), H.dev(r)]  # noqa: E731
    full = torch.empty((M, N), dtype=torch.int16, device="cuda")
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", ops(full, None)[:7], H.gemm_params(M, N, K, group)) == abi.OK
    base = torch.randint(-30000, 30000, (M, ld), dtype=torch.int16, device="cuda", generator=g)
    want = base.clone()
    assert H.launch(product_lib, "ridgefill_select", [H.dev(rows), H.dev(full, abi.BF16), abi.absent(), abi.absent(),
                                                      H.dev(want[:, c0:c0 + N], abi.BF16), abi.absent(), abi.absent()],
                    [H.pint("M", M)]) == abi.OK
    got = base.clone()
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", ops(got[:, c0:c0 + N], rows), H.gemm_params(M, N, K, group)) == abi.OK
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    sel = rows == 1
    assert torch.equal(got[~sel], base[~sel]) and torch.equal(got[sel][:, c0:c0 + N], full[sel])


def test_row_selection_refusals(cuda, product_lib):
    torch = cuda
    M, N, K = 64, 256, 256
    A, B = torch.zeros((M, K), dtype=torch.int8, device="cuda"), torch.zeros((N, K), dtype=torch.int8, device="cuda")
    SA, SB = torch.ones((M, 1), device="cuda"), torch.ones((1, N), device="cuda")
    Y = torch.zeros((M, N), dtype=torch.int16, device="cuda")
    ACC = torch.zeros((M, N, 1), dtype=torch.int32, device="cuda")
    base = [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), abi.absent(), H.dev(Y, abi.BF16), abi.absent()]
    p = H.gemm_params(M, N, K, K)
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", base + [H.dev(torch.ones(M, device="cuda"))], p) == abi.E_DTYPE
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", base + [H.dev(torch.ones(M - 1, dtype=torch.int32, device="cuda"))],
                    p) == abi.E_SHAPE
    with_acc = list(base)
    with_acc[6] = H.dev(ACC)
    assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias", with_acc + [H.dev(torch.ones(M, dtype=torch.int32, device="cuda"))],
                    p) == abi.E_UNSUPPORTED
