"""The bf16 projector / final map on B200 (ridgefill_gemm_nt_bias: y = res + act(a @ b^T + bias), bf16 after the
biased product, after the activation and after the residual; kernels/rows.cpp:155-160) against the CPU oracle.

The reference checks this row bytewise against the engine's own gemm_nt_bias row it forwards to
(tests/kernel_test.cpp:1991-2006: M 1 / 64 / 2,048, N 2,560, K 10,240 on the card, M 130 / N 48 / K 136 on the
host; bf16 and f32 bias, with and without res). That engine library is not part of the reference tree, so the
bar here is the reference's bf16 GEMM tolerance (tests/kernel_test.cpp:2121-2125): |x - y| <= 2^-7 max(|x|, |y|)
+ 2^-9 RMS(y_ref), two bf16 ulps of the larger output plus a 2^-9 RMS floor for sums that cancel. With a
residual the rounding of the pre-residual value carries into y, so its own 2^-7 |z| joins the bound. The oracle
covers sampled rows of the large shapes; a torch fp32 product (TF32 off) covers every row."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu


def _bias_params(M, N, K, act=None):
    p = [H.pint("M", M), H.pint("N", N), H.pint("K", K), H.pstr("dtype", "bf16")]
    if act is not None:
        p.append(H.pstr("act", act))
    return p


def _inputs(rng, M, N, K, bias_f32, res):
    a = H.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    b = H.f32_to_bf16_bits((rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32))
    bias = rng.standard_normal(N).astype(np.float32)
    bias = bias if bias_f32 else H.f32_to_bf16_bits(bias)
    r = H.f32_to_bf16_bits(rng.standard_normal((M, N)).astype(np.float32)) if res else None
    return a, b, bias, r


def _run(product_lib, torch, a, b, bias, r, act=None, pad_a=0, pad_y=0):
    """The device row on copies of the operands; `pad_a` / `pad_y` extra columns make a and y views with a
    row pitch wider than the matrix."""
    M, K = a.shape
    N = b.shape[0]
    A_full = torch.zeros((M, K + pad_a), dtype=torch.int16, device="cuda")
    A_full[:, :K] = torch.from_numpy(a.view(np.int16)).cuda()
    A = A_full[:, :K]
    B = torch.from_numpy(b.view(np.int16)).cuda()
    BI = torch.from_numpy(bias).cuda() if bias.dtype == np.float32 else torch.from_numpy(bias.view(np.int16)).cuda()
    R = torch.from_numpy(r.view(np.int16)).cuda() if r is not None else None
    Y_full = torch.full((M, N + pad_y), 0x5A5A, dtype=torch.int16, device="cuda")
    Y = Y_full[:, :N]
    rc = H.launch(product_lib, "ridgefill_gemm_nt_bias",
                  [H.dev(A, abi.BF16), H.dev(B, abi.BF16), H.dev(BI, abi.F32 if bias.dtype == np.float32 else abi.BF16),
                   H.dev(R, abi.BF16) if R is not None else abi.absent(), H.dev(Y, abi.BF16)],
                  _bias_params(M, N, K, act))
    assert rc == abi.OK
    if pad_y:   # the columns past N are untouched
        assert bool((Y_full[:, N:] == 0x5A5A).all())
    return Y.cpu().numpy().view(np.uint16)


def _within(y, y_ref, z_ref, res, what):
    x = H.bf16_bits_to_f32(y_ref).astype(np.float64)
    d = H.bf16_bits_to_f32(y).astype(np.float64)
    rms = np.sqrt(np.mean(x * x)) if x.size else 0.0
    tol = np.ldexp(np.maximum(np.abs(x), np.abs(d)), -7) + np.ldexp(rms, -9)
    if res:
        tol += np.ldexp(np.abs(H.bf16_bits_to_f32(z_ref).astype(np.float64)), -7)
    err = np.abs(x - d)
    assert np.all(np.isfinite(d)), what
    bad = err > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} outside the bound, worst {float((err / tol).max()):.3g}x"


def _torch_ref(torch, a, b, bias, r, act):
    """fp32 product of the bf16 operands, then the row's bf16 roundings, in torch on the device."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        A = torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16).float()
        B = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16).float()
        bv = torch.from_numpy(bias).cuda() if bias.dtype == np.float32 else \
            torch.from_numpy(bias.view(np.int16)).cuda().view(torch.bfloat16).float()
        x = (A @ B.T + bv).bfloat16()
        if act == "silu":
            xf = x.double()
            x = (xf / (1.0 + torch.exp(-xf))).float().bfloat16()
        z = x
        if r is not None:
            x = (x.float() + torch.from_numpy(r.view(np.int16)).cuda().view(torch.bfloat16).float()).bfloat16()
        torch.cuda.synchronize()
        return (x.view(torch.int16).cpu().numpy().view(np.uint16), z.view(torch.int16).cpu().numpy().view(np.uint16))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _sample_rows(M):
    if M <= 160:
        return [(0, M)]
    return [(0, 48), (M // 2 - 16, M // 2 + 16), (M - 48, M)]


@pytest.mark.parametrize("M", [1, 64, 2048])
@pytest.mark.parametrize("variant", [0, 1])
def test_projector_shape_matches_oracle(cuda, product_lib, M, variant):
    """The projector's shape on the card (N 2,560, K 10,240): bf16 bias alone, then f32 bias with res."""
    torch = cuda
    N, K = 2560, 10240
    rng = np.random.default_rng(140 + M + variant)
    a, b, bias, r = _inputs(rng, M, N, K, bias_f32=variant == 1, res=variant == 1)
    y = _run(product_lib, torch, a, b, bias, r)
    for m0, m1 in _sample_rows(M):
        y_ref, z_ref = H.oracle_gemm_bias(a, b, bias, r, rows=(m0, m1))
        _within(y[m0:m1], y_ref[m0:m1], z_ref[m0:m1], r is not None, f"oracle rows {m0}:{m1}")
    y_t, z_t = _torch_ref(torch, a, b, bias, r, None)
    _within(y, y_t, z_t, r is not None, "torch fp32, every row")


@pytest.mark.parametrize("M,N,K,bias_f32,res,act", [
    (130, 48, 136, False, False, None),     # the reference's host-row shape: N and K below a tile
    (130, 48, 136, True, True, None),
    (257, 272, 1024, False, True, "silu"),  # ragged tiles on both axes, the activation and the residual
    (200, 2560, 512, True, False, "silu"),
    (129, 520, 328, True, True, "none"),
    # the narrow form (N <= 64: M256 N64 pair tiles): the DeltaNet a|b projection's shape, and a ragged one
    (4096, 64, 2048, False, False, None),
    (515, 40, 200, True, True, "silu"),
    (300, 72, 256, False, False, None),     # a column block past the narrow form: the wide one
])
def test_ragged_shapes_match_oracle(cuda, product_lib, M, N, K, bias_f32, res, act):
    torch = cuda
    rng = np.random.default_rng(M * 3 + N + K)
    a, b, bias, r = _inputs(rng, M, N, K, bias_f32, res)
    y = _run(product_lib, torch, a, b, bias, r, act=act)
    y_ref, z_ref = H.oracle_gemm_bias(a, b, bias, r, act=1 if act == "silu" else 0)
    _within(y, y_ref, z_ref, res, f"M {M} N {N} K {K}")


def test_strided_views_match_contiguous(cuda, product_lib):
    """a and y as views with wider row pitches give the bytes of the packed call."""
    torch = cuda
    rng = np.random.default_rng(7)
    a, b, bias, r = _inputs(rng, 300, 512, 640, True, True)
    y0 = _run(product_lib, torch, a, b, bias, r, act="silu")
    y1 = _run(product_lib, torch, a, b, bias, r, act="silu", pad_a=64, pad_y=24)
    assert np.array_equal(y0, y1)


def test_refusals(cuda, product_lib):
    torch = cuda
    A = torch.zeros((4, 64), dtype=torch.int16, device="cuda")
    B = torch.zeros((16, 64), dtype=torch.int16, device="cuda")
    BI = torch.zeros(16, dtype=torch.int16, device="cuda")
    Y = torch.zeros((4, 16), dtype=torch.int16, device="cuda")
    ops = [H.dev(A, abi.BF16), H.dev(B, abi.BF16), H.dev(BI, abi.BF16), abi.absent(), H.dev(Y, abi.BF16)]
    assert H.launch(product_lib, "ridgefill_gemm_nt_bias", ops, _bias_params(4, 16, 64, "gelu")) == abi.E_UNSUPPORTED
    p = [H.pint("M", 4), H.pint("N", 16), H.pint("K", 64), H.pstr("dtype", "f16")]
    assert H.launch(product_lib, "ridgefill_gemm_nt_bias", ops, p) == abi.E_UNSUPPORTED
    A2 = torch.zeros((4, 60), dtype=torch.int16, device="cuda")   # K not a multiple of 8
    B2 = torch.zeros((16, 60), dtype=torch.int16, device="cuda")
    ops2 = [H.dev(A2, abi.BF16), H.dev(B2, abi.BF16), H.dev(BI, abi.BF16), abi.absent(), H.dev(Y, abi.BF16)]
    assert H.launch(product_lib, "ridgefill_gemm_nt_bias", ops2, _bias_params(4, 16, 60)) == abi.E_SHAPE
    assert bool((Y == 0).all())
