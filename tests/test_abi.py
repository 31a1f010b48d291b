"""The drop-in boundary, checked without a GPU: the library loads, exports every entry point its headers
declare, answers with the reference's nine schemas first (same names, parameters and operand order,
kernels/rows.cpp:44-168), has a device row with an operand description for every op, and its int8
GEMM row's stored-form hooks round-trip the folder's canonical planes (arch/ridgefill_int8.h:87-130)."""
import ctypes as C
import re

import numpy as np
import pytest

import harness as H
from harness import abi

REFERENCE_SCHEMAS = [
    ("ridgefill_mask", ["M", "share", "seed", "mode"], ["cu_last", "token_ids", "positions", "score", "mask", "bounds", "zeros"]),
    ("ridgefill_select", ["M"], ["mask", "x_src", "q_src", "s_src", "x", "q", "s"]),
    ("ridgefill_drop_rows", ["M", "top_k"], ["mask", "ids"]),
    ("ridgefill_rho_update", ["M", "n_head"], ["a", "mask", "A_log", "dt_bias", "ND", "state_idx", "bounds"]),
    ("ridgefill_state_correct", ["M", "mode", "alpha", "n_head", "sd0", "sd1"],
     ["state", "state_idx", "applied", "applied_idx", "C", "ND", "nd_idx", "bounds"]),
    ("ridgefill_state_read", ["M", "n_head", "sd0", "sd1"], ["state", "state_idx", "out"]),
    ("ridgefill_hazard", ["M"], ["cu_last", "positions", "bounds", "span", "meta", "meta_idx", "count"]),
    ("ridgefill_gemm_nt_bias", ["M", "N", "K", "dtype", "act"], ["a", "b", "bias", "res", "y"]),
    ("ridgefill_gemm_nt_q", ["M", "N", "K", "group", "dtype"], ["a", "a_scale", "b", "b_scale", "y", "a_sum", "b_ref"]),
]
NEW_OPS = ["ridgefill_gemm_nt_q_bias", "ridgefill_quant_act_i8g", "ridgefill_gdn_fill", "ridgefill_gdn_conv_prep",
           "ridgefill_gdn_in_proj", "ridgefill_attn_kv_fill"]
DEVICE_OPS = [s[0] for s in REFERENCE_SCHEMAS] + NEW_OPS


def described_params(op):
    """The geometry each op is described at (tests/kernel_test.cpp:288-299, plus the new ops)."""
    P = {"ridgefill_mask": [H.pint("M", 64), H.pf64("share", 0.25), H.pint("seed", 7), H.pstr("mode", "class")],
         "ridgefill_select": [H.pint("M", 37)], "ridgefill_drop_rows": [H.pint("M", 37), H.pint("top_k", 5)],
         "ridgefill_rho_update": [H.pint("M", 48), H.pint("n_head", 4)],
         "ridgefill_state_read": [H.pint("M", 3), H.pint("n_head", 2), H.pint("sd0", 8), H.pint("sd1", 8)],
         "ridgefill_state_correct": [H.pint("M", 3), H.pstr("mode", "apply"), H.pf64("alpha", 1.0), H.pint("n_head", 2),
                                     H.pint("sd0", 8), H.pint("sd1", 8)],
         "ridgefill_hazard": [H.pint("M", 1)],
         "ridgefill_gemm_nt_q": [H.pint("M", 64), H.pint("N", 256), H.pint("K", 256), H.pint("group", 128),
                                 H.pstr("dtype", "i8a8")],
         "ridgefill_gemm_nt_q_bias": [H.pint("M", 64), H.pint("N", 256), H.pint("K", 256), H.pint("group", 128),
                                      H.pstr("dtype", "i8a8")],
         "ridgefill_gemm_nt_bias": [H.pint("M", 64), H.pint("N", 256), H.pint("K", 256), H.pstr("dtype", "bf16")],
         "ridgefill_quant_act_i8g": [H.pint("M", 64), H.pint("n", 256), H.pint("group", 128), H.pstr("dtype", "bf16")],
         "ridgefill_gdn_fill": [H.pint("M", 130), H.pint("n_head_k", 2), H.pint("n_head_v", 4), H.pint("head_k", 128),
                                H.pint("head_v", 128), H.pint("chunk", 64)],
         "ridgefill_gdn_conv_prep": [H.pint("M", 70), H.pint("n_head_k", 1), H.pint("n_head_v", 2), H.pint("head_k", 128),
                                     H.pint("head_v", 128), H.pint("conv", 4)],
         "ridgefill_gdn_in_proj": [H.pint("M", 70), H.pint("N", 384), H.pint("K", 256), H.pint("n_head_k", 1),
                                   H.pint("n_head_v", 2), H.pint("group", 256), H.pstr("dtype", "i8a8")],
         "ridgefill_attn_kv_fill": [H.pint("M", 40), H.pint("n_head_kv", 2), H.pint("head_dim", 256), H.pint("rope_dim", 64),
                                    H.pf64("rope_theta", 1e7)]}
    return P[op]


def test_exports_every_declared_entry_point(product_lib):
    lib = product_lib.lib
    names = set()
    for header in ("ridgefill.h", "rad_plugin.h", "ridgefill_folder.h"):
        text = (H.ROOT / "include" / header).read_text()
        block = text[text.find('extern "C" {'):]
        names |= set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", block, re.M))
    names -= {"rad_arg_in", "rad_args_geti", "rad_args_gets", "rad_args_getf_or"}   # header-inline readers
    assert {"rad_plugin_abi_version", "ridgefill_mask_device", "ridgefill_gdn_fill_device", "ridgefill_attn_kv_fill_device",
            "ridgefill_folder_open", "ridgefill_folder_upload", "ridgefill_resident_map"} <= names
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_abi_version_and_info(product_lib):
    assert product_lib.lib.rad_plugin_abi_version() == abi.RAD_ABI_VERSION
    info = product_lib.info
    assert info.kind == 1 and info.name == b"ridgefill" and b"sm_100a" in info.build_target


def test_reference_schemas_first_in_order(product_lib):
    schemas = product_lib.schemas()
    assert len(schemas) == len(REFERENCE_SCHEMAS) + len(NEW_OPS)
    for sc, (op, params, operands) in zip(schemas, REFERENCE_SCHEMAS):
        assert sc.op.decode() == op
        assert [sc.params[i].key.decode() for i in range(sc.n_params)] == params
        assert [sc.operands[i].name.decode() for i in range(sc.n_operands)] == operands
    assert [s.op.decode() for s in schemas[len(REFERENCE_SCHEMAS):]] == NEW_OPS
    for sc in schemas:   # R98: no parameter carries a role (kernel_test.cpp:378-390)
        assert all(sc.params[i].role == 0 for i in range(sc.n_params))


def test_every_row_is_a_device_row(product_lib):
    rows = product_lib.rows()
    assert all(r.domain == abi.DOMAIN_DEVICE for r in rows), "the B200 library has no host rows"
    for op in DEVICE_OPS:
        assert product_lib.find_row(op, abi.DOMAIN_DEVICE) is not None, op
    assert product_lib.find_row("ridgefill_gdn_fill", abi.DOMAIN_DEVICE).scratch


def test_descriptions_cover_schemas(product_lib):
    """Every operand index has a description and one past the schema is refused (kernel_test.cpp:330-348)."""
    for op in DEVICE_OPS:
        sc = product_lib.schema(op)
        row = product_lib.find_row(op, abi.DOMAIN_DEVICE)
        params = described_params(op)
        pp = (abi.RadParam * len(params))(*params)
        for i in range(sc.n_operands):
            d = abi.RadOpdDesc()
            assert row.opd_shape(pp, len(params), i, C.byref(d)) == abi.OK, (op, i)
        d = abi.RadOpdDesc()
        assert row.opd_shape(pp, len(params), sc.n_operands, C.byref(d)) == abi.E_SHAPE


def _hook_call(row, N, K, operand, plane, dtype, stored=None):
    params = [H.pint("M", 1), H.pint("N", N), H.pint("K", K), H.pint("group", 128), H.pstr("dtype", "i8a8")]
    pp = (abi.RadParam * len(params))(*params)
    enc = abi.RadEncoding(abi.I8, abi.BF16, 1, 128)
    sel = C.c_int(0 if operand == 2 else 1)
    geom = abi.tensor(dtype, plane.shape, plane.ctypes.data)
    lay = abi.RadLayout()
    assert row.layout(pp, len(params), operand, C.byref(enc), C.byref(sel), C.byref(geom), 1, C.byref(lay)) == abi.OK
    out = np.zeros(lay.bytes, np.uint8)
    assert row.relayout(pp, len(params), operand, C.byref(enc), C.byref(sel), C.byref(geom), 1,
                        out.ctypes.data, lay.bytes) == abi.OK
    back = np.zeros(plane.nbytes, np.uint8)
    src = abi.tensor(dtype, plane.shape, out.ctypes.data)
    assert row.unrelayout(pp, len(params), operand, C.byref(enc), C.byref(sel), C.byref(src), 1,
                          back.ctypes.data, back.nbytes) == abi.OK
    return lay, out, back


def test_int8_stored_form_hooks_round_trip(product_lib):
    """The folder's canonical planes (codes i8 [N, K], scale bf16 [N, K/128]) -> the row's stored form ->
    back, byte for byte; the stored scale is f32 [K/128, N] holding the same values."""
    row = product_lib.find_row("ridgefill_gemm_nt_q", abi.DOMAIN_DEVICE)
    rng = np.random.default_rng(3)
    N, K = 48, 384
    codes = rng.integers(-127, 128, (N, K)).astype(np.int8)
    scale = H.f32_to_bf16_bits(rng.uniform(1e-3, 1e-2, (N, K // 128)).astype(np.float32))
    lay, out, back = _hook_call(row, N, K, 2, codes, abi.I8)
    assert lay.bytes == N * K and np.array_equal(back.view(np.int8).reshape(N, K), codes)
    lay, out, back = _hook_call(row, N, K, 3, scale, abi.BF16)
    assert lay.bytes == (K // 128) * N * 4
    assert np.array_equal(out.view(np.float32).reshape(K // 128, N), H.bf16_bits_to_f32(scale).T)
    assert np.array_equal(back.view(np.uint16).reshape(N, K // 128), scale)
    # every row of the op describes the same stored bytes (arch/ridgefill_int8.h:87-103)
    bias_row = product_lib.find_row("ridgefill_gemm_nt_q_bias", abi.DOMAIN_DEVICE)
    lay2, out2, _ = _hook_call(bias_row, N, K, 3, scale, abi.BF16)
    assert lay2.bytes == lay.bytes and lay2.tag == lay.tag and np.array_equal(out2, out)


def test_stored_form_hooks_refuse_other_encodings(product_lib):
    row = product_lib.find_row("ridgefill_gemm_nt_q", abi.DOMAIN_DEVICE)
    params = [H.pint("M", 1), H.pint("N", 48), H.pint("K", 384), H.pint("group", 128), H.pstr("dtype", "i8a8")]
    pp = (abi.RadParam * len(params))(*params)
    codes = np.zeros((48, 384), np.int8)
    geom = abi.tensor(abi.I8, codes.shape, codes.ctypes.data)
    lay = abi.RadLayout()
    sel = C.c_int(0)
    for enc in (abi.RadEncoding(abi.I8, abi.BF16, 1, 64), abi.RadEncoding(abi.I8, abi.F32, 1, 128)):
        assert row.layout(pp, len(params), 2, C.byref(enc), C.byref(sel), C.byref(geom), 1, C.byref(lay)) == abi.E_UNSUPPORTED
    enc = abi.RadEncoding(abi.I8, abi.BF16, 1, 128)
    assert row.layout(pp, len(params), 4, C.byref(enc), C.byref(sel), C.byref(geom), 1, C.byref(lay)) == abi.E_INVAL
