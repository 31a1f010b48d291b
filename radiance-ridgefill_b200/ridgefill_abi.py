"""ctypes binding of the RidgeFill kernel-plugin C ABI (include/rad_abi.h, include/rad_plugin.h).

This is how Python reaches the B200 library: the same entry points the radiance engine binds
(rad_kernel_count / rad_kernel_at / rad_kernel_schema_*, each row's launch hook), called with a
RadArgs of operands in schema order, exactly as the reference's harness calls its plugin
(tests/kernel_test.cpp:160-169). Nothing here computes an op: a device row launches CUDA work on the
given stream; the library has no CPU fallback and `product()` raises when it is not built.

    lib = product()                                   # radiance-ridgefill_b200/ridgefill.so
    row = lib.find_row("ridgefill_select", DOMAIN_DEVICE)
    rc = lib.launch(row, [t0, t1, ...], [pint("M", 37)], stream=torch.cuda.current_stream().cuda_stream)
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
PRODUCT_SO = HERE / "ridgefill.so"

# ----------------------------------------------------------------- constants (rad_abi.h)
RAD_ABI_VERSION = (15 << 16) | (0 << 8) | 0
OK, E_INVAL, E_DTYPE, E_SHAPE, E_STRIDE, E_UNSUPPORTED, E_DEVICE, E_NOMEM = 0, -1, -2, -3, -4, -5, -6, -7
F32, BF16, F16, I32, I8, U8, F8E4M3, I4, I64 = 1, 2, 3, 4, 5, 6, 7, 8, 9
P_INT, P_STR, P_F64 = 1, 2, 3
DOMAIN_HOST, DOMAIN_DEVICE = 0, 1
OPD_IN, OPD_OUT, OPD_INOUT, OPD_WEIGHT = 0, 1, 2, 3
FILL_NORMAL, FILL_INDEX, FILL_SIGMOID, FILL_ZERO = 0, 1, 2, 3
OPD_F_ABSENT, OPD_F_IDX_CU, OPD_F_IDX_UNIQUE = 1, 2, 4
C_IN, C_LE, C_GE, C_EQ = 1, 2, 3, 4
MAX_RANK = 8
BITS = {F32: 32, BF16: 16, F16: 16, I32: 32, I8: 8, U8: 8, F8E4M3: 8, I4: 4, I64: 64}


class RadTensor(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("rank", C.c_uint32), ("shape", C.c_int64 * MAX_RANK),
                ("stride", C.c_int64 * MAX_RANK), ("data", C.c_void_p)]


class RadParam(C.Structure):
    _fields_ = [("key", C.c_char_p), ("type", C.c_int), ("ival", C.c_longlong), ("ival_hi", C.c_longlong),
                ("sval", C.c_char_p), ("fval", C.c_double)]


class RadArgs(C.Structure):
    _fields_ = [("t", C.POINTER(RadTensor)), ("n_t", C.c_int), ("p", C.POINTER(RadParam)), ("n_p", C.c_int),
                ("rank", C.c_int), ("world_size", C.c_int), ("scratch", C.c_void_p), ("scratch_bytes", C.c_int64)]


class RadParamSpec(C.Structure):
    _fields_ = [("key", C.c_char_p), ("type", C.c_uint32), ("required", C.c_uint32), ("role", C.c_uint32)]


class RadOperandSpec(C.Structure):
    _fields_ = [("name", C.c_char_p), ("kind", C.c_uint32), ("optional", C.c_uint32)]


class RadOpSchema(C.Structure):
    _fields_ = [("op", C.c_char_p), ("params", C.POINTER(RadParamSpec)), ("n_params", C.c_int),
                ("operands", C.POINTER(RadOperandSpec)), ("n_operands", C.c_int), ("doc", C.c_char_p)]


class RadConstraint(C.Structure):
    _fields_ = [("key", C.c_char_p), ("op", C.c_int), ("ival", C.c_longlong), ("sval", C.c_char_p)]


class RadOpdDesc(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("rank", C.c_uint32), ("shape", C.c_int64 * MAX_RANK), ("fill", C.c_uint32),
                ("flags", C.c_uint32), ("idx_max", C.c_int64), ("idx_const", C.c_int64)]


class RadEncoding(C.Structure):
    _fields_ = [("codes", C.c_uint32), ("scale", C.c_uint32), ("group_rows", C.c_int32), ("group_cols", C.c_int32)]


class RadLayout(C.Structure):
    _fields_ = [("bytes", C.c_int64), ("tag", C.c_char_p), ("align", C.c_int64)]


class RadPluginInfo(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("name", C.c_char_p), ("version", C.c_char_p), ("description", C.c_char_p),
                ("build_target", C.c_char_p)]


LAUNCH = C.CFUNCTYPE(C.c_int, C.POINTER(RadArgs), C.c_void_p)
SCRATCH = C.CFUNCTYPE(C.c_int64, C.POINTER(RadArgs))
OPD_SHAPE = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadOpdDesc))
LAYOUT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadEncoding), C.POINTER(C.c_int),
                     C.POINTER(RadTensor), C.c_int, C.POINTER(RadLayout))
RELAYOUT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadEncoding), C.POINTER(C.c_int),
                       C.POINTER(RadTensor), C.c_int, C.c_void_p, C.c_int64)


class RadKernelInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("op", C.c_char_p), ("plugin", C.c_char_p), ("computes", C.c_char_p),
                ("shapes", C.c_char_p), ("dtypes", C.c_char_p), ("domain", C.c_int), ("priority", C.c_int),
                ("constraints", C.POINTER(RadConstraint)), ("n_constraints", C.c_int), ("tunables", C.c_void_p),
                ("n_tunables", C.c_int), ("init", C.c_void_p), ("fini", C.c_void_p), ("prepare", C.c_void_p),
                ("launch", LAUNCH), ("describe", C.c_void_p), ("scratch", SCRATCH), ("validate", C.c_void_p),
                ("opd_shape", OPD_SHAPE), ("layout", LAYOUT), ("relayout", RELAYOUT), ("unrelayout", RELAYOUT),
                ("replaces", C.c_char_p)]


# ----------------------------------------------------------------- helpers

def pint(key: str, v: int) -> RadParam:
    return RadParam(key.encode(), P_INT, int(v), 0, None, 0.0)


def pstr(key: str, v: str) -> RadParam:
    return RadParam(key.encode(), P_STR, 0, 0, v.encode(), 0.0)


def pf64(key: str, v: float) -> RadParam:
    return RadParam(key.encode(), P_F64, 0, 0, None, float(v))


def tensor(dtype: int, shape, data_ptr: int | None, strides=None) -> RadTensor:
    """A RadTensor over `data_ptr` (an int address; None or 0 = absent). Strides in elements; packed when
    omitted."""
    t = RadTensor()
    t.dtype = dtype
    t.rank = len(shape)
    for i, e in enumerate(shape):
        t.shape[i] = int(e)
    if strides is None:
        s = 1
        strides = [0] * len(shape)
        for i in range(len(shape) - 1, -1, -1):
            strides[i] = s
            s *= int(shape[i])
    for i, e in enumerate(strides):
        t.stride[i] = int(e)
    t.data = data_ptr if data_ptr else None
    return t


def absent() -> RadTensor:
    return RadTensor()


class Plugin:
    """A loaded kernel plugin: its schemas and rows, found by (op, domain) as the engine finds them."""

    def __init__(self, path: str | os.PathLike):
        path = Path(path)
        if not path.exists():
            raise RuntimeError(f"{path} is not built: the RidgeFill B200 library has no fallback "
                               f"(build it with radiance-ridgefill_b200/build.py)")
        self.path = path
        self.lib = C.CDLL(str(path), mode=os.RTLD_LOCAL | os.RTLD_NOW)
        L = self.lib
        L.rad_plugin_abi_version.restype = C.c_uint32
        L.rad_plugin_info.restype = C.POINTER(RadPluginInfo)
        L.rad_kernel_schema_count.restype = C.c_int
        L.rad_kernel_schema_at.restype = C.POINTER(RadOpSchema)
        L.rad_kernel_schema_at.argtypes = [C.c_int]
        L.rad_kernel_count.restype = C.c_int
        L.rad_kernel_at.restype = C.POINTER(RadKernelInfo)
        L.rad_kernel_at.argtypes = [C.c_int]
        L.rad_kernel_concurrent.restype = C.c_int
        L.rad_kernel_concurrent.argtypes = [C.c_int]
        if L.rad_plugin_abi_version() != RAD_ABI_VERSION:
            raise RuntimeError(f"{path}: ABI {L.rad_plugin_abi_version():#x}, expected {RAD_ABI_VERSION:#x}")

    @property
    def info(self) -> RadPluginInfo:
        return self.lib.rad_plugin_info().contents

    def schemas(self) -> list[RadOpSchema]:
        return [self.lib.rad_kernel_schema_at(i).contents for i in range(self.lib.rad_kernel_schema_count())]

    def schema(self, op: str) -> RadOpSchema | None:
        for s in self.schemas():
            if s.op.decode() == op:
                return s
        return None

    def rows(self) -> list[RadKernelInfo]:
        return [self.lib.rad_kernel_at(i).contents for i in range(self.lib.rad_kernel_count())]

    def find_row(self, op: str, domain: int) -> RadKernelInfo | None:
        for r in self.rows():
            if r.domain == domain and r.op.decode() == op:
                return r
        return None

    @staticmethod
    def args(tensors, params, scratch: int | None = None, scratch_bytes: int = 0):
        tt = (RadTensor * max(len(tensors), 1))(*tensors)
        pp = (RadParam * max(len(params), 1))(*params)
        a = RadArgs()
        a.t = C.cast(tt, C.POINTER(RadTensor))
        a.n_t = len(tensors)
        a.p = C.cast(pp, C.POINTER(RadParam))
        a.n_p = len(params)
        a.rank = 0
        a.world_size = 1
        a.scratch = scratch if scratch else None
        a.scratch_bytes = int(scratch_bytes)
        return a, (tt, pp)   # keep the arrays alive with the args

    def launch(self, row: RadKernelInfo, tensors, params, stream: int | None = None, scratch: int | None = None,
               scratch_bytes: int = 0) -> int:
        a, keep = self.args(tensors, params, scratch, scratch_bytes)
        rc = row.launch(C.byref(a), C.c_void_p(stream) if stream else None)
        del keep
        return rc

    def scratch_bytes(self, row: RadKernelInfo, tensors, params) -> int:
        if not row.scratch:
            return 0
        a, keep = self.args(tensors, params)
        n = row.scratch(C.byref(a))
        del keep
        return int(n)


_product: Plugin | None = None


def product() -> Plugin:
    """The B200 library (device rows only). Raises when it has not been built."""
    global _product
    if _product is None:
        _product = Plugin(PRODUCT_SO)
    return _product
