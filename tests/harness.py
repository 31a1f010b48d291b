"""Test harness: the RidgeFill rows seen the way the engine sees them (a plugin's rows, found by op and
domain, called through RadArgs with operands in schema order), after tests/kernel_test.cpp:89-250 of
the reference: seeded splitmix64 draws, host buffers that cover padded strides, sentinel-filled
outputs, and a device runner that copies every buffer to the GPU, launches the device row on a
stream, and copies every buffer back.

The expected values come from the oracle, oracle/_build/libridgefill_oracle.so (the CPU restatement), and,
when it was built from the reference sources, oracle/_ref/ridgefill_ref.so (the reference's own host rows).
"""
from __future__ import annotations

import ctypes as C
import math
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "radiance-ridgefill_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT / "oracle"))   # cpu_path: the pass on host buffers (test infrastructure)

import ridgefill_abi as abi  # noqa: E402

ORACLE_SO = ROOT / "oracle" / "_build" / "libridgefill_oracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "ridgefill_ref.so"
REF_TEST = ROOT / "oracle" / "_ref" / "kernel_test"
GOLDEN = ROOT / "tests" / "golden"


# ----------------------------------------------------------------- builds

def build_oracle() -> Path:
    if not ORACLE_SO.exists() or ORACLE_SO.stat().st_mtime < (ROOT / "oracle" / "ridgefill_oracle.cpp").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)
    return ORACLE_SO


def build_product() -> Path:
    sys.path.insert(0, str(PKG))
    import build as pkg_build  # radiance-ridgefill_b200/build.py
    return pkg_build.build()


_oracle = None
_ref = None


def oracle() -> abi.Plugin:
    global _oracle
    if _oracle is None:
        build_oracle()
        _oracle = abi.Plugin(ORACLE_SO)
        _bind_oracle_functions(_oracle.lib)
    return _oracle


def reference() -> abi.Plugin | None:
    """The reference's own host rows compiled from its sources, when they were built here."""
    global _ref
    if _ref is None and REF_SO.exists():
        _ref = abi.Plugin(REF_SO)
    return _ref


def product() -> abi.Plugin:
    build_product()
    return abi.product()


# ----------------------------------------------------------------- seeded draws (tests/kernel_test.cpp:93-107)

class Rng:
    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.s = seed & self.MASK

    def next(self) -> int:
        self.s = (self.s + 0x9E3779B97F4A7C15) & self.MASK
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.MASK
        return z ^ (z >> 31)

    def uniform(self) -> float:
        return (self.next() >> 11) * (1.0 / 9007199254740992.0)

    def below(self, n: int) -> int:
        return self.next() % n if n > 0 else 0

    def normal(self) -> float:
        u = self.uniform() + 1e-12
        v = self.uniform()
        return float(np.float32(math.sqrt(-2.0 * math.log(u)) * math.cos(6.283185307179586 * v)))


def np_rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


# ----------------------------------------------------------------- bf16

def f32_to_bf16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(np.asarray(x, np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x7FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_bits_to_f32(h) -> np.ndarray:
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------- host buffers

NP_OF = {abi.F32: np.float32, abi.I32: np.int32, abi.BF16: np.uint16, abi.I8: np.int8, abi.U8: np.uint8,
         abi.F8E4M3: np.uint8, abi.F16: np.uint16}


class Buf:
    """A host buffer and its descriptor; strides in elements (packed when omitted). The buffer covers the
    furthest element the strides reach, so a padded layout really is padded (kernel_test.cpp:113-145).
    A zero-extent buffer is present with one spare byte."""

    def __init__(self, dtype: int, shape, strides=None):
        self.dtype, self.shape = dtype, [int(e) for e in shape]
        if strides is None:
            s, strides = 1, [0] * len(self.shape)
            for i in range(len(self.shape) - 1, -1, -1):
                strides[i] = s
                s *= self.shape[i]
        self.strides = [int(e) for e in strides]
        last = sum((e - 1) * s for e, s in zip(self.shape, self.strides))
        empty = any(e == 0 for e in self.shape)
        n = 1 if empty else ((last + 1) * abi.BITS[dtype] + 7) // 8
        self.bytes = np.zeros(max(n, 1), np.uint8)

    def copy(self) -> "Buf":
        b = Buf.__new__(Buf)
        b.dtype, b.shape, b.strides, b.bytes = self.dtype, list(self.shape), list(self.strides), self.bytes.copy()
        return b

    def flat(self) -> np.ndarray:
        """The raw elements (a view of the bytes) as the dtype's numpy type."""
        np_t = NP_OF[self.dtype]
        n = len(self.bytes) // np.dtype(np_t).itemsize
        return self.bytes[: n * np.dtype(np_t).itemsize].view(np_t)

    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def host(self) -> abi.RadTensor:
        return abi.tensor(self.dtype, self.shape, self.bytes.ctypes.data, self.strides)

    def setf(self, i, v):   # element i of the raw storage as float
        f = self.flat()
        if self.dtype == abi.BF16:
            f[i] = f32_to_bf16_bits(np.float32(v))
        else:
            f[i] = v

    def getf(self, i):
        f = self.flat()
        if self.dtype == abi.BF16:
            return float(bf16_bits_to_f32(f[i]))
        return f[i]


def run_host(plugin: abi.Plugin, row, bufs, params) -> int:
    return plugin.launch(row, [b.host() if b is not None else abi.absent() for b in bufs], params)


def run_device(plugin: abi.Plugin, row, bufs, params, scratch_bytes: int | None = None) -> int:
    """The device row on device copies of `bufs` (None = absent): copy in, launch on a fresh stream,
    synchronise, copy every buffer back (tests/kernel_test.cpp:190-219)."""
    import torch
    dev, tens = [], []
    for b in bufs:
        if b is None:
            dev.append(None)
            tens.append(abi.absent())
            continue
        d = torch.from_numpy(b.bytes.copy()).to("cuda")
        dev.append(d)
        tens.append(abi.tensor(b.dtype, b.shape, d.data_ptr(), b.strides))
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    scratch = None
    n = plugin.scratch_bytes(row, tens, params) if scratch_bytes is None else scratch_bytes
    if n > 0:
        scratch = torch.empty(n, dtype=torch.uint8, device="cuda")
    with torch.cuda.stream(stream):
        rc = plugin.launch(row, tens, params, stream=stream.cuda_stream,
                           scratch=scratch.data_ptr() if scratch is not None else None, scratch_bytes=n)
    stream.synchronize()
    for b, d in zip(bufs, dev):
        if b is not None:
            b.bytes[:] = d.cpu().numpy()
    return rc


def run_row(plugin: abi.Plugin, row, bufs, params) -> int:
    return run_device(plugin, row, bufs, params) if row.domain == abi.DOMAIN_DEVICE else run_host(plugin, row, bufs, params)


def pint(k, v):
    return abi.pint(k, v)


def pstr(k, v):
    return abi.pstr(k, v)


def pf64(k, v):
    return abi.pf64(k, v)


# ----------------------------------------------------------------- new-op oracles (plain pointers)

def _bind_oracle_functions(lib):
    P = C.c_void_p
    i64 = C.c_int64
    lib.oracle_quant_act_i8g.argtypes = [P, i64, i64, i64, i64, P, i64, P, i64]
    lib.oracle_quantise_weight_i8.argtypes = [P, i64, i64, P, P]
    lib.oracle_gemm_nt_q.argtypes = [P, i64, P, i64, P, i64, P, P, P, i64, P, i64, i64, i64, i64, i64, i64]
    lib.oracle_gemm_nt_bias.argtypes = [P, i64, P, i64, P, C.c_int, P, i64, P, i64, P, i64, i64, C.c_int, i64, i64]
    lib.oracle_gdn_conv_prep.argtypes = [P, i64, P, P, P, P, P, i64, P, i64, P, P, P, P, P, P, P, P, P, i64, i64, i64]
    lib.oracle_attn_kv_fill.argtypes = [P, P, P, C.c_int, P, C.c_int, P, P, i64, P, i64, i64, i64, C.c_double, C.c_float,
                                        C.c_int, P]
    for f in (lib.oracle_gdn_fill_f64, lib.oracle_gdn_fill_f32):
        f.argtypes = [P, P, P, P, P, P, P, i64, i64, P, i64, P, i64, i64, i64, i64, C.c_float, i64, i64]
    lib.oracle_threads.restype = C.c_int


def _p(a):
    return None if a is None else a.ctypes.data


def oracle_quant(x_bits: np.ndarray, group: int):
    """x bf16 bits [M, K] -> (q i8 [M, K], s f32 [M, K/group])."""
    lib = oracle().lib
    x = np.ascontiguousarray(x_bits, np.uint16)
    M, K = x.shape
    q = np.zeros((M, K), np.int8)
    s = np.zeros((M, K // group), np.float32)
    lib.oracle_quant_act_i8g(_p(x), K, M, K, group, _p(q), K, _p(s), K // group)
    return q, s


def oracle_quantise_weight(w: np.ndarray):
    lib = oracle().lib
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    codes = np.zeros((N, K), np.int8)
    scale = np.zeros((N, K // 128), np.uint16)
    lib.oracle_quantise_weight_i8(_p(w), N, K, _p(codes), _p(scale))
    return codes, scale


def oracle_gemm(a, a_scale, b, b_scale_kn, bias=None, group=None, with_acc=False, rows=None):
    """a i8 [M, K], a_scale f32 [M, K/group], b i8 [N, K], b_scale stored f32 [K/group, N], bias bf16 bits [N]
    -> y bf16 bits [M, N] (and int32 block sums [M, N, K/group]). `rows` = (m0, m1) computes a row range."""
    lib = oracle().lib
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(b, np.int8)
    a_scale = np.ascontiguousarray(a_scale, np.float32)
    b_scale_kn = np.ascontiguousarray(b_scale_kn, np.float32)
    M, K = a.shape
    N = b.shape[0]
    group = group or K
    blocks = K // group
    y = np.zeros((M, N), np.uint16)
    acc = np.zeros((M, N, blocks), np.int32) if with_acc else None
    bias = None if bias is None else np.ascontiguousarray(bias, np.uint16)
    m0, m1 = rows or (0, M)
    lib.oracle_gemm_nt_q(_p(a), K, _p(a_scale), blocks, _p(b), K, _p(b_scale_kn), _p(bias), _p(y), N, _p(acc),
                         M, N, K, group, m0, m1)
    return (y, acc) if with_acc else y


def oracle_gemm_bias(a, b, bias, res=None, act=0, rows=None):
    """a bf16 bits [M, K], b bf16 bits [N, K], bias bf16 bits (uint16) or f32 [N], res bf16 bits [M, N] or None
    -> (y, z) bf16 bits [M, N]: y = res + act(a @ b^T + bias), z the value before the residual."""
    lib = oracle().lib
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    bias = np.ascontiguousarray(bias)
    bias_f32 = bias.dtype == np.float32
    if not bias_f32:
        bias = bias.astype(np.uint16)
    res = None if res is None else np.ascontiguousarray(res, np.uint16)
    M, K = a.shape
    N = b.shape[0]
    y = np.zeros((M, N), np.uint16)
    z = np.zeros((M, N), np.uint16)
    m0, m1 = rows or (0, M)
    lib.oracle_gemm_nt_bias(_p(a), K, _p(b), K, _p(bias), int(bias_f32), _p(res), N, _p(y), N, _p(z), N, K, act,
                            m0, m1)
    return y, z


def oracle_conv_prep(x, w, a_log, dt_bias, state, cu, a, b, idx, ctx=None, bias=None, hk=16, hv=32, out=None):
    """ridgefill_gdn_conv_prep on the CPU. x bf16 bits [T, C]; w bf16 bits [C, 4]; a_log, dt_bias f32 [Hv];
    state bf16 bits [slots, 3, C] (updated in a copy, returned); cu, idx, ctx i32; a, b bf16 bits [T, Hv].
    `out` (optional): initial (q, k, v, g, beta) arrays, for the rows the op leaves alone. Returns
    (q, k, v, g, beta, state)."""
    lib = oracle().lib
    x = np.ascontiguousarray(x, np.uint16)
    T, Cc = x.shape
    w = np.ascontiguousarray(w, np.uint16)
    a_log = np.ascontiguousarray(a_log, np.float32)
    dt_bias = np.ascontiguousarray(dt_bias, np.float32)
    st = np.ascontiguousarray(state, np.uint16).copy()
    cu = np.ascontiguousarray(cu, np.int32)
    idx = np.ascontiguousarray(idx, np.int32).reshape(-1)
    ctx = None if ctx is None else np.ascontiguousarray(ctx, np.int32)
    bias = None if bias is None else np.ascontiguousarray(bias, np.uint16)
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    if out is None:
        out = (np.zeros((T, hk, 128), np.uint16), np.zeros((T, hk, 128), np.uint16), np.zeros((T, hv, 128), np.uint16),
               np.zeros((T, hv), np.float32), np.zeros((T, hv), np.float32))
    q, k, v, g, beta = (np.ascontiguousarray(o).copy() for o in out)
    lib.oracle_gdn_conv_prep(_p(x), Cc, _p(w), _p(bias), _p(a_log), _p(dt_bias), _p(st), st.shape[0], _p(cu), len(cu) - 1,
                             _p(a), _p(b), _p(idx), _p(ctx), _p(q), _p(k), _p(v), _p(g), _p(beta), T, hk, hv)
    return q, k, v, g, beta, st


ROPE_MODES = {"neox": 0, "mrope": 1, "imrope": 2}


def oracle_attn_kv(k, v, w, pos, slots, cache, rope_dim, theta, eps=1e-6, mode="neox", sections=(0, 0, 0), k_out=False):
    """ridgefill_attn_kv_fill on the CPU. k, v bf16 bits [T, Hkv, 256]; w bf16 bits (uint16) or f32 [256];
    pos i32 [T] or [3, T]; slots i32 [T]; cache bf16 bits [2, slots, Hkv, 256] (updated in a copy). Returns
    (cache, k_out or None)."""
    lib = oracle().lib
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    T, hkv, _ = k.shape
    w = np.ascontiguousarray(w)
    pos = np.ascontiguousarray(pos, np.int32)
    slots = np.ascontiguousarray(slots, np.int32)
    cache = np.ascontiguousarray(cache, np.uint16).copy()
    sec = np.asarray(sections, np.int32)
    ko = np.zeros_like(k) if k_out else None
    lib.oracle_attn_kv_fill(_p(k), _p(v), _p(w), int(w.dtype == np.float32), _p(pos), 1 if pos.ndim == 1 else 3,
                            _p(slots), _p(cache), cache.shape[1], _p(ko), T, hkv, rope_dim, float(theta), float(eps),
                            ROPE_MODES[mode], _p(sec))
    return cache, ko


def oracle_gdn(k, v, g, beta, state, idx, cu, q=None, scale=None, f64=True, heads=None):
    """Sequential gated delta rule; state [slots, Hv, dv, dk] f32 updated in a copy, returned with o."""
    lib = oracle().lib
    T, Hk, dk = k.shape
    Hv, dv = v.shape[1], v.shape[2]
    st = np.ascontiguousarray(state, np.float32).copy()
    idx = np.ascontiguousarray(idx, np.int32).reshape(-1)
    cu = np.ascontiguousarray(cu, np.int32)
    o = np.zeros((T, Hv, dv), np.uint16) if q is not None else None
    fn = lib.oracle_gdn_fill_f64 if f64 else lib.oracle_gdn_fill_f32
    h0, h1 = heads or (0, Hv)
    # contiguous copies held here for the call (a pointer to a temporary would outlive its array)
    qc = None if q is None else np.ascontiguousarray(q, np.uint16)
    kc, vc = np.ascontiguousarray(k, np.uint16), np.ascontiguousarray(v, np.uint16)
    gc, bc = np.ascontiguousarray(g, np.float32), np.ascontiguousarray(beta, np.float32)
    fn(_p(qc), _p(kc), _p(vc), _p(gc), _p(bc), _p(st), _p(idx), 1, st.shape[0], _p(cu), len(cu) - 1, _p(o),
       Hk, Hv, dk, dv, float(scale if scale is not None else 1.0 / math.sqrt(dk)), h0, h1)
    return st, o


# ----------------------------------------------------------------- torch device operands

def dev(t, dtype: int | None = None) -> abi.RadTensor:
    """A RadTensor over a torch tensor (device or host), with its shape and element strides."""
    import torch
    if t is None:
        return abi.absent()
    code = dtype if dtype is not None else {torch.float32: abi.F32, torch.bfloat16: abi.BF16, torch.int32: abi.I32,
                                            torch.int8: abi.I8, torch.uint8: abi.U8, torch.int16: abi.BF16,
                                            torch.uint16: abi.BF16}[t.dtype]
    return abi.tensor(code, list(t.shape), t.data_ptr(), list(t.stride()))


def launch(plugin: abi.Plugin, op: str, tensors, params, scratch_bytes: int | None = None) -> int:
    """The device row of `op` on torch operands, on torch's current stream, synchronised."""
    import torch
    row = plugin.find_row(op, abi.DOMAIN_DEVICE)
    n = plugin.scratch_bytes(row, tensors, params) if scratch_bytes is None else scratch_bytes
    scratch = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda") if n > 0 else None
    rc = plugin.launch(row, tensors, params, stream=torch.cuda.current_stream().cuda_stream,
                       scratch=scratch.data_ptr() if scratch is not None else None, scratch_bytes=n)
    torch.cuda.synchronize()
    return rc


def gemm_params(M, N, K, group):
    return [pint("M", M), pint("N", N), pint("K", K), pint("group", group), pstr("dtype", "i8a8")]


def gdn_params(T, hk, hv, scale=None):
    p = [pint("M", T), pint("n_head_k", hk), pint("n_head_v", hv), pint("head_k", 128), pint("head_v", 128),
         pint("chunk", 64)]
    if scale is not None:
        p.append(pf64("scale", scale))
    return p


def gdn_inputs(seed, T, hk, hv, decay="fast", slots=3):
    """Synthetic fill inputs of the single-layer benchmark's kind: q, k L2-normalised bf16, v ~ N(0,1) bf16, beta = sigmoid(N(0,1)),
    log decay g = -softplus(N(0,1)) ("fast": decay exp(g) about 0.5 a row) or a slow decay."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((T, hk, 128)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q = rng.standard_normal((T, hk, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((T, hv, 128)).astype(np.float32)
    x = rng.standard_normal((T, hv)).astype(np.float32)
    if decay == "fast":
        g = -np.log1p(np.exp(x))
    elif decay == "slow":
        g = -0.02 * np.abs(x)
    else:
        g = -0.001 * np.abs(x)
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((T, hv))))
    state = (0.1 * rng.standard_normal((slots, hv, 128, 128))).astype(np.float32)
    return (f32_to_bf16_bits(q), f32_to_bf16_bits(k), f32_to_bf16_bits(v), g.astype(np.float32),
            beta.astype(np.float32), state)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
