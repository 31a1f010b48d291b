"""Operand builders and runners for the reference's seven ops, after tests/kernel_test.cpp:420-560 of the
reference: each builds one op's operands as host buffers (outputs pre-filled with a sentinel, so an
unwritten element shows), runs a given row (host or device, by its domain) and returns the outputs."""
from __future__ import annotations

import math

import numpy as np

import harness as H
from harness import Buf, pint, pstr, pf64, abi

SENTINEL = 0x5A5A5A5A


# ----------------------------------------------------------------- ridgefill_mask (kernel_test.cpp:424-466)

class MaskCall:
    def __init__(self, ids=(), n=0, s=0, e=0, table=None, share=0.25, seed=0, mode="class", first_pos=0,
                 components=1, n_zeros=0):
        self.ids, self.n, self.s, self.e = list(ids), n, s, e
        self.table, self.share, self.seed, self.mode = table, share, seed, mode
        self.first_pos, self.components, self.n_zeros = first_pos, components, n_zeros

    def copy(self, **kw):
        c = MaskCall(self.ids, self.n, self.s, self.e, self.table, self.share, self.seed, self.mode, self.first_pos,
                     self.components, self.n_zeros)
        for k, v in kw.items():
            setattr(c, k, v)
        return c


def run_mask(plugin, row, c: MaskCall):
    b = len(c.ids)
    vocab = len(c.table) if c.table is not None else 1
    cu, tok, score = Buf(abi.I32, [2]), Buf(abi.I32, [b]), Buf(abi.F32, [vocab])
    mask, bounds = Buf(abi.I32, [c.n]), Buf(abi.I32, [4])
    pos = Buf(abi.I32, [c.components, b]) if c.components > 1 else Buf(abi.I32, [b])
    cu.flat()[:2] = [c.s, c.e]
    tok.flat()[:b] = c.ids
    p = pos.flat()
    for i in range(c.components * b):
        p[i] = c.first_pos + i if i < b else 7777 + i
    if c.table is not None:
        score.flat()[:vocab] = np.asarray(c.table, np.float32)
    mask.flat()[:] = SENTINEL
    bounds.flat()[:] = SENTINEL
    zeros = Buf(abi.I32, [max(c.n_zeros, 1)])
    zeros.flat()[:] = SENTINEL
    rc = H.run_row(plugin, row, [cu, tok, pos, score if c.table is not None else None, mask, bounds,
                                 zeros if c.n_zeros > 0 else None],
                   [pint("M", b), pf64("share", c.share), pint("seed", c.seed), pstr("mode", c.mode)])
    return rc, mask.flat()[: c.n].copy(), bounds.flat()[:4].copy(), zeros.flat()[: c.n_zeros].copy()


def random_window(r: H.Rng, n: int, layout: int, limit: int = 8192) -> MaskCall:
    """kernel_test.cpp:1666-1680: whole step, a window inside, b before s (empty), b past e."""
    s = 0 if layout == 0 else r.below(n // 2 + 1)
    e, b = n, min(n, limit)
    if layout == 1:
        b = s + r.below(max(min(e, limit) - s, 0) + 1)
    if layout >= 2:
        e = s + r.below(n - s + 1)
    if layout == 2:
        b = s - r.below(s + 1)
    if layout == 3:
        b = e + 1 + r.below(50)
    ids = [int(r.below(1010)) - 5 for _ in range(min(max(b, 1), limit))]
    return MaskCall(ids=ids, n=n, s=s, e=e)


# ----------------------------------------------------------------- select / drop (kernel_test.cpp:468-520)

def fill_pattern(b: Buf, tag: int):
    i = np.arange(len(b.bytes), dtype=np.int64)
    b.bytes[:] = ((tag * 31 + i * 7 + 1) & 0xFF).astype(np.uint8)


def fill_sentinel(b: Buf):
    b.bytes[:] = 0xA5


def mask_buf(mask) -> Buf:
    m = Buf(abi.I32, [len(mask)])
    m.flat()[:] = np.asarray(mask, np.int32)
    return m


def run_select(plugin, row, k: dict) -> int:
    """k: mask, xs, qs, ss, x, q, s (None = absent)."""
    return H.run_row(plugin, row, [k["mask"], k["xs"], k["qs"], k["ss"], k["x"], k["q"], k["s"]],
                     [pint("M", k["mask"].shape[0])])


def selected_exactly(src: Buf, before: Buf, after: Buf, mask) -> bool:
    bytes_ = abi.BITS[src.dtype] // 8
    width = src.shape[1] * bytes_
    sp, dp = src.strides[0] * bytes_, before.strides[0] * bytes_
    at = np.arange(len(after.bytes))
    row, col = at // dp, at % dp
    m = np.asarray(mask)
    copied = (row < len(m)) & (col < width)
    copied[copied] &= m[row[copied]] == 1
    want = before.bytes.copy()
    want[copied] = src.bytes[row[copied] * sp + col[copied]]
    return bool(np.array_equal(after.bytes, want))


def run_drop(plugin, row, mask: Buf, ids: Buf, top_k: int) -> int:
    return H.run_row(plugin, row, [mask, ids], [pint("M", mask.shape[0]), pint("top_k", top_k)])


def dropped_exactly(before: Buf, after: Buf, mask, top_k: int) -> bool:
    pitch = before.strides[0]
    b, a = before.flat(), after.flat()
    at = np.arange(len(a))
    row, col = at // pitch, at % pitch
    m = np.asarray(mask)
    dropped = (row < len(m)) & (col < top_k)
    dropped[dropped] &= m[row[dropped]] == 1
    return bool(np.array_equal(a, np.where(dropped, -1, b)))


# ----------------------------------------------------------------- rho (kernel_test.cpp:522-586)

class RhoRun:
    def __init__(self):
        self.n = self.heads = 0
        self.pitch = 0
        self.col = 1
        self.slots = 4
        self.bf16 = False
        self.slot = 0
        self.a = []
        self.mask = []
        self.a_log, self.dt_bias = [], []
        self.nd = []
        self.bounds = []

    def copy(self):
        c = RhoRun()
        c.__dict__.update({k: (list(v) if isinstance(v, list) else v) for k, v in self.__dict__.items()})
        return c


def run_rho(plugin, row, c: RhoRun, bounds_as: Buf | None = None) -> int:
    pitch = c.pitch or c.heads
    a = Buf(abi.BF16 if c.bf16 else abi.F32, [c.n, c.heads], [pitch, c.col])
    mask, alog, dtb = Buf(abi.I32, [c.n]), Buf(abi.F32, [c.heads]), Buf(abi.F32, [c.heads])
    nd, sidx = Buf(abi.F32, [c.slots, c.heads, 1, 2]), Buf(abi.I32, [1, 1])
    af = a.flat()
    av = np.asarray(c.a, np.float32).reshape(c.n, c.heads) if c.n * c.heads else np.zeros((c.n, c.heads), np.float32)
    for t in range(c.n):
        idx = t * pitch + np.arange(c.heads) * c.col
        af[idx] = H.f32_to_bf16_bits(av[t]) if c.bf16 else av[t]
    mask.flat()[: c.n] = c.mask
    alog.flat()[:] = c.a_log
    dtb.flat()[:] = c.dt_bias
    nd.flat()[: len(c.nd)] = np.asarray(c.nd, np.float32)
    sidx.flat()[0] = c.slot
    bounds = Buf(abi.I32, [len(c.bounds)])
    bounds.flat()[: len(c.bounds)] = c.bounds
    if bounds_as is not None:
        bounds = bounds_as
    use_bounds = bounds if (bounds_as is not None or c.bounds) else None
    rc = H.run_row(plugin, row, [a, mask, alog, dtb, nd, sidx, use_bounds], [pint("M", c.n), pint("n_head", c.heads)])
    c.nd = list(nd.flat()[: len(c.nd)].astype(np.float32))
    return rc


def random_rho(r: H.Rng, n, heads, exact_share, bf16) -> RhoRun:
    c = RhoRun()
    c.n, c.heads, c.bf16, c.slot = n, heads, bf16, 2
    for _ in range(n * heads):
        v = np.float32(2.0 * r.normal())
        c.a.append(float(H.bf16_bits_to_f32(H.f32_to_bf16_bits(v))[0]) if bf16 else float(v))
    c.mask = [0 if r.uniform() < exact_share else 1 for _ in range(n)]
    for _ in range(heads):
        c.a_log.append(float(np.float32(-4.0 + 6.5 * r.uniform())))
        c.dt_bias.append(float(np.float32(-3.0 + 4.0 * r.uniform())))
    c.nd = [0.0] * (c.slots * heads * 2)
    return c


def nd_rho(c: RhoRun, h: int) -> float:
    n = np.float32(c.nd[(c.slot * c.heads + h) * 2])
    d = np.float32(c.nd[(c.slot * c.heads + h) * 2 + 1])
    if not d > 0:
        return 1.0
    q = np.float32(n / d)
    return 0.0 if q < 0 else (1.0 if q > 1 else float(q))


# ----------------------------------------------------------------- state_correct / state_read (kernel_test.cpp:588-645)

def slot_index(seq_slots) -> Buf:
    b = Buf(abi.I32, [len(seq_slots), 2])
    f = b.flat()
    for s, v in enumerate(seq_slots):
        f[2 * s] = v
        f[2 * s + 1] = 999
    return b


class CorrectRun:
    def __init__(self, slots, heads, sd0, sd1, seq_slots, pad):
        self.slots, self.heads, self.sd0, self.sd1 = slots, heads, sd0, sd1
        row = sd1 + pad
        head = sd0 * row + pad
        slot = heads * head + pad
        self.state = Buf(abi.F32, [slots, heads, sd0, sd1], [slot, head, row, 1])
        self.applied = Buf(abi.F32, [slots, heads, 1, 1])
        self.c = Buf(abi.F32, [heads, sd0, sd1])
        self.nd = Buf(abi.F32, [slots, heads, 1, 2])
        self.sidx = slot_index(seq_slots)
        self.aidx = slot_index(seq_slots)
        self.nidx = slot_index(seq_slots)

    def copy(self):
        k = CorrectRun.__new__(CorrectRun)
        k.__dict__.update({n: (v.copy() if isinstance(v, Buf) else v) for n, v in self.__dict__.items()})
        return k

    def st_at(self, s, h, i, j):
        st = self.state.strides
        return s * st[0] + h * st[1] + i * st[2] + j


def run_correct(plugin, row, k: CorrectRun, mode, alpha, with_nd, bounds=()) -> int:
    b = Buf(abi.I32, [len(bounds)])
    b.flat()[: len(bounds)] = bounds
    return H.run_row(plugin, row, [k.state, k.sidx, k.applied, k.aidx, k.c, k.nd if with_nd else None,
                                   k.nidx if with_nd else None, b if len(bounds) else None],
                     [pint("M", k.sidx.shape[0]), pstr("mode", mode), pf64("alpha", alpha), pint("n_head", k.heads),
                      pint("sd0", k.sd0), pint("sd1", k.sd1)])


def run_state_read(plugin, row, k: CorrectRun, index: Buf):
    out = Buf(abi.F32, [index.shape[0], k.heads, k.sd0, k.sd1])
    out.flat()[:] = 12345.0
    rc = H.run_row(plugin, row, [k.state, index, out],
                   [pint("M", index.shape[0]), pint("n_head", k.heads), pint("sd0", k.sd0), pint("sd1", k.sd1)])
    return rc, out


def random_correct(r: H.Rng, heads, seq_slots=(4, -1, 1, 5), sd=128, pad=8) -> CorrectRun:
    k = CorrectRun(6, heads, sd, sd, list(seq_slots), pad)
    sf = k.state.flat()
    sf[:] = [r.normal() for _ in range(len(sf))]
    k.c.flat()[:] = [0.01 * r.normal() for _ in range(k.c.numel())]
    k.applied.flat()[:] = [0.5 + r.normal() for _ in range(k.applied.numel())]
    nd = k.nd.flat()
    for i in range(0, k.nd.numel(), 2):
        d = np.float32(1.0 + 50.0 * r.uniform())
        nd[i] = np.float32(d * 1.2 * r.uniform())
        nd[i + 1] = d
    return k


# ----------------------------------------------------------------- hazard (kernel_test.cpp:741-767)

class HazardCall:
    def __init__(self, s=0, e=64, first_pos=0, slot=1, span=0, b=0, m0=0.0, m1=0.0, count=0.0):
        self.s, self.e, self.first_pos, self.slot, self.span, self.b = s, e, first_pos, slot, span, b
        self.m0, self.m1, self.count = m0, m1, count


def run_hazard(plugin, row, c: HazardCall):
    n = c.e if c.e > 1 else 1
    cu, pos, bounds = Buf(abi.I32, [2]), Buf(abi.I32, [n]), Buf(abi.I32, [4])
    span, meta = Buf(abi.I32, [c.span if c.span > 0 else 1]), Buf(abi.F32, [4, 1, 1, 2])
    idx, cnt = Buf(abi.I32, [1, 1]), Buf(abi.F32, [1])
    cu.flat()[:2] = [c.s, c.e]
    pos.flat()[:n] = c.first_pos + np.arange(n)
    bounds.flat()[:4] = [c.s, c.b, c.b, c.e]
    meta.flat()[2:4] = [c.m0, c.m1]
    idx.flat()[0] = c.slot
    cnt.flat()[0] = c.count
    rc = H.run_row(plugin, row, [cu, pos, bounds if c.b > 0 else None, span if c.span > 0 else None, meta, idx, cnt],
                   [pint("M", 1)])
    return rc, float(meta.flat()[2]), float(meta.flat()[3]), float(cnt.flat()[0])
