"""The refusal codes of the seven reference ops' operand parse, on randomly broken operand sets.

Each case starts from a valid operand set of one op and breaks one to three things at once -- an operand
dropped or added, its dtype, rank, an extent or a stride changed, a parameter dropped or given a bad
value -- and asks each implementation for its code: the product library's and the reference's own host
rows' (oracle/_ref, where they were built from the reference's sources) parse functions, called directly
(they read descriptors only; the product's device rows are never launched), and the oracle's host row. All must return the same code, so the product
refuses what the reference refuses and the same code wins when several rules are broken
(kernels/host_ref.cpp:16-282,435-463)."""
import ctypes as C
import random

import numpy as np
import pytest

import harness as H
from harness import abi

PARSE = ["mask", "rho", "correct", "state_read", "select", "drop", "hazard"]
DTYPES = [abi.F32, abi.I32, abi.BF16, abi.I8, abi.U8, abi.F16]


class Opd:
    """One operand descriptor: dtype, shape, strides in elements (packed when None)."""

    def __init__(self, dtype, shape, strides=None):
        self.dtype, self.shape = dtype, list(shape)
        self.strides = list(strides) if strides is not None else self.packed()

    def packed(self):
        s, out = 1, [0] * len(self.shape)
        for i in range(len(self.shape) - 1, -1, -1):
            out[i] = s
            s *= self.shape[i]
        return out

    def copy(self):
        return Opd(self.dtype, self.shape, self.strides)


def base_case(op, r):
    """A valid operand list (None = absent) and parameter dict of `op`."""
    n, H_, V = r.choice([4, 64, 300]), r.choice([1, 2, 4]), r.choice([4, 8])
    if op == "mask":
        return [Opd(abi.I32, [2]), Opd(abi.I32, [n]), Opd(abi.I32, [n]), Opd(abi.F32, [97]), Opd(abi.I32, [n]),
                Opd(abi.I32, [4]), Opd(abi.I32, [3]) if r.random() < 0.5 else None], \
            {"M": ("i", n), "share": ("f", 0.3), "seed": ("i", 7), "mode": ("s", r.choice(["class", "random", "none", "all", "step"]))}
    if op == "rho":
        return [Opd(abi.BF16, [n, H_], [2 * H_, 1]), Opd(abi.I32, [n]), Opd(abi.F32, [H_]), Opd(abi.F32, [H_]),
                Opd(abi.F32, [3, H_, 1, 2]), Opd(abi.I32, [1, 1]), Opd(abi.I32, [4]) if r.random() < 0.5 else None], \
            {"M": ("i", n), "n_head": ("i", H_)}
    if op == "correct":
        nd = r.random() < 0.5
        return [Opd(abi.F32, [3, H_, V, V]), Opd(abi.I32, [1]), Opd(abi.F32, [3, H_, 1, 1]), Opd(abi.I32, [1]),
                Opd(abi.F32, [H_, V, V]), Opd(abi.F32, [3, H_, 2, 1]) if nd else None, Opd(abi.I32, [1]) if nd else None,
                Opd(abi.I32, [4]) if r.random() < 0.5 else None], \
            {"M": ("i", 1), "mode": ("s", r.choice(["undo", "apply"])), "alpha": ("f", 0.5), "n_head": ("i", H_),
             "sd0": ("i", V), "sd1": ("i", V)}
    if op == "state_read":
        return [Opd(abi.F32, [3, H_, V, V]), Opd(abi.I32, [2]), Opd(abi.F32, [2, H_, V, V])], \
            {"M": ("i", 2), "n_head": ("i", H_), "sd0": ("i", V), "sd1": ("i", V)}
    if op == "select":
        d = r.choice([128, 256])
        q = r.random() < 0.5
        return [Opd(abi.I32, [n]), Opd(abi.BF16, [n, d]), Opd(abi.I8, [n, d]) if q else None,
                Opd(abi.F32, [n, d // 128]) if q else None, Opd(abi.BF16, [n, d], [d + 8, 1]),
                Opd(abi.I8, [n, d]) if q else None, Opd(abi.F32, [n, d // 128]) if q else None], {"M": ("i", n)}
    if op == "drop":
        return [Opd(abi.I32, [n]), Opd(abi.I32, [n, 10])], {"M": ("i", n), "top_k": ("i", r.choice([0, 4, 10]))}
    if op == "hazard":
        return [Opd(abi.I32, [2]), Opd(abi.I32, [n]), Opd(abi.I32, [4]) if r.random() < 0.5 else None,
                Opd(abi.I32, [n + 5]) if r.random() < 0.5 else None, Opd(abi.F32, [3, 1, 2]), Opd(abi.I32, [1]),
                Opd(abi.F32, [1])], {"M": ("i", 1)}
    raise AssertionError(op)


BAD_VALUES = {"mode": [("s", "classy"), ("s", ""), ("i", 1)], "share": [("f", 1.5), ("f", -0.1), ("f", float("nan"))],
              "seed": [("s", "x")], "n_head": [("i", 0), ("i", 5), ("s", "2")], "alpha": [("f", float("nan")), ("f", float("inf"))],
              "sd0": [("i", 3)], "sd1": [("i", 5)], "top_k": [("i", -1), ("i", 11), ("f", 2.0)], "M": [("i", 0)]}


def mutate(opds, params, r):
    opds, params = [o.copy() if o else None for o in opds], dict(params)
    kind = r.randrange(7)
    i = r.randrange(len(opds))
    o = opds[i]
    if kind == 0:
        opds[i] = None
    elif kind == 1 and o is None:
        opds[i] = Opd(r.choice(DTYPES), [r.choice([1, 2, 4, 64])])
    elif kind == 1 or kind == 2:
        if o is not None:
            o.dtype = r.choice(DTYPES)
    elif kind == 3 and o is not None:
        if o.shape and r.random() < 0.5:
            o.shape.pop()
        else:
            o.shape.append(r.choice([1, 2]))
        o.strides = o.packed()
    elif kind == 4 and o is not None and o.shape:
        ax = r.randrange(len(o.shape))
        o.shape[ax] = max(0, o.shape[ax] + r.choice([-1, 1, 3]))
        o.strides = o.packed()
    elif kind == 5 and o is not None and o.shape:
        ax = r.randrange(len(o.shape))
        o.strides[ax] = o.strides[ax] * 2 + (1 if r.random() < 0.3 else 0)
    elif kind == 6 and params:
        key = r.choice(list(params))
        if r.random() < 0.4:
            del params[key]
        elif key in BAD_VALUES:
            params[key] = r.choice(BAD_VALUES[key])
    return opds, params


def build_args(opds, params):
    """RadArgs over zero-filled host buffers covering every element the descriptors reach (the oracle's host
    row computes on them when its parse passes; zeros are valid values for every op)."""
    tens, bufs = [], []
    for o in opds:
        if o is None:
            tens.append(abi.absent())
            continue
        last = sum((e - 1) * abs(s) for e, s in zip(o.shape, o.strides)) if all(o.shape) else 0
        b = np.zeros(((last + 1) * abi.BITS[o.dtype] + 7) // 8 + 64, np.uint8)
        bufs.append(b)
        base = (b.ctypes.data + 15) & ~15
        tens.append(abi.tensor(o.dtype, o.shape, base, o.strides))
    pp = []
    for k, (t, v) in params.items():
        pp.append(abi.pint(k, v) if t == "i" else abi.pf64(k, v) if t == "f" else abi.pstr(k, v))
    return tens, pp, bufs


ROW = {"mask": "ridgefill_mask", "rho": "ridgefill_rho_update", "correct": "ridgefill_state_correct",
       "state_read": "ridgefill_state_read", "select": "ridgefill_select", "drop": "ridgefill_drop_rows",
       "hazard": "ridgefill_hazard"}


def parse_code(plugin, op, tens, pp):
    """The code of `op`'s parse function (exported by the product and by the reference's host rows)."""
    args, keep = abi.Plugin.args(tens, pp)
    fn = getattr(plugin.lib, f"ridgefill_{op}_parse")
    fn.restype = C.c_int
    out = (C.c_uint8 * 4096)()
    rc = fn(C.byref(args), out)
    del keep
    return rc


def oracle_code(plugin, op, tens, pp):
    """The oracle's host row (it parses, then computes on the zero-filled buffers when the parse passes)."""
    return plugin.launch(plugin.find_row(ROW[op], abi.DOMAIN_HOST), tens, pp)


@pytest.mark.parametrize("op", PARSE)
def test_refusal_codes_agree_on_broken_operand_sets(op, product_lib, oracle_lib):
    libs = [("product", product_lib), ("oracle", oracle_lib)]
    ref = H.reference()
    if ref is not None:
        libs.append(("reference", ref))
    r = random.Random(sum(map(ord, op)))
    seen = {}
    for case in range(2500):
        opds, params = base_case(op, r)
        if case:   # case 0: the valid set itself
            for _ in range(r.choice([1, 1, 2, 3])):
                opds, params = mutate(opds, params, r)
        tens, pp, bufs = build_args(opds, params)
        codes = {name: (oracle_code if name == "oracle" else parse_code)(lib, op, tens, pp) for name, lib in libs}
        del bufs
        assert len(set(codes.values())) == 1, (op, case, codes,
                                               [(o.dtype, o.shape, o.strides) if o else None for o in opds], params)
        seen[codes["product"]] = seen.get(codes["product"], 0) + 1
    # the broken sets reach every kind of refusal the op has, and the valid ones pass
    assert abi.OK in seen and abi.E_INVAL in seen and abi.E_DTYPE in seen and abi.E_SHAPE in seen, seen
