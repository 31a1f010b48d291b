"""TEST INFRASTRUCTURE and CPU baseline, not the product: one RidgeFill approximate pass on the host.

The rows the reference implements on the host -- ridgefill_mask, ridgefill_select, ridgefill_state_correct,
ridgefill_rho_update, ridgefill_hazard (kernels/host_ref.cpp) -- run as the reference's own host rows
compiled from its sources (oracle/_ref/ridgefill_ref.so) when that library was built, else as this
repository's restatement (oracle/_build/libridgefill_oracle.so). The reference has no CPU projector GEMM,
activation quantiser or DeltaNet fill (they live in radiance's absent libr4d): those run as the
restatement's oracles, OpenMP over the host's cores. Used by bench.py (cpu_baseline, --impl reference).
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "radiance-ridgefill_b200"))
import ridgefill_abi as abi  # noqa: E402

ORACLE_SO = ROOT / "oracle" / "_build" / "libridgefill_oracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "ridgefill_ref.so"


def load():
    """(rows plugin, kind, oracle plugin): the reference's host rows when built, else the restatement."""
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)
    oracle = abi.Plugin(ORACLE_SO)
    bind(oracle.lib)
    if REF_SO.exists():
        return abi.Plugin(REF_SO), "reference", oracle
    return oracle, "port", oracle


def bind(lib):
    P, i64 = C.c_void_p, C.c_int64
    lib.oracle_quant_act_i8g.argtypes = [P, i64, i64, i64, i64, P, i64, P, i64]
    lib.oracle_gemm_nt_q.argtypes = [P, i64, P, i64, P, i64, P, P, P, i64, P, i64, i64, i64, i64, i64, i64]
    lib.oracle_gdn_fill_f32.argtypes = [P, P, P, P, P, P, P, i64, i64, P, i64, P, i64, i64, i64, i64, C.c_float, i64, i64]
    lib.oracle_threads.restype = C.c_int


def _bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


class CpuStep:
    """The pass of ridgefill_step.Step on host buffers, `T` rows (a bounded sample of the 32K workload)."""

    def __init__(self, T: int, d: int = 2048, hk: int = 16, hv: int = 32, share: float = 0.30, vocab: int = 65536,
                 seed: int = 0):
        self.rows, self.kind, self.oracle = load()
        self.T, self.d, self.hk, self.hv, self.D = T, d, hk, hv, 128
        self.share = share
        rng = np.random.default_rng(seed)
        D = self.D
        self.cu_last = np.array([0, T], np.int32)
        self.token_ids = rng.integers(0, vocab, T).astype(np.int32)
        self.positions = np.arange(T, dtype=np.int32)
        score = rng.standard_normal(vocab).astype(np.float32)
        score[rng.random(vocab) < 0.5] = -np.inf
        self.score = score
        self.mask = np.zeros(T, np.int32)
        self.bounds = np.zeros(4, np.int32)
        self.h_s = _bf16(rng.standard_normal((T, d)))
        self.codes = np.zeros((T, d), np.int8)
        self.a_scale = np.zeros((T, 1), np.float32)
        self.w = rng.integers(-127, 128, (d, d)).astype(np.int8)
        self.w_scale = rng.uniform(1e-3, 1e-2, (1, d)).astype(np.float32)
        self.bias = _bf16(0.1 * rng.standard_normal(d))
        self.x_proj = np.zeros((T, d), np.uint16)
        self.x = _bf16(rng.standard_normal((T, d)))
        k = rng.standard_normal((T, hk, D)).astype(np.float32)
        self.k = _bf16(k / np.linalg.norm(k, axis=-1, keepdims=True))
        self.v = _bf16(rng.standard_normal((T, hv, D)))
        self.g = (-np.log1p(np.exp(rng.standard_normal((T, hv))))).astype(np.float32)
        self.beta = (1 / (1 + np.exp(-rng.standard_normal((T, hv))))).astype(np.float32)
        self.state = np.zeros((1, hv, D, D), np.float32)
        self.state_idx = np.zeros((1, 1), np.int32)
        self.cu = np.array([0, T], np.int32)
        self.Cm = (0.01 * rng.standard_normal((hv, D, D))).astype(np.float32)
        self.applied = np.zeros((1, hv, 1, 1), np.float32)
        self.nd = np.zeros((1, hv, 1, 2), np.float32)
        self.ab = _bf16(rng.standard_normal((T, 2 * hv)))
        self.a_log = (0.5 * rng.standard_normal(hv)).astype(np.float32)
        self.dt_bias = (0.5 * rng.standard_normal(hv)).astype(np.float32)
        self.meta = np.zeros((1, 1, 1, 2), np.float32)
        self.count = np.zeros(1, np.float32)

    @property
    def threads(self) -> int:
        return int(self.oracle.lib.oracle_threads())

    def _row(self, op):
        return self.rows.find_row(op, abi.DOMAIN_HOST)

    @staticmethod
    def _t(a: np.ndarray, code: int, shape=None, strides=None):
        if shape is None:
            shape, strides = list(a.shape), [s // a.itemsize for s in a.strides]
        return abi.tensor(code, shape, a.ctypes.data, strides)

    def run(self) -> None:
        t, P, S, F = self._t, abi.pint, abi.pstr, abi.pf64
        T, d, hv, D, L = self.T, self.d, self.hv, self.D, self.rows
        A = abi.absent()

        def go(op, tens, params):
            rc = L.launch(self._row(op), tens, params)
            if rc != abi.OK:
                raise RuntimeError(f"{op}: host row returned {rc}")

        go("ridgefill_mask", [t(self.cu_last, abi.I32), t(self.token_ids, abi.I32), t(self.positions, abi.I32),
                              t(self.score, abi.F32), t(self.mask, abi.I32), t(self.bounds, abi.I32), A],
           [P("M", T), F("share", self.share), P("seed", 0), S("mode", "class")])
        o = self.oracle.lib
        o.oracle_quant_act_i8g(self.h_s.ctypes.data, d, T, d, d, self.codes.ctypes.data, d, self.a_scale.ctypes.data, 1)
        o.oracle_gemm_nt_q(self.codes.ctypes.data, d, self.a_scale.ctypes.data, 1, self.w.ctypes.data, d,
                           self.w_scale.ctypes.data, self.bias.ctypes.data, self.x_proj.ctypes.data, d, None, T, d, d, d, 0, T)
        go("ridgefill_select", [t(self.mask, abi.I32), t(self.x_proj, abi.BF16), A, A, t(self.x, abi.BF16), A, A], [P("M", T)])
        corr = [P("M", 1), S("mode", "undo"), F("alpha", 1.0), P("n_head", hv), P("sd0", D), P("sd1", D)]
        go("ridgefill_state_correct", [t(self.state, abi.F32), t(self.state_idx, abi.I32), t(self.applied, abi.F32),
                                       t(self.state_idx, abi.I32), t(self.Cm, abi.F32), A, A, t(self.bounds, abi.I32)], corr)
        o.oracle_gdn_fill_f32(None, self.k.ctypes.data, self.v.ctypes.data, self.g.ctypes.data, self.beta.ctypes.data,
                              self.state.ctypes.data, self.state_idx.ctypes.data, 1, 1, self.cu.ctypes.data, 1, None,
                              self.hk, hv, D, D, C.c_float(1.0 / math.sqrt(D)), 0, hv)
        go("ridgefill_rho_update", [t(self.ab, abi.BF16, [T, hv], [2 * hv, 1]), t(self.mask, abi.I32), t(self.a_log, abi.F32),
                                    t(self.dt_bias, abi.F32), t(self.nd, abi.F32), t(self.state_idx, abi.I32),
                                    t(self.bounds, abi.I32)], [P("M", T), P("n_head", hv)])
        corr[1] = S("mode", "apply")
        go("ridgefill_state_correct", [t(self.state, abi.F32), t(self.state_idx, abi.I32), t(self.applied, abi.F32),
                                       t(self.state_idx, abi.I32), t(self.Cm, abi.F32), t(self.nd, abi.F32),
                                       t(self.state_idx, abi.I32), t(self.bounds, abi.I32)], corr)
        go("ridgefill_hazard", [t(self.cu_last, abi.I32), t(self.positions, abi.I32), t(self.bounds, abi.I32), A,
                                t(self.meta, abi.F32), t(self.state_idx, abi.I32), t(self.count, abi.F32)], [P("M", 1)])

    def time_steps(self, steps: int, warmup: int = 1) -> float:
        """Seconds per pass over `steps` timed passes."""
        for _ in range(warmup):
            self.run()
        t0 = time.perf_counter()
        for _ in range(steps):
            self.run()
        return (time.perf_counter() - t0) / max(steps, 1)
