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


def host_cores() -> int:
    """The host threads this process may run on (its CPU affinity), whatever OMP_NUM_THREADS says."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def load():
    """(rows plugin, kind, oracle plugin): the reference's host rows when built, else the restatement. The
    restatement's OpenMP loops are given every host core."""
    if not ORACLE_SO.exists() or ORACLE_SO.stat().st_mtime < (ROOT / "oracle" / "ridgefill_oracle.cpp").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)
    oracle = abi.Plugin(ORACLE_SO)
    bind(oracle.lib)
    oracle.lib.oracle_set_threads(host_cores())
    if REF_SO.exists():
        return abi.Plugin(REF_SO), "reference", oracle
    return oracle, "port", oracle


def bind(lib):
    P, i64 = C.c_void_p, C.c_int64
    lib.oracle_quant_act_i8g.argtypes = [P, i64, i64, i64, i64, P, i64, P, i64]
    lib.oracle_gemm_nt_q.argtypes = [P, i64, P, i64, P, i64, P, P, P, i64, P, i64, i64, i64, i64, i64, i64]
    lib.oracle_gemm_nt_bias.argtypes = [P, i64, P, i64, P, C.c_int, P, i64, P, i64, P, i64, i64, C.c_int, i64, i64]
    lib.oracle_gdn_conv_prep.argtypes = [P, i64, P, P, P, P, P, i64, P, i64, P, P, P, P, P, P, P, P, P, i64, i64, i64]
    lib.oracle_attn_kv_fill.argtypes = [P, P, P, C.c_int, P, C.c_int, P, P, i64, P, i64, i64, i64, C.c_double, C.c_float,
                                        C.c_int, P]
    for f in (lib.oracle_gdn_fill_f32, lib.oracle_gdn_fill_f64):
        f.argtypes = [P, P, P, P, P, P, P, i64, i64, P, i64, P, i64, i64, i64, i64, C.c_float, i64, i64]
    lib.oracle_threads.restype = C.c_int
    lib.oracle_set_threads.argtypes = [C.c_int]


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


# ======================================================================= the pass over every late layer

def to_host(inputs: dict) -> dict:
    """late_pass.late_inputs' torch tensors (any device) as numpy arrays, bf16 as its bits (uint16)."""
    import torch

    def one(t):
        t = t.detach().cpu()
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16).copy()
        return t.numpy().copy()

    return {k: [one(t) for t in v] if isinstance(v, list) else one(v) for k, v in inputs.items()}


def _p(a):
    return None if a is None else a.ctypes.data


class CpuLatePass:
    """late_pass.LatePass on host buffers: the same launch sequence over the same inputs (`inputs`: the numpy
    form of late_pass.late_inputs, see to_host). The reference's host rows (mask, select, state correction,
    rho, hazard) come from oracle/_ref when built, else from the restatement; the quantiser, the int8 and bf16
    GEMMs, conv_prep, the K/V cache write and the fill (f32, or f64 with `f64=True`) from the restatement.
    `layers` (optional) limits the pass to the first that many late layers (a bounded CPU sample)."""

    def __init__(self, shape, inputs: dict, f64: bool = False, layers: int | None = None):
        import copy
        self.rows, self.kind, self.oracle = load()
        self.s = s = copy.copy(shape)
        if layers is not None:
            s.layers = s.layers[:layers]
        self.x = x = inputs
        self.f64 = f64
        T, d, G, D = s.T, s.d, s.n_gdn, s.head
        self.grp = s.group or d
        hv_all = G * s.hv
        self.mask = np.zeros(T, np.int32)
        self.bounds = np.zeros(4, np.int32)
        self.codes_h = np.zeros((T, d), np.int8)
        self.scale_h = np.zeros((T, d // self.grp), np.float32)
        self.x_proj = np.zeros((T, d), np.uint16)
        self.xl = [t.copy() for t in x["x_exact"][:len(s.layers)]]
        self.codes_x = np.zeros((T, d), np.int8)
        self.scale_x = np.zeros((T, d // self.grp), np.float32)
        G_all = len([c for c in shape.layers if c == "G"])   # the inputs' DeltaNet arrays cover every layer
        self.state = np.ascontiguousarray(x["state"][:, :hv_all]).copy()
        self.C = np.ascontiguousarray(x["C"][:hv_all])
        self.applied = np.zeros((s.n_seq, hv_all, 1, 1), np.float32)
        self.nd = np.zeros((s.n_seq, hv_all, 1, 2), np.float32)
        self.meta = np.zeros((s.n_seq, 1, 1, 2), np.float32)
        self.count = np.zeros(1, np.float32)
        self.slot_last = np.array([[s.n_seq - 1]], np.int32)
        self.slots_all = np.arange(s.n_seq, dtype=np.int32)
        if s.block_inputs:
            self.ab = [np.zeros((T, 2 * s.hv), np.uint16) for _ in range(G)]
            self.k = np.zeros((T, hv_all // (s.hv // s.hk), D), np.uint16)
            self.v = np.zeros((T, hv_all, D), np.uint16)
            self.g = np.zeros((T, hv_all), np.float32)
            self.beta = np.zeros((T, hv_all), np.float32)
            self.conv_state = [t.copy() for t in x["conv_state"][:G]]
        else:
            hk_all = G * s.hk
            self.ab = x["ab"][:G]
            self.k = np.ascontiguousarray(x["k"].reshape(T, G_all * s.hk, D)[:, :hk_all])
            self.v = np.ascontiguousarray(x["v"].reshape(T, G_all * s.hv, D)[:, :hv_all])
            self.g = np.ascontiguousarray(x["g"][:, :hv_all])
            self.beta = np.ascontiguousarray(x["beta"][:, :hv_all])
        if s.n_attn:
            Ha, Dh = s.hkv, s.head_attn
            self.cache = [np.zeros((2, T + 1024, Ha, Dh), np.uint16) for _ in range(s.n_attn)]
            self.rope_pos = np.ascontiguousarray(np.broadcast_to(x["positions"], (3, T)))

    @property
    def threads(self) -> int:
        return int(self.oracle.lib.oracle_threads())

    @staticmethod
    def _t(a, code, shape=None, strides=None, offset=0):
        if shape is None:
            shape, strides = list(a.shape), [st // a.itemsize for st in a.strides]
        return abi.tensor(code, shape, a.ctypes.data + offset * a.itemsize, strides)

    def _go(self, op, tens, params):
        rc = self.rows.launch(self.rows.find_row(op, abi.DOMAIN_HOST), tens, params)
        if rc != abi.OK:
            raise RuntimeError(f"{op}: host row returned {rc}")

    def _gemm_q(self, a, sa, w, sw, bias, y, N):
        s = self.s
        self.oracle.lib.oracle_gemm_nt_q(_p(a), s.d, _p(sa), s.d // self.grp, _p(w), s.d, _p(sw), _p(bias), _p(y), N, None,
                                         s.T, N, s.d, self.grp, 0, s.T)

    def _quant(self, src, codes, scale):
        s = self.s
        self.oracle.lib.oracle_quant_act_i8g(_p(src), s.d, s.T, s.d, self.grp, _p(codes), s.d, _p(scale), s.d // self.grp)

    def _correct(self, mode):
        s, t, A = self.s, self._t, abi.absent()
        G, D = s.n_gdn, s.head
        tens = [t(self.state, abi.F32), t(self.slot_last, abi.I32), t(self.applied, abi.F32), t(self.slot_last, abi.I32),
                t(self.C, abi.F32)]
        tens += [t(self.nd, abi.F32), t(self.slot_last, abi.I32)] if mode == "apply" else [A, A]
        self._go("ridgefill_state_correct", tens + [t(self.bounds, abi.I32)],
                 [abi.pint("M", 1), abi.pstr("mode", mode), abi.pf64("alpha", s.alpha), abi.pint("n_head", G * s.hv),
                  abi.pint("sd0", D), abi.pint("sd1", D)])

    def run(self) -> None:
        s, x, t, o = self.s, self.x, self._t, self.oracle.lib
        P, S, F, A = abi.pint, abi.pstr, abi.pf64, abi.absent()
        T, d, G, hk, hv, D = s.T, s.d, s.n_gdn, s.hk, s.hv, s.head
        self._go("ridgefill_mask", [t(x["cu_last"], abi.I32), t(x["token_ids"], abi.I32), t(x["positions"], abi.I32),
                                    t(x["score"], abi.F32), t(self.mask, abi.I32), t(self.bounds, abi.I32), A],
                 [P("M", T), F("share", s.share), P("seed", 0), S("mode", "class")])
        self._quant(x["h_s"], self.codes_h, self.scale_h)
        if G:
            self._correct("undo")
        gi = ai = 0
        for li, kind in enumerate(s.layers):
            self._gemm_q(self.codes_h, self.scale_h, x["w_proj"][li], x["s_proj"][li], x["b_proj"][li], self.x_proj, d)
            self._go("ridgefill_select", [t(self.mask, abi.I32), t(self.x_proj, abi.BF16), A, A, t(self.xl[li], abi.BF16),
                                          A, A], [P("M", T)])
            if kind == "G" and s.block_inputs:
                C_ = s.conv_dim
                self._quant(self.xl[li], self.codes_x, self.scale_x)
                mixed = np.zeros((T, C_), np.uint16)
                self._gemm_q(self.codes_x, self.scale_x, x["w_in"][gi], x["s_in"][gi], None, mixed, C_)
                zero = np.zeros(2 * hv, np.uint16)
                o.oracle_gemm_nt_bias(_p(self.xl[li]), d, _p(x["w_ab"][gi]), d, _p(zero), 0, None, 0, _p(self.ab[gi]),
                                      2 * hv, None, 2 * hv, d, 0, 0, T)
                a_ = np.ascontiguousarray(self.ab[gi][:, :hv])
                b_ = np.ascontiguousarray(self.ab[gi][:, hv:])
                q = np.zeros((T, hk, D), np.uint16)
                k = np.zeros((T, hk, D), np.uint16)
                v = np.zeros((T, hv, D), np.uint16)
                g = np.zeros((T, hv), np.float32)
                beta = np.zeros((T, hv), np.float32)
                ctx = np.zeros(s.n_seq, np.int32)
                cs = self.conv_state[gi]
                o.oracle_gdn_conv_prep(_p(mixed), C_, _p(x["w_conv"][gi]), None, _p(x["a_log"][gi]), _p(x["dt_bias"][gi]),
                                       _p(cs), cs.shape[0], _p(x["cu_seqlens"]), s.n_seq, _p(a_), _p(b_), _p(self.slots_all),
                                       _p(ctx), _p(q), _p(k), _p(v), _p(g), _p(beta), T, hk, hv)
                self.k[:, gi * hk:(gi + 1) * hk] = k
                self.v[:, gi * hv:(gi + 1) * hv] = v
                self.g[:, gi * hv:(gi + 1) * hv] = g
                self.beta[:, gi * hv:(gi + 1) * hv] = beta
            elif kind == "A":
                Ha, Dh = s.hkv, s.head_attn
                self._quant(self.xl[li], self.codes_x, self.scale_x)
                kv = np.zeros((T, 2 * Ha * Dh), np.uint16)
                self._gemm_q(self.codes_x, self.scale_x, x["w_kv"][ai], x["s_kv"][ai], None, kv, 2 * Ha * Dh)
                kk = np.ascontiguousarray(kv[:, :Ha * Dh].reshape(T, Ha, Dh))
                vv = np.ascontiguousarray(kv[:, Ha * Dh:].reshape(T, Ha, Dh))
                sec = np.asarray(s.rope_sections, np.int32)
                cache = self.cache[ai]
                o.oracle_attn_kv_fill(_p(kk), _p(vv), _p(x["k_norm"][ai]), 0, _p(self.rope_pos), 3, _p(x["slot_mapping"]),
                                      _p(cache), cache.shape[1], None, T, Ha, s.rope_dim, float(s.rope_theta), 1e-6, 2,
                                      _p(sec))
                ai += 1
            if kind == "G":
                gi += 1
        if G:
            fill = o.oracle_gdn_fill_f64 if self.f64 else o.oracle_gdn_fill_f32
            fill(None, _p(self.k), _p(self.v), _p(self.g), _p(self.beta), _p(self.state), _p(self.slots_all), 1,
                 self.state.shape[0], _p(x["cu_seqlens"]), s.n_seq, None, G * hk, G * hv, D, D,
                 C.c_float(1.0 / math.sqrt(D)), 0, G * hv)
            for j in range(G):
                self._go("ridgefill_rho_update",
                         [t(self.ab[j], abi.BF16, [T, hv], [2 * hv, 1]), t(self.mask, abi.I32), t(x["a_log"][j], abi.F32),
                          t(x["dt_bias"][j], abi.F32), t(self.nd, abi.F32, [s.n_seq, hv, 1, 2],
                                                         [st // 4 for st in self.nd.strides], offset=j * hv * 2),
                          t(self.slot_last, abi.I32), t(self.bounds, abi.I32)], [P("M", T), P("n_head", hv)])
            self._correct("apply")
        self._go("ridgefill_hazard", [t(x["cu_last"], abi.I32), t(x["positions"], abi.I32), t(self.bounds, abi.I32), A,
                                      t(self.meta, abi.F32), t(self.slot_last, abi.I32), t(self.count, abi.F32)], [P("M", 1)])

    def time_passes(self, passes: int, warmup: int = 1) -> float:
        """Seconds per pass over `passes` timed passes (each pass restarts from the same state)."""
        for _ in range(warmup):
            self.run()
        t0 = time.perf_counter()
        for _ in range(passes):
            self.run()
        return (time.perf_counter() - t0) / max(passes, 1)
