"""The late-layer pass's launch list on the CPU: built over host tensors, every launch's operands and parameters
pass its device row's operand checks (the rows' exported parse functions, called directly: nothing is launched),
the pass issues the reference's op order, and its CPU twin (oracle/cpu_path.CpuLatePass) runs the same shapes."""
import collections
import ctypes as C

import numpy as np
import pytest

import harness as H  # noqa: F401  (puts the package on the path)
import late_pass as LP
import cpu_path as CP
from harness import abi

PARSE = {"ridgefill_mask": "ridgefill_mask_parse", "ridgefill_quant_act_i8g": "ridgefill_quant_parse",
         "ridgefill_select": "ridgefill_select_parse", "ridgefill_gemm_nt_bias": "ridgefill_gemm_bias_parse",
         "ridgefill_gdn_conv_prep": "ridgefill_conv_prep_parse", "ridgefill_attn_kv_fill": "ridgefill_attn_kv_parse",
         "ridgefill_state_correct": "ridgefill_correct_parse", "ridgefill_gdn_fill": "ridgefill_gdn_parse",
         "ridgefill_rho_update": "ridgefill_rho_parse", "ridgefill_hazard": "ridgefill_hazard_parse",
         "ridgefill_gdn_in_proj": "ridgefill_in_proj_parse"}

SHAPES = [LP.mini_model(), LP.LateShape(T=256, d=256, hk=2, hv=4), LP.LateShape(T=300, d=256, layers="GA", hk=2, hv=4,
                                                                              seqlens=(100, 80, 120)),
          LP.LateShape(T=256, d=256, hk=2, hv=4, group=128)]


def _parse(lib, op, tens, params):
    args, keep = abi.Plugin.args(tens, params)
    out = (C.c_uint8 * 4096)()
    if op == "ridgefill_gemm_nt_q_bias":
        fn = lib.lib.ridgefill_gemm_q_parse
        fn.restype = C.c_int
        rc = fn(C.byref(args), 1, out)
    else:
        fn = getattr(lib.lib, PARSE[op])
        fn.restype = C.c_int
        rc = fn(C.byref(args), out)
    del keep
    return rc


@pytest.mark.parametrize("shape", SHAPES, ids=["mini_model", "all24_small", "ragged", "grouped"])
def test_every_launch_passes_its_operand_checks(shape, product_lib):
    p = LP.LatePass(shape, "cpu", seed=1)
    for op, _row, tens, params, tag in p.calls:
        assert _parse(product_lib, op, tens, params) == abi.OK, (op, tag)
    counts = p.op_counts()
    G, A, L = shape.n_gdn, shape.n_attn, len(shape.layers)
    # per DeltaNet layer: the mixed projection's k|v columns (with per-row scales the fused in-projection, its
    # convolution in the epilogue), then its q columns over each sequence's last rows
    fused = shape.block_inputs and p.fused_in
    assert p.fused_in == (shape.group in (0, shape.d) and shape.head == 128)
    assert counts["ridgefill_gemm_nt_q_bias"] == L + (G * (int(not fused) + shape.n_seq) if shape.block_inputs else 0) + A
    assert counts.get("ridgefill_gdn_in_proj", 0) == (G if fused else 0)
    if fused:   # conv_prep is left the gates and the conv state, after the in-projection has read the old state
        conv = [c for c in p.calls if c[0] == "ridgefill_gdn_conv_prep"]
        assert all(dict((q.key.decode(), q.ival) for q in c[3]).get("columns") == 0 for c in conv)
        assert order_index_ok(p)
    assert counts["ridgefill_gdn_fill"] == 1 and counts["ridgefill_rho_update"] == G
    assert counts["ridgefill_state_correct"] == 2 and counts["ridgefill_mask"] == 1 and counts["ridgefill_hazard"] == 1
    order = [c[0] for c in p.calls]
    assert order[0] == "ridgefill_mask" and order[-1] == "ridgefill_hazard"
    # the projectors write the approximated rows themselves (the mask as their rows operand): no select launch
    assert "ridgefill_select" not in order
    proj = [c for c in p.calls if c[0] == "ridgefill_gemm_nt_q_bias" and c[4].startswith("proj")]
    assert len(proj) == L and all(c[2][7].data for c in proj)
    assert order.index("ridgefill_gdn_fill") > max(i for i, c in enumerate(p.calls) if c[4].startswith("proj"))


def order_index_ok(p) -> bool:
    """Each layer's conv_prep comes after its in-projection (which reads the conv state conv_prep then updates)."""
    last_in = None
    for op, _r, _t, _p, tag in p.calls:
        if op == "ridgefill_gdn_in_proj":
            last_in = tag.split()[-1]
        if op == "ridgefill_gdn_conv_prep" and last_in != tag:
            return False
    return True


def test_cpu_twin_runs_the_same_pass(oracle_lib):
    shape = LP.LateShape(T=200, d=256, layers="GGA", hk=2, hv=4, seqlens=(120, 80))
    host = CP.to_host(LP.late_inputs(shape, "cpu", 2))
    cpu = CP.CpuLatePass(shape, host)
    cpu.run()
    assert cpu.mask[:120].sum() == 0 and cpu.mask[120:].sum() > 0    # only the last sequence is approximated
    assert np.isfinite(cpu.state).all() and np.abs(cpu.nd[-1]).sum() > 0 and np.abs(cpu.nd[0]).sum() == 0
    assert (cpu.cache[0][0] != 0).any()


@pytest.mark.parametrize("shape", SHAPES[:3], ids=["mini_model", "all24_small", "ragged"])
def test_results_before_the_fill_are_final_when_the_hook_runs(shape):
    """run(before_tail=...) calls the hook once, after every layer's launches and before the fill's; the results
    it declares final there (mask, attention caches, conv states) are written by no launch after it (the mask is
    only read there: rho's row mask), and the two parts together are results()."""
    p = LP.LatePass(shape, "cpu", seed=1)
    order = []
    p._launch = lambda op, r, tens, params, stream: order.append(op)   # noqa: E731  (nothing is launched)
    p.run(0, events={}, before_tail=lambda: order.append("hook"))
    assert order.count("hook") == 1
    at = order.index("hook")
    assert order[at + 1] == "ridgefill_gdn_fill" and "ridgefill_gdn_fill" not in order[:at]
    early, late = p.results_split()
    assert sorted(map(id, early + late)) == sorted(map(id, p.results()))
    ranges = [(t.data_ptr(), t.data_ptr() + t.numel() * t.element_size()) for t in early if t.numel()]
    mask = p.mask.data_ptr()
    for op, _r, tens, _p, tag in p.tail:
        for i, a in enumerate(tens):
            ptr = getattr(a, "data", None) or 0
            if not ptr or not any(lo <= ptr < hi for lo, hi in ranges):
                continue
            assert op == "ridgefill_rho_update" and ptr == mask and i == 1, (op, tag, i)


class _Streams:
    """Stand-ins for torch.cuda's Stream, ExternalStream and Event that log what the pass asks of them."""

    def __init__(self):
        self.log = []
        outer = self

        class _S:
            def __init__(self, handle):
                self.cuda_stream = handle

            def wait_event(self, e):
                outer.log.append(("wait", self.cuda_stream, e.on))

        class _E:
            def __init__(self):
                self.on = None

            def record(self, s=None):
                self.on = s.cuda_stream
                outer.log.append(("record", s.cuda_stream))

        class _Cuda:
            Event = _E

            @staticmethod
            def Stream(device=None):
                return _S(777)

            @staticmethod
            def ExternalStream(handle, device=None):
                return _S(handle)

        self.cuda = _Cuda


SIDE_OPS = ("ridgefill_gemm_nt_bias", "ridgefill_gdn_conv_prep")


@pytest.mark.parametrize("shape", SHAPES, ids=["mini_model", "all24_small", "ragged", "grouped"])
def test_the_second_stream_plan(shape):
    """The pass's second stream, checked on its issue log:
    * each DeltaNet layer's a|b projection goes there after an event recorded once its projector is issued, and its
      conv_prep after an event recorded once its in-projection and q tails are issued; the next in-projection (or
      mixed projection) and the fill come after a wait for that conv_prep;
    * with the fill in its per-head form (head dim 128, at least 64 chains) the decay sums go there too, from an
      event recorded just before the fill, and the correction waits for them; otherwise they stay in order;
    * everything else stays on the pass's stream, and an ordered pass (`events` given) uses no second stream."""
    p = LP.LatePass(shape, "cpu", seed=1)
    fake = _Streams()
    p.torch = fake
    mixed = getattr(p, "mixed", None)   # only passes with block inputs have the mixed projection's buffer
    lo = mixed.data_ptr() if mixed is not None else 0
    hi = lo + (mixed.numel() * mixed.element_size() if mixed is not None else 0)
    writes_mixed = set()

    def launch(op, r, tens, params, stream):
        if op != "ridgefill_gdn_conv_prep" and any(lo <= (getattr(t, "data", None) or 0) < hi for t in tens):
            writes_mixed.add(len(fake.log))
        fake.log.append(("launch", op, stream))

    p._launch = launch
    p.run(5)
    log = fake.log
    launches = [(e[1], e[2]) for e in log if e[0] == "launch"]
    G, hv = shape.n_gdn, shape.hv
    beside = shape.head == 128 and G * hv * shape.n_seq >= 64
    assert p.rho_beside_fill == beside
    want = collections.Counter()
    for c in p.head:
        want[(c[0], 5)] += 1
    for proj, block in p.layers:
        attention = any(c[0] == "ridgefill_attn_kv_fill" for c in block)
        for c in proj:
            want[(c[0], 5)] += 1
        for c in block:   # an attention layer's whole block, a DeltaNet layer's a|b and conv_prep: second stream
            want[(c[0], 777 if attention or c[0] in SIDE_OPS else 5)] += 1
    for c in p.tail:
        want[(c[0], 777 if c[0] == "ridgefill_rho_update" and beside else 5)] += 1
    assert collections.Counter(launches) == want
    if shape.block_inputs and G:
        ab = [i for i, e in enumerate(log) if e[:2] == ("launch", "ridgefill_gemm_nt_bias")]
        prep = [i for i, e in enumerate(log) if e[:2] == ("launch", "ridgefill_gdn_conv_prep")]
        assert len(ab) == len(prep) == G
        for i in ab + prep:   # each side launch right after its wait on an event of the pass's stream
            assert log[i - 1] == ("wait", 777, 5) and log[i - 2] == ("record", 5)
        writers = sorted(writes_mixed)   # the in-projections and q tails (the rows conv_prep reads)
        assert len(writers) >= G
        fill = log.index(("launch", "ridgefill_gdn_fill", 5))
        for j in prep:
            stop = min([w for w in writers if w > j] + [fill])
            assert ("record", 777) in log[j:stop] and ("wait", 5, 777) in log[j:stop], (j, stop)
    if beside:
        fill = log.index(("launch", "ridgefill_gdn_fill", 5))
        assert log[fill - 2] == ("record", 5) and log[fill - 1] == ("wait", 777, 5)
        last_rho = max(i for i, e in enumerate(log) if e[:2] == ("launch", "ridgefill_rho_update"))
        corr = log.index(("launch", "ridgefill_state_correct", 5), fill)
        assert ("record", 777) in log[last_rho:corr] and ("wait", 5, 777) in log[last_rho:corr]
    # the ordered pass
    fake.log.clear()
    p.run(5, events={})
    assert all(e[0] == "launch" and e[2] == 5 for e in fake.log)
