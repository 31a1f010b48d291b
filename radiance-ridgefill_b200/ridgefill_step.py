"""One RidgeFill approximate pass over a prefill chunk, issued row by row through the library's C ABI, in
the order the reference's arch core issues it for a masked late layer (arch/ridgefill_step.h:151-175,
arch/ridgefill_layer.h:65-116, arch/qwen4exp_blocks.h:110-182):

    ridgefill_mask              which rows of the chunk stay exact (once a pass, before layer 0)
    ridgefill_quant_act_i8g     the layer-S stream's int8 codes (once a pass)
    ridgefill_gemm_nt_q_bias    the projector: y = proj(h_S) + bias, bf16
    ridgefill_select            the approximated rows of the block input take the projection
    ridgefill_state_correct     undo the previous chunk end's correction
    ridgefill_gdn_fill          the Gated DeltaNet chunk fill over the chunk, state in place
    ridgefill_rho_update        the decayed approximated share per head
    ridgefill_state_correct     apply alpha * rho * C at the bulk end
    ridgefill_hazard            the prefix-cache hazard record

Buffers live on one CUDA device (torch tensors: allocation and streams only); every op is a launch of a
sm_100a device row. `Step.run()` issues one pass on a stream, in the order above; nothing here computes on the
host. `Step.run_pipelined()` issues the same launches on two streams: the projector path (quantiser, projector) from
the top of the pass and select once the mask is written, on a lower-priority side stream; the rest on the main
stream. Every late layer projects the same h_S (arch/ridgefill_layer.h:60-63), so in a pass over the late layers
the projector path of the next layer does not wait for this layer's fill: issued beside it, it runs on the SMs
the fill's phase-1 CTAs release while the fill's chains finish.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

import ridgefill_abi as abi


@dataclass
class StepShape:
    T: int = 32768          # prefill rows in the chunk
    d: int = 2048           # projector width (hidden d = K = N)
    hk: int = 16            # DeltaNet q/k heads
    hv: int = 32            # DeltaNet v heads
    head: int = 128         # head dims
    share: float = 0.30     # share of bulk rows kept exact by the class mask
    vocab: int = 65536      # synthetic score-table size
    alpha: float = 1.0
    group: int = 0          # projector scale group: 0 = per row / per column (group = d)


class Step:
    """The buffers of one pass and the row launches that fill them."""

    def __init__(self, shape: StepShape, device: str = "cuda", seed: int = 0):
        import torch
        self.torch = torch
        self.s = shape
        self.lib = abi.product()
        T, d, hk, hv, D = shape.T, shape.d, shape.hk, shape.hv, shape.head
        self.group = shape.group or d
        g = torch.Generator(device=device).manual_seed(seed)
        dev = torch.device(device)

        def normal(*sz):
            return torch.randn(*sz, device=dev, generator=g)

        # --- mask inputs: one sequence, every row bulk
        self.cu_last = torch.tensor([0, T], dtype=torch.int32, device=dev)
        self.token_ids = torch.randint(0, shape.vocab, (T,), dtype=torch.int32, device=dev, generator=g)
        self.positions = torch.arange(T, dtype=torch.int32, device=dev)
        score = normal(shape.vocab)
        score[torch.rand(shape.vocab, device=dev, generator=g) < 0.5] = -math.inf   # half the vocabulary matches
        self.score = score.float()
        self.mask = torch.zeros(T, dtype=torch.int32, device=dev)
        self.bounds = torch.zeros(4, dtype=torch.int32, device=dev)
        # --- projector: h_S bf16 ~ N(0,1), W int8 ~ U[-127,127], per-column f32 scale ~ U(1e-3, 1e-2)
        self.h_s = normal(T, d).to(torch.bfloat16)
        self.codes = torch.empty(T, d, dtype=torch.int8, device=dev)
        self.a_scale = torch.empty(T, d // self.group, dtype=torch.float32, device=dev)
        self.w = torch.randint(-127, 128, (d, d), dtype=torch.int8, device=dev, generator=g)
        self.w_scale = (torch.rand(d // self.group, d, device=dev, generator=g) * 9e-3 + 1e-3).float()
        self.bias = (0.1 * normal(d)).to(torch.bfloat16)
        self.x_proj = torch.empty(T, d, dtype=torch.bfloat16, device=dev)
        self.x = normal(T, d).to(torch.bfloat16)          # the exact block input the select overwrites
        # --- DeltaNet (16 q/k and 32 v heads of 128): q, k L2-normalised, beta = sigmoid(N), g = -softplus(N)
        k = normal(T, hk, D)
        self.k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        self.v = normal(T, hv, D).to(torch.bfloat16)
        self.g = -torch.nn.functional.softplus(normal(T, hv)).float()
        self.beta = torch.sigmoid(normal(T, hv)).float()
        self.state = torch.zeros(1, hv, D, D, dtype=torch.float32, device=dev)
        self.state_idx = torch.zeros(1, 1, dtype=torch.int32, device=dev)
        self.cu_seqlens = torch.tensor([0, T], dtype=torch.int32, device=dev)
        # --- correction, rho, hazard
        self.C = (0.01 * normal(hv, D, D)).float()
        self.applied = torch.zeros(1, hv, 1, 1, dtype=torch.float32, device=dev)
        self.nd = torch.zeros(1, hv, 1, 2, dtype=torch.float32, device=dev)
        self.ab = normal(T, 2 * hv).to(torch.bfloat16)   # the a|b projections; rho reads the a half
        self.a_log = (normal(hv) * 0.5).float()
        self.dt_bias = (normal(hv) * 0.5).float()
        self.meta = torch.zeros(1, 1, 1, 2, dtype=torch.float32, device=dev)
        self.count = torch.zeros(1, dtype=torch.float32, device=dev)
        self._build_calls()
        self.scratch = torch.empty(max(self.gdn_scratch, 16), dtype=torch.uint8, device=dev)

    # --------------------------------------------------------------- the launch list
    def _t(self, t, dtype=None, shape=None, strides=None):
        code = dtype or {self.torch.float32: abi.F32, self.torch.bfloat16: abi.BF16, self.torch.int32: abi.I32,
                         self.torch.int8: abi.I8}[t.dtype]
        return abi.tensor(code, shape or list(t.shape), t.data_ptr(), strides or list(t.stride()))

    def _build_calls(self):
        s, t, P, S, F = self.s, self._t, abi.pint, abi.pstr, abi.pf64
        T, d, hv, D = s.T, s.d, s.hv, s.head
        row = lambda op: self.lib.find_row(op, abi.DOMAIN_DEVICE)   # noqa: E731
        self.calls = [
            ("ridgefill_mask", row("ridgefill_mask"),
             [t(self.cu_last), t(self.token_ids), t(self.positions), t(self.score), t(self.mask), t(self.bounds), abi.absent()],
             [P("M", T), F("share", s.share), P("seed", 0), S("mode", "class")]),
            ("ridgefill_quant_act_i8g", row("ridgefill_quant_act_i8g"), [t(self.h_s), t(self.codes), t(self.a_scale)],
             [P("M", T), P("n", d), P("group", self.group), S("dtype", "bf16")]),
            ("ridgefill_gemm_nt_q_bias", row("ridgefill_gemm_nt_q_bias"),
             [t(self.codes), t(self.a_scale), t(self.w), t(self.w_scale), t(self.bias), t(self.x_proj), abi.absent()],
             [P("M", T), P("N", d), P("K", d), P("group", self.group), S("dtype", "i8a8")]),
            ("ridgefill_select", row("ridgefill_select"),
             [t(self.mask), t(self.x_proj), abi.absent(), abi.absent(), t(self.x), abi.absent(), abi.absent()], [P("M", T)]),
            ("ridgefill_state_correct", row("ridgefill_state_correct"),
             [t(self.state), t(self.state_idx), t(self.applied), t(self.state_idx), t(self.C), abi.absent(), abi.absent(),
              t(self.bounds)],
             [P("M", 1), S("mode", "undo"), F("alpha", s.alpha), P("n_head", hv), P("sd0", D), P("sd1", D)]),
            ("ridgefill_gdn_fill", row("ridgefill_gdn_fill"),
             [abi.absent(), t(self.k), t(self.v), t(self.g), t(self.beta), t(self.state), t(self.state_idx),
              t(self.cu_seqlens), abi.absent()],
             [P("M", T), P("n_head_k", s.hk), P("n_head_v", hv), P("head_k", D), P("head_v", D), P("chunk", 64)]),
            ("ridgefill_rho_update", row("ridgefill_rho_update"),
             [t(self.ab, shape=[T, hv], strides=[2 * hv, 1]), t(self.mask), t(self.a_log), t(self.dt_bias), t(self.nd),
              t(self.state_idx), t(self.bounds)],
             [P("M", T), P("n_head", hv)]),
            ("ridgefill_state_correct", row("ridgefill_state_correct"),
             [t(self.state), t(self.state_idx), t(self.applied), t(self.state_idx), t(self.C), t(self.nd), t(self.state_idx),
              t(self.bounds)],
             [P("M", 1), S("mode", "apply"), F("alpha", s.alpha), P("n_head", hv), P("sd0", D), P("sd1", D)]),
            ("ridgefill_hazard", row("ridgefill_hazard"),
             [t(self.cu_last), t(self.positions), t(self.bounds), abi.absent(), t(self.meta), t(self.state_idx), t(self.count)],
             [P("M", 1)]),
        ]
        gdn = self.calls[5]
        self.gdn_scratch = self.lib.scratch_bytes(gdn[1], gdn[2], gdn[3])
        # the argument blocks are built once; a pass only calls the launch hooks
        self._args = [(name, r, tens, params) for name, r, tens, params in self.calls]
        # Beside the fill (run_pipelined) the projector is given the SMs the fill's chain CTAs leave: the fill's
        # grid is one CTA a SM, min(v heads x sequences, SMs / 4) of them chains, the rest freed by phase 1.
        sms = self.torch.cuda.get_device_properties(self.torch.cuda.current_device()).multi_processor_count
        budget = sms - min(hv, sms // 4)
        self._side_args = [(name, r, tens, params + [P("max_ctas", budget)] if name == "ridgefill_gemm_nt_q_bias" else params)
                           for name, r, tens, params in self._args]

    # kernels a pass launches (the GDN fill is two: the sequence plan, then the fill kernel)
    LAUNCHES_PER_PASS = 10
    # the issue order of `calls` (and of run())
    ORDER = ("ridgefill_mask", "ridgefill_quant_act_i8g", "ridgefill_gemm_nt_q_bias", "ridgefill_select",
             "ridgefill_state_correct", "ridgefill_gdn_fill", "ridgefill_rho_update", "ridgefill_state_correct",
             "ridgefill_hazard")
    # ops run_pipelined issues on the side stream
    SIDE_OPS = ("ridgefill_quant_act_i8g", "ridgefill_gemm_nt_q_bias", "ridgefill_select")

    def _launch(self, name, r, tens, params, stream: int) -> None:
        sb = self.gdn_scratch if name == "ridgefill_gdn_fill" else 0
        rc = self.lib.launch(r, tens, params, stream=stream, scratch=self.scratch.data_ptr() if sb else None,
                             scratch_bytes=sb)
        if rc != abi.OK:
            raise RuntimeError(f"{name}: device row refused or failed (rc {rc})")

    def run_pipelined(self, main, side, events=None) -> None:
        """Issue one pass on two torch streams. On `side` (a stream of lower priority): from the top of the pass
        the projector path (codes, projector), which reads only the pass's inputs, then, once the mask is
        written, select. The rest runs on `main` in the pass's order (mask, undo, the fill, rho, apply, the
        hazard record), and `main` then waits for `side`, so the pass is complete when `main` is. Every buffer one
        stream writes is read or written by the other only across these waits. `events` (optional) maps an op on
        `main` to a pair of CUDA events recorded around its launch."""
        torch = self.torch
        a, sa = self._args, self._side_args
        assert tuple(op[0] for op in a) == self.ORDER
        fork, masked, join = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()

        def on_main(op):
            ev = events.get(op[0]) if events else None
            if ev:
                ev[0].record(main)
            self._launch(*op, main.cuda_stream)
            if ev:
                ev[1].record(main)

        fork.record(main)                    # after the previous pass, whole
        side.wait_event(fork)
        for op in (sa[1], sa[2]):            # codes, projector
            self._launch(*op, side.cuda_stream)
        on_main(a[0])                        # mask
        masked.record(main)
        side.wait_event(masked)
        self._launch(*sa[3], side.cuda_stream)   # select
        join.record(side)
        for op in a[4:]:                     # undo, fill, rho, apply, hazard
            on_main(op)
        main.wait_event(join)

    def run(self, stream: int, events=None) -> None:
        """Issue one pass on `stream`. `events` (optional) maps an op name to a pair of CUDA events recorded
        around its launch."""
        for name, r, tens, params in self._args:
            ev = events.get(name) if events else None
            if ev:
                ev[0].record()
            self._launch(name, r, tens, params, stream)
            if ev:
                ev[1].record()

    # --------------------------------------------------------------- algorithmic work of one pass
    def algorithmic(self) -> dict:
        s = self.s
        T, d, hv, hk, D = s.T, s.d, s.hv, s.hk, s.head
        return {
            "gemm_ops": 2 * T * d * d,
            "gemm_bytes": T * d + d * d + 2 * T * d + 4 * T * (d // self.group) + 4 * d * (d // self.group),
            "quant_bytes": 2 * T * d + T * d + 4 * T * (d // self.group),
            # state-only fill: read k, v, g, beta, the state; write the state
            "gdn_bytes": 2 * T * hk * D + 2 * T * hv * D + 8 * T * hv + 2 * 4 * hv * D * D,
            # the gated delta rule's state-only arithmetic per (row, v-head): decay, S k, the rank-1 update
            "gdn_flops": T * hv * (4 * D * D),
            # the chunked form's state-only arithmetic per (64-row chunk, v-head): K K^T, W, U~ (2 C^2 d each),
            # V' and the state update (2 C d^2 each), the triangular solve (C^3 / 1.5)
            "gdn_chunk_flops": (T // 64) * hv * (6 * 64 * 64 * D + 4 * 64 * D * D + 64 ** 3 * 2 // 3),
            "select_bytes": 4 * T + 2 * 2 * d * int(T * (1 - s.share)),
        }
