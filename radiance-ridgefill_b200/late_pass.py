"""The RidgeFill approximate pass over every late layer of a prefill chunk: the lean late-layer loop of the
reference's arch core (arch/ridgefill_step.h:151-175 -> fill_layer, arch/ridgefill_layer.h:205-210), every op a
launch of this library's sm_100a device rows through the C ABI.

    ridgefill_mask                  which rows of the approximated sequence stay exact (once a pass)
    ridgefill_quant_act_i8g         the layer-S stream's codes (once a pass: every late layer projects h_S,
                                    arch/ridgefill_layer.h:60-63)
    ridgefill_state_correct undo    every DeltaNet layer's state at once (their pools are one array)
    for each late layer l:
      ridgefill_gemm_nt_q_bias      the projector x = proj_l(h_S) + bias_l
      ridgefill_select              the approximated rows of the layer's block input take the projection
      ridgefill_quant_act_i8g       the block input's codes (what the int8 block reads)
      DeltaNet layer (arch/qwen4exp_fill.h:29-61):
        ridgefill_gemm_nt_q_bias    the mixed q|k|v projection (int8, no bias)
        ridgefill_gemm_nt_bias      the a|b projection (bf16)
        ridgefill_gdn_conv_prep     conv, SiLU, q/k norm, gate and beta, into this layer's heads of the
                                    pass-wide k, v, g, beta arrays
      attention layer (arch/qwen4exp_fill.h:100-115):
        ridgefill_gemm_nt_q_bias    the k|v projection (int8, no bias)
        ridgefill_attn_kv_fill      k norm, rotary, the paged cache store
    ridgefill_gdn_fill              ONE launch for every DeltaNet layer's chunk fill (state only)
    ridgefill_rho_update            per DeltaNet layer, from its a values
    ridgefill_state_correct apply   every DeltaNet layer at once
    ridgefill_hazard                the prefix-cache hazard record

The fill is batched by laying the DeltaNet layers side by side as heads: layer j's k heads are heads
[j Hk, (j+1) Hk) of one [T, L Hk, 128] array, its v heads [j Hv, (j+1) Hv) of [T, L Hv, 128], its state
heads the same span of one [slots, L Hv, 128, 128] pool, so v-head h reads k-head h / (Hv / Hk) inside its own
layer and one launch fills L Hv chains. The correction runs over the same pool with the layers' C stacked.

Without block inputs (`block_inputs=False`, the reference's CPU mini model) the fill's k, v, g, beta and the a
values rho reads are inputs of the pass, as in the one-layer pass of ridgefill_step.py.

Buffers are torch tensors on one device (allocation and streams only); nothing here computes on the host.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import ridgefill_abi as abi

# late layers 24..47 of the 48-layer stack: full attention every fourth layer (layers 27, 31, ..., 47)
QWEN_LATE_LAYERS = "GGGA" * 6


@dataclass
class LateShape:
    T: int = 32768                 # rows of the chunk (all sequences)
    d: int = 2048                  # hidden width: the projector's K = N, the blocks' input width
    layers: str = QWEN_LATE_LAYERS # the late layers in order: G = Gated DeltaNet, A = gated attention
    hk: int = 16                   # DeltaNet q/k heads a layer
    hv: int = 32                   # DeltaNet v heads a layer
    head: int = 128                # DeltaNet head dims
    hkv: int = 2                   # attention kv heads
    head_attn: int = 256
    rope_dim: int = 64
    rope_sections: tuple = (11, 11, 10)
    rope_theta: float = 1e7
    share: float = 0.30            # the class mask keeps this share of the approximated sequence exact
    vocab: int = 65536
    alpha: float = 1.0
    block_inputs: bool = True      # DeltaNet inputs from the block input (in-projection + conv_prep); else given
    seqlens: tuple = ()            # the chunk's sequences (the approximated one last); () = one sequence of T
    group: int = 0                 # scale group of codes and weights: 0 = the whole row (per-row / per-column)

    @property
    def n_gdn(self) -> int:
        return self.layers.count("G")

    @property
    def n_attn(self) -> int:
        return self.layers.count("A")

    @property
    def conv_dim(self) -> int:
        return 2 * self.hk * self.head + self.hv * self.head

    @property
    def lengths(self) -> list[int]:
        return list(self.seqlens) if self.seqlens else [self.T]

    @property
    def n_seq(self) -> int:
        return len(self.lengths)


def config0() -> LateShape:
    """The reference's CPU mini model: d 256, 512 rows, 4 DeltaNet layers of 4 q/k and 8 v heads of 32, the fill's
    inputs given, 25 % of the rows kept exact."""
    return LateShape(T=512, d=256, layers="GGGG", hk=4, hv=8, head=32, share=0.25, vocab=4096, block_inputs=False)


def config3(T: int = 32768) -> LateShape:
    """The full step over the 24 late layers of the 48-layer stack (18 DeltaNet + 6 attention), hidden 2,048,
    DeltaNet 16 q/k and 32 v heads of 128, attention 2 kv heads of 256, 30 % of the rows exact."""
    return LateShape(T=T)


def config5(seed: int = 0, long: int = 32768, short: int = 6) -> LateShape:
    """The mixed ragged batch: six prompts of U[256, 2,048] rows, then one 32K prompt (the approximated one)."""
    import random
    r = random.Random(seed)
    lens = [r.randint(256, 2048) for _ in range(short)] + [long]
    return LateShape(T=sum(lens), seqlens=tuple(lens))


def late_inputs(s: LateShape, device, seed: int = 0) -> dict:
    """Seeded synthetic inputs and weights of one pass, with BASELINE's distributions: h_S and the exact block
    inputs ~N(0,1) bf16, int8 weights ~U[-127,127] with f32 per-column scales ~U(1e-3,1e-2), the DeltaNet and
    attention weights at the served model's scales. Torch tensors on `device` (a CPU device for the CPU arm)."""
    import torch
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    T, d = s.T, s.d
    grp = s.group or d

    def normal(*sz, scale=1.0):
        return torch.randn(*sz, device=dev, generator=g) * scale

    def bf16(x):
        return x.to(torch.bfloat16)

    def i8(*sz):
        return torch.randint(-127, 128, sz, dtype=torch.int8, device=dev, generator=g)

    def col_scale(n, k):
        return (torch.rand(k // grp, n, device=dev, generator=g) * 9e-3 + 1e-3).float()

    x = {}
    lens = s.lengths
    starts = [0]
    for n in lens:
        starts.append(starts[-1] + n)
    x["cu_seqlens"] = torch.tensor(starts, dtype=torch.int32, device=dev)
    x["cu_last"] = torch.tensor([starts[-2], starts[-1]], dtype=torch.int32, device=dev)
    x["token_ids"] = torch.randint(0, s.vocab, (T,), dtype=torch.int32, device=dev, generator=g)
    x["positions"] = torch.cat([torch.arange(n, dtype=torch.int32, device=dev) for n in lens])
    score = normal(s.vocab)
    score[torch.rand(s.vocab, device=dev, generator=g) < 0.5] = -math.inf   # half the vocabulary matches
    x["score"] = score.float()
    x["h_s"] = bf16(normal(T, d))
    L, G, A = len(s.layers), s.n_gdn, s.n_attn
    x["w_proj"] = [i8(d, d) for _ in range(L)]
    x["s_proj"] = [col_scale(d, d) for _ in range(L)]
    x["b_proj"] = [bf16(normal(d, scale=0.1)) for _ in range(L)]
    x["x_exact"] = [bf16(normal(T, d)) for _ in range(L)]   # the exact block input the select leaves on kept rows
    D, hk, hv = s.head, s.hk, s.hv
    if s.block_inputs:
        C = s.conv_dim
        x["w_in"] = [i8(C, d) for _ in range(G)]
        x["s_in"] = [(torch.rand(d // grp, C, device=dev, generator=g) * 2e-4 + 1e-4).float() for _ in range(G)]
        x["w_ab"] = [bf16(normal(2 * hv, d, scale=0.1 / math.sqrt(d))) for _ in range(G)]   # a, b ~ N(0, ~1.5)
        x["w_conv"] = [bf16(normal(C, 4, scale=0.5)) for _ in range(G)]
        x["a_log"] = [(normal(hv, scale=0.3) - 1.0).float() for _ in range(G)]
        x["dt_bias"] = [(normal(hv, scale=0.5)).float() for _ in range(G)]
        x["conv_state"] = [bf16(normal(s.n_seq, 3, C, scale=0.5)) for _ in range(G)]
    else:
        k = normal(T, G * hk, D)
        x["k"] = bf16(k / k.norm(dim=-1, keepdim=True))
        x["v"] = bf16(normal(T, G * hv, D))
        x["g"] = (-torch.nn.functional.softplus(normal(T, G * hv))).float()
        x["beta"] = torch.sigmoid(normal(T, G * hv)).float()
        x["ab"] = [bf16(normal(T, 2 * hv)) for _ in range(G)]
        x["a_log"] = [(normal(hv, scale=0.5)).float() for _ in range(G)]
        x["dt_bias"] = [(normal(hv, scale=0.5)).float() for _ in range(G)]
    x["state"] = normal(s.n_seq, G * hv, D, D, scale=0.05).float()
    x["C"] = normal(G * hv, D, D, scale=0.01).float()
    if A:
        Ha, Dh = s.hkv, s.head_attn
        x["w_kv"] = [i8(2 * Ha * Dh, d) for _ in range(A)]
        x["s_kv"] = [(torch.rand(d // grp, 2 * Ha * Dh, device=dev, generator=g) * 2e-4 + 1e-4).float() for _ in range(A)]
        x["k_norm"] = [bf16(1.0 + normal(Dh, scale=0.1)) for _ in range(A)]
        x["slot_mapping"] = torch.randperm(T + 1024, device=dev, generator=g)[:T].int()
    return x


def _code(t):
    import torch
    return {torch.float32: abi.F32, torch.bfloat16: abi.BF16, torch.int32: abi.I32, torch.int8: abi.I8,
            torch.int16: abi.BF16}[t.dtype]


def _t(t, shape=None, strides=None, offset_elems=0, dtype=None):
    return abi.tensor(dtype or _code(t), list(t.shape) if shape is None else shape,
                      t.data_ptr() + offset_elems * t.element_size(), list(t.stride()) if strides is None else strides)


class LatePass:
    """The buffers of one approximate pass over the late layers and the row launches that fill them."""

    # kernels a launch of each row starts (the fill: its sequence plan and the fused kernel; the per-row
    # form for small heads is one kernel)
    KERNELS = {"ridgefill_mask": 1, "ridgefill_quant_act_i8g": 1, "ridgefill_gemm_nt_q_bias": 1, "ridgefill_select": 1,
               "ridgefill_gemm_nt_bias": 1, "ridgefill_gdn_conv_prep": 2, "ridgefill_attn_kv_fill": 1,
               "ridgefill_state_correct": 1, "ridgefill_gdn_fill": 2, "ridgefill_rho_update": 1, "ridgefill_hazard": 1}

    def __init__(self, shape: LateShape, device: str = "cuda", seed: int = 0, inputs: dict | None = None):
        import torch
        self.torch = torch
        self.s = s = shape
        self.lib = abi.product()
        dev = torch.device(device)
        self.inp = inputs if inputs is not None else late_inputs(s, dev, seed)
        x = self.inp
        T, d, G, D = s.T, s.d, s.n_gdn, s.head
        grp = s.group or d
        self.grp = grp

        def empty(*sz, dtype):
            return torch.empty(*sz, dtype=dtype, device=dev)

        # pass outputs and intermediates
        self.mask = torch.zeros(T, dtype=torch.int32, device=dev)
        self.bounds = torch.zeros(4, dtype=torch.int32, device=dev)
        self.codes_h = empty(T, d, dtype=torch.int8)
        self.scale_h = empty(T, d // grp, dtype=torch.float32)
        self.x_proj = empty(T, d, dtype=torch.bfloat16)
        self.x = [t.clone() for t in x["x_exact"]]           # each layer's block input, the select writes into it
        self.codes_x = empty(T, d, dtype=torch.int8)
        self.scale_x = empty(T, d // grp, dtype=torch.float32)
        self.state = x["state"].clone()
        self.applied = torch.zeros(s.n_seq, G * s.hv, 1, 1, dtype=torch.float32, device=dev)
        self.nd = torch.zeros(s.n_seq, G * s.hv, 1, 2, dtype=torch.float32, device=dev)
        self.meta = torch.zeros(s.n_seq, 1, 1, 2, dtype=torch.float32, device=dev)
        self.count = torch.zeros(1, dtype=torch.float32, device=dev)
        self.slot_last = torch.tensor([[s.n_seq - 1]], dtype=torch.int32, device=dev)   # the approximated sequence
        self.slots_all = torch.arange(s.n_seq, dtype=torch.int32, device=dev).view(-1, 1)
        if s.block_inputs:
            C = s.conv_dim
            self.mixed = empty(T, C, dtype=torch.bfloat16)
            self.ab = [empty(T, 2 * s.hv, dtype=torch.bfloat16) for _ in range(G)]
            self.q = empty(T, s.hk, D, dtype=torch.bfloat16)   # the state-only fill reads no q: one buffer for all
            self.k = empty(T, G * s.hk, D, dtype=torch.bfloat16)
            self.v = empty(T, G * s.hv, D, dtype=torch.bfloat16)
            self.g = empty(T, G * s.hv, dtype=torch.float32)
            self.beta = empty(T, G * s.hv, dtype=torch.float32)
            self.conv_state = [t.clone() for t in x["conv_state"]]
            self.zero_ab = torch.zeros(2 * s.hv, dtype=torch.bfloat16, device=dev)
            self.ctx = torch.zeros(s.n_seq, dtype=torch.int32, device=dev)   # fresh prompts: no conv history
        else:
            self.ab, self.k, self.v, self.g, self.beta = x["ab"], x["k"], x["v"], x["g"], x["beta"]
        if s.n_attn:
            Ha, Dh = s.hkv, s.head_attn
            self.kv = empty(T, 2 * Ha * Dh, dtype=torch.bfloat16)
            self.cache = [torch.zeros(2, T + 1024, Ha, Dh, dtype=torch.bfloat16, device=dev) for _ in range(s.n_attn)]
            self.rope_pos = x["positions"].view(1, T).expand(3, T).contiguous()   # text rows: every plane the index
        self._build()
        self.scratch = torch.empty(max(self.fill_scratch, 16), dtype=torch.uint8, device=dev)

    # --------------------------------------------------------------- the launch list
    def _build(self):
        s, x = self.s, self.inp
        P, S, F = abi.pint, abi.pstr, abi.pf64
        A_ = abi.absent()
        T, d, G, hk, hv, D = s.T, s.d, s.n_gdn, s.hk, s.hv, s.head
        row = lambda op: self.lib.find_row(op, abi.DOMAIN_DEVICE)   # noqa: E731
        calls = []

        def add(op, tens, params, tag=""):
            calls.append((op, row(op), tens, params, tag))

        def gemm_q(a, sa, w, sw, bias, y, N, tag):
            add("ridgefill_gemm_nt_q_bias", [_t(a), _t(sa), _t(w), _t(sw), A_ if bias is None else _t(bias), y, A_],
                [P("M", T), P("N", N), P("K", d), P("group", self.grp), S("dtype", "i8a8")], tag)

        def quant(src, codes, scale, tag):
            add("ridgefill_quant_act_i8g", [_t(src), _t(codes), _t(scale)],
                [P("M", T), P("n", d), P("group", self.grp), S("dtype", "bf16")], tag)

        def correct(mode):
            tens = [_t(self.state), _t(self.slot_last), _t(self.applied), _t(self.slot_last), _t(x["C"])]
            tens += [_t(self.nd), _t(self.slot_last)] if mode == "apply" else [A_, A_]
            add("ridgefill_state_correct", tens + [_t(self.bounds)],
                [P("M", 1), S("mode", mode), F("alpha", s.alpha), P("n_head", G * hv), P("sd0", D), P("sd1", D)], mode)

        add("ridgefill_mask", [_t(x["cu_last"]), _t(x["token_ids"]), _t(x["positions"]), _t(x["score"]), _t(self.mask),
                               _t(self.bounds), A_],
            [P("M", T), F("share", s.share), P("seed", 0), S("mode", "class")])
        quant(x["h_s"], self.codes_h, self.scale_h, "h_S")
        if G:
            correct("undo")
        gi = ai = 0
        for li, kind in enumerate(s.layers):
            gemm_q(self.codes_h, self.scale_h, x["w_proj"][li], x["s_proj"][li], x["b_proj"][li], _t(self.x_proj), d, f"proj {li}")
            add("ridgefill_select", [_t(self.mask), _t(self.x_proj), A_, A_, _t(self.x[li]), A_, A_], [P("M", T)], f"{li}")
            if kind == "G" and s.block_inputs:
                quant(self.x[li], self.codes_x, self.scale_x, f"x {li}")
                C = s.conv_dim
                gemm_q(self.codes_x, self.scale_x, x["w_in"][gi], x["s_in"][gi], None, _t(self.mixed), C, f"in {li}")
                add("ridgefill_gemm_nt_bias", [_t(self.x[li]), _t(x["w_ab"][gi]), _t(self.zero_ab), A_, _t(self.ab[gi])],
                    [P("M", T), P("N", 2 * hv), P("K", d), S("dtype", "bf16")], f"ab {li}")
                ab = self.ab[gi]
                add("ridgefill_gdn_conv_prep",
                    [_t(self.mixed), _t(x["w_conv"][gi]), A_, _t(x["a_log"][gi]), _t(x["dt_bias"][gi]),
                     _t(self.conv_state[gi]), _t(x["cu_seqlens"]), _t(ab, [T, hv], [2 * hv, 1]),
                     _t(ab, [T, hv], [2 * hv, 1], offset_elems=hv), _t(self.slots_all.view(-1)), _t(self.ctx),
                     _t(self.q),
                     _t(self.k, [T, hk, D], list(self.k.stride()), offset_elems=gi * hk * D),
                     _t(self.v, [T, hv, D], list(self.v.stride()), offset_elems=gi * hv * D),
                     _t(self.g, [T, hv], [G * hv, 1], offset_elems=gi * hv),
                     _t(self.beta, [T, hv], [G * hv, 1], offset_elems=gi * hv)],
                    [P("M", T), P("n_head_k", hk), P("n_head_v", hv), P("head_k", D), P("head_v", D), P("conv", 4)], f"{li}")
            elif kind == "A":
                Ha, Dh = s.hkv, s.head_attn
                quant(self.x[li], self.codes_x, self.scale_x, f"x {li}")
                gemm_q(self.codes_x, self.scale_x, x["w_kv"][ai], x["s_kv"][ai], None, _t(self.kv), 2 * Ha * Dh, f"kv {li}")
                add("ridgefill_attn_kv_fill",
                    [_t(self.kv, [T, Ha, Dh], [2 * Ha * Dh, Dh, 1]),
                     _t(self.kv, [T, Ha, Dh], [2 * Ha * Dh, Dh, 1], offset_elems=Ha * Dh), _t(x["k_norm"][ai]),
                     _t(self.rope_pos), _t(x["slot_mapping"]), _t(self.cache[ai]), A_],
                    [P("M", T), P("n_head_kv", Ha), P("head_dim", Dh), P("rope_dim", s.rope_dim),
                     F("rope_theta", s.rope_theta), S("rope_mode", "imrope"),
                     S("rope_sections", ",".join(str(v) for v in s.rope_sections))], f"{li}")
                ai += 1
            if kind == "G":
                gi += 1
        if G:
            add("ridgefill_gdn_fill", [A_, _t(self.k), _t(self.v), _t(self.g), _t(self.beta), _t(self.state),
                                       _t(self.slots_all), _t(x["cu_seqlens"]), A_],
                [P("M", T), P("n_head_k", G * hk), P("n_head_v", G * hv), P("head_k", D), P("head_v", D), P("chunk", 64)])
            fill = calls[-1]
            self.fill_scratch = self.lib.scratch_bytes(fill[1], fill[2], fill[3])
            for j in range(G):
                add("ridgefill_rho_update",
                    [_t(self.ab[j], [T, hv], [2 * hv, 1]), _t(self.mask), _t(x["a_log"][j]), _t(x["dt_bias"][j]),
                     _t(self.nd, [s.n_seq, hv, 1, 2], list(self.nd.stride()), offset_elems=j * hv * 2),
                     _t(self.slot_last), _t(self.bounds)], [P("M", T), P("n_head", hv)], f"{j}")
            correct("apply")
        else:
            self.fill_scratch = 0
        add("ridgefill_hazard", [_t(x["cu_last"]), _t(x["positions"]), _t(self.bounds), A_, _t(self.meta),
                                 _t(self.slot_last), _t(self.count)], [P("M", 1)])
        self.calls = calls
        small = D != 128
        self.kernels = sum(1 if (c[0] == "ridgefill_gdn_fill" and small) else self.KERNELS[c[0]] for c in calls)

    def _launch(self, op, r, tens, params, stream: int) -> None:
        sb = self.fill_scratch if op == "ridgefill_gdn_fill" else 0
        rc = self.lib.launch(r, tens, params, stream=stream, scratch=self.scratch.data_ptr() if sb else None,
                             scratch_bytes=sb)
        if rc != abi.OK:
            raise RuntimeError(f"{op}: device row refused or failed (rc {rc})")

    def run(self, stream: int, events=None) -> None:
        """Issue one pass on `stream`. `events` (optional) maps an op name to a list of (start, end) CUDA event
        pairs, one pair per launch of that op, recorded on the current torch stream around each launch."""
        counts = {}
        for op, r, tens, params, _tag in self.calls:
            ev = events.get(op) if events else None
            if ev is not None:
                i = counts.get(op, 0)
                counts[op] = i + 1
                ev[i][0].record()
            self._launch(op, r, tens, params, stream)
            if ev is not None:
                ev[i][1].record()

    def op_counts(self) -> dict:
        out = {}
        for c in self.calls:
            out[c[0]] = out.get(c[0], 0) + 1
        return out

    # --------------------------------------------------------------- algorithmic work of one pass
    def algorithmic(self) -> dict:
        s = self.s
        T, d, G, A = s.T, s.d, s.n_gdn, s.n_attn
        hk, hv, D = s.hk, s.hv, s.head
        L = len(s.layers)
        n_int8_cols = L * d + (G * s.conv_dim if s.block_inputs else 0) + A * 2 * s.hkv * s.head_attn
        chunks = sum((n + 63) // 64 for n in s.lengths)
        return {
            "int8_ops": 2 * T * d * n_int8_cols,
            # the batched fill, state-only form: read k, v, g, beta and the state, write the state
            "fill_bytes": 2 * T * G * hk * D + 2 * T * G * hv * D + 8 * T * G * hv + 2 * 4 * s.n_seq * G * hv * D * D,
            "fill_chunk_flops": chunks * G * hv * (6 * 64 * 64 * D + 4 * 64 * D * D + 64 ** 3 * 2 // 3),
            "chains": G * hv * s.n_seq,
        }
