"""The RidgeFill approximate pass over every late layer of a prefill chunk: the lean late-layer loop of the
reference's arch core (arch/ridgefill_step.h:151-175 -> fill_layer, arch/ridgefill_layer.h:205-210), every op a
launch of this library's sm_100a device rows through the C ABI.

    ridgefill_mask                  which rows of the approximated sequence stay exact (once a pass)
    ridgefill_quant_act_i8g         the layer-S stream's codes (once a pass: every late layer projects h_S,
                                    arch/ridgefill_layer.h:60-63)
    ridgefill_state_correct undo    every DeltaNet layer's state at once (their pools are one array)
    for each late layer l:
      ridgefill_gemm_nt_q_bias      the projector x = proj_l(h_S) + bias_l, written straight into the approximated
                                    rows of the layer's block input (its rows operand is the mask: the select of
                                    ridgefill_select fused into the projector's epilogue)
      ridgefill_quant_act_i8g       the block input's codes (what the int8 block reads)
      DeltaNet layer (arch/qwen4exp_fill.h:29-61):
        ridgefill_gemm_nt_bias      the a|b projection (bf16)
        ridgefill_gemm_nt_q_bias    the mixed q|k|v projection (int8, no bias)
        ridgefill_gdn_conv_prep     conv, SiLU, q/k norm, gate and beta, into this layer's heads of the
                                    pass-wide k, v, g, beta arrays
      attention layer (arch/qwen4exp_fill.h:100-115):
        ridgefill_gemm_nt_q_bias    the k|v projection (int8, no bias)
        ridgefill_attn_kv_fill      k norm, rotary, the paged cache store
      (a DeltaNet layer's a|b projection and conv_prep, and an attention layer's whole block, run on a second
      stream beside the chain of projectors, codes and in-projections: LatePass._issue_block)
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


def mini_model() -> LateShape:
    """The reference's CPU mini model: d 256, 512 rows, 4 DeltaNet layers of 4 q/k and 8 v heads of 32, the fill's
    inputs given, 25 % of the rows kept exact."""
    return LateShape(T=512, d=256, layers="GGGG", hk=4, hv=8, head=32, share=0.25, vocab=4096, block_inputs=False)


def full_step(T: int = 32768) -> LateShape:
    """The full step over the 24 late layers of the 48-layer stack (18 DeltaNet + 6 attention), hidden 2,048,
    DeltaNet 16 q/k and 32 v heads of 128, attention 2 kv heads of 256, 30 % of the rows exact."""
    return LateShape(T=T)


def ragged_batch(seed: int = 0, long: int = 32768, short: int = 6) -> LateShape:
    """The mixed ragged batch: six prompts of U[256, 2,048] rows, then one 32K prompt (the approximated one)."""
    import random
    r = random.Random(seed)
    lens = [r.randint(256, 2048) for _ in range(short)] + [long]
    return LateShape(T=sum(lens), seqlens=tuple(lens))


def late_inputs(s: LateShape, device, seed: int = 0) -> dict:
    """Seeded synthetic inputs and weights of one pass, with the published benchmark's distributions: h_S and the exact block
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


# ============================================================================ tensor parallelism over one prompt

class Team:
    """The ranks of a tensor-parallel pass over one prompt (one process per GPU, torch.distributed for the
    rendezvous only): this rank, the world, and the mapping of device buffers across processes. A buffer is
    shared by `share`: every rank exports its own (CUDA IPC, ridgefill_peer_export) and maps everyone else's,
    and gets back the list of every rank's pointer as seen from here."""

    def __init__(self, world: int, rank: int, dist=None):
        self.world, self.rank, self.dist = world, rank, dist
        self.lib = abi.product().lib
        self._mapped = []   # (pointer, offset) pairs to unmap on close

    @classmethod
    def create(cls, world: int, rank: int, dist):
        return cls(world, rank, dist)

    def share(self, t) -> list[int]:
        """Every rank's pointer to its copy of the buffer `t` (one allocation per rank, the same shape
        everywhere), as device addresses valid in this process."""
        import ctypes as C
        L = self.lib
        L.ridgefill_peer_export.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_int64)]
        L.ridgefill_peer_import.argtypes = [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]
        handle = (C.c_uint8 * 64)()
        off = C.c_int64(0)
        if L.ridgefill_peer_export(C.c_void_p(t.data_ptr()), handle, C.byref(off)) != abi.OK:
            raise RuntimeError("ridgefill_peer_export failed")
        mine = (bytes(handle), off.value)
        everyone = [None] * self.world
        self.dist.all_gather_object(everyone, mine)
        ptrs = []
        for r, (h, o) in enumerate(everyone):
            if r == self.rank:
                ptrs.append(t.data_ptr())
                continue
            buf = (C.c_uint8 * 64).from_buffer_copy(h)
            out = C.c_void_p(0)
            if L.ridgefill_peer_import(buf, C.c_int64(o), C.byref(out)) != abi.OK:
                raise RuntimeError(f"ridgefill_peer_import of rank {r}'s buffer failed")
            self._mapped.append((out.value, o))
            ptrs.append(out.value)
        return ptrs

    def close(self):
        import ctypes as C
        L = self.lib
        L.ridgefill_peer_release.argtypes = [C.c_void_p, C.c_int64]
        for ptr, o in self._mapped:
            L.ridgefill_peer_release(C.c_void_p(ptr), C.c_int64(o))
        self._mapped = []


def attn_heads(hkv: int, rank: int, world: int) -> tuple[int, int]:
    """The attention kv heads [h0, h1) rank `rank` of `world` holds: an even split when world divides hkv, else one
    head each to the first hkv ranks and none to the others (ranks with no attention cache)."""
    if hkv % world == 0:
        per = hkv // world
        return rank * per, (rank + 1) * per
    return (rank, rank + 1) if rank < hkv else (0, 0)


def local_inputs(s: LateShape, x: dict, team: Team | None) -> tuple[dict, dict]:
    """This rank's slices of the pass's weights and inputs (the whole of them without a team), and the rank's
    geometry: the value and k heads of its DeltaNet span (shard.head_span, the reference's spans), its attention kv
    heads and its block of projector output columns. Every slice is a contiguous copy, so each rank's rows read
    operands laid out as a one-rank pass's are."""
    import torch
    import shard
    if team is None or team.world == 1:
        geo = {"v": (0, s.hv), "k": (0, s.hk), "a": (0, s.hkv), "cols": (0, s.d), "world": 1, "rank": 0}
        return x, geo
    world, rank = team.world, team.rank
    (v0, v1), (k0, k1) = shard.head_span(s.hk, s.hv, rank, world)
    a0, a1 = attn_heads(s.hkv, rank, world)
    if s.d % world or (s.d // world) % 16:
        raise ValueError(f"d {s.d} does not split into 16-column blocks over {world} ranks")
    c0, c1 = rank * s.d // world, (rank + 1) * s.d // world
    geo = {"v": (v0, v1), "k": (k0, k1), "a": (a0, a1), "cols": (c0, c1), "world": world, "rank": rank}
    D, hk, hv, G = s.head, s.hk, s.hv, s.n_gdn
    dev = x["h_s"].device
    y = dict(x)
    y["w_proj"] = [w[c0:c1].contiguous() for w in x["w_proj"]]
    y["s_proj"] = [t[:, c0:c1].contiguous() for t in x["s_proj"]]
    y["b_proj"] = [t[c0:c1].contiguous() for t in x["b_proj"]]
    heads_v = torch.cat([torch.arange(j * hv + v0, j * hv + v1) for j in range(G)]).to(dev)
    heads_k = torch.cat([torch.arange(j * hk + k0, j * hk + k1) for j in range(G)]).to(dev)
    y["state"] = x["state"][:, heads_v].contiguous()
    y["C"] = x["C"][heads_v].contiguous()
    if s.block_inputs:
        ch = torch.cat([torch.arange(k0 * D, k1 * D), torch.arange((hk + k0) * D, (hk + k1) * D),
                        torch.arange((2 * hk + v0) * D, (2 * hk + v1) * D)]).to(dev)
        ab_rows = torch.cat([torch.arange(v0, v1), torch.arange(hv + v0, hv + v1)]).to(dev)
        y["w_in"] = [w[ch].contiguous() for w in x["w_in"]]
        y["s_in"] = [t[:, ch].contiguous() for t in x["s_in"]]
        y["w_conv"] = [w[ch].contiguous() for w in x["w_conv"]]
        y["conv_state"] = [t[:, :, ch].contiguous() for t in x["conv_state"]]
        y["w_ab"] = [w[ab_rows].contiguous() for w in x["w_ab"]]
    else:
        y["k"] = x["k"][:, heads_k].contiguous()
        y["v"] = x["v"][:, heads_v].contiguous()
        y["g"] = x["g"][:, heads_v].contiguous()
        y["beta"] = x["beta"][:, heads_v].contiguous()
        ab_cols = torch.cat([torch.arange(v0, v1), torch.arange(hv + v0, hv + v1)]).to(dev)
        y["ab"] = [t[:, ab_cols].contiguous() for t in x["ab"]]
    y["a_log"] = [t[v0:v1].contiguous() for t in x["a_log"]]
    y["dt_bias"] = [t[v0:v1].contiguous() for t in x["dt_bias"]]
    if s.n_attn:
        Dh, Ha = s.head_attn, s.hkv
        rows_kv = torch.cat([torch.arange(a0 * Dh, a1 * Dh), torch.arange((Ha + a0) * Dh, (Ha + a1) * Dh)]).to(dev)
        y["w_kv"] = [w[rows_kv].contiguous() for w in x["w_kv"]]
        y["s_kv"] = [t[:, rows_kv].contiguous() for t in x["s_kv"]]
    return y, geo


class LatePass:
    """The buffers of one approximate pass over the late layers and the row launches that fill them, on one GPU or
    as one rank of a tensor-parallel team (`team`): the rank's DeltaNet value heads (with their k heads), its
    attention kv heads and its block of each projector's output columns, the blocks gathered into every rank's
    block input by the library's peer kernels. Each rank's state, decay sums and caches are then its heads' slices
    of the one-GPU pass's, bit for bit."""

    # kernels a launch of each row starts (the fill: its sequence plan and the fused kernel; the per-row
    # form for small heads is one kernel)
    KERNELS = {"ridgefill_mask": 1, "ridgefill_quant_act_i8g": 1, "ridgefill_gemm_nt_q_bias": 1, "ridgefill_select": 1,
               "ridgefill_gemm_nt_bias": 1, "ridgefill_gdn_conv_prep": 2, "ridgefill_attn_kv_fill": 1,
               "ridgefill_state_correct": 1, "ridgefill_gdn_fill": 2, "ridgefill_rho_update": 1, "ridgefill_hazard": 1,
               "ridgefill_gdn_in_proj": 1, "team_barrier": 1, "gather_columns": 1, "team_wait": 1}

    def __init__(self, shape: LateShape, device: str = "cuda", seed: int = 0, inputs: dict | None = None,
                 team: Team | None = None):
        import torch
        self.torch = torch
        self.s = s = shape
        self.lib = abi.product()
        dev = torch.device(device)
        self.dev = dev
        self.team = team if team is not None and team.world > 1 else None
        self.inp = inputs if inputs is not None else late_inputs(s, dev, seed)
        self.w, self.geo = local_inputs(s, self.inp, self.team)
        x = self.w
        T, d, G, D = s.T, s.d, s.n_gdn, s.head
        grp = s.group or d
        self.grp = grp
        # the DeltaNet k|v projection with conv_prep's arithmetic in its epilogue (per-row scales, 128-wide heads)
        self.fused_in = grp == d and s.head == 128 and d % 128 == 0
        (v0, v1), (k0, k1), (a0, a1), (c0, c1) = self.geo["v"], self.geo["k"], self.geo["a"], self.geo["cols"]
        self.hv_r, self.hk_r, self.hkv_r, self.cols = v1 - v0, k1 - k0, a1 - a0, c1 - c0
        hv, hk = self.hv_r, self.hk_r

        def empty(*sz, dtype):
            return torch.empty(*sz, dtype=dtype, device=dev)

        # pass outputs and intermediates
        self.mask = torch.zeros(T, dtype=torch.int32, device=dev)
        self.bounds = torch.zeros(4, dtype=torch.int32, device=dev)
        self.codes_h = empty(T, d, dtype=torch.int8)
        self.scale_h = empty(T, d // grp, dtype=torch.float32)
        # every layer's block input, one allocation (mapped by the team's peers), the exact rows copied in
        self.x_all = torch.stack(self.inp["x_exact"])
        self.x = list(self.x_all.unbind(0))
        self.codes_x = empty(T, d, dtype=torch.int8)
        self.scale_x = empty(T, d // grp, dtype=torch.float32)
        # the attention layers' block input codes: their own buffer, as their blocks run on the second stream
        self.codes_a = empty(T, d, dtype=torch.int8) if s.n_attn else None
        self.scale_a = empty(T, d // grp, dtype=torch.float32) if s.n_attn else None
        self.state = x["state"].clone()
        self.applied = torch.zeros(s.n_seq, G * hv, 1, 1, dtype=torch.float32, device=dev)
        self.nd = torch.zeros(s.n_seq, G * hv, 1, 2, dtype=torch.float32, device=dev)
        self.meta = torch.zeros(s.n_seq, 1, 1, 2, dtype=torch.float32, device=dev)
        self.count = torch.zeros(1, dtype=torch.float32, device=dev)
        self.slot_last = torch.tensor([[s.n_seq - 1]], dtype=torch.int32, device=dev)   # the approximated sequence
        self.slots_all = torch.arange(s.n_seq, dtype=torch.int32, device=dev).view(-1, 1)
        self.conv_dim_r = 2 * hk * D + hv * D
        starts = [0]
        for n in s.lengths:
            starts.append(starts[-1] + n)
        self.seq_bounds = list(zip(starts[:-1], starts[1:]))
        if s.block_inputs:
            C = self.conv_dim_r
            self.mixed = empty(T, C, dtype=torch.bfloat16)
            self.ab = [empty(T, 2 * hv, dtype=torch.bfloat16) for _ in range(G)]
            Cq = hk * D
            self.w_in_q = [w[:Cq].contiguous() for w in x["w_in"]]
            self.w_in_kv = [w[Cq:].contiguous() for w in x["w_in"]]
            self.s_in_q = [t[:, :Cq].contiguous() for t in x["s_in"]]
            self.s_in_kv = [t[:, Cq:].contiguous() for t in x["s_in"]]
            self.k = empty(T, G * hk, D, dtype=torch.bfloat16)
            self.v = empty(T, G * hv, D, dtype=torch.bfloat16)
            self.g = empty(T, G * hv, dtype=torch.float32)
            self.beta = empty(T, G * hv, dtype=torch.float32)
            self.conv_state = [t.clone() for t in x["conv_state"]]
            self.zero_ab = torch.zeros(2 * hv, dtype=torch.bfloat16, device=dev)
            self.ctx = torch.zeros(s.n_seq, dtype=torch.int32, device=dev)   # fresh prompts: no conv history
        else:
            self.ab, self.k, self.v, self.g, self.beta = x["ab"], x["k"], x["v"], x["g"], x["beta"]
        self.cache = []
        if s.n_attn and self.hkv_r:
            Dh = s.head_attn
            self.kv = empty(T, 2 * self.hkv_r * Dh, dtype=torch.bfloat16)
            self.cache = [torch.zeros(2, T + 1024, self.hkv_r, Dh, dtype=torch.bfloat16, device=dev) for _ in range(s.n_attn)]
            self.rope_pos = self.inp["positions"].view(1, T).expand(3, T).contiguous()   # text rows: every plane the index
        self.epoch = 0
        if self.team is not None:
            L = len(s.layers)
            # counters: one slot a layer (its gathered block input), then the pass barrier's
            self.counters = torch.zeros(L + 1, dtype=torch.int64, device=dev)
            self.peer_x = self.team.share(self.x_all)
            self.peer_flags = self.team.share(self.counters)
            self.comm = torch.cuda.Stream(device=dev)
        self._build()
        self.scratch = torch.empty(max(self.fill_scratch, 16), dtype=torch.uint8, device=dev)

    # --------------------------------------------------------------- the launch list
    def _build(self):
        s, x, inp = self.s, self.w, self.inp
        P, S, F = abi.pint, abi.pstr, abi.pf64
        A_ = abi.absent()
        T, d, G, D = s.T, s.d, s.n_gdn, s.head
        hk, hv = self.hk_r, self.hv_r
        row = lambda op: self.lib.find_row(op, abi.DOMAIN_DEVICE)   # noqa: E731
        c0 = self.geo["cols"][0]
        head, layers, tail = [], [], []   # the pass's launches: before the layers, per layer (list), after

        def call(op, tens, params, tag=""):
            return (op, row(op), tens, params, tag)

        def gemm_q(a, sa, w, sw, bias, y, N, tag, M=T, rows=None):
            return call("ridgefill_gemm_nt_q_bias", [a if isinstance(a, abi.RadTensor) else _t(a),
                                                     sa if isinstance(sa, abi.RadTensor) else _t(sa), _t(w), _t(sw),
                                                     A_ if bias is None else _t(bias), y, A_,
                                                     A_ if rows is None else _t(rows)],
                        [P("M", M), P("N", N), P("K", d), P("group", self.grp), S("dtype", "i8a8")], tag)

        def quant(src, codes, scale, tag):
            return call("ridgefill_quant_act_i8g", [_t(src), _t(codes), _t(scale)],
                        [P("M", T), P("n", d), P("group", self.grp), S("dtype", "bf16")], tag)

        def correct(mode):
            tens = [_t(self.state), _t(self.slot_last), _t(self.applied), _t(self.slot_last), _t(x["C"])]
            tens += [_t(self.nd), _t(self.slot_last)] if mode == "apply" else [A_, A_]
            return call("ridgefill_state_correct", tens + [_t(self.bounds)],
                        [P("M", 1), S("mode", mode), F("alpha", s.alpha), P("n_head", G * hv), P("sd0", D), P("sd1", D)], mode)

        head.append(call("ridgefill_mask", [_t(inp["cu_last"]), _t(inp["token_ids"]), _t(inp["positions"]), _t(inp["score"]),
                                            _t(self.mask), _t(self.bounds), A_],
                         [P("M", T), F("share", s.share), P("seed", 0), S("mode", "class")]))
        head.append(quant(inp["h_s"], self.codes_h, self.scale_h, "h_S"))
        if G:
            head.append(correct("undo"))
        gi = ai = 0
        for li, kind in enumerate(s.layers):
            proj = [gemm_q(self.codes_h, self.scale_h, x["w_proj"][li], x["s_proj"][li], x["b_proj"][li],
                           _t(self.x[li], [T, self.cols], list(self.x[li].stride()), offset_elems=c0), self.cols,
                           f"proj {li}", rows=self.mask)]
            block = []
            if kind == "G" and s.block_inputs:
                C, Cq = self.conv_dim_r, hk * D
                block.append(quant(self.x[li], self.codes_x, self.scale_x, f"x {li}"))
                # the a|b projection: on the second stream it starts with the codes; in an ordered pass it follows
                # them, and as the quantiser reads the block input last row first, the rows it read last (the first
                # ones) are still in L2 when this reads them in order
                block.append(call("ridgefill_gemm_nt_bias", [_t(self.x[li]), _t(x["w_ab"][gi]), _t(self.zero_ab), A_,
                                                             _t(self.ab[gi])],
                                  [P("M", T), P("N", 2 * hv), P("K", d), S("dtype", "bf16")], f"ab {li}"))
                # the mixed projection's k|v columns over every row; its q columns only over each sequence's last
                # three rows, the conv state's (the state-only fill reads no q, so conv_prep is given none). With
                # per-row scales the k|v projection carries the convolution, SiLU and k norm in its epilogue
                # (ridgefill_gdn_in_proj: k and v straight from the tiles, only the sequences' last three rows of
                # the projection to `mixed`), and conv_prep is left the gates and the conv-state update.
                kv = _t(self.mixed, [T, C - Cq], [C, 1], offset_elems=Cq)
                if self.fused_in:
                    cs = self.conv_state[gi]
                    block.append(call("ridgefill_gdn_in_proj",
                                      [_t(self.codes_x), _t(self.scale_x), _t(self.w_in_kv[gi]), _t(self.s_in_kv[gi]),
                                       _t(x["w_conv"][gi], [C - Cq, 4], [4, 1], offset_elems=Cq * 4), A_,
                                       _t(cs, [cs.shape[0], 3, C - Cq], list(cs.stride()), offset_elems=Cq),
                                       _t(inp["cu_seqlens"]), _t(self.slots_all.view(-1)), _t(self.ctx),
                                       _t(self.k, [T, hk, D], list(self.k.stride()), offset_elems=gi * hk * D),
                                       _t(self.v, [T, hv, D], list(self.v.stride()), offset_elems=gi * hv * D), kv],
                                      [P("M", T), P("N", C - Cq), P("K", d), P("n_head_k", hk), P("n_head_v", hv),
                                       P("group", self.grp), S("dtype", "i8a8")], f"in kv {li}"))
                else:
                    block.append(gemm_q(self.codes_x, self.scale_x, self.w_in_kv[gi], self.s_in_kv[gi], None, kv, C - Cq,
                                        f"in kv {li}"))
                for a_, b_ in self.seq_bounds:
                    m0 = max(a_, b_ - 3)
                    if b_ <= m0:
                        continue
                    M = b_ - m0
                    block.append(gemm_q(_t(self.codes_x, [M, d], [d, 1], offset_elems=m0 * d),
                                        _t(self.scale_x, [M, d // self.grp], [d // self.grp, 1], offset_elems=m0 * (d // self.grp)),
                                        self.w_in_q[gi], self.s_in_q[gi], None, _t(self.mixed, [M, Cq], [C, 1], offset_elems=m0 * C),
                                        Cq, f"in q {li}", M=M))
                ab = self.ab[gi]
                block.append(call("ridgefill_gdn_conv_prep",
                                  [_t(self.mixed), _t(x["w_conv"][gi]), A_, _t(x["a_log"][gi]), _t(x["dt_bias"][gi]),
                                   _t(self.conv_state[gi]), _t(inp["cu_seqlens"]), _t(ab, [T, hv], [2 * hv, 1]),
                                   _t(ab, [T, hv], [2 * hv, 1], offset_elems=hv), _t(self.slots_all.view(-1)), _t(self.ctx),
                                   A_,
                                   _t(self.k, [T, hk, D], list(self.k.stride()), offset_elems=gi * hk * D),
                                   _t(self.v, [T, hv, D], list(self.v.stride()), offset_elems=gi * hv * D),
                                   _t(self.g, [T, hv], [G * hv, 1], offset_elems=gi * hv),
                                   _t(self.beta, [T, hv], [G * hv, 1], offset_elems=gi * hv)],
                                  [P("M", T), P("n_head_k", hk), P("n_head_v", hv), P("head_k", D), P("head_v", D),
                                   P("conv", 4), P("columns", 0 if self.fused_in else 1)], f"{li}"))
            elif kind == "A" and self.hkv_r:
                Ha, Dh = self.hkv_r, s.head_attn
                block.append(quant(self.x[li], self.codes_a, self.scale_a, f"x {li}"))
                block.append(gemm_q(self.codes_a, self.scale_a, x["w_kv"][ai], x["s_kv"][ai], None, _t(self.kv), 2 * Ha * Dh,
                                    f"kv {li}"))
                block.append(call("ridgefill_attn_kv_fill",
                                  [_t(self.kv, [T, Ha, Dh], [2 * Ha * Dh, Dh, 1]),
                                   _t(self.kv, [T, Ha, Dh], [2 * Ha * Dh, Dh, 1], offset_elems=Ha * Dh), _t(inp["k_norm"][ai]),
                                   _t(self.rope_pos), _t(inp["slot_mapping"]), _t(self.cache[ai]), A_],
                                  [P("M", T), P("n_head_kv", Ha), P("head_dim", Dh), P("rope_dim", s.rope_dim),
                                   F("rope_theta", s.rope_theta), S("rope_mode", "imrope"),
                                   S("rope_sections", ",".join(str(v) for v in s.rope_sections))], f"{li}"))
            if kind == "A":
                ai += 1
            if kind == "G":
                gi += 1
            layers.append((proj, block))
        self.fill_scratch = 0
        if G:
            tail.append(call("ridgefill_gdn_fill", [A_, _t(self.k), _t(self.v), _t(self.g), _t(self.beta), _t(self.state),
                                                    _t(self.slots_all), _t(inp["cu_seqlens"]), A_],
                             [P("M", T), P("n_head_k", G * hk), P("n_head_v", G * hv), P("head_k", D), P("head_v", D),
                              P("chunk", 64)]))
            fill = tail[-1]
            self.fill_scratch = self.lib.scratch_bytes(fill[1], fill[2], fill[3])
            for j in range(G):
                tail.append(call("ridgefill_rho_update",
                                 [_t(self.ab[j], [T, hv], [2 * hv, 1]), _t(self.mask), _t(x["a_log"][j]), _t(x["dt_bias"][j]),
                                  _t(self.nd, [s.n_seq, hv, 1, 2], list(self.nd.stride()), offset_elems=j * hv * 2),
                                  _t(self.slot_last), _t(self.bounds)], [P("M", T), P("n_head", hv)], f"{j}"))
            tail.append(correct("apply"))
        tail.append(call("ridgefill_hazard", [_t(inp["cu_last"]), _t(inp["positions"]), _t(self.bounds), A_, _t(self.meta),
                                              _t(self.slot_last), _t(self.count)], [P("M", 1)]))
        self.head, self.layers, self.tail = head, layers, tail
        self.calls = head + [c for proj, block in layers for c in proj + block] + tail
        # the fill is one kernel in its per-row form (heads of at most 64 dims) and its per-head form (a state-only
        # launch of at least 64 chains), two (plan + cooperative kernel) otherwise
        one_kernel_fill = D != 128 or G * hv * s.n_seq >= 64
        self.kernels = sum(1 if (c[0] == "ridgefill_gdn_fill" and one_kernel_fill) else self.KERNELS[c[0]] for c in self.calls)
        # In the per-head form the fill's CTAs wait on nothing but their own SM, and a launch of L Hv chains over the
        # SMs leaves some of them idle in its last wave: the decay sums (which read only a, the mask and the bounds)
        # run there, on a second stream, instead of after the fill. The other forms keep the tail in order (the
        # cooperative one needs all its CTAs resident at once).
        self.rho_beside_fill = D == 128 and G * hv * s.n_seq >= 64
        if self.team is not None:   # the barrier, one gather and one wait a layer
            self.kernels += 1 + 2 * len(s.layers)

    def _launch(self, op, r, tens, params, stream: int) -> None:
        sb = self.fill_scratch if op == "ridgefill_gdn_fill" else 0
        rc = self.lib.launch(r, tens, params, stream=stream, scratch=self.scratch.data_ptr() if sb else None,
                             scratch_bytes=sb)
        if rc != abi.OK:
            raise RuntimeError(f"{op}: device row refused or failed (rc {rc})")

    def run(self, stream: int, events=None, before_tail=None) -> None:
        """Issue one pass on `stream`, with the work that can run beside the chain on this pass's second stream
        (`_issue_block`, `_issue_tail`) and, on a team, the column gathers on a third. `events` (optional) maps an
        op name to a list of (start, end) CUDA event pairs, one pair per launch of that op, recorded on the current
        torch stream around each launch; such a pass is issued in order on `stream` alone. `before_tail` (optional) is called on the host once every layer's
        launches are on `stream` and before the fill's: work the caller queues behind `stream` at that point (an
        event) sees `results_split()[0]` final, so their readback can overlap the fill."""
        counts = {}

        def emit(c, on=None):
            op = c[0]
            ev = events.get(op) if events else None
            if ev is not None:
                i = counts.get(op, 0)
                counts[op] = i + 1
                ev[i][0].record()
            self._launch(op, c[1], c[2], c[3], stream if on is None else on)
            if ev is not None:
                ev[i][1].record()

        if self.team is not None:
            self._run_team(stream, emit, before_tail, beside=events is None)
            return
        for c in self.head:
            emit(c)
        for proj, block in self.layers:
            for c in proj:
                emit(c)
            self._issue_block(stream, emit, block, beside=events is None)
        if getattr(self, "_prep_done", None) is not None or getattr(self, "_side_used", False):
            self._join_side(self.torch.cuda.ExternalStream(stream, device=self.dev))
        if before_tail is not None:
            before_tail()
        self._issue_tail(stream, emit, beside=events is None)

    def _issue_block(self, stream: int, emit, block, beside: bool) -> None:
        """One layer's block. With `beside`, a DeltaNet layer's a|b projection goes on the second stream as soon as
        the block input is complete (beside the codes and the in-projection), and its gates and conv-state update
        (conv_prep) follow it there once the layer's in-projection and q tails are done, beside the next layer's
        projector and codes; the next in-projection (which rewrites the shared tail rows conv_prep reads) and the
        fill wait for them. An attention layer's whole block goes there too (its codes in their own buffer); the
        fill waits for the second stream as a whole (`_join_side`)."""
        attention = any(c[0] == "ridgefill_attn_kv_fill" for c in block) and self.codes_a is not None
        if not (beside and (attention or any(c[0] == "ridgefill_gemm_nt_bias" for c in block))):
            for c in block:
                emit(c)
            return
        torch = self.torch
        if getattr(self, "side", None) is None:
            self.side = torch.cuda.Stream(device=self.dev)
        main, side = torch.cuda.ExternalStream(stream, device=self.dev), self.side
        ready = torch.cuda.Event()
        ready.record(main)
        side.wait_event(ready)
        if attention:
            # an attention layer's whole block (its codes in their own buffer, the k|v projection, the cache
            # write): nothing on the pass's stream reads what it writes before the fill
            for c in block:
                emit(c, side.cuda_stream)
            self._side_used = True
            return
        for c in block:
            if c[0] == "ridgefill_gemm_nt_bias":
                emit(c, side.cuda_stream)
        for c in block:
            if c[0] == "ridgefill_gemm_nt_bias":
                continue
            if c[0] == "ridgefill_gdn_conv_prep":
                issued = torch.cuda.Event()
                issued.record(main)
                side.wait_event(issued)
                emit(c, side.cuda_stream)
                self._prep_done = torch.cuda.Event()
                self._prep_done.record(side)
                continue
            if c[0] in ("ridgefill_gdn_in_proj", "ridgefill_gemm_nt_q_bias"):
                self._wait_prep(main)
            emit(c)

    def _wait_prep(self, main) -> None:
        """The pass's stream waits for the last conv_prep issued on the second stream (if one is pending)."""
        if getattr(self, "_prep_done", None) is not None:
            main.wait_event(self._prep_done)
            self._prep_done = None

    def _join_side(self, main) -> None:
        """The pass's stream waits for everything issued on the second stream so far (before the fill)."""
        self._wait_prep(main)
        if getattr(self, "_side_used", False):
            done = self.torch.cuda.Event()
            done.record(self.side)
            main.wait_event(done)
            self._side_used = False

    def _issue_tail(self, stream: int, emit, beside: bool) -> None:
        """The fill and what follows it. With `beside` (and the fill in its per-head form) the decay sums go on a
        second stream that starts with the fill; the correction waits for them."""
        if not (beside and self.rho_beside_fill):
            for c in self.tail:
                emit(c)
            return
        torch = self.torch
        if getattr(self, "side", None) is None:
            self.side = torch.cuda.Stream(device=self.dev)
        main, side = torch.cuda.ExternalStream(stream, device=self.dev), self.side
        start = torch.cuda.Event()
        start.record(main)
        side.wait_event(start)
        rho_done = None
        for c in self.tail:
            if c[0] == "ridgefill_rho_update":
                emit(c, side.cuda_stream)
                continue
            if rho_done is None and c[0] != "ridgefill_gdn_fill":
                rho_done = torch.cuda.Event()
                rho_done.record(side)
                main.wait_event(rho_done)
            emit(c)

    def _run_team(self, stream: int, emit, before_tail=None, beside: bool = False) -> None:
        """One rank's pass: the barrier (every rank has finished its previous pass), the head of the pass, then per
        layer its projector block (into the approximated rows) on `stream` and that block's gather to the peers on the comm stream,
        while `stream` goes on with the previous layer's block (after waiting for all of its columns); the fill and
        the rest once every layer is done."""
        import ctypes as C
        torch = self.torch
        team, L = self.team, self.lib.lib
        main = torch.cuda.ExternalStream(stream, device=self.dev)
        self.epoch += 1
        e, R = self.epoch, team.world
        ctas = L.ridgefill_team_gather_ctas()
        flags = (C.c_void_p * R)(*self.peer_flags)
        layer_bytes = self.s.T * self.s.d * 2
        own = C.c_void_p(self.counters.data_ptr())
        n_layers = len(self.s.layers)
        L.ridgefill_team_barrier.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_ulonglong, C.c_void_p]
        L.ridgefill_gather_columns.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int64, C.c_int64,
                                               C.c_int64, C.c_int64, C.c_int, C.c_void_p]
        L.ridgefill_team_wait.argtypes = [C.c_void_p, C.c_int, C.c_ulonglong, C.c_void_p]
        if L.ridgefill_team_barrier(flags, team.rank, R, n_layers, e * (R - 1), C.c_void_p(stream)) != abi.OK:
            raise RuntimeError("ridgefill_team_barrier failed")
        for c in self.head:
            emit(c)
        c0, c1 = self.geo["cols"]
        T, d = self.s.T, self.s.d
        comm = self.comm

        def block(li):
            if L.ridgefill_team_wait(own, li, e * (R - 1) * ctas, C.c_void_p(stream)) != abi.OK:
                raise RuntimeError("ridgefill_team_wait failed")
            self._issue_block(stream, emit, self.layers[li][1], beside)

        for li, (proj, _block) in enumerate(self.layers):
            for c in proj:
                emit(c)
            ready = torch.cuda.Event()
            ready.record(main)
            comm.wait_event(ready)
            dsts = (C.c_void_p * R)(*[ptr + li * layer_bytes for ptr in self.peer_x])   # every rank's layer-li input
            if L.ridgefill_gather_columns(C.c_void_p(self.x[li].data_ptr()), dsts, flags, team.rank, R, T, d, c0, c1, li,
                                          C.c_void_p(comm.cuda_stream)) != abi.OK:
                raise RuntimeError("ridgefill_gather_columns failed")
            if li:
                block(li - 1)
        if self.layers:
            block(len(self.layers) - 1)
        done = torch.cuda.Event()
        done.record(comm)
        main.wait_event(done)   # the last gathers read this rank's block inputs: done before the next pass writes them
        self._join_side(main)
        if before_tail is not None:
            before_tail()
        self._issue_tail(stream, emit, beside)

    def op_counts(self) -> dict:
        out = {}
        for c in self.calls:
            out[c[0]] = out.get(c[0], 0) + 1
        return out

    def inputs_per_step(self) -> list:
        """The tensors a pass reads that change from prompt to prompt: h_S, the token ids and the positions."""
        return [self.inp["h_s"], self.inp["token_ids"], self.inp["positions"]]

    def results(self) -> list:
        """The buffers a pass leaves for the engine: every DeltaNet state and conv state, every attention cache,
        the mask, the decay sums and the hazard record."""
        out = [self.state, self.mask, self.nd, self.meta, self.count] + list(self.cache)
        if self.s.block_inputs:
            out += list(self.conv_state)
        return out

    def results_split(self) -> tuple[list, list]:
        """`results()` in two parts: those final once every layer's block has run (the mask, the attention caches,
        the conv states: nothing in the fill and after it writes them), and those the fill and the ops after it
        write (the states, the decay sums, the hazard record)."""
        early = [self.mask] + list(self.cache) + (list(self.conv_state) if self.s.block_inputs else [])
        return early, [self.state, self.nd, self.meta, self.count]

    # --------------------------------------------------------------- algorithmic work of one pass
    def algorithmic(self) -> dict:
        s = self.s
        T, d, G, A = s.T, s.d, s.n_gdn, s.n_attn
        hk, hv, D = self.hk_r, self.hv_r, s.head
        L = len(s.layers)
        # the mixed projection's k|v columns over every row, its q columns over each sequence's last three rows only
        q_cols = hk * D if s.block_inputs else 0
        n_int8_cols = L * self.cols + (G * (self.conv_dim_r - q_cols) if s.block_inputs else 0) + \
            (A * 2 * self.hkv_r * s.head_attn if self.hkv_r else 0)
        q_tail_rows = sum(min(n, 3) for n in s.lengths)
        chunks = sum((n + 63) // 64 for n in s.lengths)
        # the k|v projections of the DeltaNet layers, when the fused in-projection row issues them
        in_proj_ops = 2 * T * d * G * (self.conv_dim_r - q_cols) if s.block_inputs and self.fused_in else 0
        return {
            # ridgefill_gemm_nt_q_bias launches (projectors, q tails, attention k|v; the DeltaNet k|v when not fused)
            "int8_ops": 2 * T * d * n_int8_cols + 2 * q_tail_rows * d * G * q_cols - in_proj_ops,
            "int8_ops_in_proj": in_proj_ops,
            # the batched fill, state-only form: read k, v, g, beta and the state, write the state
            "fill_bytes": 2 * T * G * hk * D + 2 * T * G * hv * D + 8 * T * G * hv + 2 * 4 * s.n_seq * G * hv * D * D,
            "fill_chunk_flops": chunks * G * hv * (6 * 64 * 64 * D + 4 * 64 * D * D + 64 ** 3 * 2 // 3),
            "chains": G * hv * s.n_seq,
        }
