"""The whole approximate pass over the late layers on the device (late_pass.LatePass, every op a device row) against
the same pass on the host (oracle/cpu_path.CpuLatePass: the reference's own host rows for mask, select, the state
correction, rho and the hazard record where oracle/_ref was built, the restatement's oracles for the rest), fed
the same seeded inputs. Every buffer the pass writes is compared:

    mask, bounds, the hazard record                    equal
    every layer's block input after select             bit for bit (the int8 projector is exact)
    attention caches, conv states                      bit for bit
    a|b projections                                    the reference's bf16 GEMM bound (2^-7 |y| + 2^-9 RMS)
    k, v (conv_prep)                                   2 bf16 ulp (2^-7 of the larger magnitude), plus the
                                                       smallest normal f32: the device flushes f32 subnormal
                                                       results (|y| < 1.2e-38) to zero, the host keeps them
    g, beta                                            1e-5 wherever a|b agree bit for bit
    DeltaNet state, every layer and slot               1e-3 relative L2 (f32 sequential rule)
    N|D decay sums, rho, applied scales                1e-4 relative on N and D, 1e-5 on rho (the reference's
                                                       bounds) for every head whose a values (from the bf16 a|b
                                                       projection) are bit for bit the host's; 1e-3 on rho for a
                                                       head that read an a value one bf16 ulp off

The shapes: the reference's CPU mini model (d 256, 512 rows, 4 DeltaNet layers of 4 / 8 heads of 32), a
2,048-row sample of the full step's first four late layers (G G G A) at full width, all 24 late layers at 256 rows
(the fill batched over 18 layers' heads), and a ragged batch of three sequences."""
import numpy as np
import pytest

import harness as H  # noqa: F401  (puts the package on the path)
import late_pass as LP
import cpu_path as CP

gpu = pytest.mark.gpu
FLT_MIN = float(np.finfo(np.float32).tiny)

SHAPES = {
    "mini_model": LP.mini_model(),
    "full_step_T2048_first4": LP.LateShape(T=2048, layers="GGGA"),
    "full_step_T256_all24": LP.LateShape(T=256),
    "ragged_3seq": LP.LateShape(T=1400, layers="GGA", seqlens=(300, 100, 1000)),
}


def _u16(t):
    import torch
    t = t.detach().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def _rel(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


@gpu
@pytest.mark.parametrize("name", list(SHAPES))
def test_late_pass_matches_the_cpu_path(name, cuda):
    torch = cuda
    shape = SHAPES[name]
    dev = LP.LatePass(shape, "cuda", seed=17)
    host = CP.to_host(dev.inp)
    cpu = CP.CpuLatePass(shape, host)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dev.run(stream.cuda_stream)
    stream.synchronize()
    cpu.run()
    s = shape
    G, hv, hk = s.n_gdn, s.hv, s.hk

    assert np.array_equal(_u16(dev.mask), cpu.mask)
    assert np.array_equal(_u16(dev.bounds), cpu.bounds)
    assert np.array_equal(_u16(dev.meta), cpu.meta) and np.array_equal(_u16(dev.count), cpu.count)
    for li in range(len(s.layers)):
        assert np.array_equal(_u16(dev.x[li]), cpu.xl[li]), f"layer {li}: block input after select"
    for ai in range(s.n_attn):
        assert np.array_equal(_u16(dev.cache[ai]), cpu.cache[ai]), f"attention layer {ai}: cache"
    same_ab = np.ones((s.T, G * hv), bool)
    if s.block_inputs:
        for j in range(G):
            assert np.array_equal(_u16(dev.conv_state[j]), cpu.conv_state[j]), f"DeltaNet layer {j}: conv state"
            got, want = _u16(dev.ab[j]), cpu.ab[j]
            xf, yf = H.bf16_bits_to_f32(got).astype(np.float64), H.bf16_bits_to_f32(want).astype(np.float64)
            rms = np.sqrt(np.mean(yf ** 2))
            assert np.all(np.abs(xf - yf) <= 2.0 ** -7 * np.maximum(np.abs(xf), np.abs(yf)) + 2.0 ** -9 * rms)
            eq = got == want
            same_ab[:, j * hv:(j + 1) * hv] = eq[:, :hv] & eq[:, hv:]
        for name, got, want in (("k", _u16(dev.k), cpu.k), ("v", _u16(dev.v), cpu.v)):
            xf, yf = H.bf16_bits_to_f32(got).astype(np.float64), H.bf16_bits_to_f32(want).astype(np.float64)
            bad = ~((got == want) | (np.abs(xf - yf) <= np.ldexp(np.maximum(np.abs(xf), np.abs(yf)), -7) + FLT_MIN))
            assert not bad.any(), (name, int(bad.sum()), [(tuple(i), xf[tuple(i)], yf[tuple(i)]) for i in np.argwhere(bad)[:4]])
        for got, want in ((_u16(dev.g), cpu.g), (_u16(dev.beta), cpu.beta)):
            err = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
            assert err[same_ab].max() <= 1e-5
    state, want_state = _u16(dev.state), cpu.state
    for sl in range(s.n_seq):
        for j in range(G):
            blk = slice(j * hv, (j + 1) * hv)
            assert _rel(state[sl, blk], want_state[sl, blk]) <= 1e-3, (sl, j)
    # decay sums and the applied scale: the reference's bounds on every head whose a values (rho's input, from the
    # bf16 a|b projection) are bit for bit the host's; a head that read an a one bf16 ulp off (the bf16 GEMM's own
    # rounding, which the reference bounds at 2 ulp) within 1e-3 of rho
    nd, want_nd = _u16(dev.nd), cpu.nd
    a_same = same_ab[:, :].all(axis=0)                      # [G hv]: every row of the head's a matched
    rho = lambda x: np.clip(x[..., 0, 0] / np.where(x[..., 0, 1] > 0, x[..., 0, 1], 1.0), 0.0, 1.0)   # noqa: E731
    exact = np.abs(nd - want_nd) <= 1e-4 * np.maximum(np.abs(want_nd), 1.0)
    assert exact.all(axis=(2, 3))[:, a_same].all()
    assert np.abs(rho(nd) - rho(want_nd))[:, a_same].max(initial=0.0) <= 1e-5
    assert np.abs(rho(nd) - rho(want_nd)).max() <= 1e-3
    ap, want_ap = _u16(dev.applied)[..., 0, 0], cpu.applied[..., 0, 0]
    assert np.abs(ap - want_ap)[:, a_same].max(initial=0.0) <= 1e-5 * max(1.0, s.alpha)
    assert np.abs(ap - want_ap).max() <= 1e-3 * max(1.0, s.alpha)


@gpu
def test_batched_fill_equals_one_fill_per_layer(cuda, product_lib):
    """The late pass's single fill launch over every DeltaNet layer's heads writes, bit for bit, what one fill
    launch per layer writes: the heads are independent chains and each is computed the same way whatever else
    the launch holds."""
    torch = cuda
    shape = LP.LateShape(T=1000, d=256, layers="GGG", block_inputs=False, seqlens=(400, 600))
    dev = LP.LatePass(shape, "cuda", seed=5)
    G, hk, hv, D, T = shape.n_gdn, shape.hk, shape.hv, shape.head, shape.T
    state0 = dev.state.clone()
    fill = [c for c in dev.calls if c[0] == "ridgefill_gdn_fill"][0]
    stream = torch.cuda.Stream()
    dev._launch(fill[0], fill[1], fill[2], fill[3], stream.cuda_stream)
    stream.synchronize()
    batched = dev.state.clone()
    per_layer = state0.clone()
    from harness import abi
    for j in range(G):
        k = dev.k[:, j * hk:(j + 1) * hk]
        v = dev.v[:, j * hv:(j + 1) * hv]
        g = dev.g[:, j * hv:(j + 1) * hv]
        b = dev.beta[:, j * hv:(j + 1) * hv]
        st = per_layer[:, j * hv:(j + 1) * hv]
        tens = [abi.absent(), H.dev(k, abi.BF16), H.dev(v, abi.BF16), H.dev(g), H.dev(b), H.dev(st), H.dev(dev.slots_all),
                H.dev(dev.inp["cu_seqlens"]), abi.absent()]
        assert H.launch(product_lib, "ridgefill_gdn_fill", tens, H.gdn_params(T, hk, hv)) == abi.OK
    torch.cuda.synchronize()
    assert torch.equal(batched, per_layer)


@gpu
def test_the_pass_and_its_fill_repeat_bit_for_bit(cuda):
    """The pass's own fill inputs (the second pass, up to its fill), the fill launched again and again from the same
    state after the pass's other kernels: every run's state equal bit for bit, and two passes from fresh objects over
    the same seeded inputs equal bit for bit. (The per-head fill once handed a chunk's gamma_L to the chain's lanes
    through a slot the next chunk of that parity could overwrite first: the first fill after other kernels then
    differed from the ones after it.)"""
    torch = cuda
    shape = LP.LateShape(T=640, layers="GGAG", seqlens=(200, 440))
    passes = []
    for _ in range(2):
        p = LP.LatePass(shape, "cuda", seed=3)
        s = torch.cuda.Stream()
        for _ in range(2):
            p.run(s.cuda_stream)
        s.synchronize()
        passes.append(p.state.clone())
    assert torch.equal(passes[0], passes[1])
    fill_i = [i for i, c in enumerate(p.calls) if c[0] == "ridgefill_gdn_fill"][0]
    for c in p.calls[:fill_i]:
        p._launch(c[0], c[1], c[2], c[3], s.cuda_stream)
    s.synchronize()
    st0 = p.state.clone()
    c = p.calls[fill_i]
    outs = []
    for _ in range(6):
        p.state.copy_(st0)
        p._launch(c[0], c[1], c[2], c[3], s.cuda_stream)
        s.synchronize()
        outs.append(p.state.clone())
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@gpu
def test_the_two_stream_pass_equals_the_ordered_pass(cuda):
    """The pass as the bench times it (a|b projections, conv_prep, attention blocks and decay sums on a second
    stream) against the same pass issued in order on one stream (`events` given), from fresh objects over the same
    seeded inputs, two passes each: every result bit for bit. And the results `results_split()` declares final when
    `before_tail` is called (mask, attention caches, conv states) are, at that point, what they are after the pass:
    copies taken on another stream from an event recorded in the hook equal the buffers at the end."""
    torch = cuda
    shape = LP.LateShape(T=640, layers="GGAG", seqlens=(200, 440))   # 3 x 32 heads x 2 sequences: the per-head fill
    two, one = LP.LatePass(shape, "cuda", seed=3), LP.LatePass(shape, "cuda", seed=3)
    assert two.rho_beside_fill
    s, copies = torch.cuda.Stream(), torch.cuda.Stream()
    early, _ = two.results_split()
    snaps = []

    def hook():
        at = torch.cuda.Event()
        at.record(s)
        copies.wait_event(at)
        with torch.cuda.stream(copies):
            snaps[:] = [t.clone() for t in early]

    for _ in range(2):
        two.run(s.cuda_stream, before_tail=hook)
        one.run(s.cuda_stream, events={})
    torch.cuda.synchronize()
    for x, y in zip(two.results(), one.results()):
        assert torch.equal(x, y)
    assert len(snaps) == len(early) and all(torch.equal(x, y) for x, y in zip(snaps, early))
