"""ridgefill_attn_kv_fill on B200 against the CPU oracle (oracle/ridgefill_oracle.cpp oracle_attn_kv_fill): the
whole cache bit for bit (k rows after k_norm and rope, v rows copied, every row no slot names untouched), k_out
bit for bit, over the three rope modes, one- and three-plane positions, bf16 and f32 k_norm weights, odd head
counts, a full-width rotation, an interleaved cache layout, in-place k_out, and the layer shape (2 kv heads x 256
at T = 32,768), where two calls over the halves of the rows write what one call writes."""
import numpy as np
import pytest

import harness as H
from harness import abi

pytestmark = pytest.mark.gpu


def _case(seed, T, hkv, n_slots, three=False, w_f32=False, skip_every=7):
    rng = np.random.default_rng(seed)
    d = {
        "k": H.f32_to_bf16_bits((3 * rng.standard_normal((T, hkv, 256))).astype(np.float32)),
        "v": H.f32_to_bf16_bits(rng.standard_normal((T, hkv, 256)).astype(np.float32)),
        "w": (1 + 0.1 * rng.standard_normal(256)).astype(np.float32),
        "pos": (rng.integers(0, 40000, (3, T)) if three else np.arange(500, 500 + T)).astype(np.int32),
        "slots": rng.permutation(n_slots)[:T].astype(np.int32),
        "cache": rng.integers(0, 1 << 16, (2, n_slots, hkv, 256)).astype(np.uint16),
    }
    if not w_f32:
        d["w"] = H.f32_to_bf16_bits(d["w"])
    if skip_every:
        d["slots"][::skip_every] = -1
        d["slots"][1] = n_slots + 3        # outside the pool: nothing stored
    return d


def _params(T, hkv, R, theta=1e7, mode=None, sections=None, eps=None):
    p = [H.pint("M", T), H.pint("n_head_kv", hkv), H.pint("head_dim", 256), H.pint("rope_dim", R),
         H.pf64("rope_theta", theta)]
    if eps is not None:
        p.append(H.pf64("eps", eps))
    if mode is not None:
        p.append(H.pstr("rope_mode", mode))
    if sections is not None:
        p.append(H.pstr("rope_sections", sections))
    return p


def _run(product_lib, torch, d, params, k_out=False, cache=None, in_place=False):
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    K, V = t16(d["k"]), t16(d["v"])
    W = torch.from_numpy(d["w"].view(np.int16) if d["w"].dtype == np.uint16 else d["w"]).cuda()
    P = torch.from_numpy(d["pos"]).cuda()
    S = torch.from_numpy(d["slots"]).cuda()
    C = cache if cache is not None else t16(d["cache"])
    KO = K if in_place else (torch.full_like(K, 0x5A5A) if k_out else None)
    ops = [H.dev(K, abi.BF16), H.dev(V, abi.BF16), H.dev(W, abi.BF16 if d["w"].dtype == np.uint16 else abi.F32), H.dev(P),
           H.dev(S), H.dev(C, abi.BF16), H.dev(KO, abi.BF16) if KO is not None else abi.absent()]
    rc = H.launch(product_lib, "ridgefill_attn_kv_fill", ops, params)
    u16 = lambda t: t.cpu().numpy().view(np.uint16)   # noqa: E731
    return rc, u16(C), (u16(KO) if KO is not None else None)


def _check(d, got, R, theta=1e7, mode="neox", sections=(0, 0, 0), eps=1e-6):
    rc, cache, ko = got
    assert rc == abi.OK
    want, want_ko = H.oracle_attn_kv(d["k"], d["v"], d["w"], d["pos"], d["slots"], d["cache"], R, theta, eps=eps, mode=mode,
                                     sections=sections, k_out=ko is not None)
    assert np.array_equal(cache[1], want[1]), "v plane"
    diff = cache[0] != want[0]
    assert not diff.any(), f"k plane: {int(diff.sum())} elements differ"
    if ko is not None:
        assert np.array_equal(ko, want_ko), "k_out"


def test_neox_one_plane(cuda, product_lib):
    torch = cuda
    d = _case(1, 300, 2, 400)
    _check(d, _run(product_lib, torch, d, _params(300, 2, 64)), 64)


def test_imrope_three_planes_f32_weight_k_out(cuda, product_lib):
    torch = cuda
    d = _case(2, 1000, 2, 1100, three=True, w_f32=True)
    got = _run(product_lib, torch, d, _params(1000, 2, 64, mode="imrope", sections="11,11,10"), k_out=True)
    _check(d, got, 64, mode="imrope", sections=(11, 11, 10))


def test_mrope_full_rotation_odd_heads(cuda, product_lib):
    """rope_dim = head_dim (every element rotates), three kv heads (a warp's second head batch holds one), the
    sections consecutive, written in brackets, and a non-default eps and theta."""
    torch = cuda
    d = _case(3, 257, 3, 300, three=True)
    got = _run(product_lib, torch, d, _params(257, 3, 256, theta=1e6, mode="mrope", sections="[40, 44, 44]", eps=1e-5),
               k_out=True)
    _check(d, got, 256, theta=1e6, mode="mrope", sections=(40, 44, 44), eps=1e-5)


def test_three_planes_plain_rope_reads_plane_zero(cuda, product_lib):
    torch = cuda
    d = _case(4, 200, 1, 256, three=True)
    _check(d, _run(product_lib, torch, d, _params(200, 1, 32)), 32)


def test_in_place_k_out_and_interleaved_cache(cuda, product_lib):
    """k_out = k itself (the in-tree k is normalised and rotated in place), and a cache kept per slot as
    [slots, 2, Hkv, D] (k and v of a slot adjacent) passed as the [2, slots, Hkv, D] view."""
    torch = cuda
    T, hkv, n = 500, 2, 640
    d = _case(5, T, hkv, n)
    inter = torch.from_numpy(np.ascontiguousarray(d["cache"].transpose(1, 0, 2, 3)).view(np.int16)).cuda()
    view = inter.permute(1, 0, 2, 3)
    rc, _, ko = _run(product_lib, torch, d, _params(T, hkv, 64), cache=view, in_place=True)
    got = inter.permute(1, 0, 2, 3).cpu().numpy().view(np.uint16)
    _check(d, (rc, got, ko), 64)


def test_layer_shape_and_split_calls(cuda, product_lib):
    """2 kv heads x 256 at T = 32,768 (the attention layers of the late stack): against the oracle, and the two
    halves of the rows as two calls (row views of every per-row operand) write the same cache bit for bit."""
    torch = cuda
    T, hkv, n = 32768, 2, 40000
    d = _case(6, T, hkv, n, three=True, skip_every=97)
    params = _params(T, hkv, 64, mode="imrope", sections="11,11,10")
    got = _run(product_lib, torch, d, params, k_out=True)
    _check(d, got, 64, mode="imrope", sections=(11, 11, 10))
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    K, V, W = t16(d["k"]), t16(d["v"]), t16(d["w"])
    P, S, C = torch.from_numpy(d["pos"]).cuda(), torch.from_numpy(d["slots"]).cuda(), t16(d["cache"])
    h = T // 2
    for r0, r1 in ((0, h), (h, T)):
        ops = [H.dev(K[r0:r1], abi.BF16), H.dev(V[r0:r1], abi.BF16), H.dev(W, abi.BF16), H.dev(P[:, r0:r1]),
               H.dev(S[r0:r1]), H.dev(C, abi.BF16), abi.absent()]
        assert H.launch(product_lib, "ridgefill_attn_kv_fill", ops,
                        _params(r1 - r0, hkv, 64, mode="imrope", sections="11,11,10")) == abi.OK
    assert np.array_equal(C.cpu().numpy().view(np.uint16), got[1])


def test_refusals(cuda, product_lib):
    torch = cuda
    T, hkv = 64, 2
    d = _case(7, T, hkv, 80)
    t16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()   # noqa: E731
    K, V, W = t16(d["k"]), t16(d["v"]), t16(d["w"])
    P, S, C = torch.from_numpy(d["pos"]).cuda(), torch.from_numpy(d["slots"]).cuda(), t16(d["cache"])

    def call(params, k=K, c=C, w_dtype=abi.BF16):
        ops = [H.dev(k, abi.BF16), H.dev(V, abi.BF16), H.dev(W, w_dtype), H.dev(P), H.dev(S), H.dev(c, abi.BF16),
               abi.absent()]
        return H.launch(product_lib, "ridgefill_attn_kv_fill", ops, params)

    assert call(_params(T, hkv, 64)) == abi.OK
    assert call(_params(T, hkv, 72)) == abi.E_UNSUPPORTED                               # rope_dim not a multiple of 16
    assert call(_params(T, hkv, 64, mode="imrope", sections="11,11,11")) == abi.E_INVAL  # sections sum != 32
    assert call(_params(T, hkv, 64, mode="yarn")) == abi.E_INVAL
    assert call(_params(T, hkv, 64, theta=0.5)) == abi.E_INVAL
    assert call(_params(T, hkv, 64), w_dtype=abi.I32) == abi.E_DTYPE
    assert call(_params(T + 1, hkv, 64)) == abi.E_SHAPE
    wide = torch.zeros((2, 80, hkv, 264), dtype=torch.int16, device="cuda")[:, :, :, :256]   # head pitch 528 B
    assert call(_params(T, hkv, 64), c=wide) == abi.OK
    odd = torch.zeros((2 * 80 * hkv * 256 + 4,), dtype=torch.int16, device="cuda")[4:].view(2, 80, hkv, 256)
    assert call(_params(T, hkv, 64), c=odd) == abi.E_STRIDE                             # base 8 bytes off
    narrow = torch.zeros((2, 80, hkv, 260), dtype=torch.int16, device="cuda")[:, :, :, :256]  # head pitch 520 B
    assert call(_params(T, hkv, 64), c=narrow) == abi.E_STRIDE
    assert call(_params(T, hkv, 64), k=K[:, :1]) == abi.E_SHAPE
