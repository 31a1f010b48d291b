"""The projector folder resident in HBM (ridgefill_folder_upload) on B200: every uploaded piece equal to the folder's
bytes in the GEMM row's stored form (codes as they lie, the bf16 scale plane widened to f32 and transposed, the bias,
a rank's span of correction heads, the row tables, the final map), and the projector GEMMs run straight from the
resident block equal, bit for bit, the same GEMMs on operands staged from the folder by hand (int8: also the
oracle). The folders are the reference-made ones under tests/golden/ and synthetic ones with a final map."""
import sys
from pathlib import Path

import numpy as np
import pytest

import harness as H
from harness import abi

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "radiance-ridgefill_b200"))
import folder as F  # noqa: E402
from test_folder import GEOM, GOLDEN, small_folder, st_bytes, view_bytes, write_folder  # noqa: E402

pytestmark = pytest.mark.gpu

NP = {abi.F32: np.float32, abi.BF16: np.uint16, abi.I8: np.int8}
TORCH_CODE = {abi.F32: "<f4", abi.BF16: "<i2", abi.I8: "|i1"}


class _DeviceArray:
    """A device pointer with a shape, readable by torch through __cuda_array_interface__."""

    def __init__(self, t: abi.RadTensor):
        shape = tuple(t.shape[i] for i in range(t.rank))
        self.__cuda_array_interface__ = {"shape": shape, "typestr": TORCH_CODE[t.dtype], "data": (t.data, False),
                                         "version": 2}


def fetch(torch, t: abi.RadTensor) -> np.ndarray:
    a = torch.as_tensor(_DeviceArray(t), device="cuda").cpu().numpy()
    return a.view(NP[t.dtype]) if t.dtype == abi.BF16 else a


def host(f: F.ProjectorFolder, name: str) -> np.ndarray:
    t = f.tensor(name)
    return np.frombuffer(view_bytes(t), NP[t.dtype]).reshape([t.shape[i] for i in range(t.rank)])


def test_int8_folder_uploads_in_the_stored_form(cuda, product_lib):
    torch = cuda
    f = F.ProjectorFolder(GOLDEN / "folder_i8")
    g = F.geometry(**GEOM)
    r = f.upload(g, stream=torch.cuda.current_stream().cuda_stream)
    assert r.bytes >= 3 * (16 * 256 + 2 * 16 * 4 + 32)
    for layer in (4, 5, 6):
        w, s, b = r.map(layer)
        assert w.dtype == abi.I8 and s.dtype == abi.F32 and b.dtype == abi.BF16
        assert np.array_equal(fetch(torch, w), host(f, f"proj.{layer}.codes"))
        scale = H.bf16_bits_to_f32(host(f, f"proj.{layer}.scale"))
        assert np.array_equal(fetch(torch, s), np.ascontiguousarray(scale.T))
        assert np.array_equal(fetch(torch, b), host(f, f"proj.{layer}.bias"))
    assert r.map(3) is None and r.map(7) is None
    for layer in (4, 6):
        assert np.array_equal(fetch(torch, r.correction(layer)), host(f, f"st.{layer}"))
    assert r.correction(5) is None   # a full-attention layer keeps none
    for name in ("score", "score_none", "score_all"):
        assert np.array_equal(fetch(torch, r.table(name)), host(f, name))
    assert r.final() is None
    r2 = f.upload(g, stream=torch.cuda.current_stream().cuda_stream, head_first=1, n_heads=1)   # a rank's span
    assert np.array_equal(fetch(torch, r2.correction(6)), host(f, "st.6")[1:2])
    with pytest.raises(F.FolderError, match="heads"):
        f.upload(g, head_first=1, n_heads=2)
    r.free()
    r2.free()


def test_int8_gemm_runs_from_the_resident_block(cuda, product_lib):
    """ridgefill_gemm_nt_q_bias on the resident codes, scale and bias = the oracle on the folder's canonical planes
    = the row on operands staged by hand."""
    torch = cuda
    f = F.ProjectorFolder(GOLDEN / "folder_i8")
    r = f.upload(F.geometry(**GEOM), stream=torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(11)
    M, N, K = 300, 16, 256
    a = rng.integers(-127, 128, (M, K)).astype(np.int8)
    sa = rng.uniform(1e-3, 1e-2, (M, K // 128)).astype(np.float32)
    A, SA = torch.from_numpy(a).cuda(), torch.from_numpy(sa).cuda()
    for layer in (4, 5, 6):
        w, s, b = r.map(layer)
        Y = torch.full((M, N), 0x5A5A, dtype=torch.int16, device="cuda")
        rc = H.launch(product_lib, "ridgefill_gemm_nt_q_bias",
                      [H.dev(A), H.dev(SA), w, s, b, H.dev(Y, abi.BF16), abi.absent()], H.gemm_params(M, N, K, 128))
        assert rc == abi.OK
        scale_kn = np.ascontiguousarray(H.bf16_bits_to_f32(host(f, f"proj.{layer}.scale")).T)
        want = H.oracle_gemm(a, sa, host(f, f"proj.{layer}.codes"), scale_kn, bias=host(f, f"proj.{layer}.bias"), group=128)
        got = Y.cpu().numpy().view(np.uint16)
        assert np.array_equal(got, want), layer
        B = torch.from_numpy(host(f, f"proj.{layer}.codes").copy()).cuda()
        SB = torch.from_numpy(scale_kn).cuda()
        BI = torch.from_numpy(host(f, f"proj.{layer}.bias").view(np.int16).copy()).cuda()
        Y2 = torch.full((M, N), 0x5A5A, dtype=torch.int16, device="cuda")
        assert H.launch(product_lib, "ridgefill_gemm_nt_q_bias",
                        [H.dev(A), H.dev(SA), H.dev(B), H.dev(SB), H.dev(BI, abi.BF16), H.dev(Y2, abi.BF16), abi.absent()],
                        H.gemm_params(M, N, K, 128)) == abi.OK
        assert torch.equal(Y, Y2)
    r.free()


def test_bf16_folder_and_final_map_run_from_the_resident_block(cuda, product_lib, tmp_path):
    """A bf16 folder with an MTP final map: ridgefill_gemm_nt_bias on the resident map and bias (and on the final
    map) = the same row on copies staged by hand, bit for bit; the views equal the folder's bytes."""
    torch = cuda
    files, manifest = small_folder(np.random.default_rng(12), int8=False, final=True)
    write_folder(tmp_path, files, manifest)
    f = F.ProjectorFolder(tmp_path)
    r = f.upload(F.geometry(**GEOM), stream=torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(13)
    M = 200
    for layer, (w, b), N in [(4, r.map(4)[::2], 16), (6, r.map(6)[::2], 16), (None, r.final(), 256)]:
        name = f"proj.{layer}" if layer is not None else "final"
        assert np.array_equal(fetch(torch, w), host(f, f"{name}.weight"))
        assert np.array_equal(fetch(torch, b), host(f, f"{name}.bias"))
        a = H.f32_to_bf16_bits(rng.standard_normal((M, 256)).astype(np.float32))
        A = torch.from_numpy(a.view(np.int16)).cuda()
        params = [H.pint("M", M), H.pint("N", N), H.pint("K", 256), H.pstr("dtype", "bf16")]
        Y = torch.zeros((M, N), dtype=torch.int16, device="cuda")
        assert H.launch(product_lib, "ridgefill_gemm_nt_bias", [H.dev(A, abi.BF16), w, b, abi.absent(), H.dev(Y, abi.BF16)],
                        params) == abi.OK
        W2 = torch.from_numpy(host(f, f"{name}.weight").view(np.int16).copy()).cuda()
        B2 = torch.from_numpy(host(f, f"{name}.bias").view(np.int16).copy()).cuda()
        Y2 = torch.zeros((M, N), dtype=torch.int16, device="cuda")
        assert H.launch(product_lib, "ridgefill_gemm_nt_bias", [H.dev(A, abi.BF16), H.dev(W2, abi.BF16), H.dev(B2, abi.BF16),
                                                                abi.absent(), H.dev(Y2, abi.BF16)], params) == abi.OK
        assert torch.equal(Y, Y2)
    assert r.map(5)[1] is None   # bf16 maps have no scale plane
    r.free()


def test_a_folder_the_row_cannot_store_is_refused_before_allocating(cuda, product_lib, tmp_path):
    """n_embd 24 is not a multiple of the stored form's 16 rows: the upload names the layer (before allocating)."""
    torch = cuda
    files, manifest = small_folder(np.random.default_rng(14))
    for layer in (4, 5, 6):   # re-shape every map to 24 rows
        rng = np.random.default_rng(layer)
        files[f"proj8.L{layer}.safetensors"] = st_bytes({
            f"proj.{layer}.codes": ("I8", (24, 256), rng.integers(-127, 128, (24, 256)).astype(np.int8).tobytes()),
            f"proj.{layer}.scale": ("BF16", (24, 2), H.f32_to_bf16_bits(np.full((24, 2), 0.01, np.float32)).tobytes()),
            f"proj.{layer}.bias": ("BF16", (24,), bytes(48))})
    write_folder(tmp_path, files, manifest)
    with pytest.raises(F.FolderError, match="cannot store proj.4") as e:
        F.ProjectorFolder(tmp_path).upload(F.geometry(**dict(GEOM, n_embd=24)),
                                           stream=torch.cuda.current_stream().cuda_stream)
    assert e.value.code == abi.E_UNSUPPORTED
