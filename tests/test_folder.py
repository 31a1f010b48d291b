"""The projector folder reader and checker (include/ridgefill_folder.h) on the CPU: the reference-made folders under
tests/golden/ (folder_i8 is the reference tool's own `int8` output) read with every manifest hash matching and every
tensor view equal to the bytes its safetensors header names; the SHA-256 against hashlib over the block-boundary lengths;
the reference loader's refusals (tests/arch_static_test.cpp:3374-3445: a missing listed file, a changed file, a
format other than 1, a name outside the folder, a tensor in two files, an unlisted README that changes nothing)
and the model checks of arch/ridgefill_projector.h:84-129 (split, dtype, map shapes, correction all or none, row
tables, the final map). No GPU: reading and checking allocate nothing on a device."""
import hashlib
import json
import shutil
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

import harness as H
from harness import abi

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "radiance-ridgefill_b200"))
import folder as F  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
GEOM = dict(n_embd=16, wide=256, n_layer=7, split_lo=1, n_vocab=40, st_heads=2, st_sd0=8, st_sd1=8)


@pytest.fixture(scope="module")
def lib():
    return H.product()


def st_bytes(tensors, metadata=None) -> bytes:
    """A safetensors file: {name: (dtype, shape, raw bytes)} in order."""
    header, data, off = {}, b"", 0
    if metadata:
        header["__metadata__"] = metadata
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        data += raw
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    return struct.pack("<Q", len(h)) + h + data


def write_folder(d: Path, files: dict, manifest: dict, listed=None):
    d.mkdir(parents=True, exist_ok=True)
    for name, raw in files.items():
        (d / name).write_bytes(raw)
    listed = files if listed is None else listed
    m = dict(manifest)
    m.setdefault("format", 1)
    m["files"] = {n: hashlib.sha256(files[n]).hexdigest() for n in listed}
    (d / "ridgefill.json").write_text(json.dumps(m))


def small_folder(rng, int8=True, layers=(4, 5, 6), full=(5,), st=(4, 6), tables=("score",), final=False):
    files, n, wide = {}, 16, 256
    for layer in layers:
        p = f"proj.{layer}"
        if int8:
            t = {f"{p}.codes": ("I8", (n, wide), rng.integers(-127, 128, (n, wide)).astype(np.int8).tobytes()),
                 f"{p}.scale": ("BF16", (n, wide // 128), H.f32_to_bf16_bits(rng.uniform(1e-3, 1e-2, (n, 2))).tobytes())}
        else:
            t = {f"{p}.weight": ("BF16", (n, wide), H.f32_to_bf16_bits(rng.standard_normal((n, wide))).tobytes())}
        t[f"{p}.bias"] = ("BF16", (n,), H.f32_to_bf16_bits(rng.standard_normal(n)).tobytes())
        files[f"proj{'8' if int8 else ''}.L{layer}.safetensors"] = st_bytes(t)
    files["correction.safetensors"] = st_bytes({f"st.{l}": ("F32", (2, 8, 8), rng.standard_normal((2, 8, 8)).astype(np.float32).tobytes())
                                                for l in st})
    files["rowsel.safetensors"] = st_bytes({t: ("F32", (40,), rng.standard_normal(40).astype(np.float32).tobytes()) for t in tables})
    manifest = {"split": layers[0], "layers": {str(l): "full_attn" if l in full else "recurrent" for l in layers},
                "projector": {"dtype": "i8" if int8 else "bf16"}}
    if final:
        files["final.safetensors"] = st_bytes({"final.weight": ("BF16", (wide, wide), H.f32_to_bf16_bits(rng.standard_normal((wide, wide))).tobytes()),
                                               "final.bias": ("BF16", (wide,), H.f32_to_bf16_bits(rng.standard_normal(wide)).tobytes())})
        manifest["final"] = {"file": "final.safetensors"}
    return files, manifest


def _header(path: Path):
    raw = path.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    return json.loads(raw[8:8 + n])


def view_bytes(t: abi.RadTensor) -> bytes:
    import ctypes
    n = int(np.prod([t.shape[i] for i in range(t.rank)]))
    width = {abi.F32: 4, abi.BF16: 2, abi.I8: 1, abi.I32: 4}[t.dtype]
    return ctypes.string_at(t.data, n * width)


@pytest.mark.parametrize("which,int8", [("folder_i8", True), ("folder_bf16", False)])
def test_reference_made_folder_reads_and_checks(lib, which, int8):
    d = GOLDEN / which
    f = F.ProjectorFolder(d)
    manifest = json.loads((d / "ridgefill.json").read_text())
    names = [n for n in manifest["files"] if n.endswith(".safetensors")]
    want = {}
    for n in names:
        h = _header(d / n)
        raw = (d / n).read_bytes()
        base = 8 + struct.unpack("<Q", raw[:8])[0]
        for k, v in h.items():
            if k != "__metadata__":
                want[k] = (v["dtype"], v["shape"], raw[base + v["data_offsets"][0]:base + v["data_offsets"][1]])
    assert f.tensor_count == len(want)
    codes = {"I8": abi.I8, "BF16": abi.BF16, "F32": abi.F32}
    for k, (dt, shape, raw) in want.items():
        t = f.tensor(k)
        assert t is not None and t.dtype == codes[dt] and [t.shape[i] for i in range(t.rank)] == shape, k
        assert view_bytes(t) == raw, k
    split, is8 = f.check(F.geometry(**GEOM))
    assert split == 4 and is8 == int8
    assert f.tensor("proj.5.weight" if int8 else "proj.5.codes") is None
    if int8:   # the reference's own quantiser wrote these: its scale rule, and an all-zero group scaled by 1
        s = np.frombuffer(view_bytes(f.tensor("proj.5.scale")), np.uint16).reshape(16, 2)
        assert H.bf16_bits_to_f32(s[2, 1]) == 1.0


@pytest.mark.parametrize("size", [1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 127, 128, 129, 1000, 65536, 1 << 20])
def test_sha256_matches_hashlib_at_every_padding_boundary(lib, tmp_path, size):
    raw = np.random.default_rng(size).integers(0, 256, size).astype(np.uint8).tobytes()
    write_folder(tmp_path, {"blob.bin": raw}, {})
    F.ProjectorFolder(tmp_path)   # opens only when our digest equals hashlib's
    (tmp_path / "blob.bin").write_bytes(raw[:-1] + bytes([raw[-1] ^ 1]))
    with pytest.raises(F.FolderError, match="blob.bin is corrupt"):
        F.ProjectorFolder(tmp_path)


def _golden_copy(tmp_path):
    d = tmp_path / "f"
    shutil.copytree(GOLDEN / "folder_i8", d)
    return d


def test_damaged_folders_are_refused_by_name(lib, tmp_path):
    cases = [
        (lambda d: (d / "rowsel.safetensors").unlink(), "lists rowsel.safetensors, which is missing"),
        (lambda d: (d / "proj8.L5.safetensors").write_bytes(b"x" + (d / "proj8.L5.safetensors").read_bytes()[1:]),
         "proj8.L5.safetensors is corrupt"),
        (lambda d: (d / "ridgefill.json").write_text('{"format": 2, "files": {}}'), "format-1"),
        (lambda d: (d / "ridgefill.json").write_text('{"format": 1, "files": {}}'), "lists no files"),
        (lambda d: (d / "ridgefill.json").write_text('{"format": 1, "files": {"../x": "00"}}'), "lists ../x"),
        (lambda d: (d / "ridgefill.json").write_text('{"format": 1, "files": '), "does not parse"),
    ]
    for damage, said in cases:
        d = _golden_copy(tmp_path)
        damage(d)
        with pytest.raises(F.FolderError, match=said.replace(".", r"\.")) as e:
            F.ProjectorFolder(d)
        assert e.value.code == abi.E_INVAL
        shutil.rmtree(d)


def test_malformed_safetensors_are_refused_naming_the_tensor(lib, tmp_path):
    good = {"score": ("F32", (5,), bytes(20))}
    cases = [
        ({"a.safetensors": st_bytes(good), "b.safetensors": st_bytes(good)}, "'score' is in two files"),
        ({"a.safetensors": st_bytes({"score": ("F32", (6,), bytes(20))})}, "tensor 'score'"),
        ({"a.safetensors": st_bytes({"score": ("F64", (5,), bytes(40))})}, "tensor 'score'"),
        ({"a.safetensors": st_bytes(good)[:-4]}, "tensor 'score'"),                       # truncated data
        ({"a.safetensors": struct.pack("<Q", 9) + b'{"x": [1,'}, "header does not parse"),
        ({"a.safetensors": b"1234"}, "shorter than a safetensors header"),
    ]
    for i, (files, said) in enumerate(cases):
        d = tmp_path / f"c{i}"
        write_folder(d, files, {})
        with pytest.raises(F.FolderError, match=said):
            F.ProjectorFolder(d)


def test_an_unlisted_readme_is_not_read(lib, tmp_path):
    d = _golden_copy(tmp_path)
    (d / "README.md").write_text("---\nlicense: apache-2.0\n---\n# a model card")
    F.ProjectorFolder(d)
    (d / "README.md").unlink()
    F.ProjectorFolder(d)


def test_model_checks_name_what_cannot_run(lib, tmp_path):
    rng = np.random.default_rng(3)
    g = F.geometry(**GEOM)
    cases = [
        (dict(), None),
        (dict(int8=False), None),
        (dict(st=()), None),                                     # no correction at all: allowed
        (dict(tables=("score", "score_none", "score_all")), None),
        (dict(final=True), None),
        (dict(st=(4,)), "covers 1 of the 2"),
        (dict(layers=(5, 6), full=(5,), st=(6,)), None),
    ]
    for i, (kw, said) in enumerate(cases):
        files, manifest = small_folder(rng, **kw)
        d = tmp_path / f"m{i}"
        write_folder(d, files, manifest)
        f = F.ProjectorFolder(d)
        if said is None:
            f.check(g)
        else:
            with pytest.raises(F.FolderError, match=said):
                f.check(g)
    files, manifest = small_folder(rng)
    for i, (edit, said) in enumerate([
            (lambda m, fl: m.update(split=0), "its split 0 is not a late layer"),
            (lambda m, fl: m.update(split=7), "its split 7 is not a late layer"),
            (lambda m, fl: m["projector"].update(dtype="i4"), "'i4' is neither bf16 nor i8"),
            (lambda m, fl: m.update(final={"file": "x"}), "its final map is not"),
            (lambda m, fl: fl.update({"proj8.L6.safetensors": st_bytes({"proj.6.codes": ("I8", (16, 128), bytes(2048)),
                                                                         "proj.6.scale": ("BF16", (16, 1), bytes(32)),
                                                                         "proj.6.bias": ("BF16", (16,), bytes(32))})}),
             r"proj\.6\.codes i8 \[16, 256\]"),
            (lambda m, fl: fl.update({"rowsel.safetensors": st_bytes({"score_all": ("F32", (41,), bytes(164))})}),
             "the row table 'score_all' is not f32 \\[40\\]")]):
        m2, f2 = json.loads(json.dumps(manifest)), dict(files)
        edit(m2, f2)
        d = tmp_path / f"e{i}"
        write_folder(d, f2, m2)
        with pytest.raises(F.FolderError, match=said):
            F.ProjectorFolder(d).check(g)
    # the full-attention flags from the model override the manifest's: with 5 and 6 full the correction on 4 alone
    # is all of it; with none full it covers 1 of 3
    d = tmp_path / "flags"
    write_folder(d, *small_folder(rng, st=(4,)))
    F.ProjectorFolder(d).check(F.geometry(**GEOM, full=[0, 0, 0, 0, 0, 1, 1]))
    with pytest.raises(F.FolderError, match="covers 1 of the 3"):
        F.ProjectorFolder(d).check(F.geometry(**GEOM, full=[0] * 7))
