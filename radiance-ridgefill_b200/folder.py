"""The projector folder through the library's C API (include/ridgefill_folder.h): read and checked as the
reference's arch plugin reads it (arch/ridgefill_folder.h:246-293, arch/ridgefill_projector.h:84-129), then held
resident in HBM in one device block instead of the reference's host block and per-pass VRAM ring
(arch/ridgefill_projector.h:10-18, 282-336).

    folder = ProjectorFolder(path)                      # RuntimeError naming the file when it is damaged
    folder.check(geom)                                  # (split, int8) or RuntimeError naming what does not fit
    res = folder.upload(geom, stream=torch.cuda.current_stream().cuda_stream)
    w, scale, bias = res.map(layer)                     # RadTensors: ridgefill_gemm_nt_q's operands 2 and 3
"""
from __future__ import annotations

import ctypes as C

import ridgefill_abi as abi


class ModelGeom(C.Structure):
    _fields_ = [("n_embd", C.c_int64), ("wide", C.c_int64), ("n_layer", C.c_int64), ("split_lo", C.c_int64),
                ("n_vocab", C.c_int64), ("st_heads", C.c_int64), ("st_sd0", C.c_int64), ("st_sd1", C.c_int64),
                ("full", C.POINTER(C.c_uint8))]


def geometry(n_embd, wide, n_layer, split_lo, n_vocab, st_heads, st_sd0, st_sd1, full=None) -> ModelGeom:
    """The model's facts. `full`: per-layer flags (1 = full-attention layer, no correction), or None to take
    them from the manifest's "layers"."""
    g = ModelGeom(n_embd, wide, n_layer, split_lo, n_vocab, st_heads, st_sd0, st_sd1, None)
    if full is not None:
        g._full = (C.c_uint8 * len(full))(*[1 if f else 0 for f in full])
        g.full = C.cast(g._full, C.POINTER(C.c_uint8))
    return g


def _bind(lib):
    if getattr(lib, "_folder_bound", False):
        return lib
    P, i64, s = C.c_void_p, C.c_int64, C.c_size_t
    T = C.POINTER(abi.RadTensor)
    G = C.POINTER(ModelGeom)
    lib.ridgefill_folder_open.argtypes = [C.c_char_p, C.POINTER(P), C.c_char_p, s]
    lib.ridgefill_folder_close.argtypes = [P]
    lib.ridgefill_folder_close.restype = None
    lib.ridgefill_folder_tensor.argtypes = [P, C.c_char_p, T]
    lib.ridgefill_folder_tensor_count.argtypes = [P]
    lib.ridgefill_folder_tensor_count.restype = i64
    lib.ridgefill_folder_file_bytes.argtypes = [P]
    lib.ridgefill_folder_file_bytes.restype = i64
    lib.ridgefill_folder_check.argtypes = [P, G, C.POINTER(i64), C.POINTER(C.c_int), C.c_char_p, s]
    lib.ridgefill_folder_upload.argtypes = [P, G, i64, i64, P, C.POINTER(P), C.c_char_p, s]
    lib.ridgefill_resident_free.argtypes = [P]
    lib.ridgefill_resident_free.restype = None
    lib.ridgefill_resident_bytes.argtypes = [P]
    lib.ridgefill_resident_bytes.restype = i64
    lib.ridgefill_resident_map.argtypes = [P, i64, T, T, T]
    lib.ridgefill_resident_correction.argtypes = [P, i64, T]
    lib.ridgefill_resident_table.argtypes = [P, C.c_char_p, T]
    lib.ridgefill_resident_final.argtypes = [P, T, T]
    lib._folder_bound = True
    return lib


class FolderError(RuntimeError):
    def __init__(self, code: int, why: str):
        super().__init__(why)
        self.code = code


class ProjectorFolder:
    def __init__(self, path, plugin: abi.Plugin | None = None):
        self.lib = _bind((plugin or abi.product()).lib)
        self.h = C.c_void_p()
        why = C.create_string_buffer(1024)
        rc = self.lib.ridgefill_folder_open(str(path).encode(), C.byref(self.h), why, len(why))
        if rc != abi.OK:
            self.h = C.c_void_p()
            raise FolderError(rc, why.value.decode(errors="replace"))

    def close(self):
        if self.h:
            self.lib.ridgefill_folder_close(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        self.close()

    @property
    def tensor_count(self) -> int:
        return self.lib.ridgefill_folder_tensor_count(self.h)

    @property
    def file_bytes(self) -> int:
        return self.lib.ridgefill_folder_file_bytes(self.h)

    def tensor(self, name: str) -> abi.RadTensor | None:
        t = abi.RadTensor()
        return t if self.lib.ridgefill_folder_tensor(self.h, name.encode(), C.byref(t)) == abi.OK else None

    def check(self, geom: ModelGeom) -> tuple[int, bool]:
        split, int8 = C.c_int64(), C.c_int()
        why = C.create_string_buffer(1024)
        rc = self.lib.ridgefill_folder_check(self.h, C.byref(geom), C.byref(split), C.byref(int8), why, len(why))
        if rc != abi.OK:
            raise FolderError(rc, why.value.decode(errors="replace"))
        return split.value, bool(int8.value)

    def upload(self, geom: ModelGeom, stream: int | None = None, head_first: int = 0, n_heads: int = -1) -> "Resident":
        h = C.c_void_p()
        why = C.create_string_buffer(1024)
        rc = self.lib.ridgefill_folder_upload(self.h, C.byref(geom), head_first, n_heads,
                                              C.c_void_p(stream) if stream else None, C.byref(h), why, len(why))
        if rc != abi.OK:
            raise FolderError(rc, why.value.decode(errors="replace"))
        return Resident(self.lib, h)


class Resident:
    """The folder in one device block; its views stay valid until free()."""

    def __init__(self, lib, h):
        self.lib, self.h = lib, h

    def free(self):
        if self.h:
            self.lib.ridgefill_resident_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        self.free()

    @property
    def bytes(self) -> int:
        return self.lib.ridgefill_resident_bytes(self.h)

    def map(self, layer: int):
        w, s, b = abi.RadTensor(), abi.RadTensor(), abi.RadTensor()
        if self.lib.ridgefill_resident_map(self.h, layer, C.byref(w), C.byref(s), C.byref(b)) != abi.OK:
            return None
        return w, (s if s.data else None), b

    def correction(self, layer: int) -> abi.RadTensor | None:
        t = abi.RadTensor()
        return t if self.lib.ridgefill_resident_correction(self.h, layer, C.byref(t)) == abi.OK else None

    def table(self, name: str) -> abi.RadTensor | None:
        t = abi.RadTensor()
        return t if self.lib.ridgefill_resident_table(self.h, name.encode(), C.byref(t)) == abi.OK else None

    def final(self):
        w, b = abi.RadTensor(), abi.RadTensor()
        return (w, b) if self.lib.ridgefill_resident_final(self.h, C.byref(w), C.byref(b)) == abi.OK else None
