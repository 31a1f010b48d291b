"""Regenerate the golden fixtures under tests/golden/ from the reference checkout (read-only).

    python tests/golden/make_golden.py --reference <reference checkout>   (or RIDGEFILL_REFERENCE in the environment)

Writes:
  rho_numpy.txt       the reference's own rho fixture, produced by running its tests/rho_ref.py (the NumPy
                      closed form of the +st rho) -- byte-identical to tests/fixtures/rho_numpy.txt.
  rowsel_keys.json    the reference's rowsel_quick9 fixture (tests/fixtures/rowsel_quick9.json, format
                      ridgefill-rowsel-fixture-1) with every token id replaced by a unique synthetic id that
                      carries the same table score. ridgefill_mask's class rule reads a row only through
                      score[token_id], so the kept rows are unchanged; the real-text ids are not copied.
  quantise_i8.npz     tools/ridgefill_projector.py quantise_i8 (the folder's i8*bf16[1x128] encoder) applied
                      to seeded weights: inputs and the reference's codes and scales.
  folder_bf16/        a small bf16 projector folder (late layers 4..6 of 7, n_embd 16, stream width 256, the
                      correction on the recurrent layers 4 and 6, the three row tables over 40 ids), its
                      manifest's hashes by the reference's own sha256_file.
  folder_i8/          the reference's `ridgefill_projector.py int8` run on folder_bf16: its proj8 files
                      (codes, bf16 scales, bias), the correction and row tables re-stamped, and its manifest.
These files are the only place the reference's outputs enter this repository; tests read them, never
the reference itself.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def rho_fixture(ref: Path) -> None:
    out = subprocess.run([sys.executable, str(ref / "tests" / "rho_ref.py")], check=True, capture_output=True, text=True)
    (HERE / "rho_numpy.txt").write_text(out.stdout)


def rowsel_fixture(ref: Path) -> None:
    fx = json.loads((ref / "tests" / "fixtures" / "rowsel_quick9.json").read_text())
    table = dict(zip(fx["kept_ids"], fx["kept_scores"]))
    docs, kept_ids, kept_scores, next_id = [], [], [], 0
    for doc in fx["docs"]:
        ids = []
        for tok in doc["token_ids"]:
            ids.append(next_id)
            if tok in table:
                kept_ids.append(next_id)
                kept_scores.append(table[tok])
            next_id += 1
        docs.append({"doc": doc["doc"], "k": doc["k"], "token_ids": ids, "rows": doc["rows"]})
    derived = {"format": fx["format"], "window": fx["window"], "share": fx["share"], "vocab": next_id,
               "kept_ids": kept_ids, "kept_scores": kept_scores, "docs": docs,
               "derived_from": "tests/fixtures/rowsel_quick9.json (ids replaced, scores and kept rows kept)"}
    (HERE / "rowsel_keys.json").write_text(json.dumps(derived, separators=(",", ":")) + "\n")


def quantise_fixture(ref: Path) -> None:
    import torch
    spec = importlib.util.spec_from_file_location("ridgefill_projector", ref / "tools" / "ridgefill_projector.py")
    sys.path.insert(0, str(ref / "tools"))
    sys.path.insert(0, str(ref / "tools" / "dev"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(20261201)
    w = (rng.standard_normal((48, 512)) * np.exp(rng.uniform(-4, 2, (48, 1)))).astype(np.float32)
    w[3, 128:256] = 0.0                       # an all-zero group: scale 1
    w[5, :128] = np.round(w[5, :128] * 4) / 4  # exact halves: round-half-even ties
    wb = torch.from_numpy(w).to(torch.bfloat16)
    codes, scale, _ = mod.quantise_i8(wb)
    np.savez_compressed(HERE / "quantise_i8.npz", w_bf16=wb.view(torch.int16).numpy().view(np.uint16),
                        codes=codes.numpy(), scale=scale.view(torch.int16).numpy().view(np.uint16))


def folder_fixture(ref: Path) -> None:
    import shutil
    import torch
    sys.path.insert(0, str(ref / "tools"))
    sys.path.insert(0, str(ref / "tools" / "dev"))
    spec = importlib.util.spec_from_file_location("ridgefill_projector", ref / "tools" / "ridgefill_projector.py")
    P = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(P)
    src, out = HERE / "folder_bf16", HERE / "folder_i8"
    for d in (src, out):
        if d.exists():
            shutil.rmtree(d)
    src.mkdir()
    gen = torch.Generator().manual_seed(20261202)
    layers = (4, 5, 6)
    for layer in layers:
        w = torch.randn(16, 256, generator=gen) * torch.exp(torch.rand(16, 1, generator=gen) * 4 - 2)
        if layer == 5:
            w[2, 128:] = 0.0   # an all-zero group: scale 1
        P.save({f"proj.{layer}.weight": w.to(torch.bfloat16),
                f"proj.{layer}.bias": torch.randn(16, generator=gen).to(torch.bfloat16)}, src / f"proj.L{layer}.safetensors")
    P.save({"st.4": torch.randn(2, 8, 8, generator=gen), "st.6": torch.randn(2, 8, 8, generator=gen)},
           src / "correction.safetensors")
    P.save({"score": torch.randn(40, generator=gen), "score_none": torch.full((40,), float("-inf")),
            "score_all": torch.zeros(40)}, src / "rowsel.safetensors")
    (src / "README.md").write_text("a small projector folder for the loader's tests\n")
    names = [f"proj.L{layer}.safetensors" for layer in layers] + ["correction.safetensors", "rowsel.safetensors"]
    manifest = {"format": 1, "adapter": "qwen4exp", "split": 4, "stream_width": 256, "block_in_width": 16,
                "layers": {"4": "recurrent", "5": "full_attn", "6": "recurrent"},
                "correction": {"kind": "gdn_terminal_state", "heads": 2, "sd": [8, 8], "layers": [4, 6]},
                "projector": {"dtype": "bf16", "layout": "plain_nk",
                              "files": {str(layer): f"proj.L{layer}.safetensors" for layer in layers}},
                "files": {n: P.S.sha256_file(src / n) for n in sorted(names)}}
    (src / "ridgefill.json").write_text(json.dumps(manifest, indent=1) + "\n")
    assert P.main(["int8", "--from", str(src), "--out", str(out)]) == 0


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RIDGEFILL_REFERENCE"), required="RIDGEFILL_REFERENCE" not in os.environ)
    ref = Path(ap.parse_args().reference)
    rho_fixture(ref)
    rowsel_fixture(ref)
    quantise_fixture(ref)
    folder_fixture(ref)
    for p in sorted(HERE.iterdir()):
        print(p.name, p.stat().st_size)
