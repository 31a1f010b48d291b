"""Regenerate the golden fixtures under tests/golden/ from the reference checkout (read-only).

    python tests/golden/make_golden.py [--reference /root/reference]

Writes:
  rho_numpy.txt       the reference's own rho fixture, produced by running its tests/rho_ref.py (the NumPy
                      closed form of the +st rho) -- byte-identical to tests/fixtures/rho_numpy.txt.
  rowsel_keys.json    the reference's rowsel_quick9 fixture (tests/fixtures/rowsel_quick9.json, format
                      ridgefill-rowsel-fixture-1) with every token id replaced by a unique synthetic id that
                      carries the same table score. ridgefill_mask's class rule reads a row only through
                      score[token_id], so the kept rows are unchanged; the real-text ids are not copied.
  quantise_i8.npz     tools/ridgefill_projector.py quantise_i8 (the folder's i8*bf16[1x128] encoder) applied
                      to seeded weights: inputs and the reference's codes and scales.
These files are the only place the reference's outputs enter this repository; tests read them, never
the reference itself.
"""
from __future__ import annotations

import argparse
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


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ref = Path(ap.parse_args().reference)
    rho_fixture(ref)
    rowsel_fixture(ref)
    quantise_fixture(ref)
    for p in sorted(HERE.iterdir()):
        print(p.name, p.stat().st_size)
