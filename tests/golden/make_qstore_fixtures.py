"""Generate the on-disk QStore fixtures from the reference implementation.

Run in a container that has the reference sources (path given as the first argument or the
MRUN_REFERENCE_SRC environment variable); the outputs are committed, so the tests need no
reference at run time:

* ``qstore_small/``: a small int8 store written in the reference's block layout (qrow
  blocks, fp32 extras and an alias) by ``mrun_b200.qstore_build.write_qstore``;
* ``qstore.npz``: what the reference's CPU path returns for it -- ``QStore.weight`` for
  every qrow block, ``QStore.fp32``, ``QStore.embed_rows`` -- opened as a legacy-schema store
  so that no provenance digests are required;
* ``qstore_layout_cases.json``: manifest and file corruptions of that store with the
  reference layout validator's verdict on each ("ok" or its error text).
"""
from __future__ import annotations

import copy
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def build_small_store(directory: Path) -> dict:
    sys.path.insert(0, str(REPO))
    from mrun_b200.qstore_build import write_qstore

    rng = np.random.default_rng(20261202)

    def qrow(rows, cols):
        w = rng.standard_normal((rows, cols)).astype(np.float32)
        scale = np.abs(w).max(axis=1) / 127.0
        codes = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
        return codes, scale.astype(np.float32)

    qrows = {
        "model.embed_tokens.weight": qrow(100, 64),
        "model.layers.0.self_attn.q_proj.weight": qrow(48, 64),
        "model.layers.0.mlp.down_proj.weight": qrow(64, 80),
        "model.layers.0.mlp.up_proj.weight": qrow(80, 64),
    }
    fp32 = {
        "model.norm.weight": (1.0 + 0.1 * rng.standard_normal(64)).astype(np.float32),
        "model.layers.0.self_attn.q_proj.bias": rng.standard_normal(48).astype(np.float32),
    }
    return write_qstore(directory, qrows=qrows, fp32=fp32, aliases={"lm_head.weight": "model.embed_tokens.weight"},
                        config={"hidden_size": 64, "vocab_size": 100}, model_name="qstore_small")


def layout_cases(manifest: dict) -> list[dict]:
    """(name, manifest edit, file edit) triples for the layout validator."""
    q = "model.layers.0.self_attn.q_proj.weight"
    e = "model.norm.weight"
    cases = [{"name": "valid", "edit": []}]

    def add(name, edit, files=None):
        cases.append({"name": name, "edit": edit, "files": files or []})

    add("weight length mismatch", [["set", q, "w_len", manifest["blocks"][q]["w_len"] + 1]])
    add("scale offset misaligned", [["set", q, "s_off", manifest["blocks"][q]["s_off"] + 2]])
    add("overlapping weight ranges", [["set", q, "w_off", max(0, manifest["blocks"][q]["w_off"] - 8)]])
    add("gap in weights", [["set", q, "w_off", manifest["blocks"][q]["w_off"] + 16]])
    add("fp32 length mismatch", [["set", e, "e_len", 12]])
    add("unknown kind", [["set", e, "kind", "int4"]])
    add("alias to missing block", [["alias", "lm_head.weight", "nope"]])
    add("alias cycle", [["alias", "a.weight", "b.weight"], ["alias", "b.weight", "a.weight"]])
    add("negative offset", [["set", q, "w_off", -1]])
    add("non-integer length", [["set", q, "w_len", 3.5]])
    add("shape with zero", [["set", q, "shape", [0, 64]]])
    add("wrong dtype", [["top", "dtype", "int4"]])
    add("no fp32 blocks", [["drop_kind", "fp32"]])
    add("weights file too long", [], [["append", "weights.i8", 16]])
    add("scales file truncated", [], [["truncate", "scales.f32", 4]])
    add("extras file missing", [], [["remove", "extras.f32"]])
    return cases


def apply_case(src: Path, dst: Path, case: dict) -> None:
    shutil.copytree(src, dst)
    manifest = json.loads((dst / "manifest.json").read_text())
    for op in case["edit"]:
        if op[0] == "set":
            manifest["blocks"][op[1]][op[2]] = op[3]
        elif op[0] == "alias":
            manifest["blocks"][op[1]] = {"alias": op[2]}
        elif op[0] == "top":
            manifest[op[1]] = op[2]
        elif op[0] == "drop_kind":
            manifest["blocks"] = {k: v for k, v in manifest["blocks"].items() if v.get("kind") != op[1]}
    (dst / "manifest.json").write_text(json.dumps(manifest))
    for op in case.get("files", []):
        path = dst / op[1]
        if op[0] == "append":
            with path.open("ab") as f:
                f.write(b"\0" * op[2])
        elif op[0] == "truncate":
            data = path.read_bytes()
            path.write_bytes(data[: len(data) - op[2]])
        elif op[0] == "remove":
            path.unlink()


def main() -> None:
    ref_src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MRUN_REFERENCE_SRC")
    if not ref_src:
        raise SystemExit("usage: make_qstore_fixtures.py <reference src directory>")
    sys.path.insert(0, ref_src)
    import torch
    from mrun.engine.kernels import qstore as ref

    store_dir = HERE / "qstore_small"
    if store_dir.exists():
        shutil.rmtree(store_dir)
    manifest = build_small_store(store_dir)

    # verdicts of the reference validator
    verdicts = []
    for case in layout_cases(manifest):
        with tempfile.TemporaryDirectory() as tmp:
            case_dir = Path(tmp) / "store"
            apply_case(store_dir, case_dir, case)
            try:
                ref._validate_int8_layout(case_dir, json.loads((case_dir / "manifest.json").read_text()))
                verdict = "ok"
            except Exception as exc:  # the reference raises RuntimeError (or KeyError/TypeError)
                verdict = f"{type(exc).__name__}: {exc}"
        verdicts.append({**case, "verdict": verdict})
    (HERE / "qstore_layout_cases.json").write_text(json.dumps(verdicts, indent=1) + "\n")

    # the reference CPU reader on a legacy-schema copy (no provenance digests needed)
    with tempfile.TemporaryDirectory() as tmp:
        legacy = Path(tmp) / "qstore_small"
        shutil.copytree(store_dir, legacy)
        man = json.loads((legacy / "manifest.json").read_text())
        man["schema_version"] = "mrun-qstore-int8-v2"
        (legacy / "manifest.json").write_text(json.dumps(man))
        store = ref.QStore("qstore_small", root=Path(tmp), explicit_device="cpu", enable_prefetch_ring=False)
        out = {}
        for name, block in manifest["blocks"].items():
            kind = block.get("kind")
            key = name.replace(".", "_")
            if kind == "qrow" or "alias" in block:
                out["weight__" + key] = store.weight(name).numpy().astype(np.float32)
            elif kind == "fp32":
                out["fp32__" + key] = store.fp32(name).numpy().astype(np.float32)
        ids = np.array([3, 99, 0, 3, 57], dtype=np.int64)
        out["embed_ids"] = ids
        out["embed_rows"] = store.embed_rows("model.embed_tokens.weight", ids).to(torch.float32).numpy()
        store.close()
    np.savez_compressed(HERE / "qstore.npz", **out)
    print(f"wrote {store_dir}, {len(verdicts)} layout cases, {len(out)} arrays")


if __name__ == "__main__":
    main()
