"""Reader and writer of the reference's float64 fixture directories.

The reference exports the released DNAGPT weights, the encrypted-input
embeddings and its float64 oracle activations as a directory of headerless
little-endian float64 arrays plus `manifest.json`
(fhe/multiblock/export_fixture.py:79-106, export_fixture_t103.py:250-470):

  manifest["arrays"][name] = {"file": name with "." -> "__" + ".bin",
                              "dtype": "float64", "endianness": "little",
                              "order": "C", "shape": [...], "elements": n,
                              "bytes": 8 n, "sha256": hex, "role": text}

with names `weights.block{L}.{ln1,attn_qkv,attn_proj,ln2,mlp_fc,mlp_proj}`
(PyTorch [out, in] layout), `weights.final_ln`, `weights.head_linear`,
`weights.head_ln`, `weights.head_readout_margin_n_minus_a`,
`input.embeddings` ([T, D]) and `oracle.*`.  `load_fixture` reads such a
directory (checking size and SHA-256 of every array) into the weight
dictionaries `EncryptedBlock`, `EncryptedHead` and `EncryptedModel` take;
`export_fixture` writes the same format.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import numpy as np

BLOCK_FIELDS = ("ln1", "attn_qkv", "attn_proj", "ln2", "mlp_fc", "mlp_proj")


def array_filename(name: str) -> str:
    return name.replace(".", "__").replace("/", "_") + ".bin"


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


class FixtureError(ValueError):
    pass


class Fixture:
    """A loaded fixture directory: `arrays` maps names to float64 arrays."""

    def __init__(self, directory, verify: bool = True):
        self.directory = Path(directory)
        with (self.directory / "manifest.json").open(encoding="utf-8") as f:
            self.manifest = json.load(f)
        if "arrays" not in self.manifest:
            raise FixtureError("manifest has no 'arrays' table")
        self.arrays: dict[str, np.ndarray] = {}
        for name, meta in self.manifest["arrays"].items():
            if meta.get("dtype", "float64") != "float64" or meta.get("endianness", "little") != "little" \
                    or meta.get("order", "C") != "C":
                raise FixtureError(f"{name}: only little-endian C-order float64 arrays are supported")
            path = self.directory / meta["file"]
            shape = tuple(int(v) for v in meta["shape"])
            n = int(np.prod(shape)) if shape else 1
            if path.stat().st_size != 8 * n or int(meta.get("bytes", 8 * n)) != 8 * n:
                raise FixtureError(f"{name}: file holds {path.stat().st_size} bytes, shape {shape} needs {8 * n}")
            if verify and "sha256" in meta and _sha256(path) != meta["sha256"]:
                raise FixtureError(f"{name}: SHA-256 differs from the manifest")
            self.arrays[name] = np.fromfile(path, dtype="<f8").reshape(shape)

    def __contains__(self, name: str) -> bool:
        return name in self.arrays

    def __getitem__(self, name: str) -> np.ndarray:
        return self.arrays[name]

    @property
    def num_blocks(self) -> int:
        n = 0
        while f"weights.block{n}.ln1" in self.arrays:
            n += 1
        return n

    def block_weights(self, layer: int) -> dict:
        return {f: self.arrays[f"weights.block{layer}.{f}"] for f in BLOCK_FIELDS}

    def head_weights(self) -> dict | None:
        names = ("weights.final_ln", "weights.head_linear", "weights.head_ln",
                 "weights.head_readout_margin_n_minus_a")
        if not all(n in self.arrays for n in names):
            return None
        return {"final_ln": self.arrays[names[0]], "head_linear": self.arrays[names[1]],
                "head_ln": self.arrays[names[2]], "readout": self.arrays[names[3]]}

    def embeddings(self) -> np.ndarray:
        return self.arrays["input.embeddings"]


def load_fixture(directory, verify: bool = True) -> Fixture:
    return Fixture(directory, verify)


def export_fixture(directory, arrays: dict, roles: dict | None = None, extra: dict | None = None) -> Path:
    """Write `arrays` (name -> array) as a fixture directory; returns the
    manifest path.  The directory must not contain a manifest yet."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    manifest_path = d / "manifest.json"
    if manifest_path.exists():
        raise FixtureError(f"{manifest_path} exists")
    table = {}
    for name, value in arrays.items():
        a = np.ascontiguousarray(np.asarray(value, dtype="<f8"))
        if a.size == 0 or not np.isfinite(a).all():
            raise FixtureError(f"refusing to export empty/non-finite array {name}")
        path = d / array_filename(name)
        with path.open("xb") as f:
            a.tofile(f)
            f.flush()
            os.fsync(f.fileno())
        table[name] = {"file": path.name, "role": (roles or {}).get(name, ""), "dtype": "float64",
                       "endianness": "little", "order": "C", "shape": list(a.shape), "elements": int(a.size),
                       "bytes": int(a.nbytes), "sha256": _sha256(path)}
    meta = dict(extra or {})
    meta["format"] = {"description": "Headerless little-endian float64 arrays; reshape in C row-major order "
                                     "using the recorded shape.", "export_dtype": "float64",
                      "endianness": "little", "order": "C"}
    meta["arrays"] = table
    with manifest_path.open("x", encoding="utf-8") as f:
        json.dump(meta, f, indent=2, allow_nan=False)
    return manifest_path


def model_arrays(blocks: list, head: dict | None = None, embeddings: np.ndarray | None = None) -> dict:
    """Fixture array names for block weight dicts, head weights and inputs."""
    out = {}
    for layer, w in enumerate(blocks):
        for f in BLOCK_FIELDS:
            out[f"weights.block{layer}.{f}"] = w[f]
    if head is not None:
        out["weights.final_ln"] = head["final_ln"]
        out["weights.head_linear"] = head["head_linear"]
        out["weights.head_ln"] = head["head_ln"]
        out["weights.head_readout_margin_n_minus_a"] = head["readout"]
    if embeddings is not None:
        out["input.embeddings"] = embeddings
    return out
