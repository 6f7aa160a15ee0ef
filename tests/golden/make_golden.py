"""Generates the golden fixtures in this directory from the reference's own
Python modules: run with DNAGPT_REFERENCE_TREE naming the reference tree
(the fixtures are committed; the tree is not needed later).

  plain_block_t8.npz  fhe/realweights/manual.py block_reference on the seeded
                      synthetic block (seed 3, T = 8) -- pins oracle/plain_block.py
  plain_head.npz      fhe/multiblock/manual.py classifier_head_reference on
                      seeded synthetic head weights and hidden states (seed
                      11 weights, seed 12 hidden, 4 tokens) with a two-row
                      readout [N, A] -- pins oracle/plain_block.py head()
  fixture_small/      a two-block + head fixture directory written by the
                      reference's own array writer (fhe/multiblock/export_fixture.py
                      _write_array, manifest "arrays" table) from seeded synthetic
                      weights at D = 16, MLP = 64, T = 3 -- pins the fixture loader
  simd_layout_b32.json + simd_layout_b32.npz
                      fhe/gpu_real_scheme_b/simd_layout.py at batch width 32,
                      one copy (the 32-tokens-per-ciphertext layout): slot map,
                      lane shift, active alignments and protocol / operation
                      counts at T = 103, a reduced-size BSGS transform and
                      score / context tiles.
"""

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("DNAGPT_REFERENCE_TREE", "")
if not REF or not os.path.isdir(REF):
    sys.exit("set DNAGPT_REFERENCE_TREE to the reference tree (fhe/ lies under it)")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(REF, "fhe", "gpu_real_scheme_b"))
sys.path.insert(0, os.path.join(REF, "fhe", "realweights"))

import manual  # noqa: E402  (reference: fhe/realweights/manual.py)
import simd_layout as sl  # noqa: E402  (reference: fhe/gpu_real_scheme_b/simd_layout.py)

from oracle.plain_block import synthetic_head_weights, synthetic_input, synthetic_weights  # noqa: E402
from tests.golden.inputs import layout_inputs  # noqa: E402


def plain_block():
    w = synthetic_weights(3)
    x = synthetic_input(4, 8)
    ref = manual.block_reference(x, {"ln1": w["ln1"], "attn_qkv": w["attn_qkv"], "attn_proj": w["attn_proj"],
                                     "ln2": w["ln2"], "mlp_fc": w["mlp_fc"], "mlp_proj": w["mlp_proj"]})
    np.savez_compressed(os.path.join(HERE, "plain_block_t8.npz"), seed_weights=3, seed_input=4,
                        block_output=ref["block_output"], ln1_output=ref["ln1_output"],
                        attention_scores=ref["attention_scores"], residual1=ref["residual1"])


def plain_head():
    import importlib.util
    spec = importlib.util.spec_from_file_location("multiblock_manual",
                                                  os.path.join(REF, "fhe", "multiblock", "manual.py"))
    mb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mb)  # reference: fhe/multiblock/manual.py
    hw = synthetic_head_weights(11)
    rng = np.random.default_rng(13)
    r_a = rng.normal(0.0, 0.02, hw["readout"].shape[0])
    readout_rows = np.stack([hw["readout"] + r_a, r_a])  # rows N and A: N - A = readout
    hidden = synthetic_input(12, 4)
    ref = mb.classifier_head_reference(hidden, {"final_ln": hw["final_ln"], "head_linear": hw["head_linear"],
                                                "head_ln": hw["head_ln"], "head_readout": readout_rows})
    np.savez_compressed(os.path.join(HERE, "plain_head.npz"), seed_weights=11, seed_hidden=12, seed_readout_a=13,
                        readout_rows=readout_rows, logits=ref["logits"], head_ln_output=ref["head_ln_output"],
                        margin=ref["logits"][:, 0] - ref["logits"][:, 1])


def fixture_small():
    import shutil
    from collections import OrderedDict

    sys.path.insert(0, REF)
    import fhe.multiblock.export_fixture as ef  # reference: fhe/multiblock/export_fixture.py
    from pathlib import Path
    out = Path(HERE) / "fixture_small"
    shutil.rmtree(out, ignore_errors=True)
    out.mkdir()
    arrays = OrderedDict()
    blocks = [synthetic_weights(60 + b, d=16, mlp=64) for b in range(2)]
    head = synthetic_head_weights(62, d=16)
    for b, w in enumerate(blocks):
        for f in ("ln1", "attn_qkv", "attn_proj", "ln2", "mlp_fc", "mlp_proj"):
            ef._write_array(out, f"weights.block{b}.{f}", w[f], "synthetic", arrays)
    ef._write_array(out, "weights.final_ln", head["final_ln"], "synthetic", arrays)
    ef._write_array(out, "weights.head_linear", head["head_linear"], "synthetic", arrays)
    ef._write_array(out, "weights.head_ln", head["head_ln"], "synthetic", arrays)
    ef._write_array(out, "weights.head_readout_margin_n_minus_a", head["readout"], "synthetic", arrays)
    ef._write_array(out, "input.embeddings", synthetic_input(63, 3, d=16), "synthetic", arrays)
    with (out / "manifest.json").open("x", encoding="utf-8") as f:
        json.dump({"schema": "synthetic test fixture", "seeds": {"blocks": [60, 61], "head": 62, "input": 63},
                   "arrays": arrays}, f, indent=2, allow_nan=False)


def layout():
    B, T = 32, 103
    out = {"batch_width": B, "tokens": T, "copies": 1}
    out["slots"] = [[c, f, t, sl.physical_slot(c, f, t, B, copies=1)] for c, f, t in
                    [(0, 0, 0), (0, 0, 31), (0, 1, 0), (0, 767, 5), (0, 1023, 31)]]
    groups = -(-T // B)
    out["active_weight_shifts"] = {
        f"{qg},{kg}": list(sl.active_weight_shifts(qg * B, min(B, T - qg * B), kg * B, min(B, T - kg * B), B))
        for qg in range(groups) for kg in range(qg + 1)}
    pc = sl.protocol_counts(T, B)
    out["protocol_counts"] = {k: getattr(pc, k) for k in ("token_groups", "score_tile_decryptions",
                                                          "weight_tile_encryptions", "layernorm1_crossings",
                                                          "layernorm2_crossings", "gelu_crossings")}
    sc = sl.server_operation_counts(T, B)
    out["server_operation_counts"] = {k: getattr(sc, k) for k in sc.__dataclass_fields__}
    vals = np.arange(19 * B, dtype=np.float64)
    arrays = {"lane_shift_in": vals}
    for d in (0, 1, 5, 31, -3):
        arrays[f"lane_shift_{d}"] = sl.lane_shift(vals, d, B)
    tok, W, q, k, weights, values = layout_inputs()
    # reduced BSGS: dimension 48 padded to 64, 8 baby steps, one copy
    arrays["bsgs_out"] = sl.bsgs_matmul_tokens(tok, W, B, dimension=48, pack_width=64, copies=1, bsgs_n1=8,
                                               max_complex_slots=64 * B)
    # score tile and context tiles at the block's head shape, one copy
    arrays["score_tile"] = sl.score_tile(q, k, B, copies=1)
    arrays["ctx_out"] = sl.context_from_weight_tiles(weights, values, B, copies=1)
    with open(os.path.join(HERE, "simd_layout_b32.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "simd_layout_b32.npz"), **arrays)


if __name__ == "__main__":
    plain_block()
    plain_head()
    fixture_small()
    layout()
    print("golden fixtures written")
